"""CPU oracle of the quantised-linear path: TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg (and its reference arm) may import this
module, and only as the checker; the product path never calls it and has no CPU fallback.

Pieces:
  * dequant_f16 / dequant_f32: ctypes over oracle/_build/liboracle.so, the C restatement of the reference's decode
    (yah_oracle.c cites gen_gemm_decode.py line by line). f16 = the tile GEMM's weights (bit-exact target);
    f32 = gguf-py's dequantize output, the reference GEMV's oracle weights (gemv_check.py:161-162).
  * gemm_ref: float64 (dequant @ x^T), the reference's checker arithmetic (gemv_check.py:161-162), laid out as the
    engine's token-major output [M][N] (gen_gemm_tile.py:1230-1231).
  * the fused epilogues of the reference kinds (gen_gemm_tile.py:309-318): kres (resid + W x) and swiglu
    (f16(silu(gate) * W x)), in float64.
  * error metrics: max-abs, relative Frobenius, and max error over max |ref| (gemv_check.py:176).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "liboracle.so")
_lib = None


def build() -> str:
    """Compile the C restatement (make in oracle/); returns the library path."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < os.path.getmtime(
                os.path.join(HERE, "yah_oracle.c")):
            build()
        L = ctypes.CDLL(LIB_PATH)
        i64 = ctypes.c_int64
        for name, outp in (("yah_oracle_dequant_f32", ctypes.c_void_p), ("yah_oracle_dequant_f16", ctypes.c_void_p)):
            fn = getattr(L, name)
            fn.argtypes = [ctypes.c_int, ctypes.c_void_p, i64, i64, i64, i64, outp]
            fn.restype = ctypes.c_int
        L.yah_oracle_superblock_bytes.argtypes = [ctypes.c_int]
        L.yah_oracle_superblock_bytes.restype = ctypes.c_int
        L.yah_oracle_f32_to_f16.argtypes = [ctypes.c_float]
        L.yah_oracle_f32_to_f16.restype = ctypes.c_uint16
        _lib = L
    return _lib


def _prep(w: np.ndarray, row_stride):
    w = np.ascontiguousarray(w)
    if w.dtype != np.uint8:
        w = w.view(np.uint8)
    if row_stride is None:
        row_stride = w.shape[1] if w.ndim == 2 else w.size
    return w, int(row_stride)


def dequant_f16(fmt: int, w: np.ndarray, rows: int, K: int, row_stride=None, kb_off: int = 0) -> np.ndarray:
    """f16 [rows][K] (as np.float16) of GGUF rows w (uint8 [rows][row_stride]) from super-block kb_off."""
    w, rs = _prep(w, row_stride)
    out = np.empty((rows, K), np.uint16)
    rc = lib().yah_oracle_dequant_f16(int(fmt), w.ctypes.data, rows, K, rs, kb_off, out.ctypes.data)
    if rc:
        raise ValueError(f"oracle dequant rejected type {fmt} K {K}")
    return out.view(np.float16)


def dequant_f32(fmt: int, w: np.ndarray, rows: int, K: int, row_stride=None, kb_off: int = 0) -> np.ndarray:
    """f32 [rows][K] before the f16 rounding (gguf-py's dequantize values)."""
    w, rs = _prep(w, row_stride)
    out = np.empty((rows, K), np.float32)
    rc = lib().yah_oracle_dequant_f32(int(fmt), w.ctypes.data, rows, K, rs, kb_off, out.ctypes.data)
    if rc:
        raise ValueError(f"oracle dequant rejected type {fmt} K {K}")
    return out


def gemm_ref(w_deq: np.ndarray, x: np.ndarray) -> np.ndarray:
    """float64 token-major y[M][N] = x[M][K] @ W[N][K]^T."""
    return x.astype(np.float64) @ w_deq.astype(np.float64).T


def epilogue_ref(acc: np.ndarray, epilogue: int, aux=None) -> np.ndarray:
    """float64 epilogue of the reference kinds: 0 kstore, 1 kres (aux = resid), 2 swiglu (aux = gate)."""
    if epilogue == 0:
        return acc
    if epilogue == 1:
        return aux.astype(np.float64) + acc
    if epilogue == 2:
        g = aux.astype(np.float64)
        return g / (1.0 + np.exp(-g)) * acc
    raise ValueError(epilogue)


def errors(y: np.ndarray, ref: np.ndarray) -> dict:
    """max-abs, relative Frobenius, and max |y - ref| / max |ref| (gemv_check.py:176)."""
    y = y.astype(np.float64)
    ref = ref.astype(np.float64)
    d = y - ref
    nref = float(np.linalg.norm(ref))
    mref = float(np.max(np.abs(ref))) if ref.size else 0.0
    return {
        "max_abs": float(np.max(np.abs(d))) if d.size else 0.0,
        "rel_fro": float(np.linalg.norm(d) / nref) if nref > 0 else float(np.linalg.norm(d)),
        "rel_max": float(np.max(np.abs(d)) / mref) if mref > 0 else 0.0,
        "finite": bool(np.all(np.isfinite(y))),
    }


def f16_half_ulp(ref: np.ndarray) -> np.ndarray:
    """Half the f16 spacing at each |ref| (the rounding bound of an f16 output)."""
    a = np.abs(ref).astype(np.float16)
    nxt = np.nextafter(a, np.float16(np.inf))
    return (nxt.astype(np.float64) - a.astype(np.float64)) * 0.5
