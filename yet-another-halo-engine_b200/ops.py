"""The quantised-linear operator, host side: the reference's kernel kinds over the C ABI.

Reference interface mirrored here:
  * tile GEMM kinds kstore / kres / swiglu (engine/gpu/loom/tools/gen_gemm_tile.py:309-322) dispatched by
    LoomPrefill::RunKstore / RunResidual / RunSwiglu (engine/model/loom_prefill.hpp:1954-2110): qgemm();
  * decode GEMV kinds plain / resid (engine/gpu/loom/tools/gen_gemv.py:16-19, LoomDecoder::Gemv
    engine/model/loom_decoder.hpp:415-439): qgemv();
  * the dequant kind (gen_gemm_tile.py:314-327): dequant().
Layouts: weights are GGUF rows [N][row bytes]; activations x f16 [M][K]; outputs token-major [M][N].
Arguments are checked twice: the footprint rule here refuses buffers smaller than the call touches (the
reference's hal_run refuses small bindings, engine/run/hal_run.cc:107-111), and the C ABI checks shapes,
alignment and kinds. Every call runs on the GPU; a missing library raises.

Two calling forms:
  *_ptr(...)  raw device pointers (the form the tensor-parallel layer, the tuner and bench.py use);
  qgemm(dev, w, fmt, x, ...) numpy in / numpy out convenience (uploads, runs, downloads, synchronises).
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import formats as F
from ._lib import EPI_RESID, EPI_STORE, EPI_SWIGLU, F16, F32, check, lib
from .device import Device, DeviceBuffer

KINDS = {"kstore": EPI_STORE, "store": EPI_STORE, "plain": EPI_STORE, "kres": EPI_RESID, "resid": EPI_RESID,
         "swiglu": EPI_SWIGLU}
DTYPES = {"f32": F32, "float32": F32, "f16": F16, "float16": F16}


def _epi(kind) -> int:
    if isinstance(kind, int):
        return kind
    if kind not in KINDS:
        raise ValueError(f"unknown kind {kind!r} (kstore, kres, swiglu)")
    return KINDS[kind]


def _dt(dtype) -> int:
    if isinstance(dtype, int):
        return dtype
    return DTYPES[str(np.dtype(dtype)) if not isinstance(dtype, str) else dtype]


def footprint(fmt, N, K, w_row_stride, kb_off, M, ldx, y_dtype, ldy):
    """(weight, input, output) bytes a call touches (yah_qgemm_footprint)."""
    wb, xb, yb = ctypes.c_int64(), ctypes.c_int64(), ctypes.c_int64()
    check(lib().yah_qgemm_footprint(F.type_of(fmt), N, K, w_row_stride, kb_off, M, ldx, _dt(y_dtype), ldy,
                                    ctypes.byref(wb), ctypes.byref(xb), ctypes.byref(yb)))
    return wb.value, xb.value, yb.value


# ----------------------------------------------------------------------------------------------- raw pointers
def qgemm_ptr(w, fmt, N, K, w_row_stride, kb_off, x, M, ldx, y, y_dtype, ldy, kind="kstore", aux=None, ldaux=0,
              stream=None, bn=0, grid=0, kchunk=0, pair=-1):
    """yah_qgemm (automatic tile: the installed tile table, else the built-in choice) unless a tile is given."""
    if bn == 0 and grid == 0 and kchunk == 0 and pair == -1:
        check(lib().yah_qgemm(w, F.type_of(fmt), N, K, w_row_stride, kb_off, x, M, ldx, y, _dt(y_dtype), ldy,
                              _epi(kind), aux, ldaux, stream))
        return
    check(lib().yah_qgemm_tile(w, F.type_of(fmt), N, K, w_row_stride, kb_off, x, M, ldx, y, _dt(y_dtype), ldy,
                               _epi(kind), aux, ldaux, bn, grid, kchunk, pair, stream))


def qgemv_ptr(w, fmt, N, K, w_row_stride, kb_off, x, M, ldx, y, y_dtype, ldy, kind="plain", aux=None, ldaux=0,
              stream=None):
    check(lib().yah_qgemv(w, F.type_of(fmt), N, K, w_row_stride, kb_off, x, M, ldx, y, _dt(y_dtype), ldy, _epi(kind),
                          aux, ldaux, stream))


def qgemv_x_ptr(w, fmt, N, K, w_row_stride, kb_off, x, M, ldx, y, y_dtype, ldy, kind="plain", aux=None, ldaux=0,
                stream=None, x_dtype="f32"):
    """yah_qgemv_x: the GEMV with the activations' element type chosen (ldx in elements of x_dtype)."""
    check(lib().yah_qgemv_x(w, F.type_of(fmt), N, K, w_row_stride, kb_off, x, _dt(x_dtype), M, ldx, y, _dt(y_dtype),
                            ldy, _epi(kind), aux, ldaux, stream))


def dequant_ptr(w, fmt, rows, K, w_row_stride, kb_off, out, ldo, stream=None):
    check(lib().yah_dequant(w, F.type_of(fmt), rows, K, w_row_stride, kb_off, out, ldo, stream))


# ----------------------------------------------------------------------------------------------- numpy helpers
def _as_dev(dev: Device, a):
    if isinstance(a, DeviceBuffer):
        return a
    return dev.upload(np.ascontiguousarray(a))


def _check_size(buf: DeviceBuffer, need: int, what: str):
    if buf.nbytes < need:
        raise ValueError(f"{what} buffer has {buf.nbytes} bytes, the call touches {need}")


def qgemm(dev: Device, w, fmt, x, N=None, K=None, kind="kstore", out_dtype="f32", aux=None, kb_off=0,
          w_row_stride=None, bn=0, grid=0, kchunk=0, pair=-1, gemv=False, x_dtype="f16"):
    """y[M][N] = kind(x @ W^T) on the GPU; w: uint8 GGUF rows (numpy or DeviceBuffer), x: f16 [M][K] numpy
    (f32 with x_dtype="f32", GEMV only)."""
    t = F.type_of(fmt)
    x32 = x_dtype == "f32"
    if x32 and not gemv:
        raise ValueError("f32 activations are a GEMV operand only")
    x = np.ascontiguousarray(x, dtype=np.float32 if x32 else np.float16)
    M = x.shape[0]
    K = K if K is not None else x.shape[1]
    if w_row_stride is None:
        w_row_stride = (w.shape[1] if isinstance(w, np.ndarray) else F.row_bytes(t, K + 256 * kb_off))
    N = N if N is not None else (w.shape[0] if isinstance(w, np.ndarray) else None)
    ep = _epi(kind)
    if ep == EPI_SWIGLU and not gemv:  # the tile GEMM's swiglu writes f16; the GEMV's f32 or f16
        out_dtype = "f16"
    if ep == EPI_RESID:
        out_dtype = "f32"
    ydt = _dt(out_dtype)
    wb, xb, yb = footprint(t, N, K, w_row_stride, kb_off, M, x.shape[1], ydt, N)
    wd = _as_dev(dev, w)
    _check_size(wd, wb, "weight")
    xd = dev.upload(x)
    yd = dev.empty(yb)
    auxd = None
    if ep != EPI_STORE:
        auxd = dev.upload(np.ascontiguousarray(aux, dtype=np.float32))
        _check_size(auxd, M * N * 4, "aux")
    fn = qgemv_ptr if gemv else qgemm_ptr
    kw = {} if gemv else {"bn": bn, "grid": grid, "kchunk": kchunk, "pair": pair}
    if x32:
        fn, kw = qgemv_x_ptr, {"x_dtype": "f32"}
    fn(wd.ptr, t, N, K, w_row_stride, kb_off, xd.ptr, M, x.shape[1], yd.ptr, ydt, N, ep,
       auxd.ptr if auxd else None, N if auxd else 0, **kw)
    dev.synchronize()
    y = yd.download(np.float16 if ydt == F16 else np.float32, (M, N))
    code = dev.status_word()
    if code:
        raise RuntimeError(f"kernel reported bounded-wait failure code {code}")
    return y


def qgemv(dev: Device, w, fmt, x, N=None, K=None, kind="plain", out_dtype="f32", aux=None, kb_off=0,
          w_row_stride=None, x_dtype="f16"):
    """Decode GEMV for M <= 32 tokens: same arguments as qgemm (kinds plain / resid / swiglu; swiglu writes the
    chosen out_dtype); x_dtype="f32" passes x as f32, the reference GEMV's operand type."""
    return qgemm(dev, w, fmt, x, N=N, K=K, kind=kind, out_dtype=out_dtype, aux=aux, kb_off=kb_off,
                 w_row_stride=w_row_stride, gemv=True, x_dtype=x_dtype)


def qgemv_swiglu_ptr(w_gate, gate_fmt, gate_row_stride, w_up, up_fmt, up_row_stride, N, K, x, M, ldx, y, ldy,
                     stream=None):
    """yah_qgemv_swiglu: y (f32) = silu(x W_gate^T) * (x W_up^T), the reference GEMV's swiglu kind (gen_gemv.py:18);
    the two tensors may differ in format."""
    check(lib().yah_qgemv_swiglu(w_gate, F.type_of(gate_fmt), gate_row_stride, w_up, F.type_of(up_fmt), up_row_stride,
                                 N, K, x, M, ldx, y, ldy, stream))


def qgemm_ffn_ptr(w_gate, w_up, fmt, N, K, w_row_stride, kb_off, x, M, ldx, y, ldy, bn=0, pair=-1, stream=None):
    """yah_qgemm_ffn: y (f16) = silu(x W_gate^T) * (x W_up^T), one tile GEMM."""
    check(lib().yah_qgemm_ffn(w_gate, w_up, F.type_of(fmt), N, K, w_row_stride, kb_off, x, M, ldx, y, ldy, bn, pair,
                              stream))


def qgemm_ffn(dev: Device, w_gate, w_up, fmt, x, N=None, K=None, kb_off=0, w_row_stride=None, bn=0, pair=-1):
    """The fused gate+up SwiGLU (the reference's ffn kind) on numpy inputs: f16 [M][N]."""
    t = F.type_of(fmt)
    x = np.ascontiguousarray(x, dtype=np.float16)
    M = x.shape[0]
    K = K if K is not None else x.shape[1]
    N = N if N is not None else w_gate.shape[0]
    if w_row_stride is None:
        w_row_stride = w_gate.shape[1] if isinstance(w_gate, np.ndarray) else F.row_bytes(t, K + 256 * kb_off)
    gd, ud, xd = _as_dev(dev, w_gate), _as_dev(dev, w_up), dev.upload(x)
    yd = dev.empty(M * N * 2)
    qgemm_ffn_ptr(gd.ptr, ud.ptr, t, N, K, w_row_stride, kb_off, xd.ptr, M, x.shape[1], yd.ptr, N, bn, pair)
    dev.synchronize()
    y = yd.download(np.float16, (M, N))
    code = dev.status_word()
    if code:
        raise RuntimeError(f"kernel reported bounded-wait failure code {code}")
    return y


def realign(dev: Device, w, stride: int | None = None, stream=None):
    """Copy GGUF rows (numpy [N][row_bytes] or a DeviceBuffer of packed rows) into rows `stride` bytes apart
    (default: row_bytes rounded up to 16), as TMA needs; returns (DeviceBuffer, stride). For tensors whose packed
    rows are not 16-byte multiples, e.g. Q6_K at K = 5120 (4200-byte rows)."""
    src = _as_dev(dev, w)
    rows, row_bytes = (w.shape[0], w.shape[1]) if isinstance(w, np.ndarray) else (None, None)
    if rows is None:
        raise ValueError("pass the host array (its shape gives rows and row bytes)")
    stride = stride or (row_bytes + 15) // 16 * 16
    dst = dev.empty(rows * stride)
    check(lib().yah_realign_rows(src.ptr, rows, row_bytes, row_bytes, dst.ptr, stride, stream))
    if stream is None:
        dev.synchronize()
    if src is not w:
        src.close()
    return dst, stride


def dequant(dev: Device, w, fmt, N=None, K=None, kb_off=0, w_row_stride=None) -> np.ndarray:
    """f16 [N][K] of GGUF rows w with the GEMM's decode (bit-exact to the reference dequant)."""
    t = F.type_of(fmt)
    if w_row_stride is None:
        w_row_stride = w.shape[1]
    N = N if N is not None else w.shape[0]
    wd = _as_dev(dev, w)
    out = dev.empty(N * K * 2)
    dequant_ptr(wd.ptr, t, N, K, w_row_stride, kb_off, out.ptr, K)
    dev.synchronize()
    return out.download(np.float16, (N, K))
