#!/usr/bin/env python3
"""Generate the committed golden vectors that pin the oracle (and through it the CUDA path) to the reference.

The reference's own dequant oracle is llama.cpp's gguf-py (engine/gpu/loom/tools/dq_bfp16_check.py:65:
quants.dequantize(...).astype(np.float16); engine/gpu/loom/tools/gemv_check.py:161-162: .astype(np.float64) @ x).
It is a third-party dependency the reference does not vendor or pin; this script ran against gguf 0.19.0.
It is run in the development container only (gguf-py and this script are never needed at test time):

    python tests/golden/make_golden.py

Per format (Q8_0, Q4_K, Q6_K, then Q5_K, Q3_K, IQ4_XS) it writes tests/golden/dequant_<fmt>.npz with
    blocks  uint8 [rows][row bytes]   the GGUF rows (seeded synthetic rows plus edge-case rows)
    K       int                       values per row
    f16     uint16 [rows][K]          gguf-py dequantize(...).astype(float16) bit patterns
    f32     float32 [rows][K]         gguf-py dequantize(...) (the f32 values before rounding)
and tests/golden/gemm_<fmt>.npz with a small token-major GEMM
    x       float16 [M][K]            activations
    y_f16w  float64 [M][N]            f16 dequant (as float64) @ x (the tile GEMM's reference)
    y_f32w  float64 [M][N]            f32 dequant (as float64) @ x (the GEMV's reference)
"""
import os
import sys

import numpy as np
from gguf import GGMLQuantizationType as T
from gguf import quants

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.abspath(os.path.join(HERE, "..", "..")))
import __graft_entry__ as ge  # noqa: E402

F = ge.load_package().formats

QT = {F.Q8_0: T.Q8_0, F.Q4_K: T.Q4_K, F.Q6_K: T.Q6_K, F.Q5_K: T.Q5_K, F.Q3_K: T.Q3_K, F.IQ4_XS: T.IQ4_XS}


def f16b(v):
    return np.array([v], np.float16).view(np.uint8)


def edge_rows(fmt, K, rng):
    """Hand-made rows: all zero, negative d, subnormal d, a d large enough to overflow f16, extreme quants."""
    rb = F.row_bytes(fmt, K)
    rows = []
    z = np.zeros(rb, np.uint8)
    rows.append(z.copy())
    for kind in ("neg", "sub", "huge", "ext"):
        r = rng.integers(0, 256, rb, dtype=np.uint8)
        if fmt == F.Q8_0:
            b = r.reshape(-1, 34)
            d = {"neg": -0.0123, "sub": 3.0e-6, "huge": 60000.0, "ext": 0.5}[kind]
            b[:, 0:2] = f16b(d)
            if kind == "ext":
                b[:, 2:] = np.where(np.arange(32) % 2, 0x80, 0x7F).astype(np.uint8)  # -128 and +127
        elif fmt == F.Q4_K:
            b = r.reshape(-1, 144)
            d, dm = {"neg": (-0.02, -0.007), "sub": (2.0e-6, 5.0e-7), "huge": (4000.0, 1.0), "ext": (0.03, 0.04)}[kind]
            b[:, 0:2] = f16b(d)
            b[:, 2:4] = f16b(dm)
            if kind == "ext":
                b[:, 4:16] = 0xFF            # every sc / m = 63
                b[:, 16:] = np.where(np.arange(128) % 2, 0xFF, 0x00).astype(np.uint8)
        elif fmt == F.Q5_K:
            b = r.reshape(-1, 176)
            d, dm = {"neg": (-0.02, -0.007), "sub": (2.0e-6, 5.0e-7), "huge": (4000.0, 1.0), "ext": (0.03, 0.04)}[kind]
            b[:, 0:2] = f16b(d)
            b[:, 2:4] = f16b(dm)
            if kind == "ext":
                b[:, 4:16] = 0xFF            # every sc / m = 63
                b[:, 16:48] = 0xFF           # every fifth bit set: quants 16..31
                b[:, 48:] = np.where(np.arange(128) % 2, 0xFF, 0x00).astype(np.uint8)
        elif fmt == F.Q3_K:
            b = r.reshape(-1, 110)
            d = {"neg": -0.015, "sub": 3.0e-6, "huge": 6000.0, "ext": 0.02}[kind]
            b[:, 108:110] = f16b(d)
            if kind == "ext":
                b[:, 96:108] = np.array([0x00, 0xFF] * 6, np.uint8)  # scales -32 and +31
                b[:, 0:32] = np.where(np.arange(32) % 2, 0xFF, 0x00).astype(np.uint8)
                b[:, 32:96] = np.where(np.arange(64) % 3, 0xFF, 0x00).astype(np.uint8)
            if kind == "sub":
                b[:, 96:104] = 0x00          # low scale bits 0 and high bits from random bytes: some scales 0
        elif fmt == F.IQ4_XS:
            b = r.reshape(-1, 136)
            d = {"neg": -0.015, "sub": 4.0e-6, "huge": 500.0, "ext": 0.02}[kind]
            b[:, 0:2] = f16b(d)
            if kind == "ext":
                b[:, 2:8] = np.array([0x00, 0x00, 0xFF, 0x00, 0xF0, 0x0F], np.uint8)  # scales -32, +31 and 0 mixed
                b[:, 8:] = np.where(np.arange(128) % 2, 0xFF, 0x00).astype(np.uint8)   # levels -127 and +113
            if kind == "neg":
                b[:, 2:4] = np.array([0xAA, 0xAA], np.uint8)  # high scale bits 2: with low bits 0, scale 0
                b[:, 4:8] = 0x00
        else:
            b = r.reshape(-1, 210)
            d = {"neg": -0.015, "sub": 4.0e-6, "huge": 50.0, "ext": 0.02}[kind]
            b[:, 208:210] = f16b(d)
            if kind == "huge":
                b[:, 192:208] = np.int8(-128).view(np.uint8)
            if kind == "ext":
                b[:, 192:208] = np.array([127, -128] * 8, np.int8).view(np.uint8)
                b[:, 0:128] = 0xFF
                b[:, 128:192] = 0xFF
        rows.append(b.reshape(rb))
    return np.stack(rows)


def main():
    rng = np.random.default_rng(20261201)
    for fmt in (F.Q8_0, F.Q4_K, F.Q6_K, F.Q5_K, F.Q3_K, F.IQ4_XS):
        name = F.NAMES[fmt].lower()
        K = 512
        syn = F.synth_weights(fmt, 8, K, seed=7 + fmt)
        blocks = np.concatenate([syn, edge_rows(fmt, K, rng)])
        rows = blocks.shape[0]
        f32 = np.stack([quants.dequantize(blocks[r], QT[fmt]).astype(np.float32) for r in range(rows)])
        with np.errstate(over="ignore"):
            f16 = f32.astype(np.float16)
        np.savez_compressed(os.path.join(HERE, f"dequant_{name}.npz"), blocks=blocks, K=K,
                            f16=f16.view(np.uint16), f32=f32)
        # GEMM: finite synthetic rows only
        N, M = 40, 7
        wq = F.synth_weights(fmt, N, K, seed=100 + fmt)
        x = F.synth_activations(M, K, seed=200 + fmt)
        w32 = np.stack([quants.dequantize(wq[r], QT[fmt]).astype(np.float32) for r in range(N)])
        w16 = w32.astype(np.float16)
        y16 = x.astype(np.float64) @ w16.astype(np.float64).T
        y32 = x.astype(np.float64) @ w32.astype(np.float64).T
        np.savez_compressed(os.path.join(HERE, f"gemm_{name}.npz"), blocks=wq, K=K, x=x, y_f16w=y16, y_f32w=y32)
        print(f"{name}: dequant rows {rows} K {K}; gemm M {M} N {N} K {K}")


if __name__ == "__main__":
    main()
