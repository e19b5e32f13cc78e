"""GGUF block-quant formats on the quantised-linear path, and the seeded synthetic tensors the benchmarks use.

Format traits follow the reference's type table (engine/core/gguf.cpp:27-35, engine/core/gguf.hpp:49-50):

    type    GGML id  elements/block  bytes/block   bytes per 256-element super-block
    Q8_0        8         32              34             272 (8 blocks, gen_gemm_decode.py:1338-1339)
    Q3_K       11        256             110             110
    Q4_K       12        256             144             144
    Q5_K       13        256             176             176
    Q6_K       14        256             210             210
    IQ4_XS     23        256             136             136

A weight tensor is stored exactly as GGUF lays it out (engine/model/weights.hpp:140-152): N rows (GGUF ne1), each
row K/block_elements blocks back to back (GGUF ne0 = K). Nothing is repacked on load.

The synthetic generators reproduce the distributions the benchmark configurations name, with numpy's
default_rng(seed) and a fixed draw order (documented per function), so a test, the bench and the CPU baseline
all see the same bytes for the same seed.
"""
from __future__ import annotations

import numpy as np

Q8_0 = 8
Q3_K = 11
Q4_K = 12
Q5_K = 13
Q6_K = 14
IQ4_XS = 23

NAMES = {Q8_0: "Q8_0", Q3_K: "Q3_K", Q4_K: "Q4_K", Q5_K: "Q5_K", Q6_K: "Q6_K", IQ4_XS: "IQ4_XS"}
BY_NAME = {v.lower(): k for k, v in NAMES.items()}
BLOCK_ELEMENTS = {Q8_0: 32, Q3_K: 256, Q4_K: 256, Q5_K: 256, Q6_K: 256, IQ4_XS: 256}
BLOCK_BYTES = {Q8_0: 34, Q3_K: 110, Q4_K: 144, Q5_K: 176, Q6_K: 210, IQ4_XS: 136}
SUPERBLOCK_BYTES = {**BLOCK_BYTES, Q8_0: 272}


def type_of(fmt) -> int:
    """GGML type id from an id or a name ("q4_k", "Q4_K", "q4k")."""
    if isinstance(fmt, (int, np.integer)):
        if int(fmt) not in NAMES:
            raise ValueError(f"unsupported GGML type {fmt}")
        return int(fmt)
    key = str(fmt).lower()
    key = {"q4k": "q4_k", "q6k": "q6_k", "q80": "q8_0", "q3k": "q3_k", "q5k": "q5_k", "iq4xs": "iq4_xs"}.get(key, key)
    if key not in BY_NAME:
        raise ValueError(f"unsupported format {fmt!r}")
    return BY_NAME[key]


def row_bytes(fmt, K: int) -> int:
    """Bytes of one weight row of K values (K a multiple of the block size)."""
    t = type_of(fmt)
    if K % BLOCK_ELEMENTS[t]:
        raise ValueError(f"K={K} is not a multiple of the {NAMES[t]} block ({BLOCK_ELEMENTS[t]})")
    return K // BLOCK_ELEMENTS[t] * BLOCK_BYTES[t]


def weight_bytes(fmt, N: int, K: int) -> int:
    return N * row_bytes(fmt, K)


def _f16_bytes(v: np.ndarray) -> np.ndarray:
    return v.astype(np.float16).view(np.uint8).reshape(v.shape + (2,))


def synth_q8_0(N: int, K: int, seed: int) -> np.ndarray:
    """Q8_0 rows [N][K/32*34]: int8 quants uniform in [-127, 127], d = |N(0, 0.02)| / 127 as f16.
    Draw order: d (N*K/32 normals), then the quants (N*K int8)."""
    rng = np.random.default_rng(seed)
    nb = N * K // 32
    d = (np.abs(rng.standard_normal(nb, dtype=np.float32)) * np.float32(0.02) / np.float32(127.0))
    q = rng.integers(-127, 128, size=(nb, 32), dtype=np.int8)
    blk = np.empty((nb, 34), np.uint8)
    blk[:, 0:2] = _f16_bytes(d)
    blk[:, 2:] = q.view(np.uint8)
    return blk.reshape(N, K // 32 * 34)


def synth_q4_k(N: int, K: int, seed: int) -> np.ndarray:
    """Q4_K rows [N][K/256*144]: the 12 scale bytes uniform (each 6-bit sc / m uniform in [0, 63]), the 128 qs bytes
    uniform (nibbles uniform in [0, 15]), d = |N(0, 0.01)| and dmin = |N(0, 0.005)| as f16.
    Draw order: d, dmin (N*K/256 normals each), scales (12 bytes per block), qs (128 bytes per block)."""
    rng = np.random.default_rng(seed)
    nb = N * K // 256
    d = np.abs(rng.standard_normal(nb, dtype=np.float32)) * np.float32(0.01)
    dmin = np.abs(rng.standard_normal(nb, dtype=np.float32)) * np.float32(0.005)
    sc = rng.integers(0, 256, size=(nb, 12), dtype=np.uint8)
    qs = rng.integers(0, 256, size=(nb, 128), dtype=np.uint8)
    blk = np.empty((nb, 144), np.uint8)
    blk[:, 0:2] = _f16_bytes(d)
    blk[:, 2:4] = _f16_bytes(dmin)
    blk[:, 4:16] = sc
    blk[:, 16:] = qs
    return blk.reshape(N, K // 256 * 144)


def synth_q6_k(N: int, K: int, seed: int) -> np.ndarray:
    """Q6_K rows [N][K/256*210]: int8 sub-scales uniform in [-32, 31], ql / qh bytes uniform (6-bit codes uniform in
    [0, 63]), d = |N(0, 0.01)| as f16.  Draw order: d (N*K/256 normals), scales (16 per block), ql (128), qh (64)."""
    rng = np.random.default_rng(seed)
    nb = N * K // 256
    d = np.abs(rng.standard_normal(nb, dtype=np.float32)) * np.float32(0.01)
    sc = rng.integers(-32, 32, size=(nb, 16), dtype=np.int8)
    ql = rng.integers(0, 256, size=(nb, 128), dtype=np.uint8)
    qh = rng.integers(0, 256, size=(nb, 64), dtype=np.uint8)
    blk = np.empty((nb, 210), np.uint8)
    blk[:, 0:128] = ql
    blk[:, 128:192] = qh
    blk[:, 192:208] = sc.view(np.uint8)
    blk[:, 208:210] = _f16_bytes(d)
    return blk.reshape(N, K // 256 * 210)


def synth_q5_k(N: int, K: int, seed: int) -> np.ndarray:
    """Q5_K rows [N][K/256*176] (no benchmark configuration names Q5_K; the Q4_K rule plus a uniform qh plane): the 12
    scale bytes uniform, qh and qs bytes uniform (5-bit quants uniform in [0, 31]), d = |N(0, 0.01)| and
    dmin = |N(0, 0.005)| as f16. Draw order: d, dmin, scales (12 per block), qh (32), qs (128)."""
    rng = np.random.default_rng(seed)
    nb = N * K // 256
    d = np.abs(rng.standard_normal(nb, dtype=np.float32)) * np.float32(0.01)
    dmin = np.abs(rng.standard_normal(nb, dtype=np.float32)) * np.float32(0.005)
    sc = rng.integers(0, 256, size=(nb, 12), dtype=np.uint8)
    qh = rng.integers(0, 256, size=(nb, 32), dtype=np.uint8)
    qs = rng.integers(0, 256, size=(nb, 128), dtype=np.uint8)
    blk = np.empty((nb, 176), np.uint8)
    blk[:, 0:2] = _f16_bytes(d)
    blk[:, 2:4] = _f16_bytes(dmin)
    blk[:, 4:16] = sc
    blk[:, 16:48] = qh
    blk[:, 48:] = qs
    return blk.reshape(N, K // 256 * 176)


def synth_q3_k(N: int, K: int, seed: int) -> np.ndarray:
    """Q3_K rows [N][K/256*110]: hmask, qs and the 12 scale bytes uniform (3-bit quants in [-4, 3], 6-bit scales in
    [-32, 31]), d = N(0, 0.01) as f16 (either sign). Draw order: d, hmask (32 per block), qs (64), scales (12)."""
    rng = np.random.default_rng(seed)
    nb = N * K // 256
    d = rng.standard_normal(nb, dtype=np.float32) * np.float32(0.01)
    hm = rng.integers(0, 256, size=(nb, 32), dtype=np.uint8)
    qs = rng.integers(0, 256, size=(nb, 64), dtype=np.uint8)
    sc = rng.integers(0, 256, size=(nb, 12), dtype=np.uint8)
    blk = np.empty((nb, 110), np.uint8)
    blk[:, 0:32] = hm
    blk[:, 32:96] = qs
    blk[:, 96:108] = sc
    blk[:, 108:110] = _f16_bytes(d)
    return blk.reshape(N, K // 256 * 110)


def synth_iq4_xs(N: int, K: int, seed: int) -> np.ndarray:
    """IQ4_XS rows [N][K/256*136]: scales_h / scales_l / qs bytes uniform (6-bit scales in [-32, 31], nibbles uniform
    over the 16 non-linear levels), d = |N(0, 0.001)| as f16 (levels reach 127, so a tenth of the K-quants' d keeps
    the weights at the Q4_K rule's magnitude). Draw order: d, scales_h (2 bytes per block), scales_l (4), qs (128)."""
    rng = np.random.default_rng(seed)
    nb = N * K // 256
    d = np.abs(rng.standard_normal(nb, dtype=np.float32)) * np.float32(0.001)
    sh = rng.integers(0, 256, size=(nb, 2), dtype=np.uint8)
    sl = rng.integers(0, 256, size=(nb, 4), dtype=np.uint8)
    qs = rng.integers(0, 256, size=(nb, 128), dtype=np.uint8)
    blk = np.empty((nb, 136), np.uint8)
    blk[:, 0:2] = _f16_bytes(d)
    blk[:, 2:4] = sh
    blk[:, 4:8] = sl
    blk[:, 8:] = qs
    return blk.reshape(N, K // 256 * 136)


def synth_weights(fmt, N: int, K: int, seed: int = 0) -> np.ndarray:
    """Seeded GGUF rows [N][row_bytes] with the benchmark configurations' distributions."""
    t = type_of(fmt)
    if K % 256:
        raise ValueError("K must be a multiple of 256")
    return {Q8_0: synth_q8_0, Q3_K: synth_q3_k, Q4_K: synth_q4_k, Q5_K: synth_q5_k, Q6_K: synth_q6_k,
            IQ4_XS: synth_iq4_xs}[t](N, K, seed)


def scale_q4k_d(w: np.ndarray, factor: float) -> np.ndarray:
    """Q4_K rows with every super-block's d and dmin multiplied by `factor` (a power of two keeps them exact unless
    they become f16 subnormals); returns a copy. The BASELINE distribution (d ~ |N(0, 0.01)|, non-negative nibbles)
    gives layer outputs of ~1e5-1e6 in the synthetic stack, beyond f16; scaled weights keep a stack's f16 partial
    sums finite."""
    out = np.array(w, copy=True)
    hdr = out.reshape(out.shape[0], -1, 144)[:, :, :4]
    hdr[...] = (hdr.copy().view(np.float16) * np.float16(factor)).view(np.uint8)
    return out


def synth_activations(M: int, K: int, seed: int = 1) -> np.ndarray:
    """f16 [M][K] activations ~ N(0, 1) (one draw of M*K f32 normals, rounded to f16)."""
    rng = np.random.default_rng(seed)
    return rng.standard_normal((M, K), dtype=np.float32).astype(np.float16)
