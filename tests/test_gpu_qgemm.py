"""Tile GEMM (tcgen05) vs the oracle's dequant-then-GEMM, through the C ABI.

Tolerances (float64 oracle of f16-dequantised weights @ f16 activations, gemv_check.py:161-162):
  f32 output:  max-abs <= 2e-2 and relative Frobenius <= 1e-3;
  f16 output:  max-abs <= 2e-2 + half an f16 ulp of the reference value (the output rounding itself), and
               relative Frobenius <= 1e-3.
"""
import os

import numpy as np
import pytest

from conftest import GOLDEN

pytestmark = pytest.mark.gpu
FMTS = ["q8_0", "q4_k", "q6_k", "q5_k", "q3_k", "iq4_xs"]
MAX_ABS, REL_FRO = 2e-2, 1e-3


def check(O, y, ref, f16=False):
    e = O.errors(y, ref)
    assert e["finite"], e
    assert e["rel_fro"] <= REL_FRO, e
    if f16:
        bound = MAX_ABS + O.f16_half_ulp(ref)
        excess = np.abs(y.astype(np.float64) - ref) - bound
        assert excess.max() <= 0, (e, float(excess.max()))
    else:
        assert e["max_abs"] <= MAX_ABS, e
    return e


@pytest.mark.parametrize("name", FMTS)
def test_golden_gemm(pkg, F, O, dev, name):
    z = np.load(os.path.join(GOLDEN, f"gemm_{name}.npz"))
    t = F.type_of(name)
    w, K, x = z["blocks"], int(z["K"]), z["x"]
    if w.shape[1] % 16:  # Q6_K at K=512: pad the rows to a 16-byte stride (same bytes, aligned view)
        wp = np.zeros((w.shape[0], (w.shape[1] + 15) // 16 * 16), np.uint8)
        wp[:, :w.shape[1]] = w
        w = wp
    y = pkg.ops.qgemm(dev, w, t, x, N=w.shape[0], K=K, out_dtype="f32")
    check(O, y, z["y_f16w"])


@pytest.mark.parametrize("name", FMTS)
@pytest.mark.parametrize("M,N,K", [(1, 128, 256), (7, 320, 1024), (48, 1000, 2048), (300, 256, 4096),
                                   (513, 384, 512), (33, 130, 768)])
def test_qgemm_shapes(pkg, F, O, dev, name, M, N, K):
    t = F.type_of(name)
    if F.row_bytes(t, K) % 16:
        K = 2048  # Q6_K rows are 16-byte aligned only at multiples of 8 super-blocks (see test_q6k_unaligned_rows)
    w = F.synth_weights(t, N, K, seed=M + N + K)
    x = F.synth_activations(M, K, seed=M)
    ref = O.gemm_ref(O.dequant_f16(t, w, N, K), x)
    y = pkg.ops.qgemm(dev, w, t, x, N=N, K=K, out_dtype="f32")
    check(O, y, ref)
    y16 = pkg.ops.qgemm(dev, w, t, x, N=N, K=K, out_dtype="f16")
    check(O, y16, ref, f16=True)


@pytest.mark.parametrize("name", FMTS)
def test_epilogues(pkg, F, O, dev, name):
    t = F.type_of(name)
    M, N, K = 40, 384, 2048
    w = F.synth_weights(t, N, K, seed=5)
    x = F.synth_activations(M, K, seed=6)
    acc = O.gemm_ref(O.dequant_f16(t, w, N, K), x)
    rng = np.random.default_rng(7)
    resid = rng.standard_normal((M, N)).astype(np.float32) * 10
    y = pkg.ops.qgemm(dev, w, t, x, N=N, K=K, kind="kres", aux=resid)
    check(O, y, O.epilogue_ref(acc, 1, resid))
    gate = rng.standard_normal((M, N)).astype(np.float32) * 3
    ys = pkg.ops.qgemm(dev, w, t, x, N=N, K=K, kind="swiglu", aux=gate)
    assert ys.dtype == np.float16
    check(O, ys, O.epilogue_ref(acc, 2, gate), f16=True)


@pytest.mark.parametrize("name", FMTS)
def test_k_window_and_strides(pkg, F, O, dev, name):
    """A K window of longer rows (KWIN) and padded activation / output strides (OSTRIDE-style)."""
    t = F.type_of(name)
    M, N, K, kb_off = 33, 256, 1024, 8   # Q6_K: 8 super-blocks keep the window 16-byte aligned
    Kfull = K + 256 * kb_off + 1024
    w = F.synth_weights(t, N, Kfull, seed=9)
    x = F.synth_activations(M, K, seed=10)
    ref = O.gemm_ref(O.dequant_f16(t, w, N, K, kb_off=kb_off), x)
    y = pkg.ops.qgemm(dev, w, t, x, N=N, K=K, kb_off=kb_off, w_row_stride=w.shape[1])
    check(O, y, ref)
    # ldx > K and ldy > N through the raw pointer API
    ldx, ldy = K + 64, N + 40
    xp = np.zeros((M, ldx), np.float16)
    xp[:, :K] = x
    wd, xd = dev.upload(w), dev.upload(xp)
    yd = dev.empty(M * ldy * 4).fill(0xFF)   # NaN sentinel: columns past N must stay untouched
    pkg.ops.qgemm_ptr(wd.ptr, t, N, K, w.shape[1], kb_off, xd.ptr, M, ldx, yd.ptr, "f32", ldy)
    dev.synchronize()
    yy = yd.download(np.float32, (M, ldy))
    check(O, yy[:, :N], ref)
    assert np.isnan(yy[:, N:]).all()


@pytest.mark.parametrize("pair,bn", [(0, 64), (0, 128), (0, 192), (1, 128), (1, 160), (1, 256)])
@pytest.mark.parametrize("grid", [0, 2, 6, 38])
@pytest.mark.parametrize("kchunk", [-1, 512])
def test_tile_choices_are_identical(pkg, F, O, dev, bn, grid, kchunk, pair):
    """Every legal tile (width, persistent grid, single CTA or 2-SM pair) gives the same bits for a given
    accumulation chunk (the reference tuner's hash check, engine/tune/tune.py:13)."""
    t = F.Q4_K
    M, N, K = 300, 640, 2048
    w = F.synth_weights(t, N, K, seed=1)
    x = F.synth_activations(M, K, seed=2)
    base = pkg.ops.qgemm(dev, w, t, x, N=N, K=K, kchunk=kchunk, pair=0)
    y = pkg.ops.qgemm(dev, w, t, x, N=N, K=K, bn=bn, grid=grid, kchunk=kchunk, pair=pair)
    assert np.array_equal(y.view(np.uint32), base.view(np.uint32))
    check(O, y, O.gemm_ref(O.dequant_f16(t, w, N, K), x))


@pytest.mark.parametrize("kchunk", [128, 256, 1152, 2048])
@pytest.mark.parametrize("pair,bn", [(0, 0), (1, 0), (1, 256)])
def test_chunked_accumulation(pkg, F, O, dev, kchunk, pair, bn):
    """Chunked accumulation (chunk sums added in f32 round-to-nearest) matches the oracle for any chunk length,
    including chunks that do not divide K, with every epilogue, also with a single accumulator region."""
    t = F.Q4_K
    M, N, K = 200, 384, 4096
    w = F.synth_weights(t, N, K, seed=8)
    x = F.synth_activations(M, K, seed=9)
    acc = O.gemm_ref(O.dequant_f16(t, w, N, K), x)
    check(O, pkg.ops.qgemm(dev, w, t, x, N=N, K=K, kchunk=kchunk, pair=pair, bn=bn), acc)
    resid = np.random.default_rng(1).standard_normal((M, N)).astype(np.float32)
    check(O, pkg.ops.qgemm(dev, w, t, x, N=N, K=K, kind="kres", aux=resid, kchunk=kchunk, pair=pair, bn=bn),
          acc + resid)


def test_invalid_tile_is_refused(pkg, F, dev):
    t = F.Q4_K
    w = F.synth_weights(t, 128, 256, seed=0)
    x = F.synth_activations(4, 256, seed=0)
    with pytest.raises(pkg.YahError):
        pkg.ops.qgemm(dev, w, t, x, N=128, K=256, bn=256, pair=0)


def test_row_shards_match_full(pkg, F, dev):
    """Column-parallel shards (a row range of the GGUF tensor) give exactly the full GEMM's columns."""
    t = F.Q4_K
    M, N, K = 64, 768, 1024
    w = F.synth_weights(t, N, K, seed=3)
    x = F.synth_activations(M, K, seed=4)
    full = pkg.ops.qgemm(dev, w, t, x, N=N, K=K)
    parts = [pkg.ops.qgemm(dev, w[r:r + 192], t, x, N=192, K=K) for r in range(0, N, 192)]
    assert np.array_equal(np.concatenate(parts, axis=1).view(np.uint32), full.view(np.uint32))


@pytest.mark.parametrize("name", FMTS)
def test_config3_k_sampled(pkg, F, O, dev, name):
    """The config 3 reduction length (K = 14336, N = 4096, M = 2048) on a sample of 128 weight rows: the longest
    f32 accumulation of the benchmark configurations stays within the bar."""
    t = F.type_of(name)
    M, N, K = 2048, 4096, 14336
    w = F.synth_weights(t, N, K, seed=2)
    x = F.synth_activations(M, K, seed=3)
    y = pkg.ops.qgemm(dev, w, t, x, N=N, K=K)
    rows = np.random.default_rng(1).choice(N, 128, replace=False)
    e = check(O, y[:, rows], O.gemm_ref(O.dequant_f16(t, w[rows], len(rows), K), x))
    print(f"config3 {name}: {e}")


@pytest.mark.parametrize("name", ["q4_k"])
def test_full_size_config2_sampled(pkg, F, O, dev, name):
    """BASELINE config 2 (Q4_K, M=2048, K=4096, N=14336) on the GPU, checked on a sample of 256 weight rows
    against the oracle and on the whole output for finiteness."""
    t = F.type_of(name)
    M, N, K = 2048, 14336, 4096
    w = F.synth_weights(t, N, K, seed=0)
    x = F.synth_activations(M, K, seed=1)
    y = pkg.ops.qgemm(dev, w, t, x, N=N, K=K, out_dtype="f16")
    assert np.isfinite(y).all()
    rows = np.random.default_rng(0).choice(N, 256, replace=False)
    ref = O.gemm_ref(O.dequant_f16(t, w[rows], len(rows), K), x)
    check(O, y[:, rows], ref, f16=True)


def test_q6k_unaligned_rows_are_refused(pkg, F, dev):
    """Q6_K rows that are not 16-byte aligned (K = 1280) are refused with YAH_ERR_UNSUPPORTED, not run."""
    t = F.Q6_K
    w = F.synth_weights(t, 128, 1280, seed=0)
    x = F.synth_activations(4, 1280, seed=0)
    with pytest.raises(pkg.YahError) as ei:
        pkg.ops.qgemm(dev, w, t, x, N=128, K=1280)
    assert ei.value.code == 2


def test_status_word_clear(pkg, dev):
    assert dev.status_word() == 0


def test_q6k_lm_head_k5120_prefill_realigned(pkg, F, O, dev):
    """Prefill GEMM on the K = 5120 Q6_K lm head after row realignment (4200 -> 4208-byte stride)."""
    t = F.Q6_K
    N, K, M = 2048, 5120, 256
    w = F.synth_weights(t, N, K, seed=53)
    wd, stride = pkg.ops.realign(dev, w)
    x = F.synth_activations(M, K, seed=54)
    y = pkg.ops.qgemm(dev, wd, t, x, N=N, K=K, w_row_stride=stride)
    e = O.errors(y, O.gemm_ref(O.dequant_f16(t, w, N, K), x))
    assert e["finite"] and e["max_abs"] <= 2e-2 and e["rel_fro"] <= 1e-3, e
    wd.close()


@pytest.mark.parametrize("name", FMTS)
@pytest.mark.parametrize("M", [1, 8, 32])
@pytest.mark.parametrize("pair", [0, 1])
def test_split_k_matches_unsplit(pkg, F, O, dev, name, M, pair):
    """Few tokens: with an automatic grid the accumulation chunks of a tile run on separate CTAs (split K) and are
    added in chunk order afterwards. Bit-identical to the unsplit GEMM (an explicit grid never splits) for every
    epilogue, and within the bar of the oracle."""
    t = F.type_of(name)
    N, K = 1024, 8192  # 4 or 8 row tiles x 4 chunks of 2048
    w = F.synth_weights(t, N, K, seed=21)
    x = F.synth_activations(M, K, seed=22)
    rng = np.random.default_rng(23)
    aux = rng.standard_normal((M, N)).astype(np.float32) * 3
    acc = O.gemm_ref(O.dequant_f16(t, w, N, K), x)
    for kind, out, ref in (("kstore", "f32", acc), ("kstore", "f16", acc), ("kres", "f32", acc + aux),
                           ("swiglu", "f16", O.epilogue_ref(acc, 2, aux))):
        a = None if kind == "kstore" else aux
        ys = pkg.ops.qgemm(dev, w, t, x, N=N, K=K, kind=kind, out_dtype=out, aux=a, pair=pair)
        yu = pkg.ops.qgemm(dev, w, t, x, N=N, K=K, kind=kind, out_dtype=out, aux=a, pair=pair, grid=dev.sm_count)
        assert ys.dtype == yu.dtype
        assert np.array_equal(ys.view(np.uint8), yu.view(np.uint8)), (kind, out)
        check(O, ys, ref, f16=ys.dtype == np.float16)


def test_split_k_config3_decode_shapes(pkg, F, O, dev):
    """The config 3 down projection (N = 4096, K = 14336: 7 chunks) at M = 32 through the automatic choice (split
    K), on a sample of 256 weight rows, and the ragged token count M = 17."""
    t = F.Q4_K
    N, K = 4096, 14336
    w = F.synth_weights(t, N, K, seed=31)
    rows = np.random.default_rng(2).choice(N, 256, replace=False)
    for M in (32, 17):
        x = F.synth_activations(M, K, seed=32 + M)
        y = pkg.ops.qgemm(dev, w, t, x, N=N, K=K)
        yu = pkg.ops.qgemm(dev, w, t, x, N=N, K=K, grid=dev.sm_count)
        assert np.array_equal(y.view(np.uint32), yu.view(np.uint32))
        check(O, y[:, rows], O.gemm_ref(O.dequant_f16(t, w[rows], len(rows), K), x))


@pytest.mark.parametrize("name", FMTS)
@pytest.mark.parametrize("pair,bn", [(-1, 0), (1, 160), (0, 192), (0, 64)])
@pytest.mark.parametrize("M,N,K", [(96, 320, 2048), (33, 200, 2048), (300, 64, 8192)])  # Q6_K rows: K % 2048
def test_ffn_matches_gate_then_up(pkg, F, O, dev, name, pair, bn, M, N, K):
    """The fused gate+up SwiGLU (one GEMM, gate and up rows in the two halves of a CTA's TMEM lanes) gives the bits
    of the gate GEMM (f32) followed by the up GEMM with the swiglu epilogue, and is within the bar of the oracle;
    ragged N (tiles of 64 output rows), ragged M, and K above 4096 (chunked accumulation)."""
    t = F.type_of(name)
    wg = F.synth_weights(t, N, K, seed=41)
    wu = F.synth_weights(t, N, K, seed=42)
    # Q4_K / Q6_K activations scaled by 2^-6 (exact) keep silu(gate) * up inside the f16 range at these K; the Q8_0
    # weights are ~50x smaller and need no scaling (scaled, its outputs would sit in f16's subnormal range)
    scale = 1.0 if name == "q8_0" else 1 / 64
    x = (F.synth_activations(M, K, seed=43).astype(np.float32) * scale).astype(np.float16)
    y = pkg.ops.qgemm_ffn(dev, wg, wu, t, x, N=N, K=K, bn=bn, pair=pair)
    g = pkg.ops.qgemm(dev, wg, t, x, N=N, K=K, out_dtype="f32")
    ref2 = pkg.ops.qgemm(dev, wu, t, x, N=N, K=K, kind="swiglu", aux=g)
    assert y.dtype == np.float16 and np.isfinite(y).all()
    assert np.array_equal(y.view(np.uint16), ref2.view(np.uint16))
    gref = O.gemm_ref(O.dequant_f16(t, wg, N, K), x)
    uref = O.gemm_ref(O.dequant_f16(t, wu, N, K), x)
    check(O, y, O.epilogue_ref(uref, 2, gref.astype(np.float32)), f16=True)


def test_ffn_k_window(pkg, F, O, dev):
    """The fused gate+up on a K window of longer rows (kb_off and the row stride)."""
    t = F.Q4_K
    M, N, K, kb_off = 40, 256, 1024, 4
    Kf = K + 256 * kb_off + 512
    wg = F.synth_weights(t, N, Kf, seed=51)
    wu = F.synth_weights(t, N, Kf, seed=52)
    x = (F.synth_activations(M, K, seed=53).astype(np.float32) / 64).astype(np.float16)
    y = pkg.ops.qgemm_ffn(dev, wg, wu, t, x, N=N, K=K, kb_off=kb_off, w_row_stride=wg.shape[1])
    gref = O.gemm_ref(O.dequant_f16(t, wg, N, K, kb_off=kb_off), x)
    uref = O.gemm_ref(O.dequant_f16(t, wu, N, K, kb_off=kb_off), x)
    check(O, y, O.epilogue_ref(uref, 2, gref.astype(np.float32)), f16=True)
