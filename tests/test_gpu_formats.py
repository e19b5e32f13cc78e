"""The GGUF formats beyond the benchmark configurations' three (Q5_K, Q3_K, IQ4_XS: the reference's FMTS entries
q5k / q3k / iq4xs, engine/gpu/loom/tools/gen_gemm_decode.py:1707-1727, and its GEMV lane setups,
engine/gpu/loom/tools/gen_gemv.py:137-230) on the same kernels, at the decode and prefill shapes of the benchmark
configurations and on K windows that start inside a 16-byte unit.

Bars as for the other formats: the tile GEMM against the float64 oracle of the f16 dequant (max-abs <= 2e-2,
relative Frobenius <= 1e-3), the GEMV against the float64 oracle of the f32 dequant with the reference checker's
max |y - ref| / max |ref| <= 1e-4 as well (gemv_check.py:176-183).
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu
NEW = ["q5_k", "q3_k", "iq4_xs"]


def check(O, y, ref, rel_max=None):
    e = O.errors(y, ref)
    assert e["finite"] and e["max_abs"] <= 2e-2 and e["rel_fro"] <= 1e-3, e
    if rel_max is not None:
        assert e["rel_max"] <= rel_max, e
    return e


@pytest.mark.parametrize("name", ["q3_k", "iq4_xs", "q6_k"])
@pytest.mark.parametrize("kb_off", [1, 3, 5])
def test_unaligned_k_window(pkg, F, O, dev, name, kb_off):
    """Super-blocks of 110 / 136 / 210 bytes: a K window starting at super-block kb_off begins inside a 16-byte
    unit; the weight copies start at the boundary below and the decode reads from the offset."""
    t = F.type_of(name)
    M, N, K = 24, 300, 2048
    Kfull = 256 * 16  # 16 super-blocks per row: rows stay 16-byte multiples for every format
    w = F.synth_weights(t, N, Kfull, seed=kb_off + 7)
    x = F.synth_activations(M, K, seed=kb_off)
    ref16 = O.gemm_ref(O.dequant_f16(t, w, N, K, kb_off=kb_off), x)
    y = pkg.ops.qgemm(dev, w, t, x, N=N, K=K, kb_off=kb_off, w_row_stride=w.shape[1])
    check(O, y, ref16)
    ref32 = O.gemm_ref(O.dequant_f32(t, w, N, K, kb_off=kb_off), x)
    for m in (1, 8, 24):
        yv = pkg.ops.qgemv(dev, w, t, x[:m], N=N, K=K, kb_off=kb_off, w_row_stride=w.shape[1])
        check(O, yv, ref32[:m], rel_max=1e-4)
    d = pkg.ops.dequant(dev, w, t, N=N, K=K, kb_off=kb_off, w_row_stride=w.shape[1]).view(np.uint16)
    assert np.count_nonzero(d != O.dequant_f16(t, w, N, K, kb_off=kb_off).view(np.uint16)) == 0


@pytest.mark.parametrize("name", NEW)
@pytest.mark.parametrize("M", [1, 8, 32])
def test_decode_gemv_config3_shape(pkg, F, O, dev, name, M):
    """The config-3 down projection shape (N = 4096, K = 14336) at 1 / 8 / 32 tokens, all rows."""
    t = F.type_of(name)
    N, K = 4096, 14336
    w = F.synth_weights(t, N, K, seed=61)
    x = F.synth_activations(M, K, seed=62 + M)
    y = pkg.ops.qgemv(dev, w, t, x, N=N, K=K)
    check(O, y, O.gemm_ref(O.dequant_f32(t, w, N, K), x), rel_max=1e-4)


@pytest.mark.parametrize("name", NEW)
def test_prefill_config2_shape_sampled(pkg, F, O, dev, name):
    """The config-2 shape (M = 2048, K = 4096, N = 14336) on a sample of 256 weight rows, plus the f32 output's
    finiteness everywhere."""
    t = F.type_of(name)
    M, N, K = 2048, 14336, 4096
    w = F.synth_weights(t, N, K, seed=71)
    x = F.synth_activations(M, K, seed=72)
    y = pkg.ops.qgemm(dev, w, t, x, N=N, K=K, out_dtype="f32")
    assert np.isfinite(y).all()
    rows = np.random.default_rng(73).choice(N, 256, replace=False)
    check(O, y[:, rows], O.gemm_ref(O.dequant_f16(t, w[rows], len(rows), K), x))


@pytest.mark.parametrize("gfmt,ufmt", [("iq4_xs", "iq4_xs"), ("q5_k", "q3_k"), ("q3_k", "q4_k")])
def test_gemv_swiglu_new_formats(pkg, F, O, dev, gfmt, ufmt):
    """The two-tensor swiglu GEMV with the new formats as gate / up."""
    tg, tu = F.type_of(gfmt), F.type_of(ufmt)
    M, N, K = 4, 2048, 4096
    wg = F.synth_weights(tg, N, K, seed=81)
    wu = F.synth_weights(tu, N, K, seed=82)
    x = F.synth_activations(M, K, seed=83)
    g = O.gemm_ref(O.dequant_f32(tg, wg, N, K), x)
    u = O.gemm_ref(O.dequant_f32(tu, wu, N, K), x)
    with np.errstate(over="ignore"):
        ref = g / (1.0 + np.exp(-g)) * u
    L = pkg.lib()
    dg, du, xd, yd = dev.upload(wg), dev.upload(wu), dev.upload(x), dev.empty(M * N * 4)
    rc = L.yah_qgemv_swiglu(dg.ptr, tg, wg.shape[1], du.ptr, tu, wu.shape[1], N, K, xd.ptr, M, K, yd.ptr, N, None)
    assert rc == 0, L.yah_last_error()
    e = O.errors(yd.download(np.float32, (M, N)), ref)
    assert e["finite"] and e["rel_fro"] <= 1e-3 and e["rel_max"] <= 1e-4, e


@pytest.mark.parametrize("name,K", [("q3_k", 1280), ("iq4_xs", 768)])
def test_unaligned_rows_are_refused(pkg, F, dev, name, K):
    """Rows that are not 16-byte multiples (Q3_K: 5 super-blocks, IQ4_XS: 3) are refused, not run."""
    t = F.type_of(name)
    w = F.synth_weights(t, 64, K, seed=0)
    x = F.synth_activations(4, K, seed=0)
    with pytest.raises(pkg.YahError) as ei:
        pkg.ops.qgemm(dev, w, t, x, N=64, K=K)
    assert ei.value.code == 2
    with pytest.raises(pkg.YahError) as ei:
        pkg.ops.qgemv(dev, w, t, x, N=64, K=K)
    assert ei.value.code == 2
