"""Decode GEMV (M <= 32 tokens) vs the oracle through the C ABI.

The GEMV multiplies the same f16 weights as the tile GEMM, so the reference is the f16 dequant-then-GEMM; the
same bars hold (max-abs <= 2e-2, relative Frobenius <= 1e-3; f32 output). Against the reference GEMV's own
oracle (f32 weights, gemv_check.py:161-162) the difference is the f16 rounding of the weights (at most 2^-11
relative per weight), so error / max |y| stays below 1e-3 there (the reference GEMV's bar is 1e-4 because it
keeps f32 weights).
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu
FMTS = ["q8_0", "q4_k", "q6_k"]


def check(O, y, ref):
    e = O.errors(y, ref)
    assert e["finite"] and e["max_abs"] <= 2e-2 and e["rel_fro"] <= 1e-3, e
    return e


@pytest.mark.parametrize("name", FMTS)
@pytest.mark.parametrize("M", [1, 2, 8, 16, 17, 32])
@pytest.mark.parametrize("N,K", [(256, 2048), (4096, 4096), (1000, 2048)])
def test_qgemv(pkg, F, O, dev, name, M, N, K):
    t = F.type_of(name)
    w = F.synth_weights(t, N, K, seed=N + K)
    x = F.synth_activations(M, K, seed=M)
    y = pkg.ops.qgemv(dev, w, t, x, N=N, K=K)
    check(O, y, O.gemm_ref(O.dequant_f16(t, w, N, K), x))
    ref32 = O.gemm_ref(O.dequant_f32(t, w, N, K), x)
    assert O.errors(y, ref32)["rel_max"] <= 1e-3


@pytest.mark.parametrize("name", FMTS)
def test_qgemv_resid_and_f16(pkg, F, O, dev, name):
    t = F.type_of(name)
    M, N, K = 5, 640, 4096
    w = F.synth_weights(t, N, K, seed=1)
    x = F.synth_activations(M, K, seed=2)
    acc = O.gemm_ref(O.dequant_f16(t, w, N, K), x)
    resid = np.random.default_rng(3).standard_normal((M, N)).astype(np.float32)
    y = pkg.ops.qgemv(dev, w, t, x, N=N, K=K, kind="resid", aux=resid)
    check(O, y, acc + resid)
    y16 = pkg.ops.qgemv(dev, w, t, x, N=N, K=K, out_dtype="f16")
    e = O.errors(y16, acc)
    assert e["rel_fro"] <= 1e-3 and (np.abs(y16 - acc) <= 2e-2 + O.f16_half_ulp(acc)).all()


def test_qgemv_and_qgemm_at_config3_k(pkg, F, O, dev):
    """Decode and prefill paths on the config 3 reduction length (K = 14336) both meet the bar."""
    t = F.Q4_K
    M, N, K = 8, 1024, 14336
    w = F.synth_weights(t, N, K, seed=11)
    x = F.synth_activations(M, K, seed=12)
    ref = O.gemm_ref(O.dequant_f16(t, w, N, K), x)
    check(O, pkg.ops.qgemv(dev, w, t, x, N=N, K=K), ref)
    check(O, pkg.ops.qgemm(dev, w, t, x, N=N, K=K), ref)


def test_qgemv_k_window(pkg, F, O, dev):
    t = F.Q8_0
    M, N, K, kb_off = 3, 300, 1024, 2
    w = F.synth_weights(t, N, K + 256 * kb_off + 512, seed=4)
    x = F.synth_activations(M, K, seed=5)
    y = pkg.ops.qgemv(dev, w, t, x, N=N, K=K, kb_off=kb_off, w_row_stride=w.shape[1])
    check(O, y, O.gemm_ref(O.dequant_f16(t, w, N, K, kb_off=kb_off), x))


def test_qgemv_repeat_deterministic(pkg, F, dev):
    """Split-K partials are reduced in a fixed order: repeated calls give identical bits."""
    t = F.Q4_K
    M, N, K = 32, 512, 14336
    w = F.synth_weights(t, N, K, seed=6)
    x = F.synth_activations(M, K, seed=7)
    a = pkg.ops.qgemv(dev, w, t, x, N=N, K=K)
    for _ in range(3):
        b = pkg.ops.qgemv(dev, w, t, x, N=N, K=K)
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
