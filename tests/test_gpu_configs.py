"""Every BASELINE configuration at its own shape on the GPU, against the oracle (tests/test_gpu_qgemm.py covers
config 2 and the config 3 reduction length; tests/test_gpu_qgemv*.py the config 3 decode sweep).

  config 1  Q8_0 prefill GEMM, M = 512, K = 4096, N = 4096: the whole output.
  config 5  Q6_K lm head, K = 4096, N = 128256 (431 MB of weights): the prefill GEMM at M = 4096 on 256 sampled
            vocabulary rows (the whole output for finiteness), and the decode GEMV at M = 1 / 8 / 32 on every row.
Bars as elsewhere: the tile GEMM (f16-rounded weights, as the reference's tile GEMM) against the f16-weight float64
oracle with max-abs <= 2e-2 (+ half an f16 ulp of the reference for f16 outputs) and relative Frobenius <= 1e-3; the
GEMV (f32 weights, as the reference GEMV) against the f32-weight oracle with the same bars plus the reference GEMV
checker's max |y - ref| / max |ref| <= 1e-4 (engine/gpu/loom/tools/gemv_check.py:176-183).
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def check(O, y, ref, f16=False, rel_max=None):
    e = O.errors(y, ref)
    assert e["finite"] and e["rel_fro"] <= 1e-3, e
    if f16:
        assert (np.abs(y.astype(np.float64) - ref) <= 2e-2 + O.f16_half_ulp(ref)).all(), e
    else:
        assert e["max_abs"] <= 2e-2, e
    if rel_max is not None:
        assert e["rel_max"] <= rel_max, e
    return e


def test_config1_q8_0_gemm_full(pkg, F, O, dev):
    t = F.Q8_0
    M, N, K = 512, 4096, 4096
    w = F.synth_weights(t, N, K, seed=101)
    x = F.synth_activations(M, K, seed=102)
    ref = O.gemm_ref(O.dequant_f16(t, w, N, K), x)
    check(O, pkg.ops.qgemm(dev, w, t, x, N=N, K=K), ref)
    check(O, pkg.ops.qgemm(dev, w, t, x, N=N, K=K, out_dtype="f16"), ref, f16=True)


@pytest.fixture(scope="module")
def lm_head(F):
    N, K = 128256, 4096
    return F.synth_weights(F.Q6_K, N, K, seed=105), N, K


def test_config5_prefill_sampled(pkg, F, O, dev, lm_head):
    w, N, K = lm_head
    t = F.Q6_K
    M = 4096
    x = F.synth_activations(M, K, seed=106)
    y = pkg.ops.qgemm(dev, w, t, x, N=N, K=K, out_dtype="f16")
    assert np.isfinite(y).all()
    # 256 sampled rows, including the ragged tail of the last 128-row tile
    rows = np.unique(np.concatenate([np.random.default_rng(5).choice(N, 248, replace=False), np.arange(N - 8, N)]))
    check(O, y[:, rows], O.gemm_ref(O.dequant_f16(t, w[rows], len(rows), K), x), f16=True)


@pytest.mark.parametrize("M", [1, 8, 32])
def test_config5_gemv_full(pkg, F, O, dev, lm_head, M):
    w, N, K = lm_head
    t = F.Q6_K
    x = F.synth_activations(M, K, seed=107 + M)
    y = pkg.ops.qgemv(dev, w, t, x, N=N, K=K)
    ref = np.empty((M, N))
    for r in range(0, N, 16384):  # the float64 oracle in row chunks (the whole f64 weight would be 4 GB)
        n = min(16384, N - r)
        ref[:, r:r + n] = O.gemm_ref(O.dequant_f32(t, w[r:r + n], n, K), x)
    check(O, y, ref, rel_max=1e-4)
