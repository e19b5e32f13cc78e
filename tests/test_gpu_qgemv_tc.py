"""The two decode GEMV kernels (tcgen05 for Q4_K, mma.sync for every format) against the oracle, the GEMV's swiglu
kind, and the two-tensor swiglu entry point (yah_qgemv_swiglu, the reference GEMV's swiglu kind with gate and up
weights that may differ in format, engine/gpu/loom/tools/gen_gemv.py:18, :97-98).

Bars as in test_gpu_qgemv.py: max-abs <= 2e-2, relative Frobenius <= 1e-3 and the reference GEMV checker's
max |y - ref| / max |ref| <= 1e-4 (engine/gpu/loom/tools/gemv_check.py:176-183) against gguf-py's f32 dequant times
x in float64. The swiglu outputs reach ~1e5, beyond any absolute f32 bar, so they are held to the relative bars.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TC, MMA = 1, 2


@pytest.fixture
def impl(pkg):
    """Select a GEMV kernel for one test and restore the automatic choice afterwards."""
    L = pkg.lib()

    def use(which):
        assert L.yah_set_gemv_impl(which) == 0

    yield use
    assert L.yah_set_gemv_impl(0) == 0


def check(O, y, ref, rel_max=1e-4, absolute=True):
    e = O.errors(y, ref)
    assert e["finite"] and e["rel_fro"] <= 1e-3 and e["rel_max"] <= rel_max, e
    if absolute:
        assert e["max_abs"] <= 2e-2, e
    return e


def silu(g):
    with np.errstate(over="ignore"):  # e^-g overflows to inf for g below about -709: silu is then -0
        return g / (1.0 + np.exp(-g))


@pytest.mark.parametrize("which", [TC, MMA])
@pytest.mark.parametrize("M", [1, 3, 8, 16, 17, 32])
@pytest.mark.parametrize("N,K", [(128, 256), (200, 2048), (1000, 4096), (4096, 14336), (14336, 4096), (333, 8192)])
def test_q4k_kernels(pkg, F, O, dev, impl, which, M, N, K):
    """Every tcgen05 work split (one CTA per K range, clusters of 2 and 4 splitting K, ragged last tiles, several
    tiles per cluster) and the mma.sync kernel on the same shapes."""
    impl(which)
    t = F.Q4_K
    w = F.synth_weights(t, N, K, seed=N + 3 * K + M)
    x = F.synth_activations(M, K, seed=M + 5)
    y = pkg.ops.qgemv(dev, w, t, x, N=N, K=K)
    check(O, y, O.gemm_ref(O.dequant_f32(t, w, N, K), x))


@pytest.mark.parametrize("which", [TC, MMA])
@pytest.mark.parametrize("M", [1, 6, 32])
def test_q4k_kinds(pkg, F, O, dev, impl, which, M):
    """resid (y = aux + W x), swiglu with a separate f32 gate (f32 and f16 out) and in place over the gate."""
    impl(which)
    t = F.Q4_K
    N, K = 768, 4096
    w = F.synth_weights(t, N, K, seed=91)
    x = F.synth_activations(M, K, seed=92)
    acc = O.gemm_ref(O.dequant_f32(t, w, N, K), x)
    rng = np.random.default_rng(93)
    resid = rng.standard_normal((M, N)).astype(np.float32)
    check(O, pkg.ops.qgemv(dev, w, t, x, N=N, K=K, kind="resid", aux=resid), acc + resid)
    gate = (rng.standard_normal((M, N)) * 4).astype(np.float32)
    ref = silu(gate.astype(np.float64)) * acc
    check(O, pkg.ops.qgemv(dev, w, t, x, N=N, K=K, kind="swiglu", aux=gate), ref, absolute=False)
    y16 = pkg.ops.qgemv(dev, w, t, x, N=N, K=K, kind="swiglu", aux=gate, out_dtype="f16")
    assert (np.abs(y16 - ref) <= 1e-4 * np.abs(ref).max() + O.f16_half_ulp(ref)).all()
    # in place: the gate buffer is the output
    L = pkg.lib()
    wd, xd, yd = dev.upload(w), dev.upload(x), dev.upload(gate)
    assert L.yah_qgemv(wd.ptr, t, N, K, w.shape[1], 0, xd.ptr, M, K, yd.ptr, 0, N, 2, yd.ptr, N, None) == 0, \
        L.yah_last_error()
    check(O, yd.download(np.float32, (M, N)), ref, absolute=False)


@pytest.mark.parametrize("which", [TC, MMA])
def test_q4k_k_window(pkg, F, O, dev, impl, which):
    """A K window of longer rows (the row-parallel shard form): kb_off super-blocks in, rows at a longer stride."""
    impl(which)
    t = F.Q4_K
    M, N, K, kb_off = 5, 640, 7168, 3
    w = F.synth_weights(t, N, K + 256 * (kb_off + 2), seed=61)
    x = F.synth_activations(M, K, seed=62)
    y = pkg.ops.qgemv(dev, w, t, x, N=N, K=K, kb_off=kb_off, w_row_stride=w.shape[1])
    check(O, y, O.gemm_ref(O.dequant_f32(t, w, N, K, kb_off=kb_off), x))


def test_tc_covers_the_decode_configs(pkg, F, dev, impl):
    """The tcgen05 kernel takes config 3 (4096 x 14336) and the gate / up shape (14336 x 4096) at 1..32 tokens: with
    only that kernel selected none of these calls is refused."""
    impl(TC)
    L = pkg.lib()
    t = F.Q4_K
    for N, K in ((4096, 14336), (14336, 4096)):
        wd = dev.empty(N * F.row_bytes(t, K)).fill(0)
        xd = dev.empty(32 * K * 2).fill(0)
        yd = dev.empty(32 * N * 4)
        for M in (1, 2, 8, 16, 17, 32):
            rc = L.yah_qgemv(wd.ptr, t, N, K, F.row_bytes(t, K), 0, xd.ptr, M, K, yd.ptr, 0, N, 0, None, 0, None)
            assert rc == 0, (N, K, M, L.yah_last_error())
        dev.synchronize()
        assert not yd.download(np.float32, (32, N)).any()


def test_tc_deterministic(pkg, F, dev, impl):
    """Cluster partial sums are added in rank order: repeated calls give identical bits."""
    impl(TC)
    t = F.Q4_K
    M, N, K = 32, 4096, 14336
    w = F.synth_weights(t, N, K, seed=71)
    x = F.synth_activations(M, K, seed=72)
    a = pkg.ops.qgemv(dev, w, t, x, N=N, K=K)
    for _ in range(2):
        assert np.array_equal(a.view(np.uint32), pkg.ops.qgemv(dev, w, t, x, N=N, K=K).view(np.uint32))


@pytest.mark.parametrize("gfmt,ufmt", [("q4_k", "q4_k"), ("q4_k", "q6_k"), ("q6_k", "q8_0"), ("q8_0", "q4_k")])
@pytest.mark.parametrize("M", [1, 8, 32])
def test_qgemv_swiglu_two_tensors(pkg, F, O, dev, gfmt, ufmt, M):
    """y = silu(G x) * (U x) with the gate and up tensors in (possibly different) formats."""
    tg, tu = F.type_of(gfmt), F.type_of(ufmt)
    N, K = 1536, 4096
    wg = F.synth_weights(tg, N, K, seed=81)
    wu = F.synth_weights(tu, N, K, seed=82)
    x = F.synth_activations(M, K, seed=83 + M)
    g = O.gemm_ref(O.dequant_f32(tg, wg, N, K), x)
    u = O.gemm_ref(O.dequant_f32(tu, wu, N, K), x)
    ref = silu(g) * u
    L = pkg.lib()
    dg, du, xd, yd = dev.upload(wg), dev.upload(wu), dev.upload(x), dev.empty(M * N * 4)
    rc = L.yah_qgemv_swiglu(dg.ptr, tg, wg.shape[1], du.ptr, tu, wu.shape[1], N, K, xd.ptr, M, K, yd.ptr, N, None)
    assert rc == 0, L.yah_last_error()
    check(O, yd.download(np.float32, (M, N)), ref, absolute=False)


def test_qgemv_swiglu_refusals(pkg, F, dev):
    L = pkg.lib()
    t = F.Q4_K
    N, K, M = 256, 256, 1
    wd, xd, yd = dev.empty(N * F.row_bytes(t, K)), dev.empty(M * K * 2), dev.empty(M * N * 4)
    assert L.yah_qgemv_swiglu(wd.ptr, t, F.row_bytes(t, K), wd.ptr, t, F.row_bytes(t, K), N, K, xd.ptr, M, K, None,
                              N, None) == 1
    # the GEMV's swiglu kind in place needs an f32 output
    assert L.yah_qgemv(wd.ptr, t, N, K, F.row_bytes(t, K), 0, xd.ptr, M, K, yd.ptr, 1, N, 2, yd.ptr, N, None) == 1
    assert L.yah_set_gemv_impl(3) == 1
    code = ctypes.c_int(-1)
    assert L.yah_status_word(ctypes.byref(code)) == 0 and code.value == 0
