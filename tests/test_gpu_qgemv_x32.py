"""The decode GEMV with f32 activations (yah_qgemv_x / yah_qgemv_swiglu_x with YAH_F32): the reference GEMV's own
binding, x f32[K] and y f32 (engine/gpu/loom/tools/gen_gemv.py:4, :729; engine/model/loom_decoder.hpp:432-434).

The oracle is the reference checker's: gguf-py's f32 dequant times the f32 activations in float64
(gemv_check.py:161-162); bars max-abs <= 2e-2, relative Frobenius <= 1e-3 and max |y - ref| / max |ref| <= 1e-4
(gemv_check.py:176-183). The activations are drawn in f32 and never rounded to f16 on the host: a GEMV that rounded
them would miss the 1e-4 bar (tests/test_oracle.py::test_rounding_x_to_f16_misses_the_gemv_bar shows it on the
oracle alone).
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
FMTS = ["q8_0", "q4_k", "q6_k", "q5_k", "q3_k", "iq4_xs"]
F16, F32 = 1, 0


def x32(M, K, seed):
    return np.random.default_rng(seed).standard_normal((M, K), dtype=np.float32)


def check(O, y, ref, absolute=True):
    e = O.errors(y, ref)
    assert e["finite"] and e["rel_fro"] <= 1e-3 and e["rel_max"] <= 1e-4, e
    if absolute:
        assert e["max_abs"] <= 2e-2, e
    return e


@pytest.mark.parametrize("name", FMTS)
@pytest.mark.parametrize("M", [1, 3, 8, 32])
@pytest.mark.parametrize("N,K", [(4096, 14336), (1000, 2048), (128, 4096)])
def test_qgemv_f32_activations(pkg, F, O, dev, name, M, N, K):
    """Config 3's shape (K = 14336: two tokens per launch, so 32 tokens take 16 launches), fewer rows than SMs hold
    row ranges for (N = 1000, 128: fewer CTAs), every format."""
    t = F.type_of(name)
    if F.row_bytes(t, K) % 16:
        pytest.skip("rows must be 16-byte multiples")
    w = F.synth_weights(t, N, K, seed=N + K + 1)
    x = x32(M, K, seed=M + 2)
    y = pkg.ops.qgemv(dev, w, t, x, N=N, K=K, x_dtype="f32")
    check(O, y, O.gemm_ref(O.dequant_f32(t, w, N, K), x))


@pytest.mark.parametrize("M", [1, 8])
def test_kinds_with_f32_activations(pkg, F, O, dev, M):
    """resid, swiglu (f32 and f16 out) and swiglu in place over the gate, with f32 x."""
    t = F.Q4_K
    N, K = 2048, 4096
    w = F.synth_weights(t, N, K, seed=5)
    x = x32(M, K, seed=6)
    acc = O.gemm_ref(O.dequant_f32(t, w, N, K), x)
    rng = np.random.default_rng(7)
    resid = rng.standard_normal((M, N)).astype(np.float32)
    check(O, pkg.ops.qgemv(dev, w, t, x, N=N, K=K, kind="resid", aux=resid, x_dtype="f32"), acc + resid)
    gate = (rng.standard_normal((M, N)) * 4).astype(np.float32)
    with np.errstate(over="ignore"):
        ref = gate / (1.0 + np.exp(-gate.astype(np.float64))) * acc
    check(O, pkg.ops.qgemv(dev, w, t, x, N=N, K=K, kind="swiglu", aux=gate, x_dtype="f32"), ref, absolute=False)
    y16 = pkg.ops.qgemv(dev, w, t, x, N=N, K=K, kind="swiglu", aux=gate, out_dtype="f16", x_dtype="f32")
    assert (np.abs(y16 - ref) <= 1e-4 * np.abs(ref).max() + O.f16_half_ulp(ref)).all()
    L = pkg.lib()
    wd, xd, yd = dev.upload(w), dev.upload(x), dev.upload(gate)
    assert L.yah_qgemv_x(wd.ptr, t, N, K, w.shape[1], 0, xd.ptr, F32, M, K, yd.ptr, F32, N, 2, yd.ptr, N, None) == 0
    check(O, yd.download(np.float32, (M, N)), ref, absolute=False)


@pytest.mark.parametrize("gfmt,ufmt", [("q4_k", "q4_k"), ("q4_k", "q6_k"), ("iq4_xs", "q5_k")])
def test_swiglu_two_tensors_f32_activations(pkg, F, O, dev, gfmt, ufmt):
    tg, tu = F.type_of(gfmt), F.type_of(ufmt)
    M, N, K = 1, 14336, 4096
    wg = F.synth_weights(tg, N, K, seed=11)
    wu = F.synth_weights(tu, N, K, seed=12)
    x = x32(M, K, seed=13)
    g = O.gemm_ref(O.dequant_f32(tg, wg, N, K), x)
    u = O.gemm_ref(O.dequant_f32(tu, wu, N, K), x)
    with np.errstate(over="ignore"):
        ref = g / (1.0 + np.exp(-g)) * u
    L = pkg.lib()
    dg, du, xd, yd = dev.upload(wg), dev.upload(wu), dev.upload(x), dev.empty(M * N * 4)
    rc = L.yah_qgemv_swiglu_x(dg.ptr, tg, wg.shape[1], du.ptr, tu, wu.shape[1], N, K, xd.ptr, F32, M, K, yd.ptr, N,
                              None)
    assert rc == 0, L.yah_last_error()
    check(O, yd.download(np.float32, (M, N)), ref, absolute=False)


def test_f16_through_the_typed_entry_point_is_yah_qgemv(pkg, F, dev):
    L = pkg.lib()
    t = F.Q4_K
    M, N, K = 4, 4096, 4096
    w = F.synth_weights(t, N, K, seed=21)
    x = F.synth_activations(M, K, seed=22)
    wd, xd = dev.upload(w), dev.upload(x)
    outs = []
    for fn, extra in ((L.yah_qgemv, ()), (L.yah_qgemv_x, (F16,))):
        yd = dev.empty(M * N * 4)
        args = (wd.ptr, t, N, K, w.shape[1], 0, xd.ptr) + extra + (M, K, yd.ptr, F32, N, 0, None, 0, None)
        assert fn(*args) == 0, L.yah_last_error()
        outs.append(yd.download(np.float32, (M, N)))
    assert np.array_equal(outs[0].view(np.uint32), outs[1].view(np.uint32))


def test_f32_activation_refusals(pkg, F, dev):
    L = pkg.lib()
    t = F.Q4_K
    M, N, K = 1, 256, 256
    wd, xd, yd = dev.empty(N * F.row_bytes(t, K)), dev.empty(M * K * 4), dev.empty(M * N * 4)
    args = lambda xdt: (wd.ptr, t, N, K, F.row_bytes(t, K), 0, xd.ptr, xdt, M, K, yd.ptr, F32, N, 0, None, 0, None)
    assert L.yah_qgemv_x(*args(7)) == 2  # x_dtype
    assert L.yah_set_gemv_impl(1) == 0
    try:
        assert L.yah_qgemv_x(*args(F32)) == 2  # the tcgen05 kernel takes f16 activations only
    finally:
        assert L.yah_set_gemv_impl(0) == 0
    code = ctypes.c_int(-1)
    assert L.yah_status_word(ctypes.byref(code)) == 0 and code.value == 0

