"""Decode GEMV (M <= 32 tokens) vs the oracle through the C ABI.

The GEMV computes with the f32 weight values of the GGUF dequant, as the reference GEMV does, so the reference is
the reference GEMV's own oracle: gguf-py's f32 dequantisation times x in float64 (gemv_check.py:112, 161). Bars:
max-abs <= 2e-2 and relative Frobenius <= 1e-3 (the path's tolerance), and the reference GEMV checker's own bar,
max |y - ref| / max |ref| <= 1e-4 (gemv_check.py:176-183), on f32 output.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu
FMTS = ["q8_0", "q4_k", "q6_k", "q5_k", "q3_k", "iq4_xs"]


def check(O, y, ref, rel_max=1e-4):
    e = O.errors(y, ref)
    assert e["finite"] and e["max_abs"] <= 2e-2 and e["rel_fro"] <= 1e-3, e
    assert e["rel_max"] <= rel_max, e
    return e


@pytest.mark.parametrize("name", FMTS)
@pytest.mark.parametrize("M", [1, 2, 8, 16, 17, 32])
@pytest.mark.parametrize("N,K", [(256, 2048), (4096, 4096), (1000, 2048), (128, 256), (2048, 6144)])
def test_qgemv(pkg, F, O, dev, name, M, N, K):
    """Shapes covering every work split: one item per CTA (128 x 256), row blocks shared by up to 8 CTAs
    (256 x 2048), CTA ranges ending inside row blocks (4096 x 4096, 2048 x 6144) and a ragged last row block."""
    t = F.type_of(name)
    if F.row_bytes(t, K) % 16:
        pytest.skip("rows must be 16-byte multiples (Q6_K / Q3_K: 8 super-blocks, IQ4_XS: 2)")
    w = F.synth_weights(t, N, K, seed=N + K)
    x = F.synth_activations(M, K, seed=M)
    y = pkg.ops.qgemv(dev, w, t, x, N=N, K=K)
    check(O, y, O.gemm_ref(O.dequant_f32(t, w, N, K), x))


@pytest.mark.parametrize("name", FMTS)
def test_qgemv_resid_and_f16(pkg, F, O, dev, name):
    t = F.type_of(name)
    M, N, K = 5, 640, 4096
    w = F.synth_weights(t, N, K, seed=1)
    x = F.synth_activations(M, K, seed=2)
    acc = O.gemm_ref(O.dequant_f32(t, w, N, K), x)
    resid = np.random.default_rng(3).standard_normal((M, N)).astype(np.float32)
    y = pkg.ops.qgemv(dev, w, t, x, N=N, K=K, kind="resid", aux=resid)
    check(O, y, acc + resid)
    y16 = pkg.ops.qgemv(dev, w, t, x, N=N, K=K, out_dtype="f16")
    e = O.errors(y16, acc)
    assert e["rel_fro"] <= 1e-3 and (np.abs(y16 - acc) <= 2e-2 + O.f16_half_ulp(acc)).all()


def test_qgemv_and_qgemm_at_down_proj_k(pkg, F, O, dev):
    """Decode and prefill paths on the down-projection reduction length (K = 14336) both meet the bar (the
    prefill GEMM multiplies f16-rounded weights, so it is held to the path's tolerance against the f16 oracle)."""
    t = F.Q4_K
    M, N, K = 8, 1024, 14336
    w = F.synth_weights(t, N, K, seed=11)
    x = F.synth_activations(M, K, seed=12)
    check(O, pkg.ops.qgemv(dev, w, t, x, N=N, K=K), O.gemm_ref(O.dequant_f32(t, w, N, K), x))
    check(O, pkg.ops.qgemm(dev, w, t, x, N=N, K=K), O.gemm_ref(O.dequant_f16(t, w, N, K), x), rel_max=1e-3)


@pytest.mark.parametrize("M", [1, 8, 32])
def test_qgemv_down_proj_full(pkg, F, O, dev, M):
    """The decode sweep of the down projection at full size: Q4_K, N = 4096, K = 14336."""
    t = F.Q4_K
    N, K = 4096, 14336
    w = F.synth_weights(t, N, K, seed=21)
    x = F.synth_activations(M, K, seed=22 + M)
    check(O, pkg.ops.qgemv(dev, w, t, x, N=N, K=K), O.gemm_ref(O.dequant_f32(t, w, N, K), x))


@pytest.mark.parametrize("M", [1, 32])
def test_qgemv_lm_head_slice(pkg, F, O, dev, M):
    """Q6_K lm-head decode on a 16032-row slice (one eighth of the 128256-row vocabulary, K = 4096)."""
    t = F.Q6_K
    N, K = 16032, 4096
    w = F.synth_weights(t, N, K, seed=23)
    x = F.synth_activations(M, K, seed=24 + M)
    check(O, pkg.ops.qgemv(dev, w, t, x, N=N, K=K), O.gemm_ref(O.dequant_f32(t, w, N, K), x))


def test_qgemv_k_window(pkg, F, O, dev):
    t = F.Q8_0
    M, N, K, kb_off = 3, 300, 1024, 2
    w = F.synth_weights(t, N, K + 256 * kb_off + 512, seed=4)
    x = F.synth_activations(M, K, seed=5)
    y = pkg.ops.qgemv(dev, w, t, x, N=N, K=K, kb_off=kb_off, w_row_stride=w.shape[1])
    check(O, y, O.gemm_ref(O.dequant_f32(t, w, N, K, kb_off=kb_off), x))


def test_qgemv_repeat_deterministic(pkg, F, dev):
    """Row blocks shared by several CTAs are summed in a fixed order: repeated calls give identical bits."""
    t = F.Q4_K
    M, N, K = 32, 512, 14336
    w = F.synth_weights(t, N, K, seed=6)
    x = F.synth_activations(M, K, seed=7)
    a = pkg.ops.qgemv(dev, w, t, x, N=N, K=K)
    for _ in range(3):
        b = pkg.ops.qgemv(dev, w, t, x, N=N, K=K)
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


@pytest.mark.parametrize("overlap", [1, 0])
@pytest.mark.parametrize("M,K", [(1, 4096), (8, 8192)])
def test_qgemv_dependent_chain(pkg, F, O, dev, overlap, M, K):
    """Back-to-back launches on one stream where each GEMV reads the previous one's f16 output (a residual-free
    layer chain) and writes the buffer the launch before it read. With programmatic launch the weights stream
    early but activations and outputs wait for the preceding kernel; the result must equal the stepwise oracle.
    Covers the resident-activation split (M = 1) and stream-K with activation copies held back (M = 8)."""
    from importlib import import_module
    L = import_module(pkg.__name__ + "._lib")
    t = F.Q4_K
    steps = 4
    ws = []
    for i in range(steps):  # d and dmin scaled by 2^-10 so the chain's activations stay near unit size
        w = F.synth_weights(t, K, K, seed=70 + i)
        hdr = w.reshape(K, K // 256, 144)[:, :, :4]
        hdr[...] = (hdr.copy().view(np.float16) * np.float16(1 / 1024)).view(np.uint8)
        ws.append(w)
    wd = [dev.upload(w) for w in ws]
    x0 = F.synth_activations(M, K, seed=69)
    bufs = [dev.upload(x0), dev.empty(M * K * 2)]
    s = pkg.Stream()
    L.check(L.lib().yah_set_launch_overlap(overlap))
    try:
        for i in range(steps):
            src, dst = bufs[i % 2], bufs[(i + 1) % 2]
            pkg.ops.qgemv_ptr(wd[i].ptr, t, K, K, ws[i].shape[1], 0, src.ptr, M, K, dst.ptr, "f16", K,
                              stream=s.handle)
        s.synchronize()
        got = bufs[steps % 2].download(np.float16, (M, K)).astype(np.float32)
    finally:
        L.check(L.lib().yah_set_launch_overlap(1))
    x = x0
    for i in range(steps):  # the oracle, step by step, rounding to f16 between steps as the device does
        acc = O.gemm_ref(O.dequant_f32(t, ws[i], K, K), x)
        x = acc.astype(np.float16)
        if i < steps - 1:
            continue
        e = O.errors(got, acc)
        assert e["finite"] and e["rel_fro"] <= 1e-3, e
    for b in wd + bufs:
        b.close()
    s.close()


@pytest.mark.parametrize("N,K", [(4096, 4096), (4098, 4096), (2500, 8192), (4096, 14336)])
@pytest.mark.parametrize("kind,out", [("plain", "f32"), ("resid", "f32"), ("plain", "f16")])
def test_qgemv_q4k_one_token(pkg, F, O, dev, N, K, kind, out):
    """The one-token Q4_K form (4 rows x 4 super-blocks per MMA): ragged row counts (4098 rows: a last CTA with a
    partial row quad), 12- and 8-super-block stages, residual epilogue and f16 output."""
    t = F.Q4_K
    w = F.synth_weights(t, N, K, seed=N + 3 * K)
    x = F.synth_activations(1, K, seed=7)
    acc = O.gemm_ref(O.dequant_f32(t, w, N, K), x)
    if kind == "resid":
        resid = np.random.default_rng(8).standard_normal((1, N)).astype(np.float32)
        check(O, pkg.ops.qgemv(dev, w, t, x, N=N, K=K, kind="resid", aux=resid), acc + resid)
    elif out == "f16":
        y16 = pkg.ops.qgemv(dev, w, t, x, N=N, K=K, out_dtype="f16")
        e = O.errors(y16, acc)
        assert e["rel_fro"] <= 1e-3 and (np.abs(y16 - acc) <= 2e-2 + O.f16_half_ulp(acc)).all()
    else:
        check(O, pkg.ops.qgemv(dev, w, t, x, N=N, K=K), acc)


@pytest.mark.parametrize("M", [1, 8, 32])
def test_q6k_lm_head_k5120_realigned(pkg, F, O, dev, M):
    """The reference's Q6_K lm head has K = 5120: packed rows of 4200 bytes, not 16-byte aligned. Rows realigned
    once to a 4208-byte stride (yah_realign_rows; blocks untouched) run through the decode GEMV unchanged."""
    t = F.Q6_K
    N, K = 2048, 5120
    w = F.synth_weights(t, N, K, seed=51)
    assert w.shape[1] == 4200
    wd, stride = pkg.ops.realign(dev, w)
    assert stride == 4208
    x = F.synth_activations(M, K, seed=52 + M)
    y = pkg.ops.qgemv(dev, wd, t, x, N=N, K=K, w_row_stride=stride)
    check(O, y, O.gemm_ref(O.dequant_f32(t, w, N, K), x))
    wd.close()
