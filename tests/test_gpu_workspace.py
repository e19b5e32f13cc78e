"""Caller-owned workspace entry points (yah_qgemm_ws, yah_qgemv_ws) against the library-owned ones.

The workspace variants run the same kernels with the same accumulation order; only where the chunk sums, split-K
chunk results and GEMV partial sums live differs. So every call must give exactly the bits of yah_qgemm_tile /
yah_qgemv with the same arguments, starting from a workspace full of garbage (it holds no state between calls), and
two calls on two streams with two workspaces may overlap. A workspace smaller than the size query says is refused
before any launch (YAH_ERR_SIZE), a misaligned one with YAH_ERR_ARG.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ERR_ARG, ERR_SIZE = 1, 3
STORE, RESID, SWIGLU = 0, 1, 2
F32, F16 = 0, 1


def gemm_size(L, t, N, K, M, y_dtype, epi, bn, grid, kchunk, pair):
    n = ctypes.c_size_t(12345)
    rc = L.yah_qgemm_workspace_size(t, N, K, M, y_dtype, epi, bn, grid, kchunk, pair, ctypes.byref(n))
    assert rc == 0, L.yah_last_error()
    return n.value


def gemv_size(L, t, N, K, M):
    n = ctypes.c_size_t(12345)
    assert L.yah_qgemv_workspace_size(t, N, K, M, ctypes.byref(n)) == 0, L.yah_last_error()
    return n.value


def bits(a):
    return a.view(np.uint32 if a.dtype == np.float32 else np.uint16)


# (type, N, K, M, y_dtype, epilogue, bn, grid, kchunk, cta_pair, expect a workspace)
GEMM_CASES = [
    ("q4_k", 1024, 8192, 64, F32, STORE, 0, 0, 0, -1, True),       # chunked, split K (few tiles)
    ("q6_k", 768, 4096, 300, F32, RESID, 0, 0, 1024, 0, True),     # explicit chunk, single CTAs, split K
    ("q8_0", 4096, 8192, 700, F16, SWIGLU, 192, 0, 0, 0, True),    # chunked, not split (enough tiles)
    ("q4_k", 2048, 4096, 200, F32, STORE, 0, 0, 0, -1, False),     # no chunking: no workspace
    ("q4_k", 512, 14336, 40, F32, STORE, 160, 37, 0, 1, True),     # explicit grid: chunked, never split
]


@pytest.mark.parametrize("case", GEMM_CASES, ids=lambda c: f"{c[0]}-{c[1]}x{c[2]}-M{c[3]}-e{c[5]}")
def test_qgemm_ws_matches_library_workspace(pkg, F, O, dev, case):
    fmt, N, K, M, ydt, epi, bn, grid, kchunk, pair, expect = case
    L = pkg.lib()
    t = F.type_of(fmt)
    w = F.synth_weights(t, N, K, seed=N + K + M)
    x = F.synth_activations(M, K, seed=M + 7)
    rng = np.random.default_rng(M)
    aux = (rng.standard_normal((M, N)) * (4 if epi == SWIGLU else 1)).astype(np.float32)
    wd, xd = dev.upload(w), dev.upload(x)
    auxd = dev.upload(aux) if epi != STORE else None
    ybytes = M * N * (2 if ydt == F16 else 4)
    nbytes = gemm_size(L, t, N, K, M, ydt, epi, bn, grid, kchunk, pair)
    assert (nbytes > 0) == expect, nbytes
    outs = []
    for use_ws in (False, True):
        yd = dev.empty(ybytes).fill(0)
        args = (wd.ptr, t, N, K, w.shape[1], 0, xd.ptr, M, K, yd.ptr, ydt, N, epi, auxd.ptr if auxd else None, N,
                bn, grid, kchunk, pair)
        if use_ws:
            ws = dev.empty(nbytes).fill(0xFF) if nbytes else None  # garbage: the workspace holds no state
            rc = L.yah_qgemm_ws(*args, ws.ptr if ws else None, nbytes, None)
        else:
            rc = L.yah_qgemm_tile(*args, None)
        assert rc == 0, L.yah_last_error()
        dev.synchronize()
        outs.append(yd.download(np.float16 if ydt == F16 else np.float32, (M, N)))
    assert np.array_equal(bits(outs[0]), bits(outs[1])), f"{np.count_nonzero(outs[0] != outs[1])} outputs differ"
    assert dev.status_word() == 0
    if epi == STORE:
        e = O.errors(outs[1], O.gemm_ref(O.dequant_f16(t, w, N, K), x))
        assert e["rel_fro"] <= 1e-3, e


def test_qgemm_ws_refusals(pkg, F, dev):
    L = pkg.lib()
    t = F.Q4_K
    N, K, M = 1024, 8192, 64
    nbytes = gemm_size(L, t, N, K, M, F32, STORE, 0, 0, 0, -1)
    assert nbytes > 0
    wd = dev.empty(N * F.row_bytes(t, K)).fill(0)
    xd, yd = dev.empty(M * K * 2).fill(0), dev.empty(M * N * 4).fill(0)
    ws = dev.empty(nbytes + 256)
    args = (wd.ptr, t, N, K, F.row_bytes(t, K), 0, xd.ptr, M, K, yd.ptr, F32, N, STORE, None, 0, 0, 0, 0, -1)
    assert L.yah_qgemm_ws(*args, ws.ptr, nbytes - 256, None) == ERR_SIZE
    assert b"workspace" in L.yah_last_error()
    assert L.yah_qgemm_ws(*args, None, 0, None) == ERR_ARG
    assert L.yah_qgemm_ws(*args, ws.ptr + 16, nbytes, None) == ERR_ARG
    dev.synchronize()
    assert dev.status_word() == 0


def test_qgemm_ws_two_streams_overlap(pkg, F, dev):
    """Two split-K GEMMs on two streams, each with its own workspace, launched back to back: both give the bits of
    the serial library-workspace calls."""
    L = pkg.lib()
    shapes = [(F.Q4_K, 1024, 8192, 64, 11), (F.Q6_K, 1536, 8192, 48, 12)]
    data, refs = [], []
    for t, N, K, M, seed in shapes:
        w = F.synth_weights(t, N, K, seed=seed)
        x = F.synth_activations(M, K, seed=seed + 1)
        wd, xd, yd = dev.upload(w), dev.upload(x), dev.empty(M * N * 4).fill(0)
        assert L.yah_qgemm_tile(wd.ptr, t, N, K, w.shape[1], 0, xd.ptr, M, K, yd.ptr, F32, N, STORE, None, 0, 0, 0,
                                0, -1, None) == 0, L.yah_last_error()
        dev.synchronize()
        refs.append(yd.download(np.float32, (M, N)))
        nbytes = gemm_size(L, t, N, K, M, F32, STORE, 0, 0, 0, -1)
        data.append((t, N, K, M, w, wd, xd, dev.empty(M * N * 4).fill(0), dev.empty(nbytes).fill(0xFF), nbytes))
    streams = [pkg.Stream(), pkg.Stream()]
    for rep in range(3):
        for (t, N, K, M, w, wd, xd, yd, ws, nbytes), s in zip(data, streams):
            rc = L.yah_qgemm_ws(wd.ptr, t, N, K, w.shape[1], 0, xd.ptr, M, K, yd.ptr, F32, N, STORE, None, 0, 0, 0, 0,
                                -1, ws.ptr, nbytes, s.handle)
            assert rc == 0, L.yah_last_error()
        for s in streams:
            s.synchronize()
        for (t, N, K, M, w, wd, xd, yd, ws, nbytes), ref in zip(data, refs):
            got = yd.download(np.float32, (M, N))
            assert np.array_equal(bits(got), bits(ref)), (rep, t)
    assert dev.status_word() == 0


@pytest.fixture
def gemv_impl(pkg):
    L = pkg.lib()
    yield lambda which: L.yah_set_gemv_impl(which)
    assert L.yah_set_gemv_impl(0) == 0


# (type, N, K, M, gemv impl) -- Q8_0 at 32 tokens of K = 4096 runs stream-K (a workspace); Q4_K at 20 tokens of
# K = 14336 on the mma.sync kernel as well; Q4_K at 32 tokens on the tcgen05 kernel needs none
GEMV_CASES = [("q8_0", 4096, 4096, 32, 0), ("q4_k", 4096, 14336, 20, 2), ("q6_k", 2000, 8192, 24, 0),
              ("q4_k", 4096, 14336, 32, 0), ("q4_k", 14336, 4096, 1, 0)]


@pytest.mark.parametrize("case", GEMV_CASES, ids=lambda c: f"{c[0]}-{c[1]}x{c[2]}-M{c[3]}-impl{c[4]}")
def test_qgemv_ws_matches_library_workspace(pkg, F, O, dev, gemv_impl, case):
    fmt, N, K, M, which = case
    assert gemv_impl(which) == 0
    L = pkg.lib()
    t = F.type_of(fmt)
    w = F.synth_weights(t, N, K, seed=N + M)
    x = F.synth_activations(M, K, seed=M + 3)
    resid = np.random.default_rng(5).standard_normal((M, N)).astype(np.float32)
    wd, xd = dev.upload(w), dev.upload(x)
    nbytes = gemv_size(L, t, N, K, M)
    outs = []
    for use_ws in (False, True, True):
        yd = dev.upload(resid)
        args = (wd.ptr, t, N, K, w.shape[1], 0, xd.ptr, M, K, yd.ptr, F32, N, RESID, yd.ptr, N)
        if use_ws:
            ws = dev.empty(nbytes).fill(0x5A) if nbytes else None  # nonzero counters must be cleared by the call
            rc = L.yah_qgemv_ws(*args, ws.ptr if ws else None, nbytes, None)
        else:
            rc = L.yah_qgemv(*args, None)
        assert rc == 0, L.yah_last_error()
        dev.synchronize()
        outs.append(yd.download(np.float32, (M, N)))
    for o in outs[1:]:
        assert np.array_equal(bits(outs[0]), bits(o)), f"{np.count_nonzero(outs[0] != o)} outputs differ"
    assert dev.status_word() == 0
    e = O.errors(outs[1], O.gemm_ref(O.dequant_f32(t, w, N, K), x) + resid)
    assert e["max_abs"] <= 2e-2 and e["rel_fro"] <= 1e-3 and e["rel_max"] <= 1e-4, e


def test_qgemv_ws_sizes_and_refusals(pkg, F, dev, gemv_impl):
    L = pkg.lib()
    t = F.Q8_0
    N, K, M = 4096, 4096, 32
    nbytes = gemv_size(L, t, N, K, M)
    assert nbytes > 0  # stream-K with split row blocks
    assert gemv_size(L, F.Q4_K, 14336, 4096, 1) == 0  # the one-token form: row ranges
    assert gemv_impl(1) == 0
    assert gemv_size(L, F.Q4_K, 4096, 14336, 32) == 0  # tcgen05: K parts meet in distributed shared memory
    assert gemv_impl(0) == 0
    wd = dev.empty(N * F.row_bytes(t, K)).fill(0)
    xd, yd = dev.empty(M * K * 2).fill(0), dev.empty(M * N * 4).fill(0)
    ws = dev.empty(nbytes + 256)
    args = (wd.ptr, t, N, K, F.row_bytes(t, K), 0, xd.ptr, M, K, yd.ptr, F32, N, STORE, None, 0)
    assert L.yah_qgemv_ws(*args, ws.ptr, nbytes - 4, None) == ERR_SIZE
    assert L.yah_qgemv_ws(*args, None, 0, None) == ERR_ARG
    assert L.yah_qgemv_ws(*args, ws.ptr + 64, nbytes, None) == ERR_ARG
    n = ctypes.c_size_t()
    assert L.yah_qgemv_workspace_size(t, N, K, 33, ctypes.byref(n)) == ERR_ARG
    dev.synchronize()
    assert dev.status_word() == 0
