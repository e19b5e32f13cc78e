"""The allocation-free decode GEMV (yah_qgemv_noalloc) against the regular one (yah_qgemv).

yah_qgemv_noalloc exists for callers that cannot allocate device memory while they run the GEMV: work recorded
inside a CUDA-graph capture, a decode loop that must stay within a fixed device-memory budget, or a host program
whose device allocator is owned by another framework. It computes the same thing as yah_qgemv but keeps its
split-K scratch in a fixed device array inside the library instead of a buffer the library allocates on demand.

Both entry points run the same kernels with the same fixed reduction order; only the scratch address differs. So
the allocation-free one, called twice in a row (the second call reuses the scratch the first one left behind, with
a different shape), must give exactly the bits of the regular entry point, and once more the GEMV tests' bars
against the float64 oracle (max-abs <= 2e-2, relative Frobenius <= 1e-3, max |y - ref| / max |ref| <= 1e-4). A
call whose scratch would not fit in the fixed array is refused with YAH_ERR_SIZE.
This file is named so that pytest collects it last; it passes alone in a fresh process as well.
"""
import ctypes
import os
import sys

import numpy as np
import pytest

sys.path.insert(0, os.path.abspath(os.path.join(os.path.dirname(__file__), "..")))
import __graft_entry__ as ge  # noqa: E402

pytestmark = pytest.mark.gpu

ERR_SIZE = 3
EPI_STORE, EPI_RESID = 0, 1


def _run(lib, fn, dev, w, t, x, N, K, resid=None):
    """Upload w and x, run one GEMV entry point (plain, or resid onto `resid`), return the f32 output [M][N]."""
    M = x.shape[0]
    wd, xd = dev.upload(w), dev.upload(x)
    if resid is None:
        yd = dev.empty(M * N * 4).fill(0)
        rc = fn(wd.ptr, t, N, K, w.shape[1], 0, xd.ptr, M, K, yd.ptr, 0, N, EPI_STORE, None, 0, None)
    else:
        yd = dev.upload(resid.astype(np.float32))
        rc = fn(wd.ptr, t, N, K, w.shape[1], 0, xd.ptr, M, K, yd.ptr, 0, N, EPI_RESID, yd.ptr, N, None)
    assert rc == 0, lib.yah_last_error()
    assert lib.yah_device_synchronize() == 0
    return yd.download(np.float32, (M, N))


def _status_clean(lib):
    code = ctypes.c_int(-1)
    assert lib.yah_qgemv_noalloc_status(ctypes.byref(code)) == 0
    return code.value == 0


def test_noalloc_gemv_matches_regular_gemv_twice():
    pkg = ge.load_package()
    F, lib = pkg.formats, pkg.lib()
    from oracle import oracle as O
    dev = pkg.Device(0)
    # Two different shapes and formats on the mma.sync kernel, both split over K (so both use the scratch): the
    # second call starts from whatever the first one left in the shared array.
    for call, (t, M, N, K, seed) in enumerate([(F.Q8_0, 8, 512, 4096, 31), (F.Q6_K, 17, 1000, 2048, 32)]):
        w = F.synth_weights(t, N, K, seed=seed)
        x = F.synth_activations(M, K, seed=seed + 100)
        ref = _run(lib, lib.yah_qgemv, dev, w, t, x, N, K)
        got = _run(lib, lib.yah_qgemv_noalloc, dev, w, t, x, N, K)
        assert np.isfinite(got).all(), f"call {call}: non-finite output"
        assert np.array_equal(got.view(np.uint32), ref.view(np.uint32)), \
            f"call {call}: {np.count_nonzero(got != ref)} outputs differ from yah_qgemv"
        assert _status_clean(lib), f"call {call}: status word set"
        if call == 0:  # the shared result against the float64 oracle of the f32 weights
            e = O.errors(got, O.gemm_ref(O.dequant_f32(t, w, N, K), x))
            assert e["max_abs"] <= 2e-2 and e["rel_fro"] <= 1e-3 and e["rel_max"] <= 1e-4, e


def test_noalloc_resid_one_token():
    """One decode token of Q4_K with the residual epilogue (the one-token form, which needs no scratch; the entry
    point then only uses its own status word): y = resid + W x, same bits."""
    pkg = ge.load_package()
    F, lib = pkg.formats, pkg.lib()
    dev = pkg.Device(0)
    t = F.Q4_K
    N, K = 16 * dev.sm_count + 96, 2048
    w = F.synth_weights(t, N, K, seed=41)
    x = F.synth_activations(1, K, seed=42)
    resid = np.random.default_rng(43).standard_normal((1, N)).astype(np.float32)
    ref = _run(lib, lib.yah_qgemv, dev, w, t, x, N, K, resid=resid)
    got = _run(lib, lib.yah_qgemv_noalloc, dev, w, t, x, N, K, resid=resid)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))
    assert _status_clean(lib)


def test_noalloc_refuses_scratch_beyond_its_array():
    """A call whose split scratch exceeds the fixed array is refused before any launch (YAH_ERR_SIZE). Only the
    mma.sync kernel uses scratch (the tcgen05 kernel adds its K parts in distributed shared memory), so Q8_0, which
    runs on it, sizes the refused call."""
    pkg = ge.load_package()
    F, lib = pkg.formats, pkg.lib()
    dev = pkg.Device(0)
    t = F.Q8_0
    # 32 tokens of K = 4096 (264 KB of activations: too many to keep resident, so stream-K) over 4141 row blocks:
    # more split counters than the array holds
    M, N, K = 32, 530_000, 4096
    wd = dev.empty(N * F.row_bytes(t, K)).fill(0)  # valid (all-zero) blocks, in case a launch did happen
    xd = dev.empty(M * K * 2).fill(0)
    yd = dev.empty(M * N * 4).fill(0)
    rc = lib.yah_qgemv_noalloc(wd.ptr, t, N, K, F.row_bytes(t, K), 0, xd.ptr, M, K, yd.ptr, 0, N, EPI_STORE, None, 0,
                               None)
    assert rc == ERR_SIZE, (rc, lib.yah_last_error())
    assert b"exceed" in lib.yah_last_error()
    assert lib.yah_device_synchronize() == 0 and _status_clean(lib)
