"""The allocation-free decode GEMV (yah_qgemv_noalloc) against the regular one (yah_qgemv).

yah_qgemv_noalloc exists for callers that cannot allocate device memory while they run the GEMV: work recorded
inside a CUDA-graph capture, a decode loop that must stay within a fixed device-memory budget, or a host program
whose device allocator is owned by another framework. It computes the same thing as yah_qgemv but keeps its
split-K scratch in a fixed device array inside the library instead of a buffer the library allocates on demand.

Both entry points are called through the C ABI on the same inputs; the allocation-free one is called twice in a
row (the second call reuses the scratch the first one left behind, with a different shape) and each result must
match the regular entry point within the GEMV tests' tolerance (max-abs <= 2e-2, relative Frobenius <= 1e-3).
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


def _run(lib, fn, dev, w, t, x, N, K):
    """Upload w and x, run one GEMV entry point, return the f32 output [M][N]."""
    M = x.shape[0]
    wd, xd = dev.upload(w), dev.upload(x)
    yd = dev.empty(M * N * 4).fill(0)
    rc = fn(wd.ptr, t, N, K, w.shape[1], 0, xd.ptr, M, K, yd.ptr, 0, N, 0, None, 0, None)
    assert rc == 0, lib.yah_last_error()
    assert lib.yah_device_synchronize() == 0
    return yd.download(np.float32, (M, N))


def test_noalloc_gemv_matches_regular_gemv_twice():
    pkg = ge.load_package()
    F, lib = pkg.formats, pkg.lib()
    dev = pkg.Device(0)
    t = F.Q4_K
    # Two different shapes, both split over K (so both use the scratch): the second call starts from whatever the
    # first one left in the shared array.
    for call, (M, N, K, seed) in enumerate([(8, 512, 4096, 31), (17, 1000, 2048, 32)]):
        w = F.synth_weights(t, N, K, seed=seed)
        x = F.synth_activations(M, K, seed=seed + 100)
        ref = _run(lib, lib.yah_qgemv, dev, w, t, x, N, K)
        got = _run(lib, lib.yah_qgemv_noalloc, dev, w, t, x, N, K)
        d = np.abs(got.astype(np.float64) - ref.astype(np.float64))
        rel_fro = np.linalg.norm(d) / np.linalg.norm(ref.astype(np.float64))
        assert np.isfinite(got).all(), f"call {call}: non-finite output"
        assert d.max() <= 2e-2 and rel_fro <= 1e-3, f"call {call}: max-abs {d.max()}, rel-Frobenius {rel_fro}"
        code = ctypes.c_int(-1)
        assert lib.yah_qgemv_noalloc_status(ctypes.byref(code)) == 0
        assert code.value == 0, f"call {call}: status word {code.value}"
