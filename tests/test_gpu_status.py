"""The failure path on the GPU, without a fault: a bounded wait that runs out reports through the status word.

Every mbarrier wait in the kernels is bounded; when one runs out, the kernel records a code in the device status word,
drains its own copies and returns, so the host can raise instead of the GPU hanging. Here a one-warp kernel waits on
an mbarrier that nothing arrives on, through the same wait routine with a short budget (no trap, no bad address);
the test checks the reported code and that the device keeps working afterwards.
"""
import ctypes
import time

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_bounded_wait_reports_timeout(pkg, F, O, dev):
    from importlib import import_module
    L = import_module(pkg.__name__ + "._lib")
    code = ctypes.c_int(-1)
    t0 = time.time()
    L.check(L.lib().yah_selftest_bounded_wait(2_000_000, ctypes.byref(code)))
    assert code.value == 1, code.value  # a consumer's wait for data ran out
    assert time.time() - t0 < 30
    assert dev.status_word() == 0  # the call cleared the word
    # the device is still usable: a decode GEMV right after it meets the bar
    N, K = 2048, 4096
    w = F.synth_weights(F.Q4_K, N, K, seed=5)
    x = F.synth_activations(1, K, seed=6)
    y = pkg.ops.qgemv(dev, w, F.Q4_K, x, N=N, K=K)
    e = O.errors(y, O.gemm_ref(O.dequant_f32(F.Q4_K, w, N, K), x))
    assert e["finite"] and e["rel_fro"] <= 1e-3, e
    assert dev.status_word() == 0


def test_bounded_wait_rejects_bad_budget(pkg):
    from importlib import import_module
    L = import_module(pkg.__name__ + "._lib")
    code = ctypes.c_int(0)
    assert L.lib().yah_selftest_bounded_wait(10, ctypes.byref(code)) != 0
    assert L.lib().yah_selftest_bounded_wait(1 << 40, ctypes.byref(code)) != 0
