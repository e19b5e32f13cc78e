"""GPU dequant vs the oracle and the golden vectors: 0 differing f16 bit patterns (dq_bfp16_check.py:87-92)."""
import os

import numpy as np
import pytest

from conftest import GOLDEN

pytestmark = pytest.mark.gpu
FMTS = ["q8_0", "q4_k", "q6_k", "q5_k", "q3_k", "iq4_xs"]


@pytest.mark.parametrize("name", FMTS)
def test_dequant_golden_bits(pkg, F, dev, name):
    z = np.load(os.path.join(GOLDEN, f"dequant_{name}.npz"))
    b, K = z["blocks"], int(z["K"])
    got = pkg.ops.dequant(dev, b, F.type_of(name), N=b.shape[0], K=K).view(np.uint16)
    assert np.count_nonzero(got != z["f16"]) == 0


@pytest.mark.parametrize("name", FMTS)
@pytest.mark.parametrize("N,K,kb_off", [(37, 2048, 0), (300, 4096, 0), (16, 1024, 3)])
def test_dequant_random_bits(pkg, F, O, dev, name, N, K, kb_off):
    t = F.type_of(name)
    Kfull = K + 256 * kb_off
    w = F.synth_weights(t, N, Kfull, seed=N + K)
    got = pkg.ops.dequant(dev, w, t, N=N, K=K, kb_off=kb_off).view(np.uint16)
    ref = O.dequant_f16(t, w, N, K, kb_off=kb_off).view(np.uint16)
    assert np.count_nonzero(got != ref) == 0


@pytest.mark.parametrize("name", FMTS)
def test_dequant_extreme_bytes(pkg, F, O, dev, name):
    """Uniformly random bytes (any d, including negative, subnormal, inf and nan scales): bit-exact except nan
    payloads, which only have to stay nan."""
    t = F.type_of(name)
    N, K = 64, 1024
    rng = np.random.default_rng(99)
    w = rng.integers(0, 256, size=(N, F.row_bytes(t, K)), dtype=np.uint8)
    got = pkg.ops.dequant(dev, w, t, N=N, K=K)
    with np.errstate(all="ignore"):
        ref = O.dequant_f16(t, w, N, K)
    both_nan = np.isnan(got) & np.isnan(ref)
    diff = (got.view(np.uint16) != ref.view(np.uint16)) & ~both_nan
    assert np.count_nonzero(diff) == 0
