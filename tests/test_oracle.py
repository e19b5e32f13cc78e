"""The CPU oracle against the committed golden vectors (gguf-py 0.19.0, the reference's own dequant oracle).

These pin the oracle before any GPU result is compared with it: f16 dequant bit patterns (dq_bfp16_check.py:87-92
counts differing bit patterns, which must be 0), the f32 values, and a small token-major GEMM.
"""
import os

import numpy as np
import pytest

from conftest import GOLDEN

FMTS = ["q8_0", "q4_k", "q6_k", "q5_k", "q3_k", "iq4_xs"]


@pytest.mark.parametrize("name", FMTS)
def test_dequant_f16_bits_match_golden(F, O, name):
    z = np.load(os.path.join(GOLDEN, f"dequant_{name}.npz"))
    t = F.type_of(name)
    b, K = z["blocks"], int(z["K"])
    got = O.dequant_f16(t, b, b.shape[0], K).view(np.uint16)
    assert np.count_nonzero(got != z["f16"]) == 0


@pytest.mark.parametrize("name", FMTS)
def test_dequant_f32_matches_golden(F, O, name):
    z = np.load(os.path.join(GOLDEN, f"dequant_{name}.npz"))
    t = F.type_of(name)
    b, K = z["blocks"], int(z["K"])
    got = O.dequant_f32(t, b, b.shape[0], K)
    assert np.array_equal(got.view(np.uint32), z["f32"].view(np.uint32))


@pytest.mark.parametrize("name", FMTS)
def test_gemm_oracle_matches_golden(F, O, name):
    z = np.load(os.path.join(GOLDEN, f"gemm_{name}.npz"))
    t = F.type_of(name)
    w, K, x = z["blocks"], int(z["K"]), z["x"]
    N = w.shape[0]
    y16 = O.gemm_ref(O.dequant_f16(t, w, N, K), x)
    y32 = O.gemm_ref(O.dequant_f32(t, w, N, K), x)
    np.testing.assert_allclose(y16, z["y_f16w"], rtol=1e-12, atol=1e-9)
    np.testing.assert_allclose(y32, z["y_f32w"], rtol=1e-12, atol=1e-9)


@pytest.mark.parametrize("name", FMTS)
def test_golden_inputs_regenerate_from_seed(F, name):
    """The synthetic generator still produces the committed bytes (the seed and draw order are stable)."""
    z = np.load(os.path.join(GOLDEN, f"gemm_{name}.npz"))
    t = F.type_of(name)
    w = F.synth_weights(t, z["blocks"].shape[0], int(z["K"]), seed=100 + t)
    assert np.array_equal(w, z["blocks"])
    x = F.synth_activations(z["x"].shape[0], int(z["K"]), seed=200 + t)
    assert np.array_equal(x.view(np.uint16), z["x"].view(np.uint16))


def test_k_window_and_row_stride(F, O):
    """kb_off / row_stride views decode the same values as slicing the full rows."""
    t = F.Q4_K
    w = F.synth_weights(t, 5, 1024, seed=3)
    full = O.dequant_f16(t, w, 5, 1024).view(np.uint16)
    win = O.dequant_f16(t, w, 5, 512, row_stride=w.shape[1], kb_off=2).view(np.uint16)
    assert np.array_equal(win, full[:, 512:])


def test_epilogue_refs(O):
    acc = np.array([[1.0, -2.0]])
    assert np.allclose(O.epilogue_ref(acc, 1, np.array([[0.5, 0.5]])), [[1.5, -1.5]])
    g = np.array([[0.0, 3.0]])
    assert np.allclose(O.epilogue_ref(acc, 2, g), [[0.0, -2.0 * 3.0 / (1 + np.exp(-3.0))]])


def test_plant_mistake_is_caught(F, O):
    """A deliberately wrong oracle value (planted on the CPU) makes the bit comparison fail."""
    z = np.load(os.path.join(GOLDEN, "dequant_q4_k.npz"))
    got = O.dequant_f16(F.Q4_K, z["blocks"], z["blocks"].shape[0], int(z["K"])).view(np.uint16).copy()
    got[3, 17] ^= 1
    assert np.count_nonzero(got != z["f16"]) == 1


def test_rounding_x_to_f16_misses_the_gemv_bar(F, O):
    """The reference GEMV takes f32 activations (gen_gemv.py:4). The same GEMV with x rounded to f16 first is off by
    more than the reference checker's max |y - ref| / max |ref| <= 1e-4 (gemv_check.py:176-183): the f32 operand has
    to be kept (the GPU path splits it into two f16 parts)."""
    t = F.Q4_K
    N, K = 512, 14336
    w = F.synth_weights(t, N, K, seed=31)
    x = np.random.default_rng(32).standard_normal((1, K), dtype=np.float32)
    wf = O.dequant_f32(t, w, N, K)
    e = O.errors(O.gemm_ref(wf, x.astype(np.float16)), O.gemm_ref(wf, x))
    assert e["rel_max"] > 1e-4, e
