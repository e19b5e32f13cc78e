"""Seeded synthetic tensors follow the benchmark configurations' distributions (checked on the decoded values)."""
import numpy as np


def test_row_bytes(F):
    assert F.row_bytes("q4_k", 4096) == 2304
    assert F.row_bytes("Q8_0", 4096) == 4352
    assert F.row_bytes(14, 4096) == 3360


def test_q8_0_distribution(F):
    w = F.synth_weights(F.Q8_0, 64, 1024, seed=0).reshape(-1, 34)
    q = w[:, 2:].view(np.int8)
    assert q.min() >= -127 and q.max() <= 127
    d = w[:, :2].copy().view(np.float16).astype(np.float32)
    assert (d >= 0).all() and 0.02 / 127 * 0.6 < d.mean() < 0.02 / 127 * 1.0


def test_q4_k_distribution(F):
    w = F.synth_weights(F.Q4_K, 64, 1024, seed=0).reshape(-1, 144)
    d = w[:, 0:2].copy().view(np.float16).astype(np.float32)
    dmin = w[:, 2:4].copy().view(np.float16).astype(np.float32)
    assert (d >= 0).all() and (dmin >= 0).all()
    assert 0.006 < d.mean() < 0.01 and 0.003 < dmin.mean() < 0.005
    sc = w[:, 4:16] & 63
    assert sc.min() == 0 and sc.max() == 63


def test_q6_k_distribution(F):
    w = F.synth_weights(F.Q6_K, 64, 1024, seed=0).reshape(-1, 210)
    sc = w[:, 192:208].view(np.int8)
    assert sc.min() == -32 and sc.max() == 31


def test_determinism(F):
    a = F.synth_weights("q4_k", 8, 512, seed=5)
    b = F.synth_weights("q4_k", 8, 512, seed=5)
    c = F.synth_weights("q4_k", 8, 512, seed=6)
    assert np.array_equal(a, b) and not np.array_equal(a, c)
