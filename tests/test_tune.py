"""Tile tuner and tile table: rule validation and table conversion on CPU; on the GPU a small search whose
candidates must all reproduce the default tile's output bit for bit, and yah_qgemm under the tuned table."""
import ctypes

import numpy as np
import pytest


def test_rule_struct_and_validation(pkg):
    L, T = pkg.lib(), pkg._lib.TileRule
    assert ctypes.sizeof(T) == 56  # 3 ints, padding, 3 int64s, 3 ints, padding (C layout)
    good = (T * 2)(T(12, 0, 1, 4096, 4096, 2048, 256, 0, 1), T(12, 1, 0, 4096, 14336, 4096, 192, 0, 0))
    assert L.yah_tile_rules_set(good, 2) == 0
    n = ctypes.c_int()
    assert L.yah_tile_rules_count(ctypes.byref(n)) == 0 and n.value == 2
    for bad in [T(12, 0, 1, 4096, 4096, 2048, 192, 0, 1),   # 192 is a single-CTA width
                T(12, 0, 1, 4096, 4096, 2048, 256, 0, 0),   # 256 is a pair width
                T(10, 0, 1, 4096, 4096, 2048, 192, 0, 0),   # unsupported format (Q2_K)
                T(12, 3, 1, 4096, 4096, 2048, 192, 0, 0),   # epilogue
                T(12, 0, 1, 4096, 4096, 0, 192, 0, 0)]:     # token bound
        assert L.yah_tile_rules_set(ctypes.byref(bad), 1) == pkg._lib.ERR_ARG
    assert L.yah_tile_rules_count(ctypes.byref(n)) == 0 and n.value == 2  # a refused set keeps the table
    assert L.yah_tile_rules_clear() == 0
    assert L.yah_tile_rules_count(ctypes.byref(n)) == 0 and n.value == 0


def test_table_to_rules(pkg):
    tu = pkg.tune
    table = {"entries": [{"fmt": 12, "epilogue": 1, "out": 0, "N": 4096, "K": 14336, "m_max": 4096, "bn": 192,
                          "grid": 0, "cta_pair": 0}]}
    r = tu.rules(table)[0]
    assert (r.ggml_type, r.epilogue, r.y_dtype, r.N, r.K, r.m_max, r.bn, r.cta_pair) == (12, 1, 0, 4096, 14336,
                                                                                         4096, 192, 0)
    sites = tu.stack_sites(pkg.tp.StackShape(), 8)
    assert [(s.name, s.N, s.K) for s in sites] == [("qkv", 768, 4096), ("o_proj", 4096, 512), ("gate", 1792, 4096),
                                                   ("up", 1792, 4096), ("down", 4096, 1792)]


@pytest.mark.gpu
def test_small_search_and_tuned_calls(pkg, F, dev, tmp_path):
    tu, ops = pkg.tune, pkg.ops
    sites = [tu.Site("plain", F.Q4_K, 512, 2048, pkg._lib.EPI_STORE, pkg._lib.F16),
             tu.Site("resid", F.Q4_K, 384, 1024, pkg._lib.EPI_RESID, pkg._lib.F32)]
    table = tu.tune(dev, sites, buckets=(64, 300), quick=1, full=2, keep=2, log=lambda *a: None)
    assert len(table["entries"]) == 4
    path = tmp_path / "tiles.json"
    tu.save(table, str(path))
    table = tu.load(str(path))
    w = F.synth_weights(F.Q4_K, 512, 2048, seed=5)
    x = F.synth_activations(300, 2048, seed=6)
    base = ops.qgemm(dev, w, F.Q4_K, x, N=512, K=2048, out_dtype="f16")
    tu.apply(table)
    try:
        tuned = ops.qgemm(dev, w, F.Q4_K, x, N=512, K=2048, out_dtype="f16")
    finally:
        tu.clear()
    assert np.array_equal(base.view(np.uint16), tuned.view(np.uint16))
