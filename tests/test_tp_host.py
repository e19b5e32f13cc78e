"""Host side of the tensor-parallel layer on CPU: shard planning, and two gloo ranks showing that column shards
concatenate to the full product and row-parallel K-window partials all-reduce to it (oracle arithmetic)."""
import multiprocessing as mp
import socket

import numpy as np
import pytest

import _tp_work as W


def test_even_range_and_k_window(pkg):
    tp = pkg.tp
    for n, parts, align in [(14336, 8, 1), (4096, 3, 1), (14336, 8, 256), (4096, 4, 256)]:
        rs = [tp.even_range(n, parts, r, align) for r in range(parts)]
        assert rs[0][0] == 0 and rs[-1][1] == n
        assert all(a[1] == b[0] for a, b in zip(rs, rs[1:]))
        assert all((hi - lo) % align == 0 for lo, hi in rs)
    assert tp.k_window(14336, 8, 7) == (12544, 14336)
    with pytest.raises(ValueError):
        tp.k_window(4096 + 128, 2, 0)


def test_qkv_rows_are_head_groups(pkg):
    tp = pkg.tp
    rows = [tp.qkv_rows(32, 8, 128, 8, r) for r in range(8)]
    assert rows[0] == [(0, 512), (4096, 4224), (5120, 5248)]
    covered = sorted(x for r in rows for a, b in r for x in range(a, b))
    assert covered == list(range(6144))
    with pytest.raises(ValueError):
        tp.qkv_rows(32, 8, 128, 3, 0)


def test_stack_flops_of_the_layer_configuration(pkg):
    tp = pkg.tp
    assert abs(tp.StackShape().flops(4096) - 57.18e12) / 57.18e12 < 1e-3  # 1.787 TFLOP per layer


def test_shard_layer_shapes(pkg):
    tp = pkg.tp
    shape = tp.StackShape(layers=1, hidden=512, n_q=4, n_kv=2, head_dim=128, ff=1024)
    full = tp.layer_weights(shape, 0)
    s = tp.shard_layer(shape, full, 2, 1)
    assert s["qkv"].shape == (shape.qkv // 2, full["qkv"].shape[1])
    assert s["o"].shape == (512, 144)  # 256 of the 512 query columns = 1 super-block
    assert s["gate"].shape == (512, full["gate"].shape[1]) and s["down"].shape == (512, 2 * 144)
    assert np.array_equal(s["up"], full["up"][512:])


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_gloo_ranks_column_and_row_parallel():
    ctx = mp.get_context("spawn")
    out_q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=W.cpu_shard_worker, args=(r, 2, port, out_q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [out_q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, col_err, row_rel in res:
        assert col_err == 0.0, (rank, col_err)
        assert row_rel <= 1e-12, (rank, row_rel)


def test_token_slices(pkg):
    tp = pkg.tp
    assert [tp.token_slice(4096, 8, r) for r in (0, 7)] == [(0, 512), (3584, 4096)]
    for bad in ((4096, 3), (96, 4)):  # not equal slices; slices of 24 tokens (not a multiple of 16)
        with pytest.raises(ValueError):
            tp.token_slice(*bad, 0)


@pytest.mark.parametrize("world", [2, 4])
def test_gloo_ranks_fused_exchange(world):
    """The fused mode's slot layout and rank-order reduction, restated with gloo ranks (W.cpu_fused_worker)."""
    ctx = mp.get_context("spawn")
    out_q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=W.cpu_fused_worker, args=(r, world, port, out_q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [out_q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, ok, err in res:
        assert ok, (rank, err)
