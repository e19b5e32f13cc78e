"""The tensor-parallel stack's shape and per-layer weights read from a GGUF file (tp.shape_from_gguf /
tp.layer_from_gguf over the C-ABI reader): a two-block Llama-style file written with gguf-py, its tensors compared
with the written arrays and sharded as the in-memory path shards them. Host code only."""
import numpy as np
import pytest

gguf = pytest.importorskip("gguf")

H, FF, NQ, NKV, HD, LAYERS = 512, 1024, 4, 2, 128, 2


def write_model(path, F, mixed=False, bad_dims=False):
    from gguf import GGMLQuantizationType as T
    w = gguf.GGUFWriter(str(path), "llama")
    w.add_uint32("llama.block_count", LAYERS)
    w.add_uint32("llama.embedding_length", H)
    w.add_uint32("llama.feed_forward_length", FF)
    w.add_uint32("llama.attention.head_count", NQ)
    w.add_uint32("llama.attention.head_count_kv", NKV)
    shapes = {"attn_q": (NQ * HD, H), "attn_k": (NKV * HD, H), "attn_v": (NKV * HD, H), "attn_output": (H, NQ * HD),
              "ffn_gate": (FF, H), "ffn_up": (FF, H), "ffn_down": (H, FF)}
    arrays = {}
    for layer in range(LAYERS):
        for i, (name, (n, k)) in enumerate(shapes.items()):
            fmt, raw = F.Q4_K, T.Q4_K
            if mixed and layer == 1 and name == "ffn_down":
                fmt, raw = F.Q6_K, T.Q6_K
            if bad_dims and layer == 0 and name == "attn_k":
                n = n + 256
            a = F.synth_weights(fmt, n, k, seed=100 * layer + i)
            arrays[(layer, name)] = a
            w.add_tensor(f"blk.{layer}.{name}.weight", a, raw_dtype=raw)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    return arrays


def test_shape_and_layers_from_gguf(pkg, F, tmp_path):
    tp = pkg.tp
    from yah_b200.gguf_file import Gguf
    path = tmp_path / "m.gguf"
    arrays = write_model(path, F)
    with Gguf(path) as g:
        shape = tp.shape_from_gguf(g)
        assert (shape.layers, shape.hidden, shape.ff, shape.n_q, shape.n_kv, shape.head_dim, shape.fmt) == \
            (LAYERS, H, FF, NQ, NKV, HD, F.Q4_K)
        for layer in range(LAYERS):
            full = tp.layer_from_gguf(g, shape, layer)
            qkv = np.concatenate([arrays[(layer, n)] for n in ("attn_q", "attn_k", "attn_v")])
            assert np.array_equal(full["qkv"], qkv)
            for part, name in (("o", "attn_output"), ("gate", "ffn_gate"), ("up", "ffn_up"), ("down", "ffn_down")):
                assert np.array_equal(full[part], arrays[(layer, name)])
            for parts in (1, 2):
                for r in range(parts):
                    a = tp.shard_layer(shape, full, parts, r)
                    b = tp.shard_layer(shape, {"qkv": qkv, "o": arrays[(layer, "attn_output")],
                                               "gate": arrays[(layer, "ffn_gate")], "up": arrays[(layer, "ffn_up")],
                                               "down": arrays[(layer, "ffn_down")]}, parts, r)
                    assert all(np.array_equal(a[k], b[k]) for k in a)
    # the arrays are copies: still readable after the mapping is closed
    assert full["qkv"].sum() == qkv.sum()


def test_mixed_formats_and_bad_dims_are_refused(pkg, F, tmp_path):
    tp = pkg.tp
    from yah_b200.gguf_file import Gguf
    p1 = tmp_path / "mixed.gguf"
    write_model(p1, F, mixed=True)
    with Gguf(p1) as g, pytest.raises(ValueError, match="one format"):
        tp.shape_from_gguf(g)
    p2 = tmp_path / "dims.gguf"
    write_model(p2, F, bad_dims=True)
    with Gguf(p2) as g:
        shape = tp.shape_from_gguf(g)
        with pytest.raises(ValueError, match="attn_k"):
            tp.layer_from_gguf(g, shape, 0)
        tp.layer_from_gguf(g, shape, 1)
