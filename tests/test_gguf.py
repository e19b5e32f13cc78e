"""The GGUF reader (yah_gguf_*, the reference's core::Gguf) on files written by gguf-py's GGUFWriter, cross-checked
with gguf-py's GGUFReader (the reference's tools read GGUF with it: engine/gpu/loom/tools/gemv_check.py:127-128),
and refusals of malformed files. Host code only: no GPU."""
import os
import struct

import numpy as np
import pytest

gguf = pytest.importorskip("gguf")


def write_file(path, F, alignment=None):
    from gguf import GGMLQuantizationType as T
    w = gguf.GGUFWriter(str(path), "llama")
    if alignment:
        w.add_custom_alignment(alignment)
    w.add_uint32("llama.block_count", 1)
    w.add_float32("llama.rope.freq_base", 10000.0)
    w.add_bool("test.flag", True)
    w.add_string("general.name", "synthetic")
    w.add_array("test.ints", [1, 2, 3])
    w.add_array("test.strs", ["a", "bc"])
    w.add_int64("test.neg", -5)
    w.add_uint64("test.big", 2 ** 40 + 7)
    w.add_float64("test.f64", 0.125)
    tensors = {
        "blk.0.ffn_gate.weight": (F.synth_weights(F.Q4_K, 64, 512, seed=1), T.Q4_K, F.Q4_K, (512, 64)),
        "blk.0.attn_q.weight": (F.synth_weights(F.Q8_0, 32, 256, seed=2), T.Q8_0, F.Q8_0, (256, 32)),
        "blk.0.ffn_down.weight": (F.synth_weights(F.Q6_K, 48, 2048, seed=3), T.Q6_K, F.Q6_K, (2048, 48)),
        "output_norm.weight": (np.arange(512, dtype=np.float32), None, 0, (512,)),
        "tok.f16": (np.arange(32, dtype=np.float16).reshape(4, 8), None, 1, (8, 4)),
    }
    for name, (arr, raw, _, _) in tensors.items():
        if raw is None:
            w.add_tensor(name, arr)
        else:
            w.add_tensor(name, arr, raw_dtype=raw)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    return tensors


@pytest.fixture(scope="module")
def gfile(tmp_path_factory, F):
    d = tmp_path_factory.mktemp("gguf")
    out = {}
    for al in (None, 64):
        p = d / f"t{al or 32}.gguf"
        out[al or 32] = (p, write_file(p, F, al))
    return out


@pytest.mark.parametrize("alignment", [32, 64])
def test_tensor_table_and_bytes(pkg, gfile, alignment):
    path, tensors = gfile[alignment]
    from yah_b200.gguf_file import Gguf
    with Gguf(path) as g:
        assert g.version == 3
        assert [t.name for t in g.tensors] == list(tensors)
        for name, (arr, _, ggml_type, dims) in tensors.items():
            t = g[name]
            assert t.ggml_type == ggml_type and t.dims == dims
            assert t.bytes == arr.nbytes and t.offset % alignment == 0
            assert np.array_equal(g.data(t).ravel(), arr.view(np.uint8).ravel())
        q4 = g["blk.0.ffn_gate.weight"]
        assert (q4.ne0, q4.ne1, q4.rows, q4.row_bytes) == (512, 64, 64, 288)
        assert g.find("missing") is None
        # the same table as gguf-py's reader: names, types, shapes and absolute data offsets
        r = gguf.GGUFReader(str(path))
        base = r.tensors[0].data_offset - g.tensors[0].offset
        assert [(t.name, int(t.tensor_type), tuple(int(x) for x in t.shape), int(t.data_offset))
                for t in r.tensors] == [(t.name, t.ggml_type, t.dims, base + t.offset) for t in g.tensors]


def test_metadata(pkg, gfile):
    from yah_b200.gguf_file import Gguf
    with Gguf(gfile[64][0]) as g:
        assert g.meta("general.architecture") == "llama"
        assert g.meta("general.alignment") == 64
        assert g.meta("llama.block_count") == 1
        assert g.meta("llama.rope.freq_base") == 10000.0
        assert g.meta("test.flag") == 1
        assert g.meta("general.name") == "synthetic"
        assert g.meta("test.ints") == ("array", 3)
        assert g.meta("test.strs") == ("array", 2)
        assert g.meta("test.neg") == -5
        assert g.meta("test.big") == 2 ** 40 + 7
        assert g.meta("test.f64") == 0.125
        with pytest.raises(pkg.YahError) as e:
            g.meta("no.such.key")
        assert e.value.code == 1
        with pytest.raises(pkg.YahError):   # a string key read as an integer
            pkg.gguf_file.check(pkg.lib().yah_gguf_meta_int(g.handle, b"general.name", pkg._lib.ctypes.byref(
                pkg._lib.ctypes.c_int64())))


def test_find_and_index_errors(pkg, gfile):
    import ctypes
    from yah_b200.gguf_file import Gguf
    L = pkg.lib()
    with Gguf(gfile[32][0]) as g:
        idx = ctypes.c_int64()
        assert L.yah_gguf_find(g.handle, b"blk.0.attn_q.weight", ctypes.byref(idx)) == 0 and idx.value == 1
        assert L.yah_gguf_find(g.handle, b"nope", ctypes.byref(idx)) == 1 and idx.value == -1
        info = pkg._lib.GgufTensorInfo()
        assert L.yah_gguf_tensor_info(g.handle, 99, ctypes.byref(info)) == 1
        assert L.yah_gguf_tensor_info(g.handle, -1, ctypes.byref(info)) == 1


def tensor_type_pos(raw: bytes, name: str) -> int:
    """Byte position of the type field of tensor `name` in a GGUF file (after its name, n_dims and dims)."""
    key = struct.pack("<Q", len(name)) + name.encode()
    i = raw.index(key) + len(key)
    nd = struct.unpack_from("<I", raw, i)[0]
    return i + 4 + 8 * nd


def open_code(pkg, path):
    import ctypes
    h = ctypes.c_void_p()
    rc = pkg.lib().yah_gguf_open(str(path).encode(), ctypes.byref(h))
    if rc == 0:
        pkg.lib().yah_gguf_close(h)
    return rc, pkg.lib().yah_last_error().decode(errors="replace")  # messages may quote a corrupt tensor name


def test_malformed_files_are_refused(pkg, gfile, tmp_path):
    src, _ = gfile[32]
    raw = open(src, "rb").read()
    ERR_ARG, ERR_UNSUPPORTED, ERR_IO = 1, 2, 7

    def write(name, data):
        p = tmp_path / name
        p.write_bytes(data)
        return p

    assert open_code(pkg, tmp_path / "absent.gguf")[0] == ERR_IO
    assert open_code(pkg, write("short.gguf", raw[:10]))[0] == ERR_IO
    assert open_code(pkg, write("magic.gguf", b"GGUX" + raw[4:]))[0] == ERR_IO
    assert open_code(pkg, write("v1.gguf", raw[:4] + struct.pack("<I", 1) + raw[8:]))[0] == ERR_IO
    pos = tensor_type_pos(raw, "blk.0.ffn_down.weight")
    rc, msg = open_code(pkg, write("table.gguf", raw[:pos - 20]))        # cut inside the tensor table
    assert rc == ERR_IO and "truncated" in msg
    rc, msg = open_code(pkg, write("data.gguf", raw[:-100]))             # the last tensor runs past the end
    assert rc == ERR_IO and "beyond the end" in msg
    bad = bytearray(raw)
    struct.pack_into("<I", bad, pos, 99)                                   # a type id of unknown block size
    rc, msg = open_code(pkg, write("type.gguf", bytes(bad)))
    assert rc == ERR_UNSUPPORTED and "99" in msg
    bad = bytearray(raw)
    struct.pack_into("<Q", bad, pos + 4, 8)                                # a tensor offset off the alignment
    assert open_code(pkg, write("align.gguf", bytes(bad)))[0] == ERR_IO
    bad = bytearray(raw)
    struct.pack_into("<Q", bad, 8, 2 ** 60)                                # a tensor count beyond the file
    assert open_code(pkg, write("count.gguf", bytes(bad)))[0] == ERR_IO
    assert open_code(pkg, src)[0] == 0 and ERR_ARG == 1
    assert os.path.getsize(src) == len(raw)


def test_fuzzed_headers_never_read_out_of_range(pkg, gfile, tmp_path):
    """Random byte flips and truncations in the header, metadata and tensor table: every open returns a status (0,
    YAH_ERR_IO or YAH_ERR_UNSUPPORTED) and never reads outside the file (the parser is bounds-checked; a read out of
    range would crash this process)."""
    import random
    src, _ = gfile[64]
    raw = open(src, "rb").read()
    head = raw.index(struct.pack("<Q", len("tok.f16")) + b"tok.f16") + 64   # past the end of the tensor table
    rng = random.Random(5)
    p = tmp_path / "fuzz.gguf"
    seen = set()
    for it in range(400):
        b = bytearray(raw)
        if it % 4 == 0:
            b = b[:rng.randrange(1, head)]
        else:
            for _ in range(rng.randrange(1, 6)):
                b[rng.randrange(0, head)] = rng.randrange(256)
        p.write_bytes(bytes(b))
        rc, _ = open_code(pkg, p)
        assert rc in (0, 2, 7), rc
        seen.add(rc)
    assert 7 in seen


def test_names_that_decode_alike_are_refused(pkg, F, tmp_path):
    """Two tensor names that differ only in bytes that are not UTF-8 decode to the same Python string; the loader
    keeps them apart, so the Python reader refuses the file instead of letting one name shadow the other."""
    from gguf import GGMLQuantizationType as T
    from yah_b200.gguf_file import Gguf
    p = tmp_path / "names.gguf"
    w = gguf.GGUFWriter(str(p), "llama")
    w.add_tensor("blk.X", F.synth_weights(F.Q4_K, 4, 256, seed=1), raw_dtype=T.Q4_K)
    w.add_tensor("blk.Y", F.synth_weights(F.Q4_K, 4, 256, seed=2), raw_dtype=T.Q4_K)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    raw = bytearray(p.read_bytes())
    for name, byte in ((b"blk.X", 0xFF), (b"blk.Y", 0xFE)):
        i = raw.index(struct.pack("<Q", len(name)) + name) + 8
        raw[i + len(name) - 1] = byte
    q = tmp_path / "names_bad.gguf"
    q.write_bytes(bytes(raw))
    with pytest.raises(ValueError, match="same name"):
        Gguf(q)
    with Gguf(p) as g:  # the unpatched file opens
        assert [t.name for t in g.tensors] == ["blk.X", "blk.Y"]
