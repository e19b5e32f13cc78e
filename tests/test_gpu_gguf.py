"""GGUF tensors uploaded to device chunks (yah_weights_upload, the reference's LoomWeights) and multiplied in place:
the GEMM and the GEMV read a tensor's rows at its device address inside a chunk, no repacking, and match the
oracle on the same bytes (tolerances as tests/test_gpu_qgemm.py and tests/test_gpu_qgemv.py)."""
import ctypes

import numpy as np
import pytest

from test_gguf import write_file

pytestmark = pytest.mark.gpu
gguf = pytest.importorskip("gguf")


@pytest.mark.parametrize("chunk_bytes", [0, 20000])
def test_uploaded_tensors_multiply_in_place(pkg, F, O, dev, tmp_path, chunk_bytes):
    path = tmp_path / "w.gguf"
    tensors = write_file(path, F, alignment=64)
    from yah_b200.gguf_file import DeviceWeights, Gguf
    with Gguf(path) as g, DeviceWeights(g, chunk_bytes=chunk_bytes) as dw:
        assert dw.chunks == (1 if chunk_bytes == 0 else 4)
        for name in ("blk.0.ffn_gate.weight", "blk.0.attn_q.weight", "blk.0.ffn_down.weight"):
            t = g[name]
            lin = dw.linear(t)
            host = tensors[name][0]
            assert lin.ptr % 16 == 0 and (lin.N, lin.K, lin.row_stride) == (host.shape[0], t.ne0, host.shape[1])
            back = np.empty_like(host)
            pkg.lib().yah_memcpy_d2h(back.ctypes.data, lin.ptr, host.nbytes, None)
            dev.synchronize()
            assert np.array_equal(back, host)
            for M in (1, 40):
                x = F.synth_activations(M, lin.K, seed=M)
                xd, yd = dev.upload(x), dev.empty(M * lin.N * 4)
                gemv = M <= 32
                fn = pkg.ops.qgemv_ptr if gemv else pkg.ops.qgemm_ptr
                fn(lin.ptr, lin.ggml_type, lin.N, lin.K, lin.row_stride, 0, xd.ptr, M, lin.K, yd.ptr, "f32", lin.N)
                dev.synchronize()
                y = yd.download(np.float32, (M, lin.N))
                w_deq = (O.dequant_f32 if gemv else O.dequant_f16)(lin.ggml_type, host, lin.N, lin.K)
                e = O.errors(y, O.gemm_ref(w_deq, x))
                assert e["finite"] and e["max_abs"] <= 2e-2 and e["rel_fro"] <= 1e-3, (name, M, e)
        if chunk_bytes:
            # a range that straddles two chunks is refused
            a, b = g["blk.0.ffn_gate.weight"], g["blk.0.attn_q.weight"]
            p = ctypes.c_void_p()
            assert pkg.lib().yah_weights_ref(dw.handle, a.offset, b.offset + b.bytes - a.offset, ctypes.byref(p)) == 1
