"""ctypes binding of libyah_b200.so (the C ABI of include/yah_qgemm.h).

Loading fails loudly: there is no CPU fallback for any entry point. `SYMBOLS` lists every function the header
declares; lib() checks that each is exported and sets its signature.
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libyah_b200.so")
HEADER = os.path.abspath(os.path.join(HERE, "..", "include", "yah_qgemm.h"))

c_int, c_i64, c_sz, c_vp, c_f = ctypes.c_int, ctypes.c_int64, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_float
P = ctypes.POINTER

# name: (restype, argtypes)
SYMBOLS = {
    "yah_version": (ctypes.c_char_p, []),
    "yah_last_error": (ctypes.c_char_p, []),
    "yah_block_elements": (c_int, [c_int]),
    "yah_block_bytes": (c_int, [c_int]),
    "yah_row_bytes": (c_i64, [c_int, c_i64]),
    "yah_device_count": (c_int, [P(c_int)]),
    "yah_set_device": (c_int, [c_int]),
    "yah_get_device": (c_int, [P(c_int)]),
    "yah_device_info": (c_int, [c_int, P(c_int), P(c_int), P(c_int), P(c_i64)]),
    "yah_malloc": (c_int, [P(c_vp), c_sz]),
    "yah_free": (c_int, [c_vp]),
    "yah_host_alloc": (c_int, [P(c_vp), c_sz]),
    "yah_host_free": (c_int, [c_vp]),
    "yah_memcpy_h2d": (c_int, [c_vp, c_vp, c_sz, c_vp]),
    "yah_memcpy_d2h": (c_int, [c_vp, c_vp, c_sz, c_vp]),
    "yah_memcpy_d2d": (c_int, [c_vp, c_vp, c_sz, c_vp]),
    "yah_memset": (c_int, [c_vp, c_int, c_sz, c_vp]),
    "yah_stream_create": (c_int, [P(c_vp)]),
    "yah_stream_destroy": (c_int, [c_vp]),
    "yah_stream_synchronize": (c_int, [c_vp]),
    "yah_device_synchronize": (c_int, []),
    "yah_event_create": (c_int, [P(c_vp)]),
    "yah_event_destroy": (c_int, [c_vp]),
    "yah_event_record": (c_int, [c_vp, c_vp]),
    "yah_event_synchronize": (c_int, [c_vp]),
    "yah_event_elapsed_ms": (c_int, [c_vp, c_vp, P(c_f)]),
    "yah_stream_begin_capture": (c_int, [c_vp]),
    "yah_stream_end_capture": (c_int, [c_vp, P(c_vp)]),
    "yah_graph_launch": (c_int, [c_vp, c_vp]),
    "yah_graph_destroy": (c_int, [c_vp]),
    "yah_set_launch_overlap": (c_int, [c_int]),
    "yah_set_sm_budget": (c_int, [c_int]),
    "yah_add_rmsnorm": (c_int, [c_vp, c_i64, c_vp, c_int, c_i64, c_i64, c_i64, c_f, c_f, c_vp, c_i64, c_vp]),
    "yah_tp_allreduce_f16": (c_int, [c_vp, c_vp, c_i64, c_vp]),
    "yah_realign_rows": (c_int, [c_vp, c_i64, c_i64, c_i64, c_vp, c_i64, c_vp]),
    "yah_selftest_bounded_wait": (c_int, [c_i64, P(c_int)]),
    "yah_stream_wait_event": (c_int, [c_vp, c_vp]),
    "yah_status_word": (c_int, [P(c_int)]),
    "yah_qgemm_footprint": (c_int, [c_int, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_int, c_i64,
                                    P(c_i64), P(c_i64), P(c_i64)]),
    "yah_qgemm_limits": (c_int, [P(c_int), P(c_int)]),
    "yah_dequant": (c_int, [c_vp, c_int, c_i64, c_i64, c_i64, c_i64, c_vp, c_i64, c_vp]),
    "yah_qgemm": (c_int, [c_vp, c_int, c_i64, c_i64, c_i64, c_i64, c_vp, c_i64, c_i64, c_vp, c_int, c_i64, c_int,
                          c_vp, c_i64, c_vp]),
    "yah_qgemm_tile": (c_int, [c_vp, c_int, c_i64, c_i64, c_i64, c_i64, c_vp, c_i64, c_i64, c_vp, c_int, c_i64,
                               c_int, c_vp, c_i64, c_int, c_int, c_i64, c_int, c_vp]),
    "yah_qgemm_workspace_size": (c_int, [c_int, c_i64, c_i64, c_i64, c_int, c_int, c_int, c_int, c_i64, c_int,
                                         P(c_sz)]),
    "yah_qgemm_ws": (c_int, [c_vp, c_int, c_i64, c_i64, c_i64, c_i64, c_vp, c_i64, c_i64, c_vp, c_int, c_i64, c_int,
                             c_vp, c_i64, c_int, c_int, c_i64, c_int, c_vp, c_sz, c_vp]),
    "yah_qgemm_ffn": (c_int, [c_vp, c_vp, c_int, c_i64, c_i64, c_i64, c_i64, c_vp, c_i64, c_i64, c_vp, c_i64, c_int,
                              c_int, c_vp]),
    "yah_qgemv": (c_int, [c_vp, c_int, c_i64, c_i64, c_i64, c_i64, c_vp, c_i64, c_i64, c_vp, c_int, c_i64, c_int,
                          c_vp, c_i64, c_vp]),
    "yah_qgemv_noalloc": (c_int, [c_vp, c_int, c_i64, c_i64, c_i64, c_i64, c_vp, c_i64, c_i64, c_vp, c_int, c_i64,
                                  c_int, c_vp, c_i64, c_vp]),
    "yah_qgemv_noalloc_status": (c_int, [P(c_int)]),
    "yah_qgemv_x": (c_int, [c_vp, c_int, c_i64, c_i64, c_i64, c_i64, c_vp, c_int, c_i64, c_i64, c_vp, c_int, c_i64,
                            c_int, c_vp, c_i64, c_vp]),
    "yah_qgemv_swiglu_x": (c_int, [c_vp, c_int, c_i64, c_vp, c_int, c_i64, c_i64, c_i64, c_vp, c_int, c_i64, c_i64,
                                   c_vp, c_i64, c_vp]),
    "yah_qgemv_workspace_size": (c_int, [c_int, c_i64, c_i64, c_i64, P(c_sz)]),
    "yah_qgemv_ws": (c_int, [c_vp, c_int, c_i64, c_i64, c_i64, c_i64, c_vp, c_i64, c_i64, c_vp, c_int, c_i64, c_int,
                             c_vp, c_i64, c_vp, c_sz, c_vp]),
    "yah_qgemv_swiglu": (c_int, [c_vp, c_int, c_i64, c_vp, c_int, c_i64, c_i64, c_i64, c_vp, c_i64, c_i64, c_vp, c_i64,
                                 c_vp]),
    "yah_set_gemv_impl": (c_int, [c_int]),
    "yah_qgemv_describe": (c_int, [c_int, c_i64, c_i64, c_i64, ctypes.c_char_p, c_i64]),
    "yah_tp_allgather_f32": (c_int, [c_vp, c_vp, c_vp, c_i64, c_vp]),
    "yah_qgemm_sliced": (c_int, [c_vp, c_int, c_i64, c_i64, c_i64, c_i64, c_vp, c_i64, c_i64, P(c_vp), c_int, c_i64,
                                 c_i64, c_vp]),
    "yah_tp_peers_create": (c_int, [c_vp, P(c_vp), c_int, c_vp, P(c_vp)]),
    "yah_tp_peers_ptr": (c_int, [c_vp, c_int, c_int, P(c_vp)]),
    "yah_tp_peers_destroy": (c_int, [c_vp]),
    "yah_tp_signal": (c_int, [c_vp, c_int, c_int, c_int, c_vp]),
    "yah_tp_wait": (c_int, [c_vp, c_int, c_int, c_int, c_int, c_vp]),
    "yah_tp_barrier": (c_int, [c_vp, c_int, c_int, c_int, c_vp]),
    "yah_tp_reduce_norm": (c_int, [c_vp, c_vp, c_i64, c_i64, c_i64, c_vp, c_int, c_i64, c_i64, c_f, c_f, c_int,
                                   c_i64, c_i64, c_vp]),
    "yah_tp_linear_row_scatter": (c_int, [c_vp, c_vp, c_int, c_i64, c_i64, c_i64, c_i64, c_vp, c_i64, c_i64, c_int,
                                          c_vp]),
    "yah_tp_available": (c_int, []),
    "yah_tp_unique_id": (c_int, [c_vp]),
    "yah_tp_init": (c_int, [P(c_vp), c_int, c_int, c_vp]),
    "yah_tp_destroy": (c_int, [c_vp]),
    "yah_tp_rank": (c_int, [c_vp, P(c_int), P(c_int)]),
    "yah_tp_allreduce_f32": (c_int, [c_vp, c_vp, c_i64, c_vp]),
    "yah_tp_linear_col": (c_int, [c_vp, c_vp, c_int, c_i64, c_i64, c_i64, c_vp, c_i64, c_i64, c_vp, c_int, c_i64,
                                  c_int, c_vp, c_i64, c_vp]),
    "yah_tp_linear_row": (c_int, [c_vp, c_vp, c_int, c_i64, c_i64, c_i64, c_i64, c_vp, c_i64, c_i64, c_vp, c_vp,
                                  c_vp]),
    "yah_rmsnorm": (c_int, [c_vp, c_i64, c_i64, c_i64, c_f, c_f, c_vp, c_i64, c_vp]),
    "yah_tile_rules_set": (c_int, [c_vp, c_int]),
    "yah_tile_rules_clear": (c_int, []),
    "yah_tile_rules_count": (c_int, [P(c_int)]),
    "yah_gguf_open": (c_int, [ctypes.c_char_p, P(c_vp)]),
    "yah_gguf_close": (c_int, [c_vp]),
    "yah_gguf_version": (c_int, [c_vp, P(ctypes.c_uint32)]),
    "yah_gguf_tensor_count": (c_int, [c_vp, P(c_i64)]),
    "yah_gguf_tensor_info": (c_int, [c_vp, c_i64, c_vp]),
    "yah_gguf_find": (c_int, [c_vp, ctypes.c_char_p, P(c_i64)]),
    "yah_gguf_data": (c_int, [c_vp, P(c_vp), P(ctypes.c_uint64)]),
    "yah_gguf_meta_kind": (c_int, [c_vp, ctypes.c_char_p, P(c_int), P(ctypes.c_uint64)]),
    "yah_gguf_meta_int": (c_int, [c_vp, ctypes.c_char_p, P(c_i64)]),
    "yah_gguf_meta_float": (c_int, [c_vp, ctypes.c_char_p, P(ctypes.c_double)]),
    "yah_gguf_meta_string": (c_int, [c_vp, ctypes.c_char_p, ctypes.c_char_p, c_i64, P(c_i64)]),
    "yah_weights_upload": (c_int, [c_vp, ctypes.c_uint64, c_vp, P(c_vp)]),
    "yah_weights_ref": (c_int, [c_vp, ctypes.c_uint64, ctypes.c_uint64, P(c_vp)]),
    "yah_weights_chunk_count": (c_int, [c_vp, P(c_i64)]),
    "yah_weights_free": (c_int, [c_vp]),
}


class GgufTensorInfo(ctypes.Structure):
    """yah_gguf_tensor (include/yah_qgemm.h)."""
    _fields_ = [("name", ctypes.c_char * 128), ("ggml_type", c_int), ("n_dims", c_int), ("dims", c_i64 * 4),
                ("offset", ctypes.c_uint64), ("bytes", ctypes.c_uint64)]


class TileRule(ctypes.Structure):
    """yah_tile_rule (include/yah_qgemm.h)."""
    _fields_ = [("ggml_type", c_int), ("epilogue", c_int), ("y_dtype", c_int), ("N", c_i64), ("K", c_i64),
                ("m_max", c_i64), ("bn", c_int), ("grid", c_int), ("cta_pair", c_int)]
TP_ID_BYTES = 128

# status codes (include/yah_qgemm.h)
OK, ERR_ARG, ERR_UNSUPPORTED, ERR_SIZE, ERR_CUDA, ERR_DEVICE, ERR_NCCL, ERR_IO = range(8)
F32, F16 = 0, 1
EPI_STORE, EPI_RESID, EPI_SWIGLU = 0, 1, 2


class YahError(RuntimeError):
    """A failed C-ABI call: .code is the status, the message comes from yah_last_error()."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"[{code}] {msg}")
        self.code = code


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is not built: run __graft_entry__.build() (make in csrc/)")
        L = ctypes.CDLL(LIB_PATH)
        missing = [n for n in SYMBOLS if not hasattr(L, n)]
        if missing:
            raise RuntimeError(f"{LIB_PATH} lacks exported symbols {missing}")
        for n, (res, args) in SYMBOLS.items():
            fn = getattr(L, n)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(rc: int) -> None:
    if rc != OK:
        raise YahError(rc, lib().yah_last_error().decode(errors="replace"))


def header_symbols() -> list:
    """Function names declared in include/yah_qgemm.h (the ABI contract)."""
    import re
    names = []
    src = open(HEADER).read()
    for m in re.finditer(r"^\s*(?:const\s+)?[a-z_0-9]+\s*\*?\s*(yah_[a-z0-9_]+)\s*\(", src, re.M):
        names.append(m.group(1))
    return names
