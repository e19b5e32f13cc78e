"""GGUF files: the quant-block loader over the C ABI (yah_gguf_*, yah_weights_*).

`Gguf` is the reference's core::Gguf (engine/core/gguf.hpp:74-105): a read-only mapping of the file with its
metadata and tensor table. `TensorInfo` carries what model::TensorRef does (engine/model/weights.hpp:15-25): GGUF
dims with ne0 = the row length (K of a linear weight) and ne1 = the row count (N). `DeviceWeights` is LoomWeights
(engine/model/loom_runtime.hpp:487-516): the tensor-data region copied to device chunks cut at tensor boundaries,
and a tensor bound as a device address inside its chunk, rows unchanged, ready for the GEMM / GEMV.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np

from ._lib import GgufTensorInfo, check, lib

KIND_STRING, KIND_ARRAY, KIND_F32, KIND_F64 = 8, 9, 6, 12


@dataclass(frozen=True)
class TensorInfo:
    name: str
    ggml_type: int
    dims: tuple        # GGUF order: dims[0] = ne0 (row length), dims[1] = ne1 (rows), ...
    offset: int        # bytes from the start of the tensor-data region
    bytes: int

    @property
    def ne0(self) -> int:
        return self.dims[0]

    @property
    def ne1(self) -> int:
        return self.dims[1] if len(self.dims) > 1 else 1

    @property
    def rows(self) -> int:
        """Rows of the tensor as a matrix (every dim past ne0)."""
        r = 1
        for d in self.dims[1:]:
            r *= d
        return r

    @property
    def row_bytes(self) -> int:
        return self.bytes // self.rows


class Gguf:
    """A GGUF file mapped read-only (yah_gguf_open); use as a context manager or call close()."""

    def __init__(self, path: str):
        h = ctypes.c_void_p()
        check(lib().yah_gguf_open(str(path).encode(), ctypes.byref(h)))
        self.handle, self.path = h.value, str(path)
        v = ctypes.c_uint32()
        check(lib().yah_gguf_version(self.handle, ctypes.byref(v)))
        self.version = v.value
        n = ctypes.c_int64()
        check(lib().yah_gguf_tensor_count(self.handle, ctypes.byref(n)))
        self.tensors = []
        info = GgufTensorInfo()
        for i in range(n.value):
            check(lib().yah_gguf_tensor_info(self.handle, i, ctypes.byref(info)))
            self.tensors.append(TensorInfo(info.name.decode(errors="replace"), info.ggml_type,
                                           tuple(info.dims[:info.n_dims]),
                                           info.offset, info.bytes))
        self._by_name = {}
        for t in self.tensors:
            # Names that are not valid UTF-8 decode with replacement characters, and ctypes' char array stops at
            # an embedded NUL, so two tensors the loader keeps apart could map to one key: refuse such a file
            # rather than let a lookup return the wrong tensor.
            if t.name in self._by_name:
                self.close()
                raise ValueError(f"{path}: two tensors decode to the same name {t.name!r}")
            self._by_name[t.name] = t

    def find(self, name: str) -> TensorInfo | None:
        return self._by_name.get(name)

    def __getitem__(self, name: str) -> TensorInfo:
        t = self.find(name)
        if t is None:
            raise KeyError(f"{self.path} has no tensor {name!r}")
        return t

    def meta(self, key: str):
        """The value of a metadata key: int (integers, bools), float, str, or ("array", element count)."""
        L, k = lib(), key.encode()
        kind, count = ctypes.c_int(), ctypes.c_uint64()
        check(L.yah_gguf_meta_kind(self.handle, k, ctypes.byref(kind), ctypes.byref(count)))
        if kind.value == KIND_ARRAY:
            return ("array", count.value)
        if kind.value == KIND_STRING:
            n = ctypes.c_int64()
            check(L.yah_gguf_meta_string(self.handle, k, None, 0, ctypes.byref(n)))
            buf = ctypes.create_string_buffer(n.value + 1)
            check(L.yah_gguf_meta_string(self.handle, k, buf, n.value + 1, None))
            return buf.raw[:n.value].decode(errors="replace")
        if kind.value in (KIND_F32, KIND_F64):
            f = ctypes.c_double()
            check(L.yah_gguf_meta_float(self.handle, k, ctypes.byref(f)))
            return f.value
        v = ctypes.c_int64()
        check(L.yah_gguf_meta_int(self.handle, k, ctypes.byref(v)))
        return v.value

    def data(self, t: TensorInfo) -> np.ndarray:
        """The tensor's bytes as a read-only uint8 view of the mapping ([rows][row_bytes]); valid until close()."""
        base, size = ctypes.c_void_p(), ctypes.c_uint64()
        check(lib().yah_gguf_data(self.handle, ctypes.byref(base), ctypes.byref(size)))
        if t.offset + t.bytes > size.value:
            raise ValueError(f"tensor {t.name} lies outside the data region")
        a = np.ctypeslib.as_array((ctypes.c_uint8 * t.bytes).from_address(base.value + t.offset))
        a.flags.writeable = False
        return a.reshape(t.rows, t.row_bytes)

    def close(self):
        if self.handle:
            check(lib().yah_gguf_close(self.handle))
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


@dataclass(frozen=True)
class Linear:
    """A weight tensor bound on the device, as yah_qgemm / yah_qgemv take it."""
    ptr: int
    ggml_type: int
    N: int             # rows (ne1)
    K: int             # row length (ne0)
    row_stride: int    # bytes


class DeviceWeights:
    """The tensor-data region of a Gguf on the current device (yah_weights_upload), in chunks of at most
    chunk_bytes (0 = 1 GiB) cut at tensor boundaries."""

    def __init__(self, gguf: Gguf, chunk_bytes: int = 0, stream=None):
        h = ctypes.c_void_p()
        check(lib().yah_weights_upload(gguf.handle, chunk_bytes, stream, ctypes.byref(h)))
        self.handle = h.value
        n = ctypes.c_int64()
        check(lib().yah_weights_chunk_count(self.handle, ctypes.byref(n)))
        self.chunks = n.value

    def ref(self, t: TensorInfo) -> int:
        p = ctypes.c_void_p()
        check(lib().yah_weights_ref(self.handle, t.offset, t.bytes, ctypes.byref(p)))
        return p.value

    def linear(self, t: TensorInfo) -> Linear:
        if len(t.dims) != 2:
            raise ValueError(f"tensor {t.name} has dims {t.dims}, not a matrix")
        return Linear(self.ref(t), t.ggml_type, t.ne1, t.ne0, t.row_bytes)

    def close(self):
        if self.handle:
            check(lib().yah_weights_free(self.handle))
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()
