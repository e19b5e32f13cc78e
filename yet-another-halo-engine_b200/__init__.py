"""B200-native quantised tile GEMM / decode GEMV (GGUF Q8_0, Q4_K, Q6_K weights x f16 activations).

Modules:
  formats  GGUF block traits and the seeded synthetic tensors of the benchmark configurations
  _lib     ctypes binding of libyah_b200.so (include/yah_qgemm.h)
  device   device memory, streams, events (the reference's LoomDevice role)
  ops      qgemm / qgemv / dequant: the reference's kernel kinds over the C ABI
  tp       tensor-parallel layer stack: shard planning, NCCL communicator, Llama-shaped linear stack
  tune     tile-configuration search and the tile table read by yah_qgemm's automatic choice
  gguf_file  GGUF reader and device weight chunks (the reference's core::Gguf / LoomWeights)
"""
from . import formats  # noqa: F401
from ._lib import YahError, lib  # noqa: F401
from . import device, gguf_file, ops, tp, tune  # noqa: F401
from .device import Device, DeviceBuffer, Event, Graph, PinnedBuffer, Stream, device_count  # noqa: F401
