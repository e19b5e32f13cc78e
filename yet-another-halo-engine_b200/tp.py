"""Tensor-parallel layer stack over the C ABI (yah_tp_*): shard planning, the NCCL communicator, and the
Llama-shaped linear stack of the benchmark's layer configuration.

The reference engine runs on one GPU; this is the sharding layer the B200 build adds. Megatron split over the
GPUs of one box, one process per GPU:
  * column-parallel QKV, gate, up: a rank holds a row range of the GGUF tensor (no re-quantisation; QKV in whole
    head groups, so the rank's query heads stay together) and writes its slice of the outputs, no collective;
  * row-parallel o_proj, down: a rank holds a K window of every row (whole super-blocks; the precedent is the
    reference's K-window GEMM form, gen_gemm_tile.py:262-264) and one ncclAllReduce(sum) of the partials gives the
    result (see the modes below).
Per layer (attention replaced by identity, so the o_proj input is the rank's query slice of the QKV output):

    xn  = rmsnorm(h)                      f16, weightless, gain 1/64
    qkv = xn Wqkv_r^T                     f16 [M][qkv_r]
    h   = h + allreduce(qkv[:, :q_r] Wo_r^T)
    xn  = rmsnorm(h)
    g   = xn Wg_r^T                       f32 [M][ff_r]
    a   = silu(g) * (xn Wu_r^T)           f16 (the GEMM's swiglu epilogue)
    h   = h + allreduce(a Wd_r^T)

Row-parallel partial sums. Parity mode: f32; rank 0's GEMM epilogue adds the residual and the allreduce sums
h + partials in place. Fused mode (the parity arithmetic without the allreduce): the tokens are split into p equal
slices, rank r owning slice r of the residual stream; each rank's row-parallel GEMM writes its f32 partial of a
token straight into the owner's memory (yah_tp_linear_row_scatter, stores over NVLink while the GEMM runs), the
owner adds the p slots in rank order into its residual slice and writes the RMSNorm of it (f16) into every rank's
activation buffer (yah_tp_reduce_norm: the all-gather), with flags in each rank's memory ordering the ranks
(yah_tp_barrier: a signal and a bounded wait in one launch). Traffic per row-parallel linear and rank: (p - 1) / p of the f32 partial
out and of the f16 activations back, against 2 (p - 1) / p of the f32 partial for the allreduce, and the scatter
overlaps its GEMM. Speed mode: every rank's GEMM stores f16 partials (no residual read), the f16 allreduce moves
half the bytes, and the next norm's pass adds the sum into the f32 residual stream (yah_add_rmsnorm). The residual
stream h is f32 [M][hidden] on every rank in both.
The reference normalises every layer input (docs/architecture.md:68); the fixed gain keeps silu(gate) * up inside
the f16 range with the synthetic weights.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np

from . import formats as F
from ._lib import EPI_RESID, EPI_STORE, EPI_SWIGLU, F16, F32, TP_ID_BYTES, check, lib  # noqa: F401
from .device import Device, DeviceBuffer, Event, Stream

NORM_GAIN = 1.0 / 64.0
NORM_EPS = 1e-6


# ----------------------------------------------------------------------------------------------- shard planning
def even_range(n: int, parts: int, part: int, align: int = 1) -> tuple:
    """[lo, hi) of part `part` when n (a multiple of align) is cut into `parts` near-equal aligned pieces."""
    if n % align:
        raise ValueError(f"{n} is not a multiple of {align}")
    units = n // align
    lo = part * units // parts
    hi = (part + 1) * units // parts
    return lo * align, hi * align


def qkv_rows(n_q: int, n_kv: int, head_dim: int, parts: int, part: int) -> list:
    """Row ranges of the fused [q | k | v] projection held by `part`: its query heads, then its key and value heads
    (whole head groups: n_q and n_kv must divide by parts)."""
    if n_q % parts or n_kv % parts:
        raise ValueError(f"{n_q} query / {n_kv} kv heads do not split over {parts} ranks")
    q0, q1 = even_range(n_q, parts, part)
    k0, k1 = even_range(n_kv, parts, part)
    kv_base = n_q * head_dim
    return [(q0 * head_dim, q1 * head_dim), (kv_base + k0 * head_dim, kv_base + k1 * head_dim),
            (kv_base + (n_kv + k0) * head_dim, kv_base + (n_kv + k1) * head_dim)]


def k_window(K: int, parts: int, part: int) -> tuple:
    """(k0, k1) of the row-parallel K window of `part`, in whole 256-value super-blocks."""
    return even_range(K, parts, part, align=256)


def token_slice(M: int, parts: int, part: int) -> tuple:
    """[lo, hi) of the tokens whose residual stream rank `part` owns in the fused mode (equal slices of a multiple of
    16 tokens: the row-parallel GEMM writes 16-token units, so a unit never straddles two owners)."""
    if M % parts or (M // parts) % 16:
        raise ValueError(f"{M} tokens do not split into {parts} slices of a multiple of 16")
    ms = M // parts
    return part * ms, (part + 1) * ms


def take_rows(w: np.ndarray, ranges: list) -> np.ndarray:
    """The rank's contiguous weight shard: the listed row ranges of GGUF rows w, stacked."""
    return np.ascontiguousarray(np.concatenate([w[a:b] for a, b in ranges], axis=0))


def take_k_window(w: np.ndarray, fmt: int, k0: int, k1: int) -> np.ndarray:
    """Compact GGUF rows of the K window [k0, k1) (whole blocks; super-block = 256 values)."""
    sb = F.SUPERBLOCK_BYTES[fmt]
    return np.ascontiguousarray(w[:, (k0 // 256) * sb:(k1 // 256) * sb])


@dataclass(frozen=True)
class StackShape:
    """The Llama-shaped stack of the layer configuration (defaults: 32 layers, hidden 4096, 32 query heads and
    8 kv heads of 128, feed-forward 14336)."""
    layers: int = 32
    hidden: int = 4096
    n_q: int = 32
    n_kv: int = 8
    head_dim: int = 128
    ff: int = 14336
    fmt: int = F.Q4_K

    @property
    def qkv(self) -> int:
        return (self.n_q + 2 * self.n_kv) * self.head_dim

    def flops(self, M: int) -> float:
        """Algorithmic FLOPs of one forward pass over M tokens (linears only)."""
        H = self.hidden
        return 2.0 * M * self.layers * (H * self.qkv + H * self.n_q * self.head_dim + 2 * H * self.ff + self.ff * H)


def layer_weights(shape: StackShape, layer: int, seed: int = 4000) -> dict:
    """Full GGUF tensors of one layer (seeded synthetic, per formats.synth_weights)."""
    H, s = shape.hidden, seed + 16 * layer
    return {
        "qkv": F.synth_weights(shape.fmt, shape.qkv, H, seed=s),
        "o": F.synth_weights(shape.fmt, H, shape.n_q * shape.head_dim, seed=s + 1),
        "gate": F.synth_weights(shape.fmt, shape.ff, H, seed=s + 2),
        "up": F.synth_weights(shape.fmt, shape.ff, H, seed=s + 3),
        "down": F.synth_weights(shape.fmt, H, shape.ff, seed=s + 4),
    }


def shard_layer(shape: StackShape, full: dict, parts: int, part: int) -> dict:
    """This rank's shards of one layer's tensors (host arrays)."""
    q0, q1 = (r * shape.head_dim for r in even_range(shape.n_q, parts, part))
    f0, f1 = even_range(shape.ff, parts, part)
    return {
        "qkv": take_rows(full["qkv"], qkv_rows(shape.n_q, shape.n_kv, shape.head_dim, parts, part)),
        "o": take_k_window(full["o"], shape.fmt, q0, q1),
        "gate": take_rows(full["gate"], [(f0, f1)]),
        "up": take_rows(full["up"], [(f0, f1)]),
        "down": take_k_window(full["down"], shape.fmt, f0, f1),
    }


# ----------------------------------------------------------------------------------------------- GGUF models
# The tensors of one Llama-style block in a GGUF file (llama.cpp's names; the reference resolves its own model's
# per-layer tensors the same way, engine/model/weights.hpp:27-52).
GGUF_LAYER_TENSORS = {"q": "attn_q", "k": "attn_k", "v": "attn_v", "o": "attn_output", "gate": "ffn_gate",
                      "up": "ffn_up", "down": "ffn_down"}


def shape_from_gguf(g) -> StackShape:
    """The stack's shape from a GGUF file's metadata ({arch}.block_count, embedding_length, feed_forward_length,
    attention.head_count, attention.head_count_kv) and its weight format. The stack runs one format for all of its
    linears, so a file whose block tensors mix formats (as some mixed-precision quantisations do) is refused."""
    arch = g.meta("general.architecture")
    key = lambda k: g.meta(f"{arch}.{k}")  # noqa: E731
    hidden, n_q = key("embedding_length"), key("attention.head_count")
    shape = StackShape(layers=key("block_count"), hidden=hidden, n_q=n_q, n_kv=key("attention.head_count_kv"),
                       head_dim=hidden // n_q, ff=key("feed_forward_length"),
                       fmt=g[f"blk.0.{GGUF_LAYER_TENSORS['gate']}.weight"].ggml_type)
    for layer in range(shape.layers):
        for part, name in GGUF_LAYER_TENSORS.items():
            t = g[f"blk.{layer}.{name}.weight"]
            if t.ggml_type != shape.fmt:
                raise ValueError(f"{t.name} is GGML type {t.ggml_type}; the stack runs one format ({shape.fmt})")
    return shape


def layer_from_gguf(g, shape: StackShape, layer: int) -> dict:
    """One block's full tensors as the stack takes them (host arrays, rows unchanged): QKV as the q, k and v rows
    one after another, o_proj, gate, up, down. Shapes are checked against `shape` (GGUF dims: ne0 = row length)."""
    H, qd, kvd = shape.hidden, shape.n_q * shape.head_dim, shape.n_kv * shape.head_dim
    want = {"q": (H, qd), "k": (H, kvd), "v": (H, kvd), "o": (qd, H), "gate": (H, shape.ff), "up": (H, shape.ff),
            "down": (shape.ff, H)}
    rows = {}
    for part, name in GGUF_LAYER_TENSORS.items():
        t = g[f"blk.{layer}.{name}.weight"]
        if t.dims != want[part]:
            raise ValueError(f"{t.name} has dims {t.dims}, the shape needs {want[part]}")
        rows[part] = np.array(g.data(t))  # a copy: the arrays outlive the mapping
    return {"qkv": np.concatenate([rows["q"], rows["k"], rows["v"]]), "o": rows["o"], "gate": rows["gate"],
            "up": rows["up"], "down": rows["down"]}


# ----------------------------------------------------------------------------------------------- communicator
class Comm:
    """An NCCL communicator of `nranks` processes, one per GPU (yah_tp_init on the current device).

    `exchange(id_bytes_or_None) -> bytes` shares rank 0's unique id with every rank (for example a broadcast over
    torch.distributed or a file); rank 0 passes its id, the others pass None."""

    def __init__(self, nranks: int, rank: int, exchange=None):
        if not lib().yah_tp_available():
            raise RuntimeError("NCCL (libnccl.so.2) is not available")
        uid = None
        if rank == 0:
            buf = ctypes.create_string_buffer(TP_ID_BYTES)
            check(lib().yah_tp_unique_id(buf))
            uid = buf.raw
        if nranks > 1:
            if exchange is None:
                raise ValueError("exchange is required for more than one rank")
            uid = exchange(uid)
        if uid is None or len(uid) != TP_ID_BYTES:
            raise ValueError("bad unique id")
        self.rank, self.nranks = rank, nranks
        h = ctypes.c_void_p()
        check(lib().yah_tp_init(ctypes.byref(h), nranks, rank, ctypes.create_string_buffer(uid, TP_ID_BYTES)))
        self.handle = h.value

    def allreduce_f32(self, ptr: int, count: int, stream=None):
        check(lib().yah_tp_allreduce_f32(self.handle, ptr, count, stream))

    def allgather_f32(self, send: int, recv: int, count: int, stream=None):
        check(lib().yah_tp_allgather_f32(self.handle, send, recv, count, stream))

    def close(self):
        if self.handle:
            check(lib().yah_tp_destroy(self.handle))
            self.handle = None


class Peers:
    """Device buffers of every rank (yah_tp_peers_*: CUDA IPC mappings exchanged over the communicator).
    Collective: every rank creates it with the same number of buffers."""

    def __init__(self, comm: Comm, bufs: list, stream=None):
        arr = (ctypes.c_void_p * len(bufs))(*[b.ptr for b in bufs])
        h = ctypes.c_void_p()
        check(lib().yah_tp_peers_create(comm.handle, arr, len(bufs), stream, ctypes.byref(h)))
        self.handle = h.value

    def ptr(self, rank: int, buf: int) -> int:
        p = ctypes.c_void_p()
        check(lib().yah_tp_peers_ptr(self.handle, rank, buf, ctypes.byref(p)))
        return p.value

    def close(self):
        if self.handle:
            check(lib().yah_tp_peers_destroy(self.handle))
            self.handle = None


# ----------------------------------------------------------------------------------------------- the stack
class LlamaStack:
    """One rank's part of the linear layer stack: its weight shards on the device and the forward pass.

    With `chunks` > 1 the M tokens go through the layers in that many row chunks, pipelined over two streams: the
    norms and GEMMs of every chunk on the caller's stream, each row-parallel allreduce on a communication stream
    once that chunk's GEMM is done, so the allreduce of chunk c runs under the GEMMs of chunk c + 1 (every op is
    row-wise in the tokens, so chunks are independent until the end). Run it with an SM budget
    (yah_set_sm_budget) below the device's SM count so that NCCL's kernels find free SMs while a GEMM runs."""

    def __init__(self, dev: Device, comm: Comm, shape: StackShape, shards: list, M: int, chunks: int = 1,
                 mode: str = "parity"):
        if chunks < 1 or M % chunks:
            raise ValueError(f"{M} tokens do not split into {chunks} chunks")
        if mode not in ("parity", "speed", "fused"):
            raise ValueError(f"mode {mode!r}: parity (f32 partial sums), speed (f16 partial sums) or fused (f32 "
                             "partial sums reduced over peer memory)")
        if mode != "parity" and chunks != 1:
            raise ValueError(f"the {mode} mode runs unchunked")
        if mode == "fused":
            token_slice(M, comm.nranks, comm.rank)  # raises when M does not split
        self.dev, self.comm, self.shape, self.M, self.chunks, self.mode = dev, comm, shape, M, chunks, mode
        p = comm.nranks
        self.q_r = shape.n_q * shape.head_dim // p
        self.qkv_r = shape.qkv // p
        self.ff_r = shape.ff // p
        self.w = [{k: dev.upload(v) for k, v in s.items()} for s in shards]
        self.row_bytes = {k: v.shape[1] for k, v in shards[0].items()}
        H = shape.hidden
        self.xn = dev.empty(M * H * 2)
        self.qkv = dev.empty(M * self.qkv_r * 2)
        self.g = dev.empty(M * self.ff_r * 4)
        self.act = dev.empty(M * self.ff_r * 2)
        # the speed mode's f16 row-parallel partial sums, added into h by the next norm's pass
        self.part = dev.empty(M * H * 2) if mode == "speed" and chunks == 1 else None
        if chunks > 1:
            self.comm_stream = Stream()
            self.ev_gemm = [Event() for _ in range(chunks)]
            self.ev_red = [Event() for _ in range(chunks)]
        self.peers = None
        if mode == "fused":
            self.ms = M // p
            self.recv = dev.empty(M * H * 4)             # [p][M/p][H] f32: slot q holds rank q's partials
            self.hs = dev.empty(self.ms * H * 4)         # this rank's slice of the residual stream
            self.flags = dev.empty(2 * 32 * 4).fill(0)   # [2][32] int epochs: 0 partials landed, 1 activations
            dev.synchronize()                            # zeroed before any rank can signal into it
            self.peers = Peers(comm, [self.recv, self.xn, self.flags])
            self.ep_r = self.ep_x = 0

    @property
    def ffn_fused(self) -> bool:
        """Whether gate and up run as one tile GEMM (yah_qgemm_ffn: the f32 gate never goes through memory; results
        identical to the two GEMMs). Measured on B200 at 4096 tokens: 137 vs 156 us for the 1792-row shards of 8
        GPUs, 248 vs 263 at 4, 477 vs 486 at 2, but 980 vs 959 for the whole 14336 rows, so only sharded."""
        return self.comm.nranks > 1 and self.M // self.chunks > 32

    @property
    def launches_per_forward(self) -> int:
        """Library kernel launches per forward pass (2 norms + 5 linears per layer and token chunk, 4 linears with
        the fused gate+up; the unchunked forward adds the final add; the fused mode adds 4 flag barriers per layer
        and its first norm)."""
        per = 7 - (1 if self.ffn_fused else 0)
        if self.mode == "fused":
            return (per + 4) * self.shape.layers + 1
        return per * self.shape.layers * self.chunks + (1 if self.part is not None else 0)

    def _gate_up(self, w, xn: int, M: int, g: int, act: int, stream):
        """act (f16 [M][ff_r]) = silu(xn W_gate^T) * (xn W_up^T) for this rank's column shards."""
        L, H, fmt = lib(), self.shape.hidden, self.shape.fmt
        if self.ffn_fused:
            check(L.yah_qgemm_ffn(w["gate"].ptr, w["up"].ptr, fmt, self.ff_r, H, self.row_bytes["gate"], 0, xn, M, H,
                                  act, self.ff_r, 0, -1, stream))
            return
        c = self.comm.handle
        check(L.yah_tp_linear_col(c, w["gate"].ptr, fmt, self.ff_r, H, self.row_bytes["gate"], xn, M, H, g, F32,
                                  self.ff_r, EPI_STORE, None, 0, stream))
        check(L.yah_tp_linear_col(c, w["up"].ptr, fmt, self.ff_r, H, self.row_bytes["up"], xn, M, H, act, F16,
                                  self.ff_r, EPI_SWIGLU, g, self.ff_r, stream))

    def forward(self, h: DeviceBuffer, stream=None):
        """h (f32 [M][hidden], the residual stream, identical on every rank) is updated in place."""
        if self.chunks > 1:
            return self._forward_chunked(h, stream)
        if self.mode == "speed":
            return self._forward_partials(h, stream)
        if self.mode == "fused":
            return self._forward_fused(h, stream)
        return self._forward_residual_epilogue(h, stream)

    def _forward_residual_epilogue(self, h: DeviceBuffer, stream=None):
        """Parity mode through yah_tp_linear_row: rank 0's GEMM epilogue adds the residual and the f32 allreduce
        sums h + partials in place (measured 3% faster at tp2 / tp4 than storing plain f32 partials and adding the
        sum in the norm pass, the speed mode's scheme)."""
        L, s, M, H, fmt = lib(), self.shape, self.M, self.shape.hidden, self.shape.fmt
        c = self.comm.handle
        for w in self.w:
            check(L.yah_rmsnorm(h.ptr, H, M, H, NORM_EPS, NORM_GAIN, self.xn.ptr, H, stream))
            check(L.yah_tp_linear_col(c, w["qkv"].ptr, fmt, self.qkv_r, H, self.row_bytes["qkv"], self.xn.ptr, M, H,
                                      self.qkv.ptr, F16, self.qkv_r, EPI_STORE, None, 0, stream))
            check(L.yah_tp_linear_row(c, w["o"].ptr, fmt, H, self.q_r, self.row_bytes["o"], 0, self.qkv.ptr, M,
                                      self.qkv_r, h.ptr, h.ptr, stream))
            check(L.yah_rmsnorm(h.ptr, H, M, H, NORM_EPS, NORM_GAIN, self.xn.ptr, H, stream))
            self._gate_up(w, self.xn.ptr, M, self.g.ptr, self.act.ptr, stream)
            check(L.yah_tp_linear_row(c, w["down"].ptr, fmt, H, self.ff_r, self.row_bytes["down"], 0, self.act.ptr, M,
                                      self.ff_r, h.ptr, h.ptr, stream))

    def _row_parallel(self, name: str, w, K_r: int, x_ptr: int, ldx: int, h_ptr: int, Mc: int, stream):
        """The GEMM half of a row-parallel linear (yah_tp_linear_row without its allreduce): rank 0 adds the
        residual (h, in place), the others store their partial into h; the allreduce follows on the communication
        stream."""
        L, fmt, H = lib(), self.shape.fmt, self.shape.hidden
        r0 = self.comm.rank == 0
        fn = L.yah_qgemv if Mc <= 32 else L.yah_qgemm
        check(fn(w.ptr, fmt, H, K_r, self.row_bytes[name], 0, x_ptr, Mc, ldx, h_ptr, F32, H,
                 EPI_RESID if r0 else EPI_STORE, h_ptr if r0 else None, H if r0 else 0, stream))

    def _forward_partials(self, h: DeviceBuffer, stream):
        """The speed mode: every rank's row-parallel GEMM stores its plain f16 partial sums (no residual read), the
        allreduce sums them in place (half the bytes of f32), and the next norm's pass adds the sum into the f32
        residual stream (yah_add_rmsnorm), the last layer's sum an add-only pass. (The same scheme with f32 partials
        was measured 3% slower than the parity mode's residual epilogue.)"""
        L, M, H, fmt = lib(), self.M, self.shape.hidden, self.shape.fmt
        c, part = self.comm.handle, self.part.ptr
        speed = self.mode == "speed"
        pdt = F16 if speed else F32
        allreduce = L.yah_tp_allreduce_f16 if speed else L.yah_tp_allreduce_f32
        pending = False
        fn = L.yah_qgemv if M <= 32 else L.yah_qgemm

        def norm():
            if pending:
                check(L.yah_add_rmsnorm(h.ptr, H, part, pdt, H, M, H, NORM_EPS, NORM_GAIN, self.xn.ptr, H, stream))
            else:
                check(L.yah_rmsnorm(h.ptr, H, M, H, NORM_EPS, NORM_GAIN, self.xn.ptr, H, stream))

        for w in self.w:
            norm()
            check(L.yah_tp_linear_col(c, w["qkv"].ptr, fmt, self.qkv_r, H, self.row_bytes["qkv"], self.xn.ptr, M, H,
                                      self.qkv.ptr, F16, self.qkv_r, EPI_STORE, None, 0, stream))
            check(fn(w["o"].ptr, fmt, H, self.q_r, self.row_bytes["o"], 0, self.qkv.ptr, M, self.qkv_r, part, pdt, H,
                     EPI_STORE, None, 0, stream))
            check(allreduce(c, part, M * H, stream))
            pending = True
            norm()
            self._gate_up(w, self.xn.ptr, M, self.g.ptr, self.act.ptr, stream)
            check(fn(w["down"].ptr, fmt, H, self.ff_r, self.row_bytes["down"], 0, self.act.ptr, M, self.ff_r, part,
                     pdt, H, EPI_STORE, None, 0, stream))
            check(allreduce(c, part, M * H, stream))
        if pending:
            check(L.yah_add_rmsnorm(h.ptr, H, part, pdt, H, M, H, NORM_EPS, NORM_GAIN, None, 0, stream))

    def _forward_fused(self, h: DeviceBuffer, stream=None):
        """The fused mode (module docstring): h (f32 [M][hidden], identical on every rank) is updated in place; the
        layers keep this rank's token slice of it and the last step gathers the slices back."""
        L, M, H, fmt = lib(), self.M, self.shape.hidden, self.shape.fmt
        c, pe, ms, rank, p = self.comm.handle, self.peers.handle, self.ms, self.comm.rank, self.comm.nranks
        RECV, XN, FLAGS = 0, 1, 2
        hs, recv = self.hs.ptr, self.recv.ptr
        check(L.yah_memcpy_d2d(hs, h.ptr + rank * ms * H * 4, ms * H * 4, stream))

        def reduce_norm(add: bool, norm: bool):
            check(L.yah_tp_reduce_norm(pe, hs, H, ms, H, recv if add else None, p if add else 0, ms * H, H, NORM_EPS,
                                       NORM_GAIN, XN if norm else -1, rank * ms, H, stream))

        def exchange_partials():  # every rank's scatter into this rank's slots has landed
            self.ep_r += 1
            check(L.yah_tp_barrier(pe, FLAGS, 0, self.ep_r, stream))

        def publish_activations():  # every rank's normalised slice is in this rank's xn
            self.ep_x += 1
            check(L.yah_tp_barrier(pe, FLAGS, 32, self.ep_x, stream))

        reduce_norm(False, True)
        publish_activations()
        n = len(self.w)
        for i, w in enumerate(self.w):
            check(L.yah_tp_linear_col(c, w["qkv"].ptr, fmt, self.qkv_r, H, self.row_bytes["qkv"], self.xn.ptr, M, H,
                                      self.qkv.ptr, F16, self.qkv_r, EPI_STORE, None, 0, stream))
            check(L.yah_tp_linear_row_scatter(pe, w["o"].ptr, fmt, H, self.q_r, self.row_bytes["o"], 0, self.qkv.ptr,
                                              M, self.qkv_r, RECV, stream))
            exchange_partials()
            reduce_norm(True, True)
            publish_activations()
            self._gate_up(w, self.xn.ptr, M, self.g.ptr, self.act.ptr, stream)
            check(L.yah_tp_linear_row_scatter(pe, w["down"].ptr, fmt, H, self.ff_r, self.row_bytes["down"], 0,
                                              self.act.ptr, M, self.ff_r, RECV, stream))
            exchange_partials()
            last = i == n - 1
            reduce_norm(True, not last)
            if not last:
                publish_activations()
        self.comm.allgather_f32(hs, h.ptr, ms * H, stream)

    def _forward_chunked(self, h: DeviceBuffer, stream):
        L, s, H, fmt, C = lib(), self.shape, self.shape.hidden, self.shape.fmt, self.chunks
        Mc = self.M // C
        c_h, cs = self.comm.handle, self.comm_stream
        first = True
        for w in self.w:
            for half in (0, 1):
                for c in range(C):
                    hp = h.ptr + c * Mc * H * 4
                    xn = self.xn.ptr + c * Mc * H * 2
                    if not first:  # this chunk's previous allreduce is done before its rows are read again
                        check(L.yah_stream_wait_event(stream, self.ev_red[c].handle))
                    check(L.yah_rmsnorm(hp, H, Mc, H, NORM_EPS, NORM_GAIN, xn, H, stream))
                    if half == 0:
                        qkv = self.qkv.ptr + c * Mc * self.qkv_r * 2
                        check(L.yah_tp_linear_col(c_h, w["qkv"].ptr, fmt, self.qkv_r, H, self.row_bytes["qkv"], xn,
                                                  Mc, H, qkv, F16, self.qkv_r, EPI_STORE, None, 0, stream))
                        self._row_parallel("o", w["o"], self.q_r, qkv, self.qkv_r, hp, Mc, stream)
                    else:
                        g = self.g.ptr + c * Mc * self.ff_r * 4
                        act = self.act.ptr + c * Mc * self.ff_r * 2
                        self._gate_up(w, xn, Mc, g, act, stream)
                        self._row_parallel("down", w["down"], self.ff_r, act, self.ff_r, hp, Mc, stream)
                    self.ev_gemm[c].record(stream)
                    cs.wait(self.ev_gemm[c])
                    check(L.yah_tp_allreduce_f32(c_h, hp, Mc * H, cs.handle))
                    self.ev_red[c].record(cs.handle)
                first = False
        for c in range(C):
            check(L.yah_stream_wait_event(stream, self.ev_red[c].handle))

    def close(self):
        for w in self.w:
            for b in w.values():
                b.close()
        for b in (self.xn, self.qkv, self.g, self.act) + ((self.part,) if self.part else ()):
            b.close()
        if self.chunks > 1:
            for e in self.ev_gemm + self.ev_red:
                e.close()
            self.comm_stream.close()
        if self.peers is not None:
            self.peers.close()
            for b in (self.recv, self.hs, self.flags):
                b.close()
