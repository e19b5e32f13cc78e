"""Reference math and spawned worker processes of the tensor-parallel tests (not collected by pytest).

stack_ref restates the layer stack of yet-another-halo-engine_b200/tp.py in float64 with the same f16 / f32
rounding points (normalised input, QKV output and SwiGLU output are f16; the residual stream is f32), on the
oracle's f16 dequantisation of the full (unsharded) weights.
"""
import os
import sys
from datetime import timedelta

import numpy as np

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def rmsnorm_ref(h, gain, eps):
    h = h.astype(np.float64)
    return (h * gain / np.sqrt((h * h).mean(axis=1, keepdims=True) + eps)).astype(np.float16)


def stack_ref(O, shape, layers, h, gain, eps):
    """float64 restatement of LlamaStack.forward over full weights; returns the final f32 residual stream."""
    fmt, H, q = shape.fmt, shape.hidden, shape.n_q * shape.head_dim
    h = h.astype(np.float32)
    for W in layers:
        deq = {k: O.dequant_f16(fmt, v, v.shape[0], (v.shape[1] // {8: 272, 12: 144, 14: 210}[fmt]) * 256)
               for k, v in W.items()}
        xn = rmsnorm_ref(h, gain, eps)
        qkv = O.gemm_ref(deq["qkv"], xn).astype(np.float16)
        h = (h.astype(np.float64) + O.gemm_ref(deq["o"], qkv[:, :q])).astype(np.float32)
        xn = rmsnorm_ref(h, gain, eps)
        g = O.gemm_ref(deq["gate"], xn).astype(np.float32).astype(np.float64)
        act = (g / (1.0 + np.exp(-g)) * O.gemm_ref(deq["up"], xn)).astype(np.float16)
        h = (h.astype(np.float64) + O.gemm_ref(deq["down"], act)).astype(np.float32)
    return h


def cpu_shard_worker(rank, world, port, out_q):
    """gloo rank: column shards concatenate to the full product, row-parallel partials all-reduce to it (oracle)."""
    import torch
    import torch.distributed as dist
    import __graft_entry__ as ge
    from oracle import oracle as O
    pkg = ge.load_package()
    F, tp = pkg.formats, pkg.tp
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=60))
    try:
        N, K, M = 96, 1024, 5
        w = F.synth_weights(F.Q4_K, N, K, seed=70)
        x = F.synth_activations(M, K, seed=71)
        full = O.gemm_ref(O.dequant_f16(F.Q4_K, w, N, K), x)
        # column-parallel: this rank's rows; gather the slices
        r0, r1 = tp.even_range(N, world, rank)
        ws = tp.take_rows(w, [(r0, r1)])
        part = torch.from_numpy(O.gemm_ref(O.dequant_f16(F.Q4_K, ws, r1 - r0, K), x))
        slices = [None] * world
        dist.all_gather_object(slices, (r0, r1, part.numpy()))
        col = np.concatenate([s[2] for s in sorted(slices, key=lambda s: s[0])], axis=1)
        # row-parallel: this rank's K window, summed over ranks
        k0, k1 = tp.k_window(K, world, rank)
        wk = tp.take_k_window(w, F.Q4_K, k0, k1)
        partial = torch.from_numpy(O.gemm_ref(O.dequant_f16(F.Q4_K, wk, N, k1 - k0), x[:, k0:k1]))
        dist.all_reduce(partial)
        out_q.put((rank, float(np.abs(col - full).max()), float(np.abs(partial.numpy() - full).max() /
                                                                    np.abs(full).max())))
    finally:
        dist.destroy_process_group()


def cpu_fused_worker(rank, world, port, out_q):
    """gloo rank: the fused mode's exchange restated on the CPU (oracle arithmetic). Each rank's row-parallel K-window
    partial goes, token slice by token slice, to the slice's owner as slot `rank`; the owner adds the slots in rank
    order into its slice of the residual stream and normalises it; the normalised slices gathered in owner order
    must equal the single-rank result (residual + full product, then RMSNorm)."""
    import torch.distributed as dist
    import __graft_entry__ as ge
    from oracle import oracle as O
    pkg = ge.load_package()
    F, tp = pkg.formats, pkg.tp
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=60))
    try:
        N, K, M = 256, 1024, 64
        w = F.synth_weights(F.Q4_K, N, K, seed=80)
        x = F.synth_activations(M, K, seed=81)
        h = np.random.default_rng(82).standard_normal((M, N))
        full = O.gemm_ref(O.dequant_f16(F.Q4_K, w, N, K), x)
        want = rmsnorm_ref(h + full, 1 / 64, 1e-6)
        k0, k1 = tp.k_window(K, world, rank)
        partial = O.gemm_ref(O.dequant_f16(F.Q4_K, tp.take_k_window(w, F.Q4_K, k0, k1), N, k1 - k0), x[:, k0:k1])
        parts = [None] * world
        dist.all_gather_object(parts, partial)  # stands in for the GEMM's stores into the owners' slots
        lo, hi = tp.token_slice(M, world, rank)
        slots = np.stack([parts[q][lo:hi] for q in range(world)])  # [world][M / world][N]: slot q = rank q's partial
        hs = h[lo:hi].copy()
        for q in range(world):
            hs = hs + slots[q]
        mine = rmsnorm_ref(hs, 1 / 64, 1e-6)
        gathered = [None] * world
        dist.all_gather_object(gathered, (lo, mine))
        got = np.concatenate([g[1] for g in sorted(gathered, key=lambda g: g[0])])
        err = np.abs(got.astype(np.float64) - want.astype(np.float64))
        ulp = np.spacing(np.abs(want).astype(np.float16)).astype(np.float64)
        out_q.put((rank, bool((err <= ulp).all()), float(err.max())))
    finally:
        dist.destroy_process_group()


def gpu_stack_worker(rank, world, id_q, out_q, mode="parity"):
    """NCCL rank on GPU `rank`: the small stack sharded over `world` ranks vs the float64 reference."""
    import __graft_entry__ as ge
    from oracle import oracle as O
    pkg = ge.load_package()
    tp = pkg.tp
    from ctypes import c_int
    dev = pkg.Device(rank)
    shape = tp.StackShape(layers=2, hidden=512, n_q=4, n_kv=2, head_dim=128, ff=1024)
    M = 64

    def exchange(uid):
        if rank == 0:
            for _ in range(world - 1):
                id_q.put(uid)
            return uid
        return id_q.get(timeout=60)

    comm = tp.Comm(world, rank, exchange)
    full = [tp.layer_weights(shape, i) for i in range(shape.layers)]
    if mode == "speed":  # f16 partial sums need weights whose layer outputs fit f16 (d, dmin scaled by 2^-6)
        full = [{k: pkg.formats.scale_q4k_d(v, 1 / 64) for k, v in f.items()} for f in full]
    stack = tp.LlamaStack(dev, comm, shape, [tp.shard_layer(shape, f, world, rank) for f in full], M, mode=mode)
    h0 = np.random.default_rng(72).standard_normal((M, shape.hidden)).astype(np.float32)
    h = dev.upload(h0)
    stack.forward(h)
    got = h.download(np.float32, (M, shape.hidden))
    ref = stack_ref(O, shape, full, h0, tp.NORM_GAIN, tp.NORM_EPS)
    e = O.errors(got, ref)
    status = c_int(0)
    pkg.lib().yah_status_word(status)
    stack.close()
    comm.close()
    out_q.put((rank, e["rel_fro"], e["finite"], status.value))
