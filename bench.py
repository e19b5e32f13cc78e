#!/usr/bin/env python3
"""Benchmark of the quantised-linear hot path on B200 (one JSON line on rank 0).

Workloads (--workload):
  gemm   (default) BASELINE config 2: Q4_K prefill tile GEMM, M=2048 tokens, K=4096, N=14336, f16 out; TFLOP/s.
  gemv   BASELINE config 3 decode GEMV: Q4_K 4096 x 14336 weights, M tokens (--tokens, default 1); HBM GB/s.
  lmhead BASELINE config 5: Q6_K lm head, 128256 x 4096 weights (431 MB); --tokens <= 32: decode GEMV, HBM GB/s;
         above: prefill GEMM, TFLOP/s.
  stack  BASELINE config 4: the Llama-shaped Q4_K linear stack (32 layers, hidden 4096, QKV 6144, FF 14336) over
         M=4096 tokens, tensor-parallel over the N GPUs (column-parallel QKV/gate/up, row-parallel o_proj/down with
         one NCCL allreduce each; yet-another-halo-engine_b200/tp.py); TFLOP/s of the whole job, strong scaling.
A step is one launch of the kernel over one batch. Inputs are resident in HBM when the timed region starts; the
step rotates through input copies whose total exceeds L2 (126 MB), so no step reads inputs another step left in
L2. Timing: W warm-up steps, then exactly K steps between a barrier + device synchronise on both sides, CUDA
events on the launching stream, max over ranks; gemm / gemv / lmhead replay the K steps as one CUDA graph. `e2e` repeats
the metric through the public API with pinned host buffers: every step copies its activations host->device and its
output device->host inside the timed region.

Multi-GPU (torchrun, one process per GPU): for gemm / gemv every rank runs the same workload on its own batch
(replicas, weak scaling; the single GEMM / GEMV has no exchange step); the stack is sharded (the allreduces go
through the library's own NCCL communicator). torch.distributed (gloo, CPU tensors) is used only for the barrier,
the max over ranks and handing rank 0's NCCL id to the others.

--impl reference: the reference's CPU path for the same metric (its test-suite oracle: gguf-py
quants.dequantize -> f16 -> numpy matmul, engine/gpu/loom/tools/gemv_check.py:161-162), on the host cores, rank 0.
"""
from __future__ import annotations

import argparse
import importlib
import json
import os
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

L2_BYTES = 126 * 2 ** 20


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return {"hbm_gbs": d["hbm_gbs"], "tflops": d["bf16_tflops"], "tflops_sustained": d["bf16_tflops_sustained"],
                "src": "measured"}
    return {"hbm_gbs": 6650.0, "tflops": 1590.0, "tflops_sustained": 1400.0, "src": "fallback"}


class Clocks:
    """nvidia-smi sampling during the timed region (median SM clock, throttle reasons seen)."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-i", str(self.index), "-lms", "100"], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self):
        if not self.proc:
            return None
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [v.strip() for v in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = max(mx, float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


def dist_init(n):
    if n <= 1 or "RANK" not in os.environ:
        return None
    import datetime

    import torch.distributed as dist
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=600))
    return dist


def barrier(dist):
    if dist:
        dist.barrier()


def max_over_ranks(dist, v):
    if not dist:
        return v
    import torch
    t = torch.tensor([v], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def cpu_cores():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


# ------------------------------------------------------------------------------------------------ workloads
def workload_of(args):
    """The single-kernel workloads: config 2 (Q4_K gate/up prefill GEMM), config 3 (Q4_K down decode GEMV at
    --tokens), config 5 (Q6_K lm head, 128256 x 4096: decode GEMV for --tokens <= 32, prefill GEMM above)."""
    if args.workload == "gemv":
        return dict(name="q4k_decode_gemv", fmt=12, fmt_name="Q4_K", M=args.tokens, K=14336, N=4096, out="f32",
                    gemv=True, metric=f"Q4_K decode GEMV HBM GB/s (M={args.tokens})")
    if args.workload == "lmhead":
        gemv = args.tokens <= 32
        return dict(name="q6k_lm_head_" + ("decode_gemv" if gemv else "prefill_gemm"), fmt=14, fmt_name="Q6_K",
                    M=args.tokens, K=4096, N=128256, out="f32" if gemv else "f16", gemv=gemv,
                    metric=(f"Q6_K lm-head decode GEMV HBM GB/s (M={args.tokens})" if gemv
                            else f"Q6_K lm-head prefill TFLOP/s (M={args.tokens})"))
    return dict(name="q4k_prefill_gemm", fmt=12, fmt_name="Q4_K", M=2048, K=4096, N=14336, out="f16", gemv=False,
                metric="Q4_K dequant-GEMM prefill TFLOP/s")


def run_ours(args, dist, rank, local_rank):
    import __graft_entry__ as ge
    pkg = ge.load_package()
    F, ops = pkg.formats, pkg.ops
    dev = pkg.Device(local_rank)
    wl = workload_of(args)
    t, M, K, N = wl["fmt"], wl["M"], wl["K"], wl["N"]
    gemv = wl["gemv"]
    w = F.synth_weights(t, N, K, seed=0)
    x = F.synth_activations(M, K, seed=1 + rank)
    wbytes, xbytes = w.nbytes, x.nbytes
    ydt = 1 if wl["out"] == "f16" else 0
    ybytes = M * N * (2 if ydt else 4)
    per_copy = wbytes + xbytes
    copies = max(2, int(np.ceil(2.2 * L2_BYTES / per_copy)))
    wd = [dev.upload(w) for _ in range(copies)]
    xd = [dev.upload(x) for _ in range(copies)]
    yd = [dev.empty(ybytes) for _ in range(2)]
    stream = pkg.Stream()
    s = stream.handle
    fn = ops.qgemv_ptr if gemv else ops.qgemm_ptr

    def step(i):
        j = i % copies
        fn(wd[j].ptr, t, N, K, w.shape[1], 0, xd[j].ptr, M, K, yd[i & 1].ptr, ydt, N, stream=s)

    for i in range(args.warmup):
        step(i)
    stream.synchronize()
    # The K timed steps as one CUDA graph (one kernel node per step, rotating inputs): a decode GEMV lasts a few
    # microseconds, less than the host needs to issue a call, and an engine replays such loops as graphs.
    graph = pkg.Graph(stream)
    graph.begin()
    for i in range(args.steps):
        step(i)
    graph.end()
    graph.launch()  # one untimed replay
    stream.synchronize()
    e0, e1 = pkg.Event(), pkg.Event()
    clocks = Clocks(local_rank)
    barrier(dist)
    dev.synchronize()
    clocks.start()
    time.sleep(0.3)  # the sampler's first reading precedes the timed region
    e0.record(s)
    graph.launch()
    e1.record(s)
    e1.synchronize()
    dev.synchronize()
    clk = clocks.stop()
    graph.close()
    if clk is not None:
        clk["timed_region_ms"] = None
    barrier(dist)
    ms_local = e0.elapsed_ms(e1)
    ms = max_over_ranks(dist, ms_local)
    status = dev.status_word()
    if status:
        raise RuntimeError(f"kernel status word {status}")

    # ---------------- e2e: pinned host activations in, output out, every step
    xh = pkg.PinnedBuffer(xbytes)
    xh.array(np.float16, x.shape)[...] = x
    yh = pkg.PinnedBuffer(ybytes)
    xdev = dev.empty(xbytes)

    def e2e_step(i):
        pkg.lib().yah_memcpy_h2d(xdev.ptr, xh.ptr, xbytes, s)
        fn(wd[0].ptr, t, N, K, w.shape[1], 0, xdev.ptr, M, K, yd[0].ptr, ydt, N, stream=s)
        pkg.lib().yah_memcpy_d2h(yh.ptr, yd[0].ptr, ybytes, s)

    for i in range(max(1, args.warmup)):
        e2e_step(i)
    stream.synchronize()
    barrier(dist)
    e2 = pkg.Event()
    e3 = pkg.Event()
    e2.record(s)
    for i in range(args.steps):
        e2e_step(i)
    e3.record(s)
    e3.synchronize()
    ms_e2e = max_over_ranks(dist, e2.elapsed_ms(e3))

    world = int(os.environ.get("WORLD_SIZE", "1"))
    pk = peaks()
    per_step_ms = ms / args.steps
    if gemv:
        alg_bytes = wbytes + xbytes + ybytes
        value = world * alg_bytes / (per_step_ms * 1e-3) / 1e9
        unit, metric = "GB/s", wl["metric"]
        achieved = alg_bytes / (ms_local / args.steps * 1e-3) / 1e9
        roof = {"bound": "hbm", "achieved": round(achieved, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
                "frac": round(achieved / pk["hbm_gbs"], 4), "traffic": None, "peak_src": pk["src"],
                "algorithmic_bytes_per_launch": alg_bytes}
        e2e_val = world * alg_bytes / (ms_e2e / args.steps * 1e-3) / 1e9
    else:
        flops = 2.0 * M * N * K
        value = world * flops / (per_step_ms * 1e-3) / 1e12
        unit, metric = "TFLOP/s", wl["metric"]
        achieved = flops / (ms_local / args.steps * 1e-3) / 1e12
        roof = {"bound": "tensor", "achieved": round(achieved, 1), "peak": pk["tflops"], "unit": "TFLOP/s",
                "frac": round(achieved / pk["tflops"], 4), "traffic": None, "peak_src": pk["src"],
                "frac_of_sustained": round(achieved / pk["tflops_sustained"], 4),
                "algorithmic_flops_per_launch": flops}
        e2e_val = world * flops / (ms_e2e / args.steps * 1e-3) / 1e12
    traffic = load_traffic(wl["name"])
    if traffic is not None:
        roof["traffic"] = traffic
    line = {
        "metric": metric, "value": round(value, 2), "unit": unit, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(per_step_ms, 5), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": f"f16 x GGUF-{wl['fmt_name']} -> f32 acc",
        "data": "synthetic",
        "config": {"workload": wl["name"], "M_tokens": M, "K": K, "N": N, "weight_format": wl["fmt_name"],
                   "out_dtype": wl["out"], "parallelism": f"replicas x{world}",
                   "launch_overlap": bool(args.launch_overlap),
                   "l2": f"rotating {copies} input copies ({copies * per_copy / 2**20:.0f} MiB > L2)"},
        "e2e": {"value": round(e2e_val, 2), "unit": unit, "h2d_bytes_per_step": xbytes, "d2h_bytes_per_step": ybytes},
        "gpu_launches": args.steps,
        "roofline": roof,
        "clocks": clk,
    }
    return line


def run_stack(args, dist, rank, local_rank):
    """The tensor-parallel layer stack: one step = one forward pass of all layers over M tokens."""
    import __graft_entry__ as ge
    pkg = ge.load_package()
    F, tp = pkg.formats, pkg.tp
    dev = pkg.Device(local_rank)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    shape = tp.StackShape(layers=args.layers)
    M, H = args.stack_tokens, shape.hidden

    def exchange(uid):
        obj = [uid]
        dist.broadcast_object_list(obj, src=0)
        return obj[0]

    comm = tp.Comm(world, rank, exchange if world > 1 else None)
    # Each rank generates its own shards (seeded per rank; the full tensors would be their concatenation). Four
    # distinct weight sets cycle over the layers: 4 x 122.7 MB / world > L2 at one GPU, and no layer finds the
    # weights it reads in L2.
    p = world
    sets = []
    # The speed mode's f16 partial sums overflow with the BASELINE weight distribution (layer outputs ~1e5-1e6), so
    # it runs on weights whose d and dmin are scaled by 2^-8 (same bytes and work; reported in `data`).
    scale = (lambda w: F.scale_q4k_d(w, 1 / 256)) if args.stack_mode == "speed" else (lambda w: w)
    for k in range(min(4, shape.layers)):
        s0 = 5000 + 64 * k + 8 * rank
        sets.append({"qkv": scale(F.synth_weights(shape.fmt, shape.qkv // p, H, seed=s0)),
                     "o": scale(F.synth_weights(shape.fmt, H, shape.n_q * shape.head_dim // p, seed=s0 + 1)),
                     "gate": scale(F.synth_weights(shape.fmt, shape.ff // p, H, seed=s0 + 2)),
                     "up": scale(F.synth_weights(shape.fmt, shape.ff // p, H, seed=s0 + 3)),
                     "down": scale(F.synth_weights(shape.fmt, H, shape.ff // p, seed=s0 + 4))})
    chunks = args.stack_chunks
    if chunks > 1:
        pkg.lib().yah_set_sm_budget(dev.sm_count - args.stack_nccl_sms)
    stack = tp.LlamaStack(dev, comm, shape, [sets[i % len(sets)] for i in range(shape.layers)], M, chunks=chunks,
                          mode=args.stack_mode)
    h0 = np.random.default_rng(7).standard_normal((M, H)).astype(np.float32)
    h0d, h = dev.upload(h0), dev.empty(M * H * 4)
    stream = pkg.Stream()
    s = stream.handle

    def step():
        pkg.lib().yah_memcpy_d2d(h.ptr, h0d.ptr, M * H * 4, s)  # every step starts from the same residual stream
        stack.forward(h, s)

    for _ in range(args.warmup):
        step()
    stream.synchronize()
    e0, e1 = pkg.Event(), pkg.Event()
    clocks = Clocks(local_rank)
    barrier(dist)
    dev.synchronize()
    clocks.start()
    time.sleep(0.3)
    e0.record(s)
    for _ in range(args.steps):
        step()
    e1.record(s)
    e1.synchronize()
    clk = clocks.stop()
    barrier(dist)
    ms_local = e0.elapsed_ms(e1)
    ms = max_over_ranks(dist, ms_local)
    if dev.status_word():
        raise RuntimeError(f"kernel status word {dev.status_word()}")
    # e2e: the residual stream in from pinned host memory and out again every step
    hh = pkg.PinnedBuffer(M * H * 4)
    hh.array(np.float32, (M, H))[...] = h0
    barrier(dist)
    e2, e3 = pkg.Event(), pkg.Event()
    e2.record(s)
    for _ in range(args.steps):
        pkg.lib().yah_memcpy_h2d(h.ptr, hh.ptr, M * H * 4, s)
        stack.forward(h, s)
        pkg.lib().yah_memcpy_d2h(hh.ptr, h.ptr, M * H * 4, s)
    e3.record(s)
    e3.synchronize()
    ms_e2e = max_over_ranks(dist, e2.elapsed_ms(e3))
    out = h.download(np.float32, (M, H))
    if not np.isfinite(out).all():
        raise RuntimeError("non-finite residual stream")
    flops = shape.flops(M)
    per_step_ms = ms / args.steps
    value = flops / (per_step_ms * 1e-3) / 1e12
    pk = peaks()
    achieved = flops / world / (ms_local / args.steps * 1e-3) / 1e12
    line = {
        "metric": "Q4_K layer-stack prefill TFLOP/s (tensor-parallel)", "value": round(value, 2), "unit": "TFLOP/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(per_step_ms, 4),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "f16 x GGUF-Q4_K -> f32 acc, f32 residual stream",
        "data": ("synthetic" if args.stack_mode == "parity" else
                 "synthetic, Q4_K rule with d and dmin scaled by 2^-8 (f16 partial sums stay finite)"),
        "config": {"workload": "q4k_layer_stack_tp", "layers": shape.layers, "hidden": H, "qkv": shape.qkv,
                   "ff": shape.ff, "M_tokens": M, "parallelism": f"tp{world}", "token_chunks": chunks,
                   "partial_sums": "f32 (parity mode)" if args.stack_mode == "parity" else "f16 (speed mode)",
                   "gemm_sms": (dev.sm_count - args.stack_nccl_sms) if chunks > 1 else dev.sm_count,
                   "l2": "4 distinct weight sets cycled over the layers (> L2 per GPU at tp1)"},
        "e2e": {"value": round(flops / (ms_e2e / args.steps * 1e-3) / 1e12, 2), "unit": "TFLOP/s",
                "h2d_bytes_per_step": M * H * 4, "d2h_bytes_per_step": M * H * 4},
        "gpu_launches": args.steps * stack.launches_per_forward,
        "roofline": {"bound": "tensor", "achieved": round(achieved, 1), "peak": pk["tflops_sustained"],
                     "unit": "TFLOP/s", "frac": round(achieved / pk["tflops_sustained"], 4), "traffic": None,
                     "peak_src": pk["src"] + " (sustained)", "per_gpu": True},
        "clocks": clk,
    }
    stack.close()
    comm.close()
    return line


def load_traffic(name):
    """Per-launch DRAM bytes of the dominant kernel from the committed ncu summary (profiles/*.json)."""
    p = os.path.join(ROOT, "profiles", f"{name}.traffic.json")
    if os.path.exists(p):
        try:
            return json.load(open(p))["dram_bytes_per_launch"]
        except (ValueError, KeyError):
            return None
    return None


# ------------------------------------------------------------------------------------------------ CPU paths
CPU_PHASES = {"dequant": 0.0, "gemm": 0.0}  # seconds spent in each phase of cpu_reference_step since the last reset


def cpu_reference_step(fmt, w, x, K, use_gguf=True):
    """One dequant-then-GEMM on the host: gguf-py's dequantize (the reference's oracle) -> f16 -> f32 matmul. The two
    phases are timed separately into CPU_PHASES."""
    N = w.shape[0]
    t0 = time.perf_counter()
    if use_gguf:
        from gguf import GGMLQuantizationType as T
        from gguf import quants
        qt = {8: T.Q8_0, 12: T.Q4_K, 14: T.Q6_K}[fmt]
        wq = quants.dequantize(w, qt).astype(np.float16)
    else:
        from oracle import oracle as O
        wq = O.dequant_f16(fmt, w, N, K)
    t1 = time.perf_counter()
    y = x.astype(np.float32) @ wq.astype(np.float32).T
    CPU_PHASES["dequant"] += t1 - t0
    CPU_PHASES["gemm"] += time.perf_counter() - t1
    return y


def cpu_phases_reset():
    CPU_PHASES["dequant"] = CPU_PHASES["gemm"] = 0.0


def cpu_phases_ms(runs):
    """Milliseconds per run of the two phases since the last reset."""
    return {"dequant_ms": round(CPU_PHASES["dequant"] / runs * 1e3, 3),
            "gemm_ms": round(CPU_PHASES["gemm"] / runs * 1e3, 3)}


def cpu_jobs(args, frac):
    """The bounded CPU sample of the workload: a list of (format, weight rows, activations, K, full rows) and its
    algorithmic size (FLOPs, bytes). `frac` is the fraction of every weight's rows taken, so a stack sample keeps
    the stack's FLOP mix (QKV, o_proj, gate, up, down of one layer over all M tokens)."""
    import __graft_entry__ as ge
    F = ge.load_package().formats
    if args.workload == "stack":
        shape = ge.load_package().tp.StackShape(layers=args.layers)
        M, H = args.stack_tokens, shape.hidden
        mats = [(shape.qkv, H), (H, shape.n_q * shape.head_dim), (shape.ff, H), (shape.ff, H), (H, shape.ff)]
        fmt = shape.fmt
    else:
        wl = workload_of(args)
        M, fmt = wl["M"], wl["fmt"]
        mats = [(wl["N"], wl["K"])]
    xs, jobs = {}, []
    for i, (n, k) in enumerate(mats):
        rows = max(16, min(n, int(round(n * frac))))
        if k not in xs:
            xs[k] = F.synth_activations(M, k, seed=1 + k)
        jobs.append((fmt, F.synth_weights(fmt, rows, k, seed=i), xs[k], k, n))
    flops = sum(2.0 * M * w.shape[0] * k for _, w, _, k, _ in jobs)
    nbytes = sum(w.nbytes + x.nbytes + M * w.shape[0] * 4 for _, w, x, _, _ in jobs)
    return jobs, flops, nbytes


def cpu_run(jobs, use_gguf):
    for fmt, w, x, k, _ in jobs:
        cpu_reference_step(fmt, w, x, k, use_gguf)


def cpu_sample_text(args, jobs, use_gguf, runs_note):
    M = jobs[0][2].shape[0]
    mats = ", ".join(f"{w.shape[0]} of {n} rows x K={k}" for _, w, _, k, n in jobs)
    what = "one layer of the stack: " if args.workload == "stack" else ""
    return (f"{'gguf-py dequantize' if use_gguf else 'oracle C dequant'} + numpy f32 matmul, {what}{mats}, "
            f"{M} tokens; {runs_note}; OPENBLAS_NUM_THREADS={os.environ.get('OPENBLAS_NUM_THREADS', 'unset')}")


def cpu_kind():
    try:
        import gguf  # noqa: F401
        return True, "reference"
    except ImportError:
        return False, "port"


def cpu_metric(args, flops, nbytes, per):
    gemv = args.workload != "stack" and workload_of(args)["gemv"]
    return (nbytes / per / 1e9, "GB/s") if gemv else (flops / per / 1e12, "TFLOP/s")


def cpu_baseline(args, seconds=10.0):
    """The CPU path timed on a bounded sample (rows of each weight) for the same metric."""
    use_gguf, kind = cpu_kind()
    frac = 1 / 16 if args.workload == "stack" else min(1.0, 2048 / workload_of(args)["N"])
    jobs, flops, nbytes = cpu_jobs(args, frac)
    cpu_run(jobs, use_gguf)  # warm-up
    cpu_phases_reset()
    n, t0 = 0, time.perf_counter()
    while True:
        cpu_run(jobs, use_gguf)
        n += 1
        el = time.perf_counter() - t0
        if el >= seconds or n >= 50:
            break
    per = el / n
    val, unit = cpu_metric(args, flops, nbytes, per)
    return {"value": round(val, 5), "unit": unit, "cores": cpu_cores(), "kind": kind,
            "sample": cpu_sample_text(args, jobs, use_gguf, f"{n} runs, {per * 1e3:.1f} ms each"), **cpu_phases_ms(n)}


def run_reference(args, rank, budget_s=150.0):
    """The reference's CPU path on the same metric and config, rank 0 only. Each step is one bounded sample; when
    the first warm-up step shows that K steps would take more than `budget_s`, every weight's sampled rows shrink
    by the same factor so that the run still ends within a few minutes."""
    if rank != 0:
        return None
    use_gguf, kind = cpu_kind()
    frac = 1 / 16 if args.workload == "stack" else min(1.0, 1024 / workload_of(args)["N"])
    jobs, flops, nbytes = cpu_jobs(args, frac)
    t0 = time.perf_counter()
    cpu_run(jobs, use_gguf)
    first = time.perf_counter() - t0
    if first * (args.steps + args.warmup) > budget_s:
        frac *= budget_s / (first * (args.steps + args.warmup))
        jobs, flops, nbytes = cpu_jobs(args, frac)
    for _ in range(args.warmup):
        cpu_run(jobs, use_gguf)
    cpu_phases_reset()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        cpu_run(jobs, use_gguf)
    el = time.perf_counter() - t0
    per = el / args.steps
    val, unit = cpu_metric(args, flops, nbytes, per)
    sample = cpu_sample_text(args, jobs, use_gguf, "per step")
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if args.workload == "stack":
        import __graft_entry__ as ge
        shape = ge.load_package().tp.StackShape(layers=args.layers)
        metric = "Q4_K layer-stack prefill TFLOP/s (tensor-parallel)"
        config = {"workload": "q4k_layer_stack_tp", "layers": shape.layers, "hidden": shape.hidden,
                  "qkv": shape.qkv, "ff": shape.ff, "M_tokens": args.stack_tokens, "parallelism": f"tp{world}"}
        scaling = "strong"
    else:
        wl = workload_of(args)
        metric = wl["metric"]
        config = {"workload": wl["name"], "M_tokens": wl["M"], "K": wl["K"], "N": wl["N"],
                  "weight_format": wl["fmt_name"]}
        scaling = "weak"
    return {"impl": "reference", "metric": metric, "value": round(val, 5), "unit": unit,
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(per * 1e3, 3), "higher_is_better": True, "scaling": scaling, "vs_baseline": None,
            "dtype": "f16 weights (dequantised) x f16 -> f32", "data": "synthetic", "config": config,
            "cpu_baseline": {"value": round(val, 5), "unit": unit, "cores": cpu_cores(), "kind": kind,
                             "sample": sample, **cpu_phases_ms(args.steps)},
            "e2e": {"value": round(val, 5), "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="gemm", choices=["gemm", "gemv", "lmhead", "stack"])
    ap.add_argument("--layers", type=int, default=32, help="stack layers")
    ap.add_argument("--stack-tokens", type=int, default=4096, help="stack tokens M")
    ap.add_argument("--stack-chunks", type=int, default=1,
                    help="token chunks pipelined over a compute and a communication stream (measured slower at tp1 "
                         "and tp2 on B200: the smaller GEMMs lose more than the overlapped allreduces gain)")
    ap.add_argument("--stack-mode", default="parity", choices=["parity", "speed"],
                    help="row-parallel partial sums in f32 (parity) or f16 (speed: half the allreduce bytes)")
    ap.add_argument("--stack-nccl-sms", type=int, default=8,
                    help="SMs left to NCCL while chunked GEMMs run (the GEMMs' SM budget is the rest)")
    ap.add_argument("--tile-table", default=None, help="tile table (tune.py output) installed before the run")
    ap.add_argument("--tokens", type=int, default=1, help="gemv tokens (1..32)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--launch-overlap", type=int, default=1, choices=[0, 1],
                    help="programmatic dependent launch of the GEMV (1, the library default) or plain stream order")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        line = run_reference(args, rank)
        if line is not None:
            print(json.dumps(line), flush=True)
        return
    dist = dist_init(args.gpus)
    import __graft_entry__ as ge
    lib_mod = importlib.import_module(ge.load_package().__name__ + "._lib")
    lib_mod.check(lib_mod.lib().yah_set_launch_overlap(args.launch_overlap))
    if args.tile_table:
        import __graft_entry__ as ge
        tune = ge.load_package().tune
        tune.apply(tune.load(args.tile_table))
    if args.workload == "stack":
        line = run_stack(args, dist, rank, local_rank)
    else:
        line = run_ours(args, dist, rank, local_rank)
    if rank == 0:
        if not args.no_cpu_baseline and int(os.environ.get("WORLD_SIZE", "1")) == 1:
            line["cpu_baseline"] = cpu_baseline(args)
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
