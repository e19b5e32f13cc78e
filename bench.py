#!/usr/bin/env python3
"""Benchmark of the quantised-linear hot path on B200 (one JSON line on rank 0).

Default line (--workload gemm): BASELINE config 2, the Q4_K prefill tile GEMM (M=2048 tokens, K=4096, N=14336, f16
out), TFLOP/s of the whole job. On N GPUs the weight rows are column-sharded (each rank holds N/p consecutive rows
of the GGUF tensor and computes them for all M tokens, no collective: the reference's OSTRIDE row-range form,
engine/gpu/loom/tools/gen_gemm_tile.py:246-250), so the N-GPU value is strong scaling of the same GEMM. Nested in
the same line:
  decode    BASELINE config 3 decode GEMV (Q4_K 4096 x 14336, M = 1 / 8 / 32 tokens): HBM GB/s and its fraction of
            the measured copy bandwidth, timed like the GEMM (N = 1 only).
  tp_stack  BASELINE config 4, the Llama-shaped Q4_K linear stack (32 layers, hidden 4096, QKV 6144, FF 14336,
            4096 tokens) tensor-parallel over the N GPUs on the BASELINE weight distribution with f32 partial sums:
            column-parallel QKV / gate / up, row-parallel o_proj / down, timed in the parity mode (one ncclAllReduce
            of the f32 partials through the library's own NCCL communicator, whose rank count is reported) and in the
            fused mode (the row-parallel GEMM writes its partials into the token-slice owners' memory over NVLink;
            reduce + RMSNorm + all-gather by the owner); the faster mode is the record's figure, both are listed,
            with the allreduces' time alone and the per-site GEMM rates at the shard shapes.
  lm_head   BASELINE config 5's decode lm head (Q6_K 128256 x 4096, M = 1 and 32), vocab-column sharded over the
            N GPUs (16032 rows per rank at N = 8, ragged last row tiles): whole-job GB/s, max over ranks.
  sustained the config-2 GEMM over >= 2000 back-to-back launches (about half a second) with the SM clocks of that
            window: the figure under the power cap, beside the short run's burst figure.
Other workloads (--workload): gemv (config 3, --tokens M), lmhead (config 5, Q6_K 128256 x 4096: GEMV for
--tokens <= 32, prefill GEMM above), stack (config 4 alone).

A step is one launch of the kernel over one batch. Inputs are resident in HBM when the timed region starts; steps
rotate through input copies whose total exceeds L2 (126 MB), so no step reads inputs another step left in L2.
Timing: W warm-up steps, then exactly K steps between a barrier + device synchronise on both sides, CUDA events on
the launching stream, max over ranks; single-kernel workloads replay the K steps as one CUDA graph. SM clocks and
throttle reasons are sampled through NVML (the device matched by UUID) every millisecond inside the timed region.
`e2e` is the same metric through the public C ABI with pinned host buffers: every step copies its activations
host->device and its output device->host inside the timed region, pipelined over three streams (the copy-in of
step i + 1 and the copy-out of step i - 1 overlap the GEMM of step i; double-buffered pinned and device buffers,
weights rotating as in the device-timed leg).

Multi-GPU (torchrun, one process per GPU): torch.distributed (gloo, CPU tensors) carries the barrier, the max over
ranks and rank 0's NCCL id; the stack's allreduces go through the library's communicator (NCCL_DEBUG=INFO with the
INIT subsystem is set unless the caller set NCCL_DEBUG, so NCCL's own log shows the communicator's nranks; the
JSON line is the last line of stdout: the process ends right after it, before NCCL's exit-time log).

--impl reference: the reference's CPU path for the same metric (its test-suite oracle: gguf-py
quants.dequantize -> f16 -> numpy matmul, engine/gpu/loom/tools/gemv_check.py:161-162) on the host cores, rank 0
only, with the BLAS thread pool pinned to every core this process may use (torchrun's OMP_NUM_THREADS=1 would
otherwise make it single-threaded).
"""
from __future__ import annotations

import argparse
import importlib
import json
import os
import subprocess
import sys
import threading
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


def cpu_cores():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def pin_blas_threads():
    """Let numpy's BLAS use every core this process may use (torchrun exports OMP_NUM_THREADS=1). Returns the
    thread count set."""
    n = cpu_cores()
    try:
        from threadpoolctl import threadpool_limits
        threadpool_limits(limits=n, user_api="blas")
    except ImportError:
        pass
    return n


# ------------------------------------------------------------------------------------------------ clocks
class Clocks:
    """SM clock and throttle reasons of one CUDA device, sampled through NVML every `period` seconds while a
    region runs (start() ... stop()). The NVML device is found by the CUDA device's UUID, so the sampler reads the
    GPU the process runs on whatever CUDA_VISIBLE_DEVICES says; without NVML it falls back to nvidia-smi."""

    REASONS = {"hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40, "sw_power_cap": 0x4,
               "hw_power_brake_slowdown": 0x80}

    def __init__(self, cuda_index, period=0.001):
        self.cuda_index, self.period = cuda_index, period
        self.handle = None
        self.samples = []
        self.thread = None
        self.stop_flag = threading.Event()
        try:
            import pynvml
            import torch
            pynvml.nvmlInit()
            uuid = "GPU-" + str(torch.cuda.get_device_properties(cuda_index).uuid)
            self.nvml = pynvml
            self.handle = pynvml.nvmlDeviceGetHandleByUUID(uuid.encode())
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(self.handle, pynvml.NVML_CLOCK_SM))
        except Exception:  # noqa: BLE001 - no NVML / torch.cuda: sampled by nvidia-smi instead
            self.handle = None
            self.max_mhz = 0.0

    def _poll(self):
        n = self.nvml
        while not self.stop_flag.is_set():
            try:
                sm = n.nvmlDeviceGetClockInfo(self.handle, n.NVML_CLOCK_SM)
                rs = n.nvmlDeviceGetCurrentClocksEventReasons(self.handle)
                self.samples.append((float(sm), int(rs)))
            except Exception:  # noqa: BLE001
                pass
            time.sleep(self.period)

    def start(self):
        self.samples = []
        self.stop_flag.clear()
        if self.handle is not None:
            self.thread = threading.Thread(target=self._poll, daemon=True)
            self.thread.start()
            t0 = time.perf_counter()
            while not self.samples and time.perf_counter() - t0 < 0.2:  # a first reading before the region
                time.sleep(self.period / 4)
        else:
            q = ("index,clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,clocks_event_reasons.sw_power_cap,"
                 "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown")
            try:
                self.thread = subprocess.Popen(["nvidia-smi", f"--query-gpu={q}", "--format=csv,noheader,nounits",
                                                "-i", str(self.cuda_index), "-lms", "20"], stdout=subprocess.PIPE,
                                               stderr=subprocess.DEVNULL, text=True)
            except OSError:
                self.thread = None

    def stop(self):
        if self.thread is None:
            return None
        if self.handle is not None:
            self.stop_flag.set()
            self.thread.join()
            sm = [s for s, _ in self.samples]
            mask = 0
            for _, r in self.samples:
                mask |= r
            reasons = sorted(k for k, b in self.REASONS.items() if mask & b)
            mx = self.max_mhz
        else:
            self.thread.terminate()
            out, _ = self.thread.communicate()
            sm, reasons, mx = [], set(), 0.0
            names = ["hw_slowdown", "sw_power_cap", "hw_thermal_slowdown", "sw_thermal_slowdown"]
            for line in out.strip().splitlines():
                f = [v.strip() for v in line.split(",")]
                try:
                    sm.append(float(f[1]))
                    mx = max(mx, float(f[2]))
                except (ValueError, IndexError):
                    continue
                for nm, v in zip(names, f[3:7]):
                    if v.lower() == "active":
                        reasons.add(nm)
            reasons = sorted(reasons)
        if not sm:
            return None
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": mx, "reasons": reasons, "samples": len(sm),
                "sm_mhz_min": float(min(sm)), "source": "nvml" if self.handle is not None else "nvidia-smi"}


# ------------------------------------------------------------------------------------------------ ranks
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


def world_size():
    return int(os.environ.get("WORLD_SIZE", "1"))


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


def shard_rows(N, world, rank, align=256):
    """[lo, hi) of this rank's column shard: consecutive weight rows, whole 2-SM tiles where N allows."""
    a = align if N % (align * world) == 0 else (128 if N % (128 * world) == 0 else 1)
    units = N // a
    return rank * units // world * a, (rank + 1) * units // world * a


class Kernel:
    """One single-kernel workload on this rank's device: its resident input copies (rotating, > L2), the launch of
    one step through the C ABI, a CUDA-graph timer and the pipelined end-to-end leg."""

    def __init__(self, pkg, dev, fmt, N, K, M, out, gemv, seed_w=0, seed_x=1, rows=None):
        """N weight rows x K (a column shard: rows = (lo, hi) of an N-row tensor generated whole, so the shards of
        the ranks tile the same tensor), M tokens."""
        F = pkg.formats
        w = F.synth_weights(fmt, N, K, seed=seed_w)
        if rows is not None:
            w = w[rows[0]:rows[1]]
            N = rows[1] - rows[0]
        self.pkg, self.dev, self.fmt, self.N, self.K, self.M, self.gemv = pkg, dev, fmt, N, K, M, gemv
        self.fn = pkg.ops.qgemv_ptr if gemv else pkg.ops.qgemm_ptr
        self.w = np.ascontiguousarray(w)
        self.x = F.synth_activations(M, K, seed=seed_x)
        self.ydt = 1 if out == "f16" else 0
        self.wbytes, self.xbytes = self.w.nbytes, self.x.nbytes
        self.ybytes = M * N * (2 if self.ydt else 4)
        per_copy = self.wbytes + self.xbytes
        self.copies = max(2, int(np.ceil(2.2 * L2_BYTES / per_copy)))
        self.l2_note = f"rotating {self.copies} input copies ({self.copies * per_copy / 2**20:.0f} MiB > L2)"
        self.wd = [dev.upload(self.w) for _ in range(self.copies)]
        self.xd = [dev.upload(self.x) for _ in range(self.copies)]
        self.yd = [dev.empty(self.ybytes) for _ in range(2)]
        self.stream = pkg.Stream()

    def step(self, i, x_ptr=None, y_ptr=None, stream=None, j=None):
        j = i % self.copies if j is None else j
        self.fn(self.wd[j].ptr, self.fmt, self.N, self.K, self.w.shape[1], 0,
                self.xd[j].ptr if x_ptr is None else x_ptr, self.M, self.K,
                self.yd[i & 1].ptr if y_ptr is None else y_ptr, self.ydt, self.N,
                stream=self.stream.handle if stream is None else stream)

    def graph(self, n, start=0):
        g = self.pkg.Graph(self.stream)
        g.begin()
        for i in range(start, start + n):
            self.step(i)
        g.end()
        return g

    def time_graph(self, g, dist=None, clocks=None, replays=1):
        """ms of `replays` launches of graph g between barrier + synchronise on both sides (max over ranks); the
        local ms too."""
        s = self.stream.handle
        e0, e1 = self.pkg.Event(), self.pkg.Event()
        barrier(dist)
        self.dev.synchronize()
        if clocks:
            clocks.start()
        e0.record(s)
        for _ in range(replays):
            g.launch()
        e1.record(s)
        e1.synchronize()
        self.dev.synchronize()
        clk = clocks.stop() if clocks else None
        barrier(dist)
        ms_local = e0.elapsed_ms(e1)
        return max_over_ranks(dist, ms_local), ms_local, clk

    def e2e(self, steps, warmup, dist=None):
        """ms of `steps` end-to-end steps through the C ABI: pinned host activations -> device, the kernel, output
        -> pinned host, on three streams (copy-in, compute, copy-out) with double buffers, max over ranks."""
        pkg, lib = self.pkg, self.pkg.lib()
        xh = [pkg.PinnedBuffer(self.xbytes) for _ in range(2)]
        yh = [pkg.PinnedBuffer(self.ybytes) for _ in range(2)]
        for b in xh:
            b.array(np.float16, self.x.shape)[...] = self.x
        xdev = [self.dev.empty(self.xbytes) for _ in range(2)]
        ydev = [self.dev.empty(self.ybytes) for _ in range(2)]
        s_in, s_k, s_out = pkg.Stream(), self.stream, pkg.Stream()
        ev = {k: [pkg.Event() for _ in range(2)] for k in ("x_ready", "x_free", "y_ready", "y_free")}
        used = set()

        def one(i):
            b = i & 1
            if ("x_free", b) in used:
                s_in.wait(ev["x_free"][b])
            pkg._lib.check(lib.yah_memcpy_h2d(xdev[b].ptr, xh[b].ptr, self.xbytes, s_in.handle))
            ev["x_ready"][b].record(s_in.handle)
            s_k.wait(ev["x_ready"][b])
            if ("y_free", b) in used:
                s_k.wait(ev["y_free"][b])
            self.step(i, x_ptr=xdev[b].ptr, y_ptr=ydev[b].ptr, stream=s_k.handle, j=i % self.copies)
            ev["x_free"][b].record(s_k.handle)
            ev["y_ready"][b].record(s_k.handle)
            s_out.wait(ev["y_ready"][b])
            pkg._lib.check(lib.yah_memcpy_d2h(yh[b].ptr, ydev[b].ptr, self.ybytes, s_out.handle))
            ev["y_free"][b].record(s_out.handle)
            used.update({("x_free", b), ("y_free", b)})

        for i in range(warmup):
            one(i)
        self.dev.synchronize()
        barrier(dist)
        e0, e1 = pkg.Event(), pkg.Event()
        e0.record(s_in.handle)
        for i in range(steps):
            one(warmup + i)
        e1.record(s_out.handle)
        e1.synchronize()
        self.dev.synchronize()
        ms = max_over_ranks(dist, e0.elapsed_ms(e1))
        for b in xh + yh + xdev + ydev:
            b.close()
        s_in.close()
        s_out.close()
        return ms

    def close(self):
        for b in self.wd + self.xd + self.yd:
            b.close()
        self.stream.close()


def run_gemm_line(args, dist, rank, local_rank):
    """The default line: config 2, column-sharded over the ranks (strong scaling of one GEMM)."""
    import __graft_entry__ as ge
    pkg = ge.load_package()
    dev = pkg.Device(local_rank)
    world = world_size()
    wl = workload_of(args)
    lo, hi = shard_rows(wl["N"], world, rank)
    # every rank generates the full tensor's seed stream and keeps its rows, so the shards tile the same tensor
    k = Kernel(pkg, dev, wl["fmt"], wl["N"], wl["K"], wl["M"], wl["out"], False, seed_w=0, seed_x=1, rows=(lo, hi))
    for i in range(args.warmup):
        k.step(i)
    k.stream.synchronize()
    g = k.graph(args.steps)
    g.launch()  # one untimed replay
    k.stream.synchronize()
    clocks = Clocks(local_rank)
    ms, ms_local, clk = k.time_graph(g, dist, clocks)
    g.close()
    status = dev.status_word()
    if status:
        raise RuntimeError(f"kernel status word {status}")
    flops_total = 2.0 * wl["M"] * wl["N"] * wl["K"]
    flops_local = 2.0 * wl["M"] * (hi - lo) * wl["K"]
    per_step_ms = ms / args.steps
    value = flops_total / (per_step_ms * 1e-3) / 1e12
    pk = peaks()
    achieved = flops_local / (ms_local / args.steps * 1e-3) / 1e12
    roof = {"bound": "tensor", "achieved": round(achieved, 1), "peak": pk["tflops"], "unit": "TFLOP/s",
            "frac": round(achieved / pk["tflops"], 4), "traffic": None, "peak_src": pk["src"] + " (burst)",
            "frac_of_sustained": round(achieved / pk["tflops_sustained"], 4),
            "algorithmic_flops_per_launch": flops_local}
    if world == 1:
        t = load_traffic(wl["name"])
        if t is not None:
            roof["traffic"] = t
    ms_e2e = k.e2e(args.steps, max(3, args.warmup), dist)
    line = {
        "metric": wl["metric"], "value": round(value, 2), "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(per_step_ms, 5), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": f"f16 x GGUF-{wl['fmt_name']} -> f32 acc",
        "data": "synthetic",
        "config": {"workload": wl["name"], "M_tokens": wl["M"], "K": wl["K"], "N": wl["N"],
                   "weight_format": wl["fmt_name"], "out_dtype": wl["out"],
                   "parallelism": f"column-sharded x{world} ({hi - lo} weight rows per GPU, no collective)",
                   "launch_overlap": bool(args.launch_overlap), "l2": k.l2_note},
        "e2e": {"value": round(flops_total / (ms_e2e / args.steps * 1e-3) / 1e12, 2), "unit": "TFLOP/s",
                "h2d_bytes_per_step": k.xbytes, "d2h_bytes_per_step": k.ybytes,
                "pipeline": "copy-in / GEMM / copy-out on three streams, double-buffered, weights rotating"},
        "gpu_launches": args.steps,
        "roofline": roof,
        "clocks": clk,
    }
    if args.sustained:
        launches = 200
        gs = k.graph(launches)
        gs.launch()
        k.stream.synchronize()
        reps = 10
        ms_s, ms_s_local, clk_s = k.time_graph(gs, dist, Clocks(local_rank), replays=reps)
        gs.close()
        ach = flops_local / (ms_s_local / (launches * reps) * 1e-3) / 1e12
        line["sustained"] = {"launches": launches * reps, "ms": round(ms_s, 3),
                             "tflops_total": round(flops_total / (ms_s / (launches * reps) * 1e-3) / 1e12, 2),
                             "tflops_per_gpu": round(ach, 1), "frac_of_burst_peak": round(ach / pk["tflops"], 4),
                             "frac_of_sustained_peak": round(ach / pk["tflops_sustained"], 4), "clocks": clk_s}
        line["gpu_launches_sustained"] = launches * reps
    k.close()
    if dev.status_word():
        raise RuntimeError("kernel status word set")
    return line


def run_decode_record(args, local_rank, launches=200):
    """Config 3 decode GEMV at M = 1 / 8 / 32 (GB/s of weight + activation + output bytes per launch)."""
    import __graft_entry__ as ge
    pkg = ge.load_package()
    dev = pkg.Device(local_rank)
    pk = peaks()
    out = {"workload": "q4k_decode_gemv (config 3: Q4_K 4096 x 14336)", "launches_per_M": launches,
           "timing": "CUDA graph of the launches, rotating input copies > L2, CUDA events", "by_M": {}}
    for M in args.decode_tokens:
        k = Kernel(pkg, dev, 12, 4096, 14336, M, "f32", True, seed_w=0, seed_x=1)
        for i in range(3):
            k.step(i)
        k.stream.synchronize()
        g = k.graph(launches)
        g.launch()
        k.stream.synchronize()
        ms, _, clk = k.time_graph(g, None, Clocks(local_rank))
        g.close()
        if dev.status_word():
            raise RuntimeError("kernel status word set")
        alg = k.wbytes + k.xbytes + k.ybytes
        us = ms / launches * 1e3
        import ctypes
        desc = ctypes.create_string_buffer(512)
        pkg._lib.check(pkg.lib().yah_qgemv_describe(12, 4096, 14336, M, desc, 512))
        gbs = alg / (us * 1e-6) / 1e9
        out["by_M"][str(M)] = {"us_per_launch": round(us, 3), "GB/s": round(gbs, 1),
                               "GB/s_weights_only": round(k.wbytes / (us * 1e-6) / 1e9, 1),
                               "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": pk["hbm_gbs"],
                                            "unit": "GB/s", "frac": round(gbs / pk["hbm_gbs"], 4),
                                            "peak_src": pk["src"], "algorithmic_bytes_per_launch": alg},
                               "clocks": clk, "kernel": desc.value.decode()}
        k.close()
    return out


def run_lmhead_record(args, dist, rank, local_rank, launches=50):
    """Config 5's decode lm head (Q6_K 128256 x 4096, f32 logits) vocab-column sharded over the N GPUs: rank r
    computes rows [r N / p, (r + 1) N / p) for all tokens, no collective (16032 rows at p = 8: ragged last row
    tiles). GB/s of the whole job (the head's bytes once) over the max over ranks of the per-launch time."""
    import __graft_entry__ as ge
    pkg = ge.load_package()
    dev = pkg.Device(local_rank)
    pk = peaks()
    world = world_size()
    N, K = 128256, 4096
    lo, hi = shard_rows(N, world, rank)
    out = {"workload": "q6k_lm_head_decode_gemv (config 5: Q6_K 128256 x 4096)", "parallelism":
           f"vocab column shards x{world}", "rows_per_rank": hi - lo, "launches_per_M": launches,
           "scaling": "strong", "by_M": {}}
    for M in args.lmhead_tokens:
        k = Kernel(pkg, dev, 14, N, K, M, "f32", True, seed_w=0, seed_x=1, rows=(lo, hi))
        for i in range(3):
            k.step(i)
        k.stream.synchronize()
        g = k.graph(launches)
        g.launch()
        k.stream.synchronize()
        ms, ms_local, clk = k.time_graph(g, dist, Clocks(local_rank))
        g.close()
        if dev.status_word():
            raise RuntimeError("kernel status word set")
        job = pkg.formats.row_bytes(14, K) * N + M * K * 2 + M * N * 4
        shard = k.wbytes + k.xbytes + k.ybytes
        us, us_local = ms / launches * 1e3, ms_local / launches * 1e3
        rank_gbs = shard / (us_local * 1e-6) / 1e9
        out["by_M"][str(M)] = {"us_per_launch": round(us, 3), "GB/s": round(job / (us * 1e-6) / 1e9, 1),
                               "roofline_rank0": {"bound": "hbm", "achieved": round(rank_gbs, 1),
                                                  "peak": pk["hbm_gbs"], "unit": "GB/s",
                                                  "frac": round(rank_gbs / pk["hbm_gbs"], 4), "peak_src": pk["src"],
                                                  "algorithmic_bytes_per_launch": shard},
                               "clocks": clk}
        k.close()
    return out


def stack_weights(F, shape, world, rank, scale=None):
    """Four distinct weight sets of this rank's shards (cycled over the layers: > L2 per GPU at tp1)."""
    p, H = world, shape.hidden
    sets = []
    sc = scale or (lambda w: w)
    for k in range(min(4, shape.layers)):
        s0 = 5000 + 64 * k + 8 * rank
        sets.append({"qkv": sc(F.synth_weights(shape.fmt, shape.qkv // p, H, seed=s0)),
                     "o": sc(F.synth_weights(shape.fmt, H, shape.n_q * shape.head_dim // p, seed=s0 + 1)),
                     "gate": sc(F.synth_weights(shape.fmt, shape.ff // p, H, seed=s0 + 2)),
                     "up": sc(F.synth_weights(shape.fmt, shape.ff // p, H, seed=s0 + 3)),
                     "down": sc(F.synth_weights(shape.fmt, H, shape.ff // p, seed=s0 + 4))})
    return sets


def make_comm(pkg, dist, world, rank):
    def exchange(uid):
        obj = [uid]
        dist.broadcast_object_list(obj, src=0)
        return obj[0]
    return pkg.tp.Comm(world, rank, exchange if world > 1 else None)


def run_stack_record(args, dist, rank, local_rank, steps=3, warmup=2):
    """Config 4 at tp-N on the BASELINE weights with f32 partial sums: the forward's time in the parity mode
    (ncclAllReduce after each row-parallel GEMM) and in the fused mode (the GEMM's epilogue scatters its partials
    into the token-slice owners' memory over NVLink; reduce + RMSNorm + all-gather by the owner), the faster one as
    the record's figure, the allreduces' time alone, and each GEMM site's rate at this degree's shard shapes."""
    import __graft_entry__ as ge
    pkg = ge.load_package()
    F, tp, L = pkg.formats, pkg.tp, pkg.lib()
    dev = pkg.Device(local_rank)
    world = world_size()
    shape = tp.StackShape(layers=args.layers)
    M, H = args.stack_tokens, shape.hidden
    comm = make_comm(pkg, dist, world, rank)
    import ctypes
    r_, n_ = ctypes.c_int(), ctypes.c_int()
    pkg._lib.check(L.yah_tp_rank(comm.handle, ctypes.byref(r_), ctypes.byref(n_)))
    sets = stack_weights(F, shape, world, rank)
    h0 = np.random.default_rng(7).standard_normal((M, H)).astype(np.float32)
    h0d, h = dev.upload(h0), dev.empty(M * H * 4)
    stream = pkg.Stream()
    s = stream.handle
    e0, e1 = pkg.Event(), pkg.Event()
    modes = ["parity", "fused"] if args.stack_mode == "auto" else [args.stack_mode]
    timed = {}
    for mode in modes:  # the same steps on every rank, in the same order
        stack = tp.LlamaStack(dev, comm, shape, [sets[i % len(sets)] for i in range(shape.layers)], M, mode=mode)

        def fwd():
            L.yah_memcpy_d2d(h.ptr, h0d.ptr, M * H * 4, s)  # every step starts from the same residual stream
            stack.forward(h, s)

        for _ in range(warmup):
            fwd()
        stream.synchronize()
        barrier(dist)
        dev.synchronize()
        clocks = Clocks(local_rank, period=0.005)
        clocks.start()
        e0.record(s)
        for _ in range(steps):
            fwd()
        e1.record(s)
        e1.synchronize()
        clk_m = clocks.stop()
        barrier(dist)
        ms_m = max_over_ranks(dist, e0.elapsed_ms(e1)) / steps
        if dev.status_word():
            raise RuntimeError(f"kernel status word set ({mode} mode)")
        out = h.download(np.float32, (M, H))
        timed[mode] = {"ms": ms_m, "finite": bool(np.isfinite(out).all()), "clocks": clk_m,
                       "launches": stack.launches_per_forward, "out": out}
        stack.close()
    best = min(timed, key=lambda m: timed[m]["ms"])
    ms, finite, clk = timed[best]["ms"], timed[best]["finite"], timed[best]["clocks"]
    # both modes compute the same sums in a different order: their outputs agree to f32 rounding
    agree = None
    if len(timed) == 2:
        a, b = timed["parity"]["out"].astype(np.float64), timed["fused"]["out"].astype(np.float64)
        agree = float(np.linalg.norm(a - b) / max(np.linalg.norm(a), 1e-30))
    stack = tp.LlamaStack(dev, comm, shape, [sets[0]], M, mode="parity")  # buffers and shards for the site timings
    # the allreduces alone: the forward's 2 x layers ncclAllReduce of the f32 [M][hidden] residual stream
    nred = 2 * shape.layers
    for _ in range(2):
        comm.allreduce_f32(h.ptr, M * H, s)
    stream.synchronize()
    barrier(dist)
    dev.synchronize()
    e0.record(s)
    for _ in range(nred):
        comm.allreduce_f32(h.ptr, M * H, s)
    e1.record(s)
    e1.synchronize()
    barrier(dist)
    ms_red = max_over_ranks(dist, e0.elapsed_ms(e1))
    # the GEMM sites at this degree's shard shapes (one weight set, 5 launches each, local time)
    w = stack.w[0]
    sites = {}
    fmt = shape.fmt
    q_r, qkv_r, ff_r = stack.q_r, stack.qkv_r, stack.ff_r
    site_calls = {
        "qkv": (qkv_r, H, lambda: L.yah_qgemm(w["qkv"].ptr, fmt, qkv_r, H, stack.row_bytes["qkv"], 0, stack.xn.ptr, M,
                                               H, stack.qkv.ptr, 1, qkv_r, 0, None, 0, s)),
        "o_proj": (H, q_r, lambda: L.yah_qgemm(w["o"].ptr, fmt, H, q_r, stack.row_bytes["o"], 0, stack.qkv.ptr, M,
                                                qkv_r, h.ptr, 0, H, 1 if rank == 0 else 0,
                                                h.ptr if rank == 0 else None, H if rank == 0 else 0, s)),
        "gate": (ff_r, H, lambda: L.yah_qgemm(w["gate"].ptr, fmt, ff_r, H, stack.row_bytes["gate"], 0, stack.xn.ptr,
                                               M, H, stack.g.ptr, 0, ff_r, 0, None, 0, s)),
        "up_swiglu": (ff_r, H, lambda: L.yah_qgemm(w["up"].ptr, fmt, ff_r, H, stack.row_bytes["up"], 0, stack.xn.ptr,
                                                    M, H, stack.act.ptr, 1, ff_r, 2, stack.g.ptr, ff_r, s)),
        "down": (H, ff_r, lambda: L.yah_qgemm(w["down"].ptr, fmt, H, ff_r, stack.row_bytes["down"], 0, stack.act.ptr,
                                               M, ff_r, h.ptr, 0, H, 1 if rank == 0 else 0,
                                               h.ptr if rank == 0 else None, H if rank == 0 else 0, s)),
    }
    for name, (n, kk, call) in site_calls.items():
        for _ in range(2):
            pkg._lib.check(call())
        stream.synchronize()
        e0.record(s)
        for _ in range(5):
            pkg._lib.check(call())
        e1.record(s)
        e1.synchronize()
        us = e0.elapsed_ms(e1) / 5 * 1e3
        sites[name] = {"N": n, "K": kk, "us": round(us, 1), "tflops": round(2.0 * M * n * kk / (us * 1e-6) / 1e12, 1)}
    if dev.status_word():
        raise RuntimeError("kernel status word set")
    flops = shape.flops(M)
    pk = peaks()
    tfl = flops / (ms * 1e-3) / 1e12
    limiting = min(sites, key=lambda k: sites[k]["tflops"])
    rec = {
        "workload": "q4k_layer_stack_tp (config 4: 32 layers, hidden 4096, QKV 6144, FF 14336, linears only)",
        "mode": (f"{best} (f32 residual stream and f32 partial sums; BASELINE Q4_K weight distribution)"),
        "ms_per_forward_by_mode": {m: round(v["ms"], 3) for m, v in timed.items()},
        "modes_rel_fro_difference": agree,
        "M_tokens": M, "layers": shape.layers, "parallelism": f"tp{world}",
        "nccl_comm_nranks": n_.value, "nccl_comm_rank": r_.value,
        "steps": steps, "warmup": warmup, "ms_per_forward": round(ms, 3), "tflops": round(tfl, 1),
        "tflops_per_gpu": round(tfl / world, 1),
        "frac_of_sustained_peak_per_gpu": round(tfl / world / pk["tflops_sustained"], 4),
        "allreduce": {"calls_per_forward": nred, "bytes_each": M * H * 4, "ms_alone": round(ms_red, 3),
                      "share_of_forward": round(ms_red / ms, 4) if world > 1 else 0.0,
                      "busbw_GBs": (round(2 * (world - 1) / world * M * H * 4 * nred / (ms_red * 1e-3) / 1e9, 1)
                                    if world > 1 else None)},
        "sites": sites, "limiting_kernel": f"{limiting} shard GEMM ({sites[limiting]['N']} x {sites[limiting]['K']})",
        "limiting_collective": ((f"ncclAllReduce(sum) f32 [{M}][{H}] x {nred} per forward" if best == "parity" else
                                 f"reduce-scatter of f32 [{M}][{H}] written by the row-parallel GEMMs over NVLink + "
                                 f"all-gather of the f16 RMSNorm output, x {nred} per forward")
                                if world > 1 else None),
        "finite": finite, "gpu_launches_per_forward": timed[best]["launches"], "clocks": clk,
        "l2": "4 distinct weight sets cycled over the layers",
    }
    stack.close()
    comm.close()
    for b in (h0d, h):
        b.close()
    stream.close()
    return rec


def run_ours(args, dist, rank, local_rank):
    """--workload gemv: one kernel, replicas on every rank (weak scaling). --workload lmhead: on N GPUs the
    128256-row head is vocab-column sharded (rank r computes rows [r N / p, (r + 1) N / p) of the one tensor for all
    tokens, no collective; 16032 rows at p = 8, so the last row tile of each shard is ragged), strong scaling."""
    import __graft_entry__ as ge
    pkg = ge.load_package()
    dev = pkg.Device(local_rank)
    wl = workload_of(args)
    world = world_size()
    shard = args.workload == "lmhead" and world > 1
    rows = shard_rows(wl["N"], world, rank) if shard else None
    k = Kernel(pkg, dev, wl["fmt"], wl["N"], wl["K"], wl["M"], wl["out"], wl["gemv"], seed_w=0,
               seed_x=1 + (0 if shard else rank), rows=rows)
    for i in range(args.warmup):
        k.step(i)
    k.stream.synchronize()
    g = k.graph(args.steps)
    g.launch()
    k.stream.synchronize()
    ms, ms_local, clk = k.time_graph(g, dist, Clocks(local_rank))
    g.close()
    if dev.status_word():
        raise RuntimeError("kernel status word set")
    ms_e2e = k.e2e(args.steps, max(3, args.warmup), dist)
    pk = peaks()
    per_step_ms = ms / args.steps
    M, N, K = wl["M"], wl["N"], wl["K"]
    copies = 1 if shard else world  # the whole job: one head split over the ranks, or one head per rank
    if wl["gemv"]:
        alg = k.wbytes + k.xbytes + k.ybytes
        job = (pkg.formats.row_bytes(wl["fmt"], K) * N + M * K * 2 + M * N * 4) if shard else alg
        value = copies * job / (per_step_ms * 1e-3) / 1e9
        unit = "GB/s"
        achieved = alg / (ms_local / args.steps * 1e-3) / 1e9
        roof = {"bound": "hbm", "achieved": round(achieved, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
                "frac": round(achieved / pk["hbm_gbs"], 4), "traffic": load_traffic(wl["name"]),
                "peak_src": pk["src"], "algorithmic_bytes_per_launch": alg}
        e2e_val = copies * job / (ms_e2e / args.steps * 1e-3) / 1e9
    else:
        flops = 2.0 * M * k.N * K
        job = 2.0 * M * N * K if shard else flops
        value = copies * job / (per_step_ms * 1e-3) / 1e12
        unit = "TFLOP/s"
        achieved = flops / (ms_local / args.steps * 1e-3) / 1e12
        roof = {"bound": "tensor", "achieved": round(achieved, 1), "peak": pk["tflops"], "unit": "TFLOP/s",
                "frac": round(achieved / pk["tflops"], 4), "traffic": load_traffic(wl["name"]),
                "peak_src": pk["src"], "frac_of_sustained": round(achieved / pk["tflops_sustained"], 4),
                "algorithmic_flops_per_launch": flops}
        e2e_val = copies * job / (ms_e2e / args.steps * 1e-3) / 1e12
    line = {
        "metric": wl["metric"], "value": round(value, 2), "unit": unit, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(per_step_ms, 5), "higher_is_better": True,
        "scaling": "strong" if shard else "weak",
        "vs_baseline": None, "dtype": f"f16 x GGUF-{wl['fmt_name']} -> f32 acc", "data": "synthetic",
        "config": {"workload": wl["name"], "M_tokens": M, "K": K, "N": N, "weight_format": wl["fmt_name"],
                   "out_dtype": wl["out"],
                   "parallelism": (f"vocab column shards x{world} ({k.N} rows on rank {rank})" if shard
                                   else f"replicas x{world}"),
                   "launch_overlap": bool(args.launch_overlap), "l2": k.l2_note},
        "e2e": {"value": round(e2e_val, 2), "unit": unit, "h2d_bytes_per_step": k.xbytes,
                "d2h_bytes_per_step": k.ybytes},
        "gpu_launches": args.steps, "roofline": roof, "clocks": clk,
    }
    k.close()
    return line


def run_stack_line(args, dist, rank, local_rank):
    """--workload stack: config 4 as the line itself (tp over the N GPUs, strong scaling)."""
    rec = run_stack_record(args, dist, rank, local_rank, steps=args.steps, warmup=args.warmup)
    pk = peaks()
    world = world_size()
    return {
        "metric": "Q4_K layer-stack prefill TFLOP/s (tensor-parallel)", "value": rec["tflops"], "unit": "TFLOP/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": rec["ms_per_forward"],
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "f16 x GGUF-Q4_K -> f32 acc, f32 residual stream", "data": "synthetic",
        "config": {"workload": "q4k_layer_stack_tp", "layers": rec["layers"], "hidden": 4096, "qkv": 6144,
                   "ff": 14336, "M_tokens": rec["M_tokens"], "parallelism": f"tp{world}",
                   "partial_sums": "f32 (" + rec["mode"].split(" ")[0] + " mode)", "l2": rec["l2"]},
        "e2e": None, "gpu_launches": args.steps * rec["gpu_launches_per_forward"],
        "roofline": {"bound": "tensor", "achieved": rec["tflops_per_gpu"], "peak": pk["tflops_sustained"],
                     "unit": "TFLOP/s", "frac": rec["frac_of_sustained_peak_per_gpu"], "traffic": None,
                     "peak_src": pk["src"] + " (sustained)", "per_gpu": True},
        "clocks": rec["clocks"], "tp_stack": rec,
    }


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


def cpu_sample_text(args, jobs, use_gguf, runs_note, threads):
    M = jobs[0][2].shape[0]
    mats = ", ".join(f"{w.shape[0]} of {n} rows x K={k}" for _, w, _, k, n in jobs)
    what = "one layer of the stack: " if args.workload == "stack" else ""
    return (f"{'gguf-py dequantize' if use_gguf else 'oracle C dequant'} + numpy f32 matmul, {what}{mats}, "
            f"{M} tokens; {runs_note}; BLAS threads {threads} (threadpoolctl)")


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
    threads = pin_blas_threads()
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
    return {"value": round(val, 5), "unit": unit, "cores": threads, "kind": kind,
            "sample": cpu_sample_text(args, jobs, use_gguf, f"{n} runs, {per * 1e3:.1f} ms each", threads),
            **cpu_phases_ms(n)}


def run_reference(args, rank, budget_s=150.0):
    """The reference's CPU path on the same metric and config, rank 0 only. Each step is one bounded sample; when
    the first warm-up step shows that K steps would take more than `budget_s`, every weight's sampled rows shrink
    by the same factor so that the run still ends within a few minutes."""
    if rank != 0:
        return None
    threads = pin_blas_threads()
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
    sample = cpu_sample_text(args, jobs, use_gguf, "per step", threads)
    world = world_size()
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
        scaling = "strong" if args.workload == "gemm" else "weak"
    return {"impl": "reference", "metric": metric, "value": round(val, 5), "unit": unit,
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(per * 1e3, 3), "higher_is_better": True, "scaling": scaling, "vs_baseline": None,
            "dtype": "f16 weights (dequantised) x f16 -> f32", "data": "synthetic", "config": config,
            "cpu_baseline": {"value": round(val, 5), "unit": unit, "cores": threads, "kind": kind,
                             "sample": sample, **cpu_phases_ms(args.steps)},
            "e2e": {"value": round(val, 5), "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="gemm", choices=["gemm", "gemv", "lmhead", "stack"])
    ap.add_argument("--layers", type=int, default=32, help="stack layers")
    ap.add_argument("--stack-tokens", type=int, default=4096, help="stack tokens M")
    ap.add_argument("--stack-mode", default="auto", choices=["auto", "parity", "fused"],
                    help="row-parallel reduction of the stack: ncclAllReduce (parity), the GEMM-written reduce-scatter "
                         "over peer memory (fused), or both timed and the faster reported (auto)")
    ap.add_argument("--no-stack", dest="stack", action="store_false",
                    help="leave the nested config-4 tp_stack record out of the default line")
    ap.add_argument("--no-lmhead", dest="lmhead", action="store_false",
                    help="skip the nested config-5 vocab-sharded lm-head record")
    ap.add_argument("--lmhead-tokens", type=int, nargs="+", default=[1, 32])
    ap.add_argument("--no-decode", dest="decode", action="store_false",
                    help="leave the nested config-3 decode record out of the default line")
    ap.add_argument("--no-sustained", dest="sustained", action="store_false",
                    help="leave the >= 2000-launch sustained figure out of the default line")
    ap.add_argument("--decode-tokens", type=int, nargs="+", default=[1, 8, 32])
    ap.add_argument("--tile-table", default=None, help="tile table (tune.py output) installed before the run")
    ap.add_argument("--tokens", type=int, default=1, help="gemv / lmhead tokens")
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
    # NCCL's own log of the communicator (rank, nRanks) is wanted in the output: raise NCCL_DEBUG to INFO (an
    # environment default of VERSION or WARN would hide it) and keep it to the INIT subsystem.
    if os.environ.get("NCCL_DEBUG", "").upper() not in ("INFO", "TRACE"):
        os.environ["NCCL_DEBUG"] = "INFO"
    os.environ.setdefault("NCCL_DEBUG_SUBSYS", "INIT")
    dist = dist_init(args.gpus)
    import __graft_entry__ as ge
    lib_mod = importlib.import_module(ge.load_package().__name__ + "._lib")
    lib_mod.check(lib_mod.lib().yah_set_launch_overlap(args.launch_overlap))
    if args.tile_table:
        tune = ge.load_package().tune
        tune.apply(tune.load(args.tile_table))
    world = world_size()
    if args.workload == "stack":
        line = run_stack_line(args, dist, rank, local_rank)
    elif args.workload == "gemm":
        line = run_gemm_line(args, dist, rank, local_rank)
        if args.decode and world == 1:
            line["decode"] = run_decode_record(args, local_rank)
        if args.lmhead:
            line["lm_head"] = run_lmhead_record(args, dist, rank, local_rank)
        if args.stack:
            line["tp_stack"] = run_stack_record(args, dist, rank, local_rank)
    else:
        line = run_ours(args, dist, rank, local_rank)
    if rank == 0:
        if not args.no_cpu_baseline and world == 1:
            line["cpu_baseline"] = cpu_baseline(args)
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    # End the process here: NCCL's teardown at interpreter exit logs (under NCCL_DEBUG=INFO) after the JSON line,
    # which must stay the last line of stdout. Every communicator, graph and buffer is released above.
    sys.stdout.flush()
    sys.stderr.flush()
    os._exit(0)


if __name__ == "__main__":
    main()
