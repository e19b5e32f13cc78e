"""Tile-configuration search for the tile GEMM on this GPU, and the table that yah_qgemm's automatic choice reads.

The B200 counterpart of the reference's tuner (engine/tune/tune.py): for every GEMM a model runs (its "sites") and
every token bucket, measure each tile the library instantiates (2-SM pairs of width 256 / 160 / 128 tokens, single
CTAs of 192 / 128 / 64), first briefly, then the best few again with more repetitions (successive halving), and
keep the fastest. Every candidate's output must hash the same as the default tile's (the reference's rule,
tune.py:12): tiles only move work between CTAs, the accumulation chunks stay the same, so results are identical.
Weights rotate through copies larger than L2, so every launch reads them from DRAM, as a layer stack does.

The table (JSON) lists the best tile per (site, bucket); `apply` installs it with yah_tile_rules_set, after which
every yah_qgemm (the tensor-parallel layer included) uses it.

    python yet-another-halo-engine_b200/tune.py --out tiles.json [--parts P] [--buckets 256,2048,4096]
"""
from __future__ import annotations

if __name__ == "__main__" and not __package__:  # run as a script: import the package, then its main
    import os
    import sys
    sys.path.insert(0, os.path.abspath(os.path.join(os.path.dirname(os.path.abspath(__file__)), "..")))
    import __graft_entry__
    __graft_entry__.load_package().tune.main()
    raise SystemExit(0)

import hashlib
import json
import time
from dataclasses import asdict, dataclass

import numpy as np

from . import formats as F
from ._lib import EPI_RESID, EPI_STORE, EPI_SWIGLU, F16, F32, TileRule, check, lib
from .device import Device, Event, Stream

TILES = [(1, 256), (1, 160), (1, 128), (0, 192), (0, 128), (0, 64)]  # (cta_pair, bn)
BUCKETS = (256, 2048, 4096)
L2_BYTES = 126 * 2 ** 20


@dataclass(frozen=True)
class Site:
    """One GEMM of a model: N x K weights of `fmt`, epilogue, output dtype."""
    name: str
    fmt: int
    N: int
    K: int
    epilogue: int = EPI_STORE
    out: int = F16


def stack_sites(shape, parts: int = 1) -> list:
    """The five GEMMs of the tensor-parallel layer stack (yet-another-halo-engine_b200/tp.py) at degree `parts`."""
    H, q = shape.hidden, shape.n_q * shape.head_dim
    return [Site("qkv", shape.fmt, shape.qkv // parts, H, EPI_STORE, F16),
            Site("o_proj", shape.fmt, H, q // parts, EPI_RESID, F32),
            Site("gate", shape.fmt, shape.ff // parts, H, EPI_STORE, F32),
            Site("up", shape.fmt, shape.ff // parts, H, EPI_SWIGLU, F16),
            Site("down", shape.fmt, H, shape.ff // parts, EPI_RESID, F32)]


class _Bench:
    """Device buffers of one (site, M): rotating weight copies, activations, aux operand, output."""

    def __init__(self, dev: Device, site: Site, M: int, seed: int = 90):
        self.dev, self.site, self.M = dev, site, M
        w = F.synth_weights(site.fmt, site.N, site.K, seed=seed)
        self.row = w.shape[1]
        copies = max(2, int(np.ceil(2.2 * L2_BYTES / w.nbytes)))
        self.w = [dev.upload(w) for _ in range(copies)]
        self.x = dev.upload(F.synth_activations(M, site.K, seed=seed + 1))
        rng = np.random.default_rng(seed + 2)
        self.aux = dev.upload(rng.standard_normal((M, site.N)).astype(np.float32)) if site.epilogue else None
        self.esz = 2 if site.out == F16 else 4
        self.y = dev.empty(M * site.N * self.esz)
        self.stream = Stream()
        self.i = 0

    def launch(self, pair: int, bn: int):
        s = self.site
        w = self.w[self.i % len(self.w)]
        self.i += 1
        check(lib().yah_qgemm_tile(w.ptr, s.fmt, s.N, s.K, self.row, 0, self.x.ptr, self.M, s.K, self.y.ptr, s.out,
                                   s.N, s.epilogue, self.aux.ptr if self.aux else None, s.N if self.aux else 0,
                                   bn, 0, 0, pair, self.stream.handle))

    def time_us(self, pair: int, bn: int, reps: int) -> float:
        self.launch(pair, bn)  # warm-up (also the first-use set-up of the tile)
        e0, e1 = Event(), Event()
        e0.record(self.stream.handle)
        for _ in range(reps):
            self.launch(pair, bn)
        e1.record(self.stream.handle)
        e1.synchronize()
        return e0.elapsed_ms(e1) * 1e3 / reps

    def digest(self, pair: int, bn: int) -> str:
        self.launch(pair, bn)
        self.stream.synchronize()
        return hashlib.sha1(self.y.download(np.uint8, (self.M * self.site.N * self.esz,)).tobytes()).hexdigest()

    def close(self):
        for b in self.w + [self.x, self.y] + ([self.aux] if self.aux else []):
            b.close()
        self.stream.close()


def tune(dev: Device, sites: list, buckets=BUCKETS, quick: int = 3, full: int = 10, keep: int = 3, log=print) -> dict:
    """Measure every tile for every (site, bucket); returns the table (see `save`)."""
    entries = []
    for site in sites:
        for M in buckets:
            b = _Bench(dev, site, M)
            try:
                ref = b.digest(-1 if site.epilogue == EPI_STORE else 0, 0)
                cands = []
                for pair, bn in TILES:
                    if b.digest(pair, bn) != ref:
                        raise RuntimeError(f"{site.name} M={M}: tile ({pair}, {bn}) changes the result")
                    cands.append((b.time_us(pair, bn, quick), pair, bn))
                cands.sort()
                final = sorted((b.time_us(pair, bn, full), pair, bn) for _, pair, bn in cands[:keep])
                us, pair, bn = final[0]
                flops = 2.0 * M * site.N * site.K
                entries.append({"site": site.name, "fmt": site.fmt, "N": site.N, "K": site.K,
                                "epilogue": site.epilogue, "out": site.out, "m_max": M, "cta_pair": pair, "bn": bn,
                                "grid": 0, "us": round(us, 2), "tflops": round(flops / us / 1e6, 1),
                                "candidates_us": {f"{p}:{n}": round(t, 2) for t, p, n in cands}})
                log(f"{site.name:8s} M {M:5d}: pair {pair} bn {bn:3d} {us:9.1f} us {flops / us / 1e6:7.1f} TFLOP/s")
            finally:
                b.close()
    info = ctypes_device_info(dev)
    return {"device": info, "tiles": [list(t) for t in TILES], "buckets": list(buckets),
            "sites": [asdict(s) for s in sites], "entries": entries, "time": time.strftime("%Y-%m-%d %H:%M:%S")}


def ctypes_device_info(dev: Device) -> dict:
    return {"ordinal": dev.ordinal, "sms": dev.sm_count}


def save(table: dict, path: str):
    with open(path, "w") as f:
        json.dump(table, f, indent=1)


def load(path: str) -> dict:
    with open(path) as f:
        return json.load(f)


def rules(table: dict) -> list:
    """The table's entries as yah_tile_rule values."""
    return [TileRule(e["fmt"], e["epilogue"], e["out"], e["N"], e["K"], e["m_max"], e["bn"], e["grid"],
                     e["cta_pair"]) for e in table["entries"]]


def apply(table: dict):
    """Install the table for this process's yah_qgemm calls."""
    rs = rules(table)
    arr = (TileRule * len(rs))(*rs)
    check(lib().yah_tile_rules_set(arr, len(rs)))


def clear():
    check(lib().yah_tile_rules_clear())


def main(argv=None):
    import argparse

    from .tp import StackShape
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--out", required=True)
    ap.add_argument("--parts", type=int, default=1, help="tensor-parallel degree of the stack's shards")
    ap.add_argument("--buckets", default=",".join(map(str, BUCKETS)))
    ap.add_argument("--device", type=int, default=0)
    args = ap.parse_args(argv)
    dev = Device(args.device)
    table = tune(dev, stack_sites(StackShape(), args.parts), [int(v) for v in args.buckets.split(",")])
    save(table, args.out)

