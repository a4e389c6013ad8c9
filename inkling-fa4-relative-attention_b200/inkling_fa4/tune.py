"""Tile-configuration sweep of the sm_100a prefill (the measurement behind ``autotune_configs``).

    python -m inkling_fa4.tune [--seq 32768] [--tile-configs 0,1,2,3,7] [--reps 2] [--steps 30]

The reference tunes its Triton kernels with a grid search over BLOCK_Q x BLOCK_K x warps x
stages (benchmarks/autotune.py:1-140, writing outputs/autotune_results.csv).  Here the kernel
shape is fixed by the hardware design (128-row sub-tiles, 128-key KV tiles, 12 warps, TMEM
S0 | S1 | O0 | O1), and the variants behind ``tile_config`` differ in where the exponentials of
the single-pass interior tiles run (FMA-pipe polynomial, SFU f16x2 or SFU fp32).  This sweep
times each variant on the benchmark workloads (causal, window 4096, R = 1024, R = 512 with window
511, ragged config 2, chunked config 4), interleaving variants within each repetition, and prints
TFLOP/s (algorithmic FLOPs / median step) as JSON: {workload: {tile_config: [per rep]}}.
"""
from __future__ import annotations

import argparse
import json

import torch

from . import _ops
from .workloads import causal_visible_pairs, config_chunked, config_ragged, make_case

HEAD_DIM = 128


def _median_ms(fn, steps, warmup):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(steps + 1)]
    ev[0].record()
    for i in range(steps):
        fn()
        ev[i + 1].record()
    torch.cuda.synchronize()
    ts = sorted(ev[i].elapsed_time(ev[i + 1]) for i in range(steps))
    return ts[len(ts) // 2]


def workloads(seq: int, device):
    """(name, case, keyword arguments, algorithmic FLOPs) of the swept workloads."""
    out = []
    for name, hq, hkv, rext, win in (("causal", 32, 8, 128, None),
                                     ("window4096", 32, 8, 128, 4096),
                                     ("global_rel1024", 32, 8, 1024, None),
                                     ("local_rel512_w511", 32, 8, 512, 511)):
        c = make_case([seq], [seq], hq, hkv, rext, seed=0, device=device, rel_std=0.5,
                      gen_device=device)
        kw = {} if win is None else {"window_size": (win, 0)}
        fl = 4 * HEAD_DIM * hq * causal_visible_pairs([seq], [seq], window_left=win)
        out.append((name, c, kw, fl))
    for name, make, align in (("ragged", config_ragged, "reference"),
                              ("chunked", config_chunked, "bottom_right")):
        c = make(device=device, seed=0, gen_device=device)
        fl = 4 * HEAD_DIM * 32 * causal_visible_pairs(c.seqlens_q, c.seqlens_k, causal_align=align)
        out.append((name, c, {"causal_align": align}, fl))
    return out


def sweep(seq=32768, tile_configs=(0, 1, 2, 3, 7), reps=2, steps=30, warmup=5, device="cuda"):
    device = torch.device(device)
    cases = workloads(seq, device)
    res = {}
    for _ in range(reps):
        for tc in tile_configs:
            for name, c, kw, fl in cases:
                ms = _median_ms(lambda: _ops.prefill(c.q, c.k, c.v, c.rel, c.cu_q, c.cu_k,
                                                     c.max_q, c.max_k, c.rel_extent,
                                                     tile_config=tc, **kw), steps, warmup)
                res.setdefault(name, {}).setdefault(str(tc), []).append(round(fl / ms / 1e9, 1))
    return res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--seq", type=int, default=32768)
    ap.add_argument("--tile-configs", default="0,1,2,3,7")
    ap.add_argument("--reps", type=int, default=2)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=5)
    a = ap.parse_args()
    tcs = [int(x) for x in a.tile_configs.split(",")]
    print(json.dumps(sweep(a.seq, tcs, a.reps, a.steps, a.warmup)))


if __name__ == "__main__":
    main()
