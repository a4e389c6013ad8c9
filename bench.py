#!/usr/bin/env python
"""Benchmark of the relative-bias flash-attention hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...      (one rank per GPU, NCCL)

Headline (``value``): prefill TFLOP/s on the 32k causal GQA 32/8, d=128, R=128 configuration
(full causal), aggregated over all ranks.  A "step" is one prefill call over
one 32768-token sequence with all 32 query heads; exactly K steps are timed after W warm-up
steps.  FLOPs are algorithmic: 4 * head_dim * n_heads * (visible query/key pairs), the bias
gather and masking excluded.  Scaling is weak: every rank owns an independent 32k sequence
(work shards by sequence / KV-head group with no data-path collective); ``value`` = all ranks'
FLOPs / the slowest rank's time.

Every other BASELINE configuration is a secondary object of the same JSON line, each with its
roofline fraction and, at N = 1, its CPU baseline (the oracle, on a bounded sample):
config 1 (S=128, Hq=Hkv=4, scale 1/sqrt(128), per-head distance table), config 2 (ragged
16 x U[1, 4096]), config 3b (window 4096), config 4 (chunked 8 x (16384 + 2048), contiguous
and paged), config 5 (batched decode, contiguous and paged, GB/s against HBM); plus the shapes
the reference itself benchmarks and the model uses (R = 1024 global layer, R = 512 with window
511 local layer, and the reference benchmark's own S=4096 Hq=Hkv=4 R=1024 shape), the
backward, the rel_logits producer, and the end-to-end number through the public API with host
buffers (``e2e``).  Secondary legs time max(K, 50) steps after max(W, 10) warm-up steps and
report the median step as well as the mean.  SM clocks are sampled with nvidia-smi from the
headline's warm-up to the end of the last GPU leg.

At N > 1 two more legs split ONE problem over the ranks by KV-head group (strong scaling):
the 32k prefill and the config-5 decode, each timed without and with the all-gather of the
output heads, and each checked against the rank's own unsharded call (``parity_ok``).

``--impl reference`` times the reference's algorithm on the host CPU (the oracle port; the
reference itself is a Python/Triton package whose CPU path is the torch oracle ref_rel_attn)
on the same bounded sample as the headline's ``cpu_baseline``; rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "inkling-fa4-relative-attention_b200"))
sys.path.insert(0, ROOT)

METRIC = "prefill TFLOP/s at 32k GQA 32/8 d128 bf16; decode HBM GB/s & us/step"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
DATASHEET = {"bf16_tflops": 2250.0, "hbm_gbs": 7700.0}
SEQ, HQ, HKV, D, R = 32768, 32, 8, 128, 128
# Published latency of the reference on its own benchmark shape (S=4096, Hq=Hkv=4, d=128,
# R=1024, causal; RTX 3090, after tuning): README.md:14 of the reference.
REF_PUBLISHED_MS_S4096 = 1.037

# DRAM bytes per launch (dram__bytes_read.sum + dram__bytes_write.sum) from one-pass ncu
# captures of this script's own workloads (command:
#   ncu --metrics dram__bytes_read.sum,dram__bytes_write.sum,gpu__time_duration.sum
#       --clock-control none -k regex:<kernel> -s 3 -c 1 python bench.py --only <leg> ...).
# The decode figure is a batch-16 capture (1.0066 x its algorithmic bytes) scaled to the
# batch-128 step by K/V bytes; the others are full-size launches.
NCU_DRAM_BYTES_PER_LAUNCH = {
    "prefill_causal32k": 951016448,
    "rel_logits32k": 248236032,
    "decode128": 9576854379,
}

LEGS = ("e2e", "window", "ragged", "chunked", "global_rel1024", "local_rel512",
        "refbench", "config1", "backward", "backward_rel1024", "rel_logits", "decode")


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            j = json.load(f)
        return {k: float(j[k]) for k in FALLBACK_PEAKS}, "measured"
    return dict(FALLBACK_PEAKS), "fallback"


def visible_pairs_causal(seq, window=None):
    if window is None:
        return seq * (seq + 1) // 2
    w = window + 1  # keys i-window .. i
    full = max(0, seq - w)
    return w * (w + 1) // 2 + full * w if seq >= w else seq * (seq + 1) // 2


class c_stdout_to_stderr:
    """Point file descriptor 1 at stderr for the duration (C-level writes included)."""

    def __enter__(self):
        sys.stdout.flush()
        self.saved = os.dup(1)
        os.dup2(2, 1)
        return self

    def __exit__(self, *exc):
        sys.stdout.flush()
        try:
            import ctypes
            ctypes.CDLL(None).fflush(None)  # C stdio buffers written inside go to stderr too
        except OSError:
            pass
        os.dup2(self.saved, 1)
        os.close(self.saved)
        return False


# ---------------------------------------------------------------------------------------
class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons while the GPU legs run."""

    FIELDS = ("index,uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, uuids):
        self.uuids = [u.lower() for u in uuids]
        self.proc = None
        self.lines = []
        self.first = threading.Event()

    def _drain(self):
        for line in self.proc.stdout:
            self.lines.append(line)
            self.first.set()

    def start(self, wait_s=3.0):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.reader = threading.Thread(target=self._drain, daemon=True)
            self.reader.start()
            self.first.wait(wait_s)  # sampling has begun before the timed work starts
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.reader.join(timeout=5)
        rows = []
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 10:
                continue
            uuid = parts[1].lower()
            if self.uuids and not any(u in uuid or uuid in u for u in self.uuids):
                continue
            rows.append(parts)
        if not rows:
            return None

        def num(s):
            try:
                return float(s)
            except ValueError:
                return None

        sm = [num(r[2]) for r in rows]
        pw = [num(r[4]) for r in rows]
        smax = [x for x in (num(r[3]) for r in rows) if x is not None]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        loaded_rows = [i for i, p in enumerate(pw) if p is not None and p > 300]
        reasons = sorted({names[i] for k in (loaded_rows or range(len(rows)))
                          for i in range(4) if rows[k][6 + i].lower() == "active"})
        loaded = [sm[i] for i in loaded_rows if sm[i] is not None] or \
            [x for x in sm if x is not None]
        return {"sm_mhz": statistics.median(loaded) if loaded else None,
                "sm_max_mhz": max(smax) if smax else None, "reasons": reasons,
                "samples": len(rows), "samples_under_load": len(loaded_rows),
                "power_w_max": max((p for p in pw if p is not None), default=None),
                "window": "from the headline's warm-up to the end of the last GPU leg"}


# ---------------------------------------------------------------------------------------
# CPU baselines: the torch-CPU twin of reference.py's algorithm (the oracle port), all host
# threads, on bounded samples of each configuration.  Inputs have the configuration's shapes
# and distributions (seeded, generated on the CPU); every sample scores its rows densely
# against all keys, as reference.py computes them, and is credited with algorithmic FLOPs
# (or bytes) only.

def _cpu_threads():
    import torch

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    return threads


class CausalSample:
    """The headline's CPU sample: one head of the 32k causal sequence, 128-row blocks taken in
    a fixed order spread over the sequence (block i at rows ((97 i) mod 256) * 128)."""

    BLK = 128

    def __init__(self, window=None):
        from inkling_fa4.workloads import make_case

        c = make_case([SEQ], [SEQ], 1, 1, R, seed=123, rel_std=0.5)
        self.q, self.k, self.v, self.rel = (t[:, 0].float().contiguous()
                                            for t in (c.q, c.k, c.v, c.rel))
        self.window = window
        self.n_blocks = SEQ // self.BLK

    def block(self, i):
        """Run block i; returns (its algorithmic FLOPs, seconds)."""
        import torch

        import oracle

        r0 = ((i * 97) % self.n_blocks) * self.BLK
        lo = lambda r: 0 if self.window is None else max(0, r - self.window)
        flops = sum(4 * D * (r + 1 - lo(r)) for r in range(r0, r0 + self.BLK))
        pos = torch.arange(r0, r0 + self.BLK)
        return _clocked(lambda: oracle.rel_attn_rows_torch(
            self.q[r0:r0 + self.BLK], self.k, self.v, self.rel[r0:r0 + self.BLK], pos, SEQ, SEQ,
            1.0 / D, R, True, self.window, "reference"), flops)

    def describe(self, blocks):
        w = "" if self.window is None else f", window {self.window}"
        return (f"1 of {HQ} heads, {blocks * self.BLK} of {SEQ} query rows ({blocks} blocks of "
                f"{self.BLK} spread over the sequence{w}), dense scores against all {SEQ} keys as "
                "reference.py computes them; algorithmic FLOPs")


def _run_for(seconds, fn, start=0):
    """Call fn(i) for i = start, start+1, ... until `seconds` of timed CPU work; fn returns
    (units of work, seconds it timed), so input preparation stays outside the count.  Returns
    (total units, seconds, calls)."""
    units, used, i = 0, 0.0, start
    while used < seconds:
        u, dt = fn(i)
        units += u
        used += dt
        i += 1
    return units, used, i - start


def _clocked(run, units):
    t0 = time.perf_counter()
    run()
    return units, time.perf_counter() - t0


def cpu_causal32k(seconds, window=None):
    threads = _cpu_threads()
    s = CausalSample(window)
    s.block(0)  # warm-up (thread pool, allocator)
    flops, used, n = _run_for(seconds, s.block, start=1)
    return {"value": flops / used / 1e12, "unit": "TFLOP/s", "cores": threads, "kind": "port",
            "sample": s.describe(n), "seconds": used}


def cpu_config1(seconds):
    """Config 1 in full (S=128, Hq=Hkv=4, scale 1/sqrt(128), per-head table), repeated."""
    import oracle
    from inkling_fa4.workloads import config_cpu_reference

    threads = _cpu_threads()
    c = config_cpu_reference()
    args = [t.float() for t in (c.q, c.k, c.v, c.rel)]
    fl = 4 * D * 4 * visible_pairs_causal(128)

    def call(_):
        return _clocked(lambda: oracle.rel_attn_torch(*args, c.cu_q, c.cu_k, 128 ** -0.5, 128), fl)

    call(0)
    flops, used, n = _run_for(seconds, call)
    return {"value": flops / used / 1e12, "unit": "TFLOP/s", "cores": threads, "kind": "port",
            "ms_per_call": used * 1e3 / n, "sample": f"the whole configuration, {n} calls"}


def cpu_ragged(seconds):
    """Config 2: (sequence, head) pairs of the seeded ragged batch in a fixed order, each a
    full dense per-head attention of that sequence."""
    import torch

    import oracle
    from inkling_fa4.workloads import make_case, ragged_batch_lengths

    threads = _cpu_threads()
    lens = ragged_batch_lengths()
    cases = []
    for b, L in enumerate(lens):  # one head per sequence (heads are independent and alike)
        c = make_case([L], [L], 1, 1, R, seed=50 + b, rel_std=0.5)
        cases.append(tuple(t[:, 0].float().contiguous() for t in (c.q, c.k, c.v, c.rel)))

    def call(i):
        b = i % len(lens)
        q, k, v, rel = cases[b]
        L = lens[b]
        return _clocked(lambda: oracle.rel_attn_rows_torch(
            q, k, v, rel, torch.arange(L), L, L, 1.0 / D, R, True, None, "reference"),
            4 * D * visible_pairs_causal(L))

    call(0)
    flops, used, n = _run_for(seconds, call, start=1)
    return {"value": flops / used / 1e12, "unit": "TFLOP/s", "cores": threads, "kind": "port",
            "sample": f"{n} (sequence, head) attentions over the 16 seeded lengths (one head "
                      "per sequence, sequences in order, repeated), dense as reference.py "
                      "computes them; algorithmic causal FLOPs"}


def cpu_chunked(seconds):
    """Config 4: 128-row blocks of one sequence's 2048-token chunk (one head) against its
    18432 keys, bottom-right alignment."""
    import torch

    import oracle
    from inkling_fa4.workloads import make_case

    threads = _cpu_threads()
    cache, chunk = 16384, 2048
    sk = cache + chunk
    c = make_case([chunk], [sk], 1, 1, R, seed=60, rel_std=0.5)
    q, k, v, rel = (t[:, 0].float().contiguous() for t in (c.q, c.k, c.v, c.rel))

    def call(i):
        r0 = ((i * 5) % (chunk // 128)) * 128
        return _clocked(lambda: oracle.rel_attn_rows_torch(
            q[r0:r0 + 128], k, v, rel[r0:r0 + 128], torch.arange(r0, r0 + 128), chunk, sk,
            1.0 / D, R, True, None, "bottom_right"),
            sum(4 * D * (cache + r + 1) for r in range(r0, r0 + 128)))

    call(0)
    flops, used, n = _run_for(seconds, call, start=1)
    return {"value": flops / used / 1e12, "unit": "TFLOP/s", "cores": threads, "kind": "port",
            "sample": f"{n} blocks of 128 query rows of one 2048-token chunk (one head) against "
                      f"its {sk} keys, bottom-right alignment; algorithmic FLOPs"}


def cpu_decode(seconds, lens):
    """Config 5: whole sequences of the seeded decode batch (all 32 heads, one query each)
    in a fixed order; GB/s of algorithmic bytes (K/V once per GQA group, q/rel/out).  The keys
    of a sequence of length L are the first L of one seeded 32768-key pool."""
    import torch

    import oracle
    from inkling_fa4.workloads import make_case

    threads = _cpu_threads()
    order = [(i * 37) % len(lens) for i in range(len(lens))]
    pool = make_case([1], [max(lens)], HQ, HKV, R, seed=70, rel_std=0.5)
    q, rel = pool.q.float(), pool.rel.float()
    ks = [pool.k[:, kh].float().contiguous() for kh in range(HKV)]
    vs = [pool.v[:, kh].float().contiguous() for kh in range(HKV)]
    g = HQ // HKV
    pos = torch.tensor([0])

    def call(i):
        L = lens[order[i % len(order)]]

        def run():
            for h in range(HQ):
                oracle.rel_attn_rows_torch(q[:, h], ks[h // g][:L], vs[h // g][:L], rel[:, h],
                                           pos, 1, L, 1.0 / D, R, True, None, "bottom_right")

        return _clocked(run, L * HKV * D * 2 * 2 + HQ * (D * 2 * 2 + R * 2))

    nbytes, used, n = _run_for(seconds, call)
    gbs = nbytes / used / 1e9
    total = sum(lens) * HKV * D * 2 * 2 + len(lens) * HQ * (D * 2 * 2 + R * 2)
    return {"value": gbs, "unit": "GB/s", "cores": threads, "kind": "port",
            "us_per_step_extrapolated": total / (gbs * 1e9) * 1e6,
            "sample": f"{n} whole sequences of the 128 seeded lengths (all 32 heads, one query), "
                      "oracle port; algorithmic bytes (K/V counted once per GQA group)"}


def run_reference_arm(args, rank, world):
    """The reference's algorithm on the host cores, on the headline's configuration: each step
    runs `blocks_per_step` blocks of the same CPU sample as the headline's cpu_baseline."""
    if rank != 0:
        return
    threads = _cpu_threads()
    s = CausalSample()
    per = args.ref_blocks_per_step
    for i in range(args.warmup):
        for j in range(per):
            s.block(i * per + j)
    flops, t0 = 0, time.perf_counter()
    base = args.warmup * per
    for i in range(args.steps):
        for j in range(per):
            flops += s.block(base + i * per + j)[0]
    dt = time.perf_counter() - t0
    value = flops / dt / 1e12
    sample = (f"per step: {per} blocks of the headline's CPU sample; "
              f"{s.describe(args.steps * per)}; oracle port, torch CPU, {threads} threads")
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "TFLOP/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": dt * 1e3 / max(1, args.steps), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "causal32k_gqa32_8_d128_rel128", "seq_len": SEQ,
                       "n_heads": HQ, "kv_heads": HKV, "head_dim": D, "rel_extent": R},
            "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": threads, "kind": "port",
                             "sample": sample},
            "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------------------
def timed(fn, steps, warmup, stream, dist=None, barrier=None):
    """Warm up, then time `steps` calls between a barrier + synchronize on both sides with one
    CUDA event per step on the launching stream.  Returns (total ms, median step ms), each the
    max over ranks."""
    import torch

    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    if barrier:
        barrier()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(steps + 1)]
    ev[0].record(stream)
    for i in range(steps):
        fn()
        ev[i + 1].record(stream)
    torch.cuda.synchronize()
    if barrier:
        barrier()
    ms = ev[0].elapsed_time(ev[-1])
    med = statistics.median(ev[i].elapsed_time(ev[i + 1]) for i in range(steps))
    if dist is not None:
        t = torch.tensor([ms, med], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, med = float(t[0].item()), float(t[1].item())
    return ms, med


def graph_replay_us(fn, calls=10, reps=100):
    """Device time per call of `fn` replayed from a CUDA graph of `calls` calls (the calls'
    host-side Python and ctypes work is paid once, at capture), so launch-latency-bound calls
    show their device time rather than the host's."""
    import torch

    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(3):
            fn()
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for _ in range(calls):
            fn()
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(reps):
        graph.replay()
    b.record()
    torch.cuda.synchronize()
    us = a.elapsed_time(b) * 1e3 / (reps * calls)
    del graph
    return us


def read_stream_peak(dev, stream):
    """The read-only HBM stream ceiling of this GPU, measured in the run: the library's
    measurement hook (16-byte non-coherent loads, four in flight per thread) over a 4 GiB
    buffer, best of 10 after 3 warm-up passes, CUDA events on the launching stream.  Decode
    reads ~99 % and writes ~1 % of its bytes, so a read stream, not the read+write copy of
    MEASURED_PEAKS.json, is its ceiling."""
    import ctypes

    import torch

    from inkling_fa4 import _lib

    L = _lib.lib()
    nbytes = 4 << 30
    x = torch.ones(nbytes // 2, dtype=torch.bfloat16, device=dev)
    sink = torch.zeros(1, dtype=torch.int32, device=dev)
    h = ctypes.c_void_p(stream.cuda_stream)
    best = float("inf")
    for i in range(13):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        _lib.check(L.ifa4_measure_read_stream(ctypes.c_void_p(x.data_ptr()),
                                              ctypes.c_size_t(nbytes),
                                              ctypes.c_void_p(sink.data_ptr()), h))
        b.record(stream)
        torch.cuda.synchronize()
        if i >= 3:
            best = min(best, a.elapsed_time(b))
    del x, sink
    torch.cuda.empty_cache()
    return nbytes / (best / 1e3) / 1e9


def parse_args(argv=None):
    """(args, the set of legs to skip, whether the headline runs)."""
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-seconds", type=float, default=6.0,
                    help="CPU work per configuration's cpu_baseline sample")
    ap.add_argument("--ref-blocks-per-step", type=int, default=8,
                    help="reference arm: 128-row blocks of the CPU sample per step")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--skip", default="", help=f"comma-separated legs to skip, of {LEGS}")
    ap.add_argument("--only", default="all",
                    help="'headline', or one leg name (profiling runs); 'all' runs everything")
    ap.add_argument("--no-shard", action="store_true",
                    help="skip the head-sharded legs (N > 1 only)")
    ap.add_argument("--peer-stores", type=int, default=1,
                    help="N > 1: also time the head-sharded prefill whose kernel stores its rows "
                         "into every rank's output (1) or not (0)")
    ap.add_argument("--prefill-seq", type=int, default=SEQ,
                    help="sequence length of the headline workload (32768 = BASELINE config 3)")
    ap.add_argument("--tile-config", type=int, default=0,
                    help="prefill kernel variant (0 = default; see autotune_configs)")
    ap.add_argument("--decode-batch", type=int, default=128,
                    help="decode batch (128 = BASELINE config 5)")
    # earlier spellings, kept so that the capture commands recorded with the profiles still run:
    # --no-<leg> is --skip <leg>, --only prefill is --only headline
    for leg in ("e2e", "decode", "window", "backward", "rel-logits"):
        ap.add_argument(f"--no-{leg}", action="append_const", dest="old_skip",
                        const=leg.replace("-", "_"), help=argparse.SUPPRESS)
    args = ap.parse_args(argv)
    if args.warmup < 3:
        args.warmup = 3
    if args.only == "prefill":
        args.only = "headline"
    skip = {s for s in args.skip.split(",") if s} | set(args.old_skip or ())
    bad = skip - set(LEGS)
    if bad:
        ap.error(f"unknown legs {sorted(bad)}")
    if args.only != "all":
        if args.only != "headline" and args.only not in LEGS:
            ap.error(f"--only must be 'all', 'headline' or one of {LEGS}")
        skip = set(LEGS) - {args.only}
        args.no_shard = True
        args.no_cpu_baseline = True
    return args, skip, args.only in ("all", "headline", "e2e")


def main():
    args, skip, run_headline = parse_args()
    want = lambda leg: leg not in skip

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        run_reference_arm(args, rank, world)
        return

    import torch

    torch.cuda.set_device(local_rank)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as tdist

        # NCCL prints its version banner (with NCCL_DEBUG set) on the process's C stdout when the
        # communicator is created, and debug lines to its debug file (stdout by default); rank 0's
        # stdout must hold only the JSON result line, so both go to stderr.
        os.environ.setdefault("NCCL_DEBUG_FILE", "/dev/stderr")
        with c_stdout_to_stderr():
            tdist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180),
                                     device_id=torch.device("cuda", local_rank))
            tdist.barrier()  # the communicator exists (and has printed) before stdout returns
        dist = tdist
    barrier = (lambda: dist.barrier()) if dist else None

    from inkling_fa4 import (_lib, _ops, inkling_fa4_rel_attention_decode_triton,
                             inkling_fa4_rel_attention_triton)
    from inkling_fa4.workloads import (causal_visible_pairs, config_chunked, config_decode,
                                       config_long, config_ragged, make_case, page_kv)

    peaks, peak_kind = load_peaks()
    dev = torch.device("cuda", local_rank)
    stream = torch.cuda.current_stream(dev)
    steps2, warm2 = max(args.steps, 50), max(args.warmup, 10)  # secondary legs
    cpu_on = rank == 0 and world == 1 and not args.no_cpu_baseline

    def prefill_call(*pa, **kw):
        """The public prefill entry point, or the same call pinned to --tile-config (for tile
        sweeps; paged caches exist for tile configs 0 to 3)."""
        if args.tile_config and (kw.get("block_table") is None or args.tile_config <= 3):
            return _ops.prefill(*pa, tile_config=args.tile_config, **kw)
        return inkling_fa4_rel_attention_triton(*pa, **kw)

    def tensor_roofline(flops_per_step, ms_step, traffic=None, kernel="rel_attn_prefill_kernel"):
        achieved = flops_per_step / (ms_step / 1e3) / 1e12
        return {"bound": "tensor", "achieved": achieved, "peak": peaks["bf16_tflops"],
                "unit": "TFLOP/s", "frac": achieved / peaks["bf16_tflops"],
                "peak_source": f"bf16_tflops (burst) of {peak_kind}",
                "frac_of_sustained": achieved / peaks["bf16_tflops_sustained"],
                "frac_of_datasheet_2250": achieved / DATASHEET["bf16_tflops"],
                "traffic": traffic, "kernel": f"{kernel} (1 launch per step)"}

    def prefill_leg(name, case, flops, steps, warmup, extra_cfg, **kw):
        def step():
            return prefill_call(case.q, case.k, case.v, case.rel, case.cu_q, case.cu_k,
                                case.max_q, case.max_k, case.rel_extent, **kw)

        ms, med = timed(step, steps, warmup, stream, dist, barrier)
        ms_step = ms / steps
        cfg = {"rel_extent": case.rel_extent, "batch": len(case.seqlens_q),
               "total_q": int(case.q.shape[0]), "total_k": int(case.cu_k[-1].item()),
               "n_heads": int(case.q.shape[1]),
               "kv_heads": int(case.k.shape[-2]), "flops_per_step_per_gpu": flops}
        cfg.update(extra_cfg)
        return {"value": world * flops * steps / (ms / 1e3) / 1e12, "unit": "TFLOP/s",
                "ms_per_step": ms_step, "ms_per_step_median": med, "steps": steps,
                "warmup": warmup, "config": cfg,
                "roofline": tensor_roofline(flops, med), "gpu_launches": steps}

    uuids = []
    try:
        uuids = [str(torch.cuda.get_device_properties(dev).uuid)]
    except Exception:
        pass
    sampler = ClockSampler(uuids) if rank == 0 else None
    if sampler:
        sampler.start()

    # ---------------- headline: 32k causal prefill, inputs resident in HBM
    S = args.prefill_seq
    c = config_long(device=dev, seed=rank, seq=S, gen_device=dev)
    flops = 4 * D * HQ * visible_pairs_causal(S)

    def prefill_step():
        return prefill_call(c.q, c.k, c.v, c.rel, c.cu_q, c.cu_k, S, S, R)

    if run_headline:
        ms, med = timed(prefill_step, args.steps, args.warmup, stream, dist, barrier)
    else:
        ms, med = float("nan"), float("nan")
    ms_step = ms / args.steps
    value = world * flops * args.steps / (ms / 1e3) / 1e12
    status = _lib.read_device_status(stream.cuda_stream)

    result = {
        "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
        "ms_per_step_median": med,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: seeded N(0,1) q/k/v and N(0,0.5) per-token rel logits, generated on "
                "the device (rank r uses seed r)",
        "config": {"workload": ("causal32k_gqa32_8_d128_rel128" if S == SEQ else
                                f"causal{S}_gqa32_8_d128_rel128"), "batch": 1, "seq_len": S,
                   "n_heads": HQ, "kv_heads": HKV, "head_dim": D, "rel_extent": R,
                   "causal": True, "window_left": None, "causal_align": "reference",
                   "flops_per_step_per_gpu": flops,
                   "l2": (f"no flush; inputs of {(S * (HQ * (2 * D + 2 * R) + HKV * 4 * D)) >> 20} MB "
                          "per step exceed the 126 MB L2"),
                   "parallelism": f"{world} independent {S}-token sequences, one per rank (weak)"},
        "roofline": dict(tensor_roofline(flops, ms_step,
                                         NCU_DRAM_BYTES_PER_LAUNCH["prefill_causal32k"]
                                         if S == SEQ else None),
                         traffic_note="ncu one-pass capture of the full-size 32k launch "
                                      "(dram__bytes_read.sum + dram__bytes_write.sum)",
                         tile_config=args.tile_config),
        "gpu_launches": args.steps if run_headline else 0,
        "device_status": status,
    }

    # ---------------- end to end through the public API with host buffers
    # Every step uploads its own inputs from pinned host memory, runs the public API call and
    # downloads its output to pinned host memory.  Three streams and two buffer sets let the
    # upload of step i+1 and the download of step i-1 overlap the kernel of step i, as a
    # serving pipeline would; the timed region spans the first upload to the last download.
    if run_headline and want("e2e"):
        names = ("q", "k", "v", "rel", "cu_q", "cu_k")
        host = {n: getattr(c, n).cpu().pin_memory() for n in names}
        dbuf = [{n: torch.empty_like(getattr(c, n)) for n in names} for _ in range(2)]
        dout = [torch.empty((S, HQ, D), dtype=torch.bfloat16, device=dev) for _ in range(2)]
        hout = [torch.empty((S, HQ, D), dtype=torch.bfloat16).pin_memory() for _ in range(2)]
        h2d = sum(t.numel() * t.element_size() for t in host.values())
        d2h = hout[0].numel() * hout[0].element_size()
        s_up, s_run, s_down = (torch.cuda.Stream(dev) for _ in range(3))
        ev = {k: [torch.cuda.Event() for _ in range(2)] for k in ("up", "run", "down")}
        e_steps = max(4, min(args.steps, 20))

        def pipeline(nsteps):
            for i in range(nsteps):
                b = i % 2
                with torch.cuda.stream(s_up):
                    if i >= 2:
                        s_up.wait_event(ev["run"][b])      # kernel i-2 done with dbuf[b]
                    for n in names:
                        dbuf[b][n].copy_(host[n], non_blocking=True)
                    ev["up"][b].record(s_up)
                with torch.cuda.stream(s_run):
                    s_run.wait_event(ev["up"][b])
                    if i >= 2:
                        s_run.wait_event(ev["down"][b])    # download i-2 done with dout[b]
                    d = dbuf[b]
                    inkling_fa4_rel_attention_triton(d["q"], d["k"], d["v"], d["rel"], d["cu_q"],
                                                     d["cu_k"], S, S, R, out=dout[b])
                    ev["run"][b].record(s_run)
                with torch.cuda.stream(s_down):
                    s_down.wait_event(ev["run"][b])
                    hout[b].copy_(dout[b], non_blocking=True)
                    ev["down"][b].record(s_down)
            for st in (s_up, s_run, s_down):
                stream.wait_stream(st)

        pipeline(2)
        torch.cuda.synchronize()
        if barrier:
            barrier()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        for st in (s_up, s_run, s_down):
            st.wait_stream(stream)
        pipeline(e_steps)
        t1.record(stream)
        torch.cuda.synchronize()
        if barrier:
            barrier()
        ems = t0.elapsed_time(t1)
        if dist is not None:
            tt = torch.tensor([ems], dtype=torch.float64, device=dev)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            ems = float(tt.item())
        ok = torch.equal(hout[(e_steps - 1) % 2], dout[(e_steps - 1) % 2].cpu())
        result["e2e"] = {"value": world * flops * e_steps / (ems / 1e3) / 1e12, "unit": "TFLOP/s",
                         "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                         "ms_per_step": ems / e_steps, "steps": e_steps,
                         "output_roundtrip_ok": bool(ok),
                         "path": "pinned host -> device upload of q/k/v/rel/cu_seqlens, "
                                 "inkling_fa4_rel_attention_triton (C ABI), device -> pinned host "
                                 "download of the output; 3 streams, 2 buffer sets, every step "
                                 "moves its own inputs and output"}
        del host, dbuf, dout, hout

    # ---------------- config 3b: sliding window 4096 at 32k
    if want("window"):
        wflops = 4 * D * HQ * visible_pairs_causal(S, 4096)
        result["window32k"] = prefill_leg("window32k", c, wflops, steps2, warm2,
                                          {"workload": "window4096_32k_gqa32_8_d128_rel128",
                                           "window_left": 4096}, window_size=(4096, 0))

    # ---------------- backward of a prefill (not in the reference)
    def backward_leg(bc, rext, bflops):
        from inkling_fa4 import inkling_fa4_rel_attention_backward

        bout, blse = inkling_fa4_rel_attention_triton(bc.q, bc.k, bc.v, bc.rel, bc.cu_q, bc.cu_k,
                                                      S, S, rext, return_lse=True)
        gen = torch.Generator(device=dev)
        gen.manual_seed(1000 + rank)
        bdout = torch.randn(bc.q.shape, generator=gen, device=dev).to(torch.bfloat16)
        bws = torch.empty(HQ * S * 4, dtype=torch.uint8, device=dev)
        bufs = (torch.empty_like(bc.q), torch.empty_like(bc.k), torch.empty_like(bc.v),
                torch.empty_like(bc.rel))

        def bwd_step():
            return inkling_fa4_rel_attention_backward(
                bdout, bc.q, bc.k, bc.v, bc.rel, bout, blse, bc.cu_q, bc.cu_k, S, S, rext,
                dq=bufs[0], dk=bufs[1], dv=bufs[2], drel=bufs[3], workspace=bws)

        bsteps = max(5, args.steps // 2)
        bms, bmed = timed(bwd_step, bsteps, args.warmup, stream, dist, barrier)
        leg = {
            "value": world * bflops * bsteps / (bms / 1e3) / 1e12, "unit": "TFLOP/s",
            "ms_per_step": bms / bsteps, "ms_per_step_median": bmed, "steps": bsteps,
            "rel_extent": rext, "flops_per_step_per_gpu": bflops,
            "flops_note": "algorithmic 2.5x forward (S, dP, dV, dK, dQ); the kernels execute "
                          "3.5x (S and dP are recomputed by the dQ kernel to avoid atomics)",
            "roofline": dict(tensor_roofline(bflops, bmed), kernel="rel_attn_bwd_prep_kernel, "
                             "rel_attn_bwd_dkdv_kernel, rel_attn_bwd_dq_kernel (3 launches per "
                             "step; algorithmic FLOPs over the whole step)"),
            "gpu_launches": 3 * bsteps}
        del bout, blse, bdout, bws, bufs
        return leg

    if want("backward"):  # of the headline prefill
        result["backward32k"] = backward_leg(c, R, 2.5 * flops)

    # ---------------- rel_logits producer for the headline shape (the step before the path)
    if want("rel_logits"):
        from inkling_fa4 import inkling_rel_logits

        gen = torch.Generator(device=dev)
        gen.manual_seed(2000 + rank)
        rr = torch.randn((S, HQ, 16), generator=gen, device=dev).to(torch.bfloat16)
        rw = (0.5 * torch.randn((HQ, 16, R), generator=gen, device=dev)).to(torch.bfloat16)
        rout = torch.empty((S, HQ, R), dtype=torch.bfloat16, device=dev)

        def rl_step():
            return inkling_rel_logits(rr, rw, alpha=0.1, nf=4096.0, out=rout)

        rms, rmed = timed(rl_step, steps2, warm2, stream, dist, barrier)
        rbytes = rr.numel() * 2 + rw.numel() * 2 + rout.numel() * 2
        rgbs = rbytes * steps2 / (rms / 1e3) / 1e9
        # Write-stream reference on the same box: torch's fill_ of the same output buffer, same
        # protocol (the producer's traffic is 89 % writes).
        fms, _ = timed(lambda: rout.fill_(1.0), steps2, warm2, stream, dist, barrier)
        fill_gbs = rout.numel() * 2 * steps2 / (fms / 1e3) / 1e9
        write_gbs = rout.numel() * 2 * steps2 / (rms / 1e3) / 1e9
        result["rel_logits32k"] = {
            "value": world * rgbs, "unit": "GB/s", "us_per_step": rms * 1e3 / steps2,
            "us_per_step_median": rmed * 1e3, "steps": steps2,
            "config": {"workload": "rel_logits_32k_h32_r128", "tokens": S, "n_heads": HQ,
                       "d_rel": 16, "rel_extent": R, "weight": "per head", "alpha": 0.1,
                       "nf": 4096.0, "bytes_per_step_per_gpu": rbytes,
                       "l2": "working set 302 MB > 126 MB L2 (the 268 MB output streams out "
                             "every step)"},
            "roofline": {"bound": "hbm", "achieved": rgbs, "peak": peaks["hbm_gbs"],
                         "unit": "GB/s", "frac": rgbs / peaks["hbm_gbs"],
                         "peak_source": f"hbm_gbs of {peak_kind}",
                         "write_gbs": write_gbs, "fill_gbs_same_buffer": fill_gbs,
                         "write_frac_of_fill": write_gbs / fill_gbs,
                         "traffic": (NCU_DRAM_BYTES_PER_LAUNCH["rel_logits32k"]
                                     if S == SEQ else None),
                         "traffic_note": "one cold ncu launch: reads + writes performed before "
                                         "it ended (54 MB of output still dirty in L2)"},
            "kernel": "rel_logits_kernel (1 launch per step)", "gpu_launches": steps2}
        del rr, rw, rout
    del c
    torch.cuda.empty_cache()

    # ---------------- config 2: ragged 16 x U[1, 4096], config 4: chunked 8 x (16384 + 2048)
    for name, make, align in (("ragged", config_ragged, "reference"),
                              ("chunked", config_chunked, "bottom_right")):
        if not want(name):
            continue
        cc = make(device=dev, seed=rank, gen_device=dev)
        fl = 4 * D * HQ * causal_visible_pairs(cc.seqlens_q, cc.seqlens_k, causal_align=align)
        cfg = {"workload": cc.meta["name"], "causal_align": align}
        if name == "ragged":
            cfg["seqlens"] = cc.seqlens_q
        result[name] = prefill_leg(name, cc, fl, steps2, warm2, cfg, causal_align=align)
        if name == "chunked":  # the same chunks against a 16-token paged cache
            pc = page_kv(cc, page_size=16, seed=rank)
            del cc
            cc = pc
            leg = prefill_leg("chunked_paged", pc, fl, steps2, warm2,
                              dict(cfg, page_size=16, num_pages=pc.meta["num_pages"]),
                              causal_align=align, block_table=pc.meta["block_table"])
            result["chunked_paged"] = leg
        del cc
        torch.cuda.empty_cache()

    # ---------------- the rel extents the model and the reference's benchmark use
    # Global layers: R = 1024, full causal; local layers: R = 512 with window (511, 0)
    # (the reference's architecture notes); the reference's benchmark: S = 4096, Hq = Hkv = 4,
    # R = 1024, causal (its only published numbers).
    # The global layers' backward (same inputs as the R = 1024 forward leg) as backward_rel1024.
    for name, seq, hq, hkv, rext, win in (("global_rel1024", S, HQ, HKV, 1024, None),
                                          ("local_rel512", S, HQ, HKV, 512, 511),
                                          ("refbench", 4096, 4, 4, 1024, None)):
        with_bwd = name == "global_rel1024" and want("backward_rel1024")
        if not want(name) and not with_bwd:
            continue
        gc = make_case([seq], [seq], hq, hkv, rext, seed=rank, device=dev, rel_std=0.5,
                       gen_device=dev)
        fl = 4 * D * hq * visible_pairs_causal(seq, win)
        kw = {} if win is None else {"window_size": (win, 0)}
        key = {"global_rel1024": f"global{seq}_rel1024", "local_rel512": f"local{seq}_rel512_window511",
               "refbench": "refbench4096_h4_rel1024"}[name]
        if want(name):
            leg = prefill_leg(key, gc, fl, steps2, warm2,
                              {"workload": f"{key}_gqa{hq}_{hkv}_d128", "seq_len": seq,
                               "window_left": win}, **kw)
            if name == "refbench":
                leg["reference_published_ms_rtx3090"] = REF_PUBLISHED_MS_S4096
                leg["speedup_vs_published"] = REF_PUBLISHED_MS_S4096 / leg["ms_per_step_median"]
            result[key] = leg
        if with_bwd:
            result[f"backward{seq}_rel1024"] = backward_leg(gc, rext, 2.5 * fl)
        del gc
        torch.cuda.empty_cache()

    # ---------------- config 1 on the GPU (bf16 inputs; the configuration is the CPU case)
    if want("config1"):
        from inkling_fa4.workloads import config_cpu_reference

        c1 = config_cpu_reference(device=dev)
        fl1 = 4 * D * 4 * visible_pairs_causal(128)
        leg = prefill_leg("config1", c1, fl1, steps2, warm2,
                          {"workload": "cpu_reference_s128_h4_4_rel128_table",
                           "softmax_scale": 128 ** -0.5, "rel": "per-head table (token stride 0)",
                           "note": "launch-latency bound: one 128-row tile per head"},
                          softmax_scale=128 ** -0.5)
        # eager calls of this size are bound by the host (Python + ctypes, about 40 us per call);
        # replayed from a CUDA graph they show the kernel's own time
        leg["graph_replay_us_per_call"] = graph_replay_us(
            lambda: prefill_call(c1.q, c1.k, c1.v, c1.rel, c1.cu_q, c1.cu_k, c1.max_q, c1.max_k,
                                 c1.rel_extent, softmax_scale=128 ** -0.5))
        result["config1"] = leg
        del c1

    # ---------------- one problem split over the ranks by KV-head group (N > 1 only)
    # Strong scaling of a single call: rank r runs the heads of kv groups [r*8/N, (r+1)*8/N)
    # (head-slice views, no copies), timed without and with the NCCL all-gather that assembles
    # the full output on every rank, and checked against the rank's own unsharded call on the
    # same inputs (the per-head arithmetic is identical, so the outputs are equal bit for bit).
    if world > 1 and not args.no_shard and HKV % world == 0:
        from inkling_fa4.sharding import gather_heads, head_shard, shard_tensors

        sh = head_shard(HQ, HKV, world, rank)
        sc = config_long(device=dev, seed=0, seq=S, gen_device=dev)  # same sequence on all ranks
        q_s, k_s, v_s, rel_s = shard_tensors(sh, sc.q, sc.k, sc.v, sc.rel)
        shard_step = lambda: inkling_fa4_rel_attention_triton(q_s, k_s, v_s, rel_s, sc.cu_q,
                                                               sc.cu_k, S, S, R)
        gather_step = lambda: gather_heads(shard_step(), world)
        ms_ng, _ = timed(shard_step, args.steps, args.warmup, stream, dist, barrier)
        ms_g, _ = timed(gather_step, args.steps, args.warmup, stream, dist, barrier)
        full = gather_step()
        ref = inkling_fa4_rel_attention_triton(sc.q, sc.k, sc.v, sc.rel, sc.cu_q, sc.cu_k, S, S,
                                               R)
        diff = float((full.float() - ref.float()).abs().max().item())
        ok = torch.tensor([1 if torch.equal(full, ref) else 0], device=dev)
        dist.all_reduce(ok, op=dist.ReduceOp.MIN)
        # the same split with the output assembled during the call: each rank's kernel stores its
        # heads' finished rows into every rank's output buffer (CUDA IPC mappings), then one
        # one-element all-reduce orders the reads
        fused = peers = None
        if args.peer_stores:
            from inkling_fa4.sharding import PeerOutputs, prefill_to_all_ranks

            peers = PeerOutputs((S, HQ, D), dtype=torch.bfloat16, device=dev)
            fused_step = lambda: prefill_to_all_ranks(peers, sh, q_s, k_s, v_s, rel_s, sc.cu_q,
                                                      sc.cu_k, S, S, R)
            peers.local.fill_(float("nan"))
            peers.barrier()
            ms_f, _ = timed(fused_step, args.steps, args.warmup, stream, dist, barrier)
            peers.local.fill_(float("nan"))  # every element must come from this call's stores
            peers.barrier()
            fused = fused_step()
            torch.cuda.synchronize()
            fdiff = float((fused.float() - ref.float()).abs().max().item())
            fok = torch.tensor([1 if torch.equal(fused, ref) else 0], device=dev)
            dist.all_reduce(fok, op=dist.ReduceOp.MIN)
        full_flops = 4 * D * HQ * visible_pairs_causal(S)
        # NCCL's own time for the 32 MB-per-rank all-gather alone (the output of this rank)
        src = torch.empty((S, sh.n_q, D), dtype=torch.bfloat16, device=dev)
        gbuf = torch.empty((world, S, sh.n_q, D), dtype=torch.bfloat16, device=dev)
        ag_ms, _ = timed(lambda: dist.all_gather_into_tensor(gbuf, src), args.steps, args.warmup,
                         stream, dist, barrier)
        ag_bytes = gbuf.numel() * 2
        result["head_sharded32k"] = {
            "unit": "TFLOP/s", "scaling": "strong",
            "value_no_gather": full_flops * args.steps / (ms_ng / 1e3) / 1e12,
            "value_with_gather": full_flops * args.steps / (ms_g / 1e3) / 1e12,
            "ms_per_step_no_gather": ms_ng / args.steps,
            "ms_per_step_with_gather": ms_g / args.steps,
            "parity_ok": bool(ok.item() == 1), "max_abs_diff_vs_unsharded": diff,
            "nccl_all_gather_alone": {"ms": ag_ms / args.steps,
                                      "bus_gbs": ag_bytes * (world - 1) / world
                                      / (ag_ms / args.steps / 1e3) / 1e9,
                                      "bytes_per_rank": src.numel() * 2},
            "config": {"workload": "causal32k_gqa32_8_d128_rel128, one sequence",
                       "heads_per_rank": sh.n_q, "kv_heads_per_rank": sh.n_kv,
                       "collective": "one NCCL all_gather_into_tensor of the output heads "
                                     f"({S * HQ * D * 2 >> 20} MB assembled per step)"},
            "gpu_launches": args.steps}
        if args.peer_stores:
            result["head_sharded32k"].update({
                "value_with_peer_stores": full_flops * args.steps / (ms_f / 1e3) / 1e12,
                "ms_per_step_with_peer_stores": ms_f / args.steps,
                "peer_stores_parity_ok": bool(fok.item() == 1),
                "peer_stores_max_abs_diff_vs_unsharded": fdiff,
                "peer_stores": "each rank's prefill kernel stores its heads' output rows into "
                               "every rank's [T, 32, 128] buffer (CUDA IPC peer mappings, plain "
                               "16-byte stores over NVLink) as its tiles finish; one 4-byte NCCL "
                               "all-reduce per step orders the reads"})
        if peers is not None:
            peers.close()  # every rank unmaps the others' buffers before any rank frees its own
        del sc, q_s, k_s, v_s, rel_s, full, ref, src, gbuf, fused, peers
        torch.cuda.empty_cache()

        # config 5 decode with its KV heads split 8/N per rank (same batch on every rank)
        dcs = config_decode(device=dev, seed=0, batch=args.decode_batch, gen_device=dev)
        lens = dcs.seqlens_k
        p = _ops._decode_params(dcs.q, dcs.k, dcs.v, dcs.rel, dcs.q, dcs.cu_q, dcs.cu_k, HQ, HKV,
                                R, True, -1, "bottom_right", max(lens), 1.0 / D, 0, 0)
        _, nsplit, chunk = _ops.decode_plan(p)
        dq, dk, dv, drel = shard_tensors(sh, dcs.q, dcs.k, dcs.v, dcs.rel)
        ws = torch.empty(64 << 20, dtype=torch.uint8, device=dev)

        def dshard_step():
            return inkling_fa4_rel_attention_decode_triton(
                dq, dk, dv, drel, dcs.cu_q, dcs.cu_k, 1, max(lens), R, causal_align="bottom_right",
                num_splits=nsplit, chunk_len=chunk, workspace=ws)

        dgather_step = lambda: gather_heads(dshard_step(), world)
        dms_ng, dmed_ng = timed(dshard_step, steps2, warm2, stream, dist, barrier)
        dms_g, _ = timed(dgather_step, steps2, warm2, stream, dist, barrier)
        dfull = dgather_step()
        dref = inkling_fa4_rel_attention_decode_triton(
            dcs.q, dcs.k, dcs.v, dcs.rel, dcs.cu_q, dcs.cu_k, 1, max(lens), R,
            causal_align="bottom_right", num_splits=nsplit, chunk_len=chunk, workspace=ws)
        ddiff = float((dfull.float() - dref.float()).abs().max().item())
        dok = torch.tensor([1 if torch.equal(dfull, dref) else 0], device=dev)
        dist.all_reduce(dok, op=dist.ReduceOp.MIN)
        total_bytes = sum(lens) * HKV * D * 2 * 2 + len(lens) * HQ * (D * 2 * 2 + R * 2)
        rank_bytes = total_bytes // world
        rank_gbs = rank_bytes / (dmed_ng / 1e3) / 1e9
        result["decode_head_sharded"] = {
            "unit": "GB/s", "scaling": "strong",
            "value_no_gather": total_bytes * steps2 / (dms_ng / 1e3) / 1e9,
            "value_with_gather": total_bytes * steps2 / (dms_g / 1e3) / 1e9,
            "us_per_step_no_gather": dms_ng * 1e3 / steps2,
            "us_per_step_with_gather": dms_g * 1e3 / steps2,
            "per_rank_gbs": rank_gbs, "per_rank_frac_of_hbm": rank_gbs / peaks["hbm_gbs"],
            "parity_ok": bool(dok.item() == 1), "max_abs_diff_vs_unsharded": ddiff,
            "config": {"workload": "decode128_u1024_32768_gqa32_8_d128_rel128",
                       "kv_heads_per_rank": sh.n_kv, "heads_per_rank": sh.n_q,
                       "num_splits": nsplit, "chunk_len": chunk,
                       "bytes_per_step_total": total_bytes,
                       "collective": "one NCCL all_gather_into_tensor of the output heads "
                                     f"({len(lens) * HQ * D * 2 >> 10} KB assembled per step)"},
            "gpu_launches": steps2 * (2 if nsplit > 1 else 1)}
        del dcs, dq, dk, dv, drel, ws, dfull, dref
        torch.cuda.empty_cache()

    # ---------------- config 5: batched decode (contiguous and paged)
    if want("decode"):
        read_gbs = read_stream_peak(dev, stream)
        dc = config_decode(device=dev, seed=rank, batch=args.decode_batch, gen_device=dev)
        lens = dc.seqlens_k
        kv_bytes = sum(lens) * HKV * D * 2 * 2
        other = len(lens) * HQ * (D * 2 * 2 + R * 2)
        dbytes = kv_bytes + other
        ws = torch.empty(64 << 20, dtype=torch.uint8, device=dev)

        def dec_step():
            return inkling_fa4_rel_attention_decode_triton(
                dc.q, dc.k, dc.v, dc.rel, dc.cu_q, dc.cu_k, 1, max(lens), R,
                causal_align="bottom_right", workspace=ws)

        p = _ops._decode_params(dc.q, dc.k, dc.v, dc.rel, dc.q, dc.cu_q, dc.cu_k, HQ, HKV, R,
                                True, -1, "bottom_right", max(lens), 1.0 / D, 0, 0)
        _, nsplit, chunk = _ops.decode_plan(p)
        dms, dmed = timed(dec_step, steps2, warm2, stream, dist, barrier)
        us = dms * 1e3 / steps2
        gbs = world * dbytes * steps2 / (dms / 1e3) / 1e9
        per_gpu = dbytes / (dmed / 1e3) / 1e9

        def hbm_roofline(achieved):
            return {"bound": "hbm", "achieved": achieved, "peak": read_gbs, "unit": "GB/s",
                    "frac": achieved / read_gbs,
                    "peak_source": "read-only stream measured in this run "
                                   "(ifa4_measure_read_stream over 4 GiB, best of 10)",
                    "frac_of_copy_peak": achieved / peaks["hbm_gbs"],
                    "copy_peak": peaks["hbm_gbs"],
                    "copy_peak_source": f"hbm_gbs (read+write copy) of {peak_kind}",
                    "frac_of_datasheet_7700": achieved / DATASHEET["hbm_gbs"]}

        # host-side cost of one call at small batch: wall clock around the Python call
        # (argument checks, ctypes, workspace planning) against the device time of the same call
        small = config_decode(device=dev, seed=rank, batch=1, gen_device=dev)
        sws = torch.empty(8 << 20, dtype=torch.uint8, device=dev)
        small_step = lambda: inkling_fa4_rel_attention_decode_triton(
            small.q, small.k, small.v, small.rel, small.cu_q, small.cu_k, 1, small.max_k, R,
            causal_align="bottom_right", workspace=sws)
        for _ in range(20):
            small_step()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(200):
            small_step()
        host_us = (time.perf_counter() - t0) / 200 * 1e6
        torch.cuda.synchronize()
        sms, smed = timed(small_step, steps2, warm2, stream)
        sgraph = graph_replay_us(small_step)
        result["decode"] = {
            "value": gbs, "unit": "GB/s", "us_per_step": us, "us_per_step_median": dmed * 1e3,
            "steps": steps2,
            "config": {"workload": "decode128_u1024_32768_gqa32_8_d128_rel128",
                       "batch": len(lens), "kv_tokens": sum(lens),
                       "causal_align": "bottom_right", "num_splits": nsplit, "chunk_len": chunk,
                       "bytes_per_step_per_gpu": dbytes},
            "roofline": dict(hbm_roofline(per_gpu),
                             traffic=(NCU_DRAM_BYTES_PER_LAUNCH["decode128"]
                                      if args.decode_batch == 128 else None),
                             traffic_note="batch-16 ncu capture scaled to batch 128 by K/V bytes"),
            "host_call_overhead_b1": {
                "host_us_per_call": host_us, "device_us_per_call_median": smed * 1e3,
                "device_us_per_call_graph_replay": sgraph,
                "kv_tokens": small.max_k,
                "note": "wall clock of 200 back-to-back Python calls (argument checks, one "
                        "torch-operator call that fills the C ABI's parameter block, plans, "
                        "allocates the workspace and makes 2 launches) vs CUDA-event device "
                        "time; the host cost hides behind the device when it is the smaller"},
            "gpu_launches": steps2 * (2 if nsplit > 1 else 1)}
        del small, sws
        # the same step against a 16-token paged cache (pages handed out in random order)
        pdc = page_kv(dc, page_size=16, seed=rank)
        del dc
        torch.cuda.empty_cache()

        def paged_step():
            return inkling_fa4_rel_attention_decode_triton(
                pdc.q, pdc.k, pdc.v, pdc.rel, pdc.cu_q, pdc.cu_k, 1, max(lens), R,
                causal_align="bottom_right", workspace=ws, block_table=pdc.meta["block_table"])

        pms, pmed = timed(paged_step, steps2, warm2, stream, dist, barrier)
        pbytes = dbytes + 4 * sum((n + 15) // 16 for n in lens)
        result["decode_paged"] = {
            "value": world * pbytes * steps2 / (pms / 1e3) / 1e9, "unit": "GB/s",
            "us_per_step": pms * 1e3 / steps2, "us_per_step_median": pmed * 1e3,
            "page_size": 16, "num_pages": pdc.meta["num_pages"],
            "bytes_per_step_per_gpu": pbytes,
            "roofline": hbm_roofline(pbytes / (pmed / 1e3) / 1e9),
            "gpu_launches": steps2 * (2 if nsplit > 1 else 1)}
        del pdc, ws
        torch.cuda.empty_cache()

    result["device_status"] = _lib.read_device_status(stream.cuda_stream)
    clocks = sampler.stop() if sampler else None
    if clocks:
        result["clocks"] = clocks

    # ---------------- CPU baselines (rank 0, N = 1): the oracle port on bounded samples
    if cpu_on:
        from inkling_fa4.workloads import decode_batch_lengths

        secs = args.cpu_seconds
        if run_headline:
            result["cpu_baseline"] = cpu_causal32k(secs)
        if "window32k" in result:
            result["window32k"]["cpu_baseline"] = cpu_causal32k(secs / 2, window=4096)
        if "ragged" in result:
            result["ragged"]["cpu_baseline"] = cpu_ragged(secs)
        if "chunked" in result:
            result["chunked"]["cpu_baseline"] = cpu_chunked(secs)
        if "config1" in result:
            result["config1"]["cpu_baseline"] = cpu_config1(secs / 3)
        if "decode" in result:
            result["decode"]["cpu_baseline"] = cpu_decode(
                secs, decode_batch_lengths(batch=args.decode_batch))

    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(result), flush=True)


if __name__ == "__main__":
    main()
