#!/usr/bin/env python
"""Benchmark of the relative-bias flash-attention hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...      (one rank per GPU, NCCL)

Headline (``value``): prefill TFLOP/s on the 32k causal GQA 32/8, d=128, R=128 configuration
(full causal), aggregated over all ranks.  A "step" is one prefill call over
one 32768-token sequence with all 32 query heads.  FLOPs are algorithmic:
4 * head_dim * n_heads * (causally visible query/key pairs), the bias gather and masking
excluded.  Scaling is weak: every rank owns an independent 32k sequence (work shards by
sequence / KV-head group with no data-path collective); ``value`` = all ranks' FLOPs / the
slowest rank's time.

Secondary objects in the same JSON line: the sliding-window variant (window 4096), the backward,
the rel_logits producer for the headline shape (GB/s against HBM), batched
decode (GB/s and us/step against HBM), the end-to-end number through the
public API with host buffers (``e2e``), the CPU baseline (the oracle on host cores, bounded
sample) and SM clocks sampled during the timed region.

``--impl reference`` times the reference's algorithm on the host CPU (the oracle port; the
reference itself is a Python/Triton package whose CPU path is the torch oracle ref_rel_attn),
on bounded samples of the same workload; rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "inkling-fa4-relative-attention_b200"))
sys.path.insert(0, ROOT)

METRIC = "prefill TFLOP/s at 32k GQA 32/8 d128 bf16; decode HBM GB/s & us/step"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
SEQ, HQ, HKV, D, R = 32768, 32, 8, 128, 128


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            j = json.load(f)
        return {k: float(j[k]) for k in FALLBACK_PEAKS}, "measured"
    return dict(FALLBACK_PEAKS), "fallback"


def profile_traffic(name):
    """dram bytes per launch recorded from an ncu capture in profiles/<name> (a line
    'dram_bytes_per_launch_full: <int>'), or None."""
    p = os.path.join(ROOT, "profiles", name)
    if not os.path.exists(p):
        return None
    for line in open(p):
        if line.startswith("dram_bytes_per_launch_full:"):
            try:
                return int(float(line.split(":", 1)[1].strip()))
            except ValueError:
                return None
    return None


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
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed region."""

    FIELDS = ("index,uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, uuids):
        self.uuids = [u.lower() for u in uuids]
        self.proc = None
        self.lines = []

    def _drain(self):
        for line in self.proc.stdout:
            self.lines.append(line)

    def start(self):
        import threading
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.reader = threading.Thread(target=self._drain, daemon=True)
            self.reader.start()
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
        sm = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        smax = [float(r[3]) for r in rows if r[3].replace(".", "").isdigit()]
        pw = [float(r[4]) for r in rows if r[4].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[6 + i].lower() == "active"})
        loaded = [s for s, p in zip(sm, pw) if p > 300] or sm
        return {"sm_mhz": statistics.median(loaded) if loaded else None,
                "sm_max_mhz": max(smax) if smax else None, "reasons": reasons,
                "samples": len(rows), "power_w_max": max(pw) if pw else None}


# ---------------------------------------------------------------------------------------
def cpu_baseline_prefill(seconds, window=None, threads=None):
    """The oracle (torch twin of reference.py's algorithm, all host threads) on a bounded
    sample of the 32k workload: one head, 128-row blocks spread over the sequence, each row
    scored densely against all keys as the reference does.  Returns (TFLOP/s, cores, sample)."""
    import torch

    import oracle
    from inkling_fa4.workloads import make_case

    threads = threads or os.cpu_count() or 1
    torch.set_num_threads(threads)
    c = make_case([SEQ], [SEQ], 1, 1, R, seed=123, rel_std=0.5)
    q, k, v, rel = (t[:, 0].float().contiguous() for t in (c.q, c.k, c.v, c.rel))
    blk = 128
    order = [((i * 97) % (SEQ // blk)) * blk for i in range(SEQ // blk)]
    flops, t_used, rows = 0, 0.0, 0
    for r0 in order:
        t0 = time.perf_counter()
        oracle.rel_attn_rows_torch(q[r0:r0 + blk], k, v, rel[r0:r0 + blk],
                                   torch.arange(r0, r0 + blk), SEQ, SEQ, 1.0 / D, R, True,
                                   window, "reference")
        t_used += time.perf_counter() - t0
        for i in range(r0, r0 + blk):
            lo = 0 if window is None else max(0, i - window)
            flops += 4 * D * (i + 1 - lo)
        rows += blk
        if t_used >= seconds:
            break
    sample = (f"1 of {HQ} heads, {rows} of {SEQ} query rows ({rows // blk} blocks of {blk} "
              f"spread over the sequence), dense scores against all {SEQ} keys as reference.py "
              "computes them; algorithmic causal FLOPs")
    return flops / t_used / 1e12, threads, sample


def run_reference_arm(args, rank, world):
    if rank != 0:
        return
    import torch

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    import oracle
    from inkling_fa4.workloads import make_case

    c = make_case([SEQ], [SEQ], 1, 1, R, seed=123, rel_std=0.5)
    q, k, v, rel = (t[:, 0].float().contiguous() for t in (c.q, c.k, c.v, c.rel))
    blk = 64
    positions = [((i * 97) % (SEQ // blk)) * blk for i in range(SEQ // blk)]

    def step(i):
        r0 = positions[i % len(positions)]
        oracle.rel_attn_rows_torch(q[r0:r0 + blk], k, v, rel[r0:r0 + blk],
                                   torch.arange(r0, r0 + blk), SEQ, SEQ, 1.0 / D, R, True, None,
                                   "reference")
        return sum(4 * D * (j + 1) for j in range(r0, r0 + blk))

    for i in range(args.warmup):
        step(i)
    flops, t0 = 0, time.perf_counter()
    for i in range(args.steps):
        flops += step(args.warmup + i)
    dt = time.perf_counter() - t0
    value = flops / dt / 1e12
    sample = (f"per step: 1 of {HQ} heads x {blk} query rows of the 32k causal sequence, dense "
              f"scores against all {SEQ} keys (reference.py's algorithm, oracle port, torch CPU, "
              f"{threads} threads); algorithmic causal FLOPs")
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
    import torch

    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    if barrier:
        barrier()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(steps):
        fn()
    end.record(stream)
    torch.cuda.synchronize()
    if barrier:
        barrier()
    ms = start.elapsed_time(end)
    if dist is not None:
        t = torch.tensor([ms], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    return ms


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-decode", action="store_true")
    ap.add_argument("--no-window", action="store_true")
    ap.add_argument("--no-backward", action="store_true")
    ap.add_argument("--no-rel-logits", action="store_true")
    ap.add_argument("--no-shard", action="store_true",
                    help="skip the head-sharded single-sequence leg (N > 1 only)")
    ap.add_argument("--extra-configs", action="store_true",
                    help="also time BASELINE configs 2 (ragged) and 4 (chunked)")
    ap.add_argument("--only", choices=["all", "prefill", "decode", "rel_logits"], default="all",
                    help="prefill: headline + window only; decode: decode only; rel_logits: the "
                         "producer only (profiling runs)")
    ap.add_argument("--prefill-seq", type=int, default=SEQ,
                    help="sequence length of the prefill workload (32768 = BASELINE config 3)")
    ap.add_argument("--tile-config", type=int, default=0,
                    help="prefill kernel variant (0 = default; see autotune_configs)")
    ap.add_argument("--decode-batch", type=int, default=128,
                    help="decode batch (128 = BASELINE config 5)")
    args = ap.parse_args()
    if args.only == "prefill":
        args.no_decode = args.no_rel_logits = args.no_shard = True
    if args.only == "decode":
        args.no_e2e = args.no_window = args.no_backward = args.no_rel_logits = True
        args.no_shard = True
    if args.only == "rel_logits":
        args.no_e2e = args.no_window = args.no_backward = args.no_decode = True
        args.no_shard = True
    if args.warmup < 3:
        args.warmup = 3

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

    from inkling_fa4 import (_lib, inkling_fa4_rel_attention_decode_triton,
                             inkling_fa4_rel_attention_triton)
    from inkling_fa4.workloads import config_decode, config_long

    peaks, peak_kind = load_peaks()
    dev = torch.device("cuda", local_rank)
    stream = torch.cuda.current_stream(dev)

    # ---------------- headline: 32k causal prefill, inputs resident in HBM
    S = args.prefill_seq
    c = config_long(device=dev, seed=rank, seq=S, gen_device=dev)
    flops = 4 * D * HQ * visible_pairs_causal(S)

    from inkling_fa4 import _ops

    def prefill_call(*pa, **kw):
        """The public prefill entry point, or the same call pinned to --tile-config (for tile
        sweeps; applies to the headline, window, ragged and chunked legs)."""
        if args.tile_config:
            return _ops.prefill(*pa, tile_config=args.tile_config, **kw)
        return inkling_fa4_rel_attention_triton(*pa, **kw)

    def prefill_step():
        return prefill_call(c.q, c.k, c.v, c.rel, c.cu_q, c.cu_k, S, S, R)

    uuids = []
    try:
        uuids = [str(torch.cuda.get_device_properties(dev).uuid)]
    except Exception:
        pass
    sampler = ClockSampler(uuids) if rank == 0 else None
    if args.only in ("decode", "rel_logits"):
        ms, clocks = float("nan"), None
    else:
        if sampler:
            sampler.start()
        ms = timed(prefill_step, args.steps, args.warmup, stream, dist, barrier)
        clocks = sampler.stop() if sampler else None
    ms_step = ms / args.steps
    value = world * flops * args.steps / (ms / 1e3) / 1e12
    achieved = flops / (ms_step / 1e3) / 1e12
    status = _lib.read_device_status(stream.cuda_stream)

    result = {
        "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
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
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peaks["bf16_tflops"],
                     "unit": "TFLOP/s", "frac": achieved / peaks["bf16_tflops"],
                     "peak_source": f"bf16_tflops (burst) of {peak_kind}",
                     "frac_of_sustained": achieved / peaks["bf16_tflops_sustained"],
                     "frac_of_datasheet_2250": achieved / 2250.0,
                     "traffic": profile_traffic("prefill_dram_traffic.md") if S == SEQ else None,
                     "traffic_note": "one-pass ncu capture of the 32k launch "
                                     "(profiles/prefill_dram_traffic.md)",
                     "kernel": "rel_attn_prefill_kernel (1 launch per step)",
                     "tile_config": args.tile_config},
        "gpu_launches": args.steps,
        "device_status": status,
    }
    if clocks:
        result["clocks"] = clocks

    # ---------------- end to end through the public API with host buffers
    # Every step uploads its own inputs from pinned host memory, runs the public API call and
    # downloads its output to pinned host memory.  Three streams and two buffer sets let the
    # upload of step i+1 and the download of step i-1 overlap the kernel of step i, as a
    # serving pipeline would; the timed region spans the first upload to the last download.
    if not args.no_e2e:
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

    # ---------------- sliding window 4096 at 32k (BASELINE config 3b)
    if not args.no_window:
        wflops = 4 * D * HQ * visible_pairs_causal(S, 4096)

        def win_step():
            return prefill_call(c.q, c.k, c.v, c.rel, c.cu_q, c.cu_k, S, S, R,
                                window_size=(4096, 0))

        wms = timed(win_step, args.steps, args.warmup, stream, dist, barrier)
        result["window32k"] = {"value": world * wflops * args.steps / (wms / 1e3) / 1e12,
                               "unit": "TFLOP/s", "ms_per_step": wms / args.steps,
                               "window_left": 4096, "flops_per_step_per_gpu": wflops}

    # ---------------- backward of the headline prefill (not in the reference)
    if not args.no_backward:
        from inkling_fa4 import inkling_fa4_rel_attention_backward

        bout, blse = inkling_fa4_rel_attention_triton(c.q, c.k, c.v, c.rel, c.cu_q, c.cu_k, S, S,
                                                      R, return_lse=True)
        gen = torch.Generator(device=dev)
        gen.manual_seed(1000 + rank)
        bdout = torch.randn(c.q.shape, generator=gen, device=dev).to(torch.bfloat16)
        bws = torch.empty(HQ * S * 4, dtype=torch.uint8, device=dev)
        bufs = (torch.empty_like(c.q), torch.empty_like(c.k), torch.empty_like(c.v),
                torch.empty_like(c.rel))

        def bwd_step():
            return inkling_fa4_rel_attention_backward(
                bdout, c.q, c.k, c.v, c.rel, bout, blse, c.cu_q, c.cu_k, S, S, R, dq=bufs[0],
                dk=bufs[1], dv=bufs[2], drel=bufs[3], workspace=bws)

        bsteps = max(5, args.steps // 5)
        bms = timed(bwd_step, bsteps, args.warmup, stream, dist, barrier)
        bflops = 2.5 * flops  # 5 matrix products of the forward's size (the usual convention)
        result["backward32k"] = {
            "value": world * bflops * bsteps / (bms / 1e3) / 1e12, "unit": "TFLOP/s",
            "ms_per_step": bms / bsteps, "steps": bsteps,
            "flops_per_step_per_gpu": bflops,
            "flops_note": "algorithmic 2.5x forward (S, dP, dV, dK, dQ); the kernels execute "
                          "3.5x (S and dP are recomputed by the dQ kernel to avoid atomics)",
            "kernels": "rel_attn_bwd_prep_kernel, rel_attn_bwd_dkdv_kernel, "
                       "rel_attn_bwd_dq_kernel (3 launches per step)",
            "gpu_launches": 3 * bsteps}
        del bout, blse, bdout, bws, bufs

    # ---------------- rel_logits producer for the headline shape (the step before the path)
    if not args.no_rel_logits:
        from inkling_fa4 import inkling_rel_logits

        gen = torch.Generator(device=dev)
        gen.manual_seed(2000 + rank)
        rr = torch.randn((S, HQ, 16), generator=gen, device=dev).to(torch.bfloat16)
        rw = (0.5 * torch.randn((HQ, 16, R), generator=gen, device=dev)).to(torch.bfloat16)
        rout = torch.empty((S, HQ, R), dtype=torch.bfloat16, device=dev)

        def rl_step():
            return inkling_rel_logits(rr, rw, alpha=0.1, nf=4096.0, out=rout)

        rms = timed(rl_step, args.steps, args.warmup, stream, dist, barrier)
        rbytes = rr.numel() * 2 + rw.numel() * 2 + rout.numel() * 2
        rgbs = rbytes * args.steps / (rms / 1e3) / 1e9
        # Write-stream reference on the same box: torch's fill_ of the same output buffer, same
        # protocol (the producer's traffic is 89 % writes; a plain write stream reaches well
        # below the read+write copy peak).
        fms = timed(lambda: rout.fill_(1.0), args.steps, args.warmup, stream, dist, barrier)
        fill_gbs = rout.numel() * 2 * args.steps / (fms / 1e3) / 1e9
        write_gbs = rout.numel() * 2 * args.steps / (rms / 1e3) / 1e9
        result["rel_logits32k"] = {
            "value": world * rgbs, "unit": "GB/s", "us_per_step": rms * 1e3 / args.steps,
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
                         "traffic": (profile_traffic("rel_logits_32k_ncu.md")
                                     if S == SEQ else None),
                         "traffic_note": "one cold ncu launch: reads + writes performed before "
                                         "it ended (54 MB of output still dirty in L2)"},
            "kernel": "rel_logits_kernel (1 launch per step)", "gpu_launches": args.steps}
        del rr, rw, rout
    del c
    torch.cuda.empty_cache()

    # ---------------- one 32k sequence sharded by KV-head group over the ranks (N > 1 only)
    # Strong scaling of a single call: rank r runs the heads of kv groups [r*8/N, (r+1)*8/N) of
    # the same sequence (head-slice views, no copies), timed without and with the NCCL
    # all-gather that assembles the [T, 32, 128] output on every rank.
    if world > 1 and not args.no_shard and HKV % world == 0:
        from inkling_fa4.sharding import gather_heads, head_shard, shard_tensors

        sc = config_long(device=dev, seed=0, seq=S, gen_device=dev)  # same sequence on all ranks
        sh = head_shard(HQ, HKV, world, rank)
        q_s, k_s, v_s, rel_s = shard_tensors(sh, sc.q, sc.k, sc.v, sc.rel)
        shard_step = lambda: inkling_fa4_rel_attention_triton(q_s, k_s, v_s, rel_s, sc.cu_q,
                                                               sc.cu_k, S, S, R)
        gather_step = lambda: gather_heads(shard_step(), world)
        ms_ng = timed(shard_step, args.steps, args.warmup, stream, dist, barrier)
        ms_g = timed(gather_step, args.steps, args.warmup, stream, dist, barrier)
        full_flops = 4 * D * HQ * visible_pairs_causal(S)
        result["head_sharded32k"] = {
            "unit": "TFLOP/s", "scaling": "strong",
            "value_no_gather": full_flops * args.steps / (ms_ng / 1e3) / 1e12,
            "value_with_gather": full_flops * args.steps / (ms_g / 1e3) / 1e12,
            "ms_per_step_no_gather": ms_ng / args.steps,
            "ms_per_step_with_gather": ms_g / args.steps,
            "config": {"workload": "causal32k_gqa32_8_d128_rel128, one sequence",
                       "heads_per_rank": sh.n_q, "kv_heads_per_rank": sh.n_kv,
                       "collective": "one NCCL all_gather_into_tensor of the output heads "
                                     f"({S * HQ * D * 2 >> 20} MB assembled per step)"},
            "gpu_launches": args.steps}
        del sc, q_s, k_s, v_s, rel_s
        torch.cuda.empty_cache()

    # ---------------- ragged (config 2) and chunked (config 4) prefill, on request
    if args.extra_configs:
        from inkling_fa4.workloads import (causal_visible_pairs, config_chunked, config_ragged,
                                           page_kv)

        for name, make, align in (("ragged", config_ragged, "reference"),
                                  ("chunked", config_chunked, "bottom_right")):
            cc = make(device=dev, seed=rank, gen_device=dev)
            fl = 4 * D * HQ * causal_visible_pairs(cc.seqlens_q, cc.seqlens_k,
                                                   causal_align=align)

            def step(cc=cc, align=align):
                return prefill_call(cc.q, cc.k, cc.v, cc.rel, cc.cu_q, cc.cu_k, cc.max_q,
                                    cc.max_k, R, causal_align=align)

            xms = timed(step, args.steps, args.warmup, stream, dist, barrier)
            result[name] = {"value": world * fl * args.steps / (xms / 1e3) / 1e12,
                            "unit": "TFLOP/s", "ms_per_step": xms / args.steps,
                            "flops_per_step_per_gpu": fl, "causal_align": align,
                            "seqlens_q": cc.seqlens_q if name == "ragged" else None}
            if name == "chunked":  # the same chunks against a 16-token paged cache
                pc = page_kv(cc, page_size=16, seed=rank)
                del cc

                # paged caches exist for tile configs 0 to 3; other sweep values run the default
                paged_call = prefill_call if args.tile_config <= 3 else \
                    inkling_fa4_rel_attention_triton

                def pstep(pc=pc):
                    return paged_call(
                        pc.q, pc.k, pc.v, pc.rel, pc.cu_q, pc.cu_k, pc.max_q, pc.max_k, R,
                        causal_align="bottom_right", block_table=pc.meta["block_table"])

                pms = timed(pstep, args.steps, args.warmup, stream, dist, barrier)
                result["chunked_paged"] = {
                    "value": world * fl * args.steps / (pms / 1e3) / 1e12, "unit": "TFLOP/s",
                    "ms_per_step": pms / args.steps, "flops_per_step_per_gpu": fl,
                    "page_size": 16, "num_pages": pc.meta["num_pages"]}
                cc = pc
            del cc
        torch.cuda.empty_cache()

    # ---------------- batched decode
    if not args.no_decode:
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

        from inkling_fa4 import _ops
        p = _ops._decode_params(dc.q, dc.k, dc.v, dc.rel, dc.q, dc.cu_q, dc.cu_k, HQ, HKV, R,
                                True, -1, "bottom_right", max(lens), 1.0 / D, 0, 0)
        _, nsplit, chunk = _ops.decode_plan(p)
        dms = timed(dec_step, args.steps, args.warmup, stream, dist, barrier)
        us = dms * 1e3 / args.steps
        gbs = world * dbytes * args.steps / (dms / 1e3) / 1e9
        per_gpu = dbytes / (us / 1e6) / 1e9
        result["decode"] = {
            "value": gbs, "unit": "GB/s", "us_per_step": us,
            "config": {"workload": "decode128_u1024_32768_gqa32_8_d128_rel128",
                       "batch": len(lens), "kv_tokens": sum(lens),
                       "causal_align": "bottom_right", "num_splits": nsplit, "chunk_len": chunk,
                       "bytes_per_step_per_gpu": dbytes},
            "roofline": {"bound": "hbm", "achieved": per_gpu, "peak": peaks["hbm_gbs"],
                         "unit": "GB/s", "frac": per_gpu / peaks["hbm_gbs"],
                         "peak_source": f"hbm_gbs of {peak_kind}",
                         "traffic": (profile_traffic("decode_dram_traffic.md")
                                     if args.decode_batch == 128 else None)},
            "gpu_launches": args.steps * (2 if nsplit > 1 else 1)}
        # the same step against a 16-token paged cache (pages handed out in random order)
        from inkling_fa4.workloads import page_kv
        pdc = page_kv(dc, page_size=16, seed=rank)
        del dc
        torch.cuda.empty_cache()

        def paged_step():
            return inkling_fa4_rel_attention_decode_triton(
                pdc.q, pdc.k, pdc.v, pdc.rel, pdc.cu_q, pdc.cu_k, 1, max(lens), R,
                causal_align="bottom_right", workspace=ws, block_table=pdc.meta["block_table"])

        pms = timed(paged_step, args.steps, args.warmup, stream, dist, barrier)
        pus = pms * 1e3 / args.steps
        result["decode_paged"] = {
            "value": world * dbytes * args.steps / (pms / 1e3) / 1e9, "unit": "GB/s",
            "us_per_step": pus, "page_size": 16, "num_pages": pdc.meta["num_pages"],
            "frac": dbytes / (pus / 1e6) / 1e9 / peaks["hbm_gbs"],
            "bytes_per_step_per_gpu": dbytes + 4 * sum((n + 15) // 16 for n in lens)}
        dc = pdc
        del dc, ws
        torch.cuda.empty_cache()

    result["device_status"] = _lib.read_device_status(stream.cuda_stream)

    # ---------------- CPU baseline (rank 0, N = 1)
    if rank == 0 and world == 1 and not args.no_cpu_baseline and args.only == "all":
        v, cores, sample = cpu_baseline_prefill(args.cpu_seconds)
        result["cpu_baseline"] = {"value": v, "unit": "TFLOP/s", "cores": cores, "kind": "port",
                                  "sample": sample}

    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(result), flush=True)


if __name__ == "__main__":
    main()
