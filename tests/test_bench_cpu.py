"""bench.py's host-side pieces that need no GPU: the algorithmic FLOP count of the headline
configurations, and the stdout guard that keeps NCCL's C-level banner off rank 0's JSON line."""
import os
import subprocess
import sys

import bench
from inkling_fa4.workloads import causal_visible_pairs

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_visible_pairs_match_the_workload_counter():
    # 32k causal and the 4096 window (BASELINE config 3a / 3b), and small edge cases
    for seq, window in ((32768, None), (32768, 4096), (1, None), (5000, 4096), (4097, 4096)):
        want = causal_visible_pairs([seq], [seq], window_left=window)
        assert bench.visible_pairs_causal(seq, window) == want, (seq, window)
    assert 4 * 128 * 32 * bench.visible_pairs_causal(32768) == 8796361457664


def test_c_level_stdout_goes_to_stderr_inside_the_guard():
    code = (
        "import ctypes, sys\n"
        f"sys.path.insert(0, {REPO!r})\n"
        "import bench\n"
        "libc = ctypes.CDLL(None)\n"
        "with bench.c_stdout_to_stderr():\n"
        "    libc.printf(b'NCCL version banner\\n')\n"
        "    print('python inside')\n"
        "print('{\"metric\": 1}')\n")
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    assert r.stdout.strip().splitlines() == ['{"metric": 1}']
    assert "NCCL version banner" in r.stderr and "python inside" in r.stderr


def test_recorded_profile_commands_parse_to_the_legs_they_ran():
    """The capture commands kept with the ncu summaries use the earlier --no-<leg> and
    --only prefill spellings; they still select the same legs."""
    args, skip, headline = bench.parse_args(
        "--steps 5 --warmup 3 --no-e2e --no-cpu-baseline --no-decode --no-window --no-backward "
        "--no-rel-logits".split())
    assert headline and args.no_cpu_baseline and args.steps == 5
    assert {"e2e", "decode", "window", "backward", "rel_logits"} <= skip
    args, skip, headline = bench.parse_args(
        "--only prefill --prefill-seq 8192 --steps 2 --warmup 3 --no-e2e --no-window".split())
    assert headline and args.prefill_seq == 8192 and skip == set(bench.LEGS)
    args, skip, headline = bench.parse_args([])
    assert headline and not skip and args.warmup == 5
    args, skip, headline = bench.parse_args(["--only", "decode"])
    assert not headline and skip == set(bench.LEGS) - {"decode"}
