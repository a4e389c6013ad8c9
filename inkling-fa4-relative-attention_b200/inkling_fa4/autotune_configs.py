"""Tile-configuration table (drop-in for src/inkling_fa4/autotune_configs.py).

The reference maps (seq_len, arch) to Triton launch parameters (autotune_configs.py:17-85),
tuned by a grid search on an RTX 3090 (benchmarks/autotune.py).  Here only sm_100a kernels
exist, so every architecture key resolves to the sm100 table, whose entries describe the
hand-written kernels:

* prefill: two 128-row query sub-tiles per CTA (BLOCK_Q = 128 each) against 128-key KV tiles,
  12 warps (TMA, MMA, TMEM owner, spare, two softmax warpgroups), a 2-stage K and a 2-stage V
  ring; ``tile_config`` is the id passed through the C ABI.  The variants differ only in where
  the exponentials of the single-pass interior tiles run.
* decode: 64-key tiles through a 3-stage TMA ring, 4 consumer warps + 1 producer warp, chunk
  length and split count chosen by the library from max_seqlen_k and the SM count
  (``ifa4_decode_workspace_size`` reports them).

Every number below was measured on one B200 of this build's pool: TFLOP/s (algorithmic FLOPs /
median step, two interleaved repetitions of ``python -m inkling_fa4.tune``) and the tensor pipe's
active fraction of the same launches (ncu ``sm__pipe_tensor_cycles_active``, one pass).
"""
from __future__ import annotations

import torch

# Prefill variants behind tile_config: how many of every 16 score columns of a single-pass
# interior tile take their exponential from the FMA-pipe polynomial / the SFU in f16x2 instead of
# the SFU in fp32.  tile_config 0 resolves to the measured best, 2.
TILE_CONFIGS = {
    0: {"note": "automatic: tile_config 2"},
    1: {"emulated_exp_of_16": 0, "sfu_f16x2_of_16": 0},
    2: {"emulated_exp_of_16": 2, "sfu_f16x2_of_16": 0},
    3: {"emulated_exp_of_16": 4, "sfu_f16x2_of_16": 0},
    4: {"emulated_exp_of_16": 6, "sfu_f16x2_of_16": 0},
    5: {"emulated_exp_of_16": 8, "sfu_f16x2_of_16": 0},
    6: {"emulated_exp_of_16": 0, "sfu_f16x2_of_16": 16},
    7: {"emulated_exp_of_16": 0, "sfu_f16x2_of_16": 8},
    8: {"emulated_exp_of_16": 4, "sfu_f16x2_of_16": 8},
}

# Per workload: the chosen tile_config and the measurements behind it: TFLOP/s per variant (mean
# of two interleaved repetitions; variants within about 2 % are run-to-run noise) and the tensor
# pipe's active percentage of the elapsed cycles (ncu, mean over three launches).
# Workloads: 32k tokens, GQA 32/8, d = 128; R = rel_extent.
WORKLOAD_TABLE = {
    "causal":            {"tile_config": 0, "tflops": {0: 1064.2, 1: 1045.8, 2: 1048.6, 3: 1032.5, 7: 1022.6},
                         "tensor_pipe_pct": {0: 57.4, 1: 56.0, 2: 57.4, 3: 56.2, 7: 54.8}},
    "window4096":        {"tile_config": 0, "tflops": {0: 894.5, 1: 881.0, 2: 877.2, 3: 860.5, 7: 865.8},
                         "tensor_pipe_pct": {0: 47.3, 1: 46.9, 2: 47.3, 3: 47.1, 7: 45.9}},
    "global_rel1024":    {"tile_config": 0, "tflops": {0: 910.9, 1: 907.1, 2: 912.0, 3: 894.6, 7: 884.3},
                         "tensor_pipe_pct": {0: 47.2, 1: 46.4, 2: 47.3, 3: 46.3, 7: 44.8}},
    "local_rel512_w511": {"tile_config": 0, "tflops": {0: 222.7, 1: 226.9, 2: 216.1, 3: 216.9, 7: 229.6},
                         "tensor_pipe_pct": {0: 13.7, 1: 13.8, 2: 13.7, 3: 13.7, 7: 13.9}},
    "ragged":            {"tile_config": 0, "tflops": {0: 660.5, 1: 661.5, 2: 639.8, 3: 648.2, 7: 651.8},
                         "tensor_pipe_pct": {0: 33.0, 1: 32.9, 2: 33.1, 3: 32.5, 7: 32.2}},
    "chunked":           {"tile_config": 0, "tflops": {0: 1026.0, 1: 1018.2, 2: 1025.3, 3: 1005.6, 7: 1002.1},
                         "tensor_pipe_pct": {0: 56.0, 1: 54.6, 2: 56.1, 3: 55.0, 7: 53.5}},
}
# Reading: the variants only change the interior tiles, so on band-tile-bound workloads
# (local_rel512_w511: every tile carries bias) they differ by noise alone; where interior tiles
# dominate, 2 FMA-pipe exponentials of 16 (tile_config 2 = 0) lead or tie, and 4 of 16 or the
# f16x2 mixes trail by 1-4 %.  No workload has a variant ahead by more than the noise, so the
# automatic choice is the same for all of them.

# (max_seq_len, BLOCK_Q, BLOCK_K, num_warps, num_stages, tile_config), as in the reference's
# PRESETS layout; one kernel shape serves every length on sm_100a.
PRESETS = {
    "sm100": {
        "default": (128, 128, 12, 2, 0),
        "buckets": [
            (4096, 128, 128, 12, 2, 0),    # the reference benchmark's 4k shape: 0.113 ms
            (32768, 128, 128, 12, 2, 0),   # 1087 TFLOP/s causal
        ],
        "workloads": WORKLOAD_TABLE,
    },
}

# Decode (batch 128, K/V lengths U[1024, 32768], GQA 32/8): 6950 GB/s of
# algorithmic bytes, 0.98 of the read-only HBM stream measured in the same run (7126 GB/s) and
# 1.06 of the read+write copy peak; 16-token paged cache 6555 GB/s.
DECODE_PRESET = {"BLOCK_K": 64, "num_warps": 5, "num_stages": 3, "chunk_len": 0, "num_splits": 0,
                 "measured_gbs": 6950.0, "measured_frac_of_read_stream": 0.98}


def _detect_arch() -> str:
    """Compute-capability key of the current GPU, e.g. 'sm100' (reference :53-58)."""
    if not torch.cuda.is_available():
        return "sm100"
    cap = torch.cuda.get_device_capability()
    return f"sm{cap[0]}{cap[1]}"


def get_preset(seq_len: int, arch: str | None = None, workload: str | None = None) -> dict:
    """Tile configuration for a query length (reference :61-85).  Every arch resolves to sm100.
    ``workload`` (a key of WORKLOAD_TABLE) selects that workload's measured choice."""
    table = PRESETS["sm100"]
    if seq_len == 1:
        return dict(DECODE_PRESET, BLOCK_Q=1)
    entry = table["default"]
    for bucket in table["buckets"]:
        if seq_len <= bucket[0]:
            entry = bucket[1:]
            break
    bq, bk, nw, ns, tc = entry
    if workload is not None:
        if workload not in table["workloads"]:
            raise KeyError(f"unknown workload {workload!r}; one of {sorted(table['workloads'])}")
        tc = table["workloads"][workload]["tile_config"]
    return {"BLOCK_Q": bq, "BLOCK_K": bk, "num_warps": nw, "num_stages": ns, "tile_config": tc}


get_config = get_preset  # name used in the reference module docstring
