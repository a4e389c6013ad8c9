"""Tile-configuration table (drop-in for src/inkling_fa4/autotune_configs.py).

The reference maps (seq_len, arch) to Triton launch parameters (autotune_configs.py:17-85).
Here only sm_100a kernels exist, so every architecture key resolves to the sm100 table, whose
entries describe the hand-written kernels:

* prefill: two 128-row query sub-tiles per CTA (BLOCK_Q = 128 each) against 128-key KV tiles,
  12 warps (TMA, MMA, TMEM owner, spare, two softmax warpgroups), a 2-stage K and a 2-stage V
  ring; ``tile_config`` is the id passed through the C ABI.
* decode: 64-key tiles through a 3-stage TMA ring, 4 consumer warps + 1 producer warp, chunk
  length and split count chosen by the library from max_seqlen_k and the SM count
  (``ifa4_decode_workspace_size`` reports them).
"""
from __future__ import annotations

import torch

# (max_seq_len, BLOCK_Q, BLOCK_K, num_warps, num_stages, tile_config)
PRESETS = {
    "sm100": {
        "default": (128, 128, 12, 2, 0),
        "buckets": [],
    },
}

# Prefill kernel variants behind tile_config (all: two 128-row query sub-tiles per CTA, 128-key
# KV tiles, 12 warps, 2-stage K and V rings).  They differ in how many of every 16 score columns
# take their exponential from the FMA-pipe polynomial instead of the SFU.  Measured on one B200,
# bench.py --only prefill (32k causal, GQA 32/8): TFLOP/s per variant.  tile_config 0 resolves
# to the fastest.
TILE_CONFIGS = {
    0: {"note": "automatic: tile_config 2 (2 FMA-pipe exponentials of 16)"},
    1: {"emulated_exp_of_16": 0, "sfu_f16x2_of_16": 0},
    2: {"emulated_exp_of_16": 2, "sfu_f16x2_of_16": 0},
    3: {"emulated_exp_of_16": 4, "sfu_f16x2_of_16": 0},
    4: {"emulated_exp_of_16": 6, "sfu_f16x2_of_16": 0},
    5: {"emulated_exp_of_16": 8, "sfu_f16x2_of_16": 0},
    6: {"emulated_exp_of_16": 0, "sfu_f16x2_of_16": 16},
    7: {"emulated_exp_of_16": 0, "sfu_f16x2_of_16": 8},
    8: {"emulated_exp_of_16": 4, "sfu_f16x2_of_16": 8},
}
# Interleaved A/B on one B200 (5 rounds, medians), GQA 32/8, R = 128, TFLOP/s, with interior
# tiles taking their exponentials against the running max (no row-max pass):
#   causal 32k:   tc1 1034.6  tc2 1039.8  tc3 993.5  tc7 1011.7  tc8 973.5
#   window 4096:  tc1  863.3  tc2  894.2  tc3 862.8  tc7  859.2  tc8 850.0
#   ragged (config 2): tc1 597.3  tc2 606.6  tc3 585.1  tc7 598.0  tc8 563.7
# Paged caches: tile configs 0 to 3.
DECODE_PRESET = {"BLOCK_K": 64, "num_warps": 5, "num_stages": 3, "chunk_len": 0, "num_splits": 0}


def _detect_arch() -> str:
    """Compute-capability key of the current GPU, e.g. 'sm100' (reference :53-58)."""
    if not torch.cuda.is_available():
        return "sm100"
    cap = torch.cuda.get_device_capability()
    return f"sm{cap[0]}{cap[1]}"


def get_preset(seq_len: int, arch: str | None = None) -> dict:
    """Tile configuration for a query length (reference :61-85).  Every arch resolves to sm100."""
    table = PRESETS["sm100"]
    entry = table["default"]
    for bucket in table["buckets"]:
        if seq_len <= bucket[0]:
            entry = bucket[1:]
            break
    bq, bk, nw, ns, tc = entry
    if seq_len == 1:
        return dict(DECODE_PRESET, BLOCK_Q=1)
    return {"BLOCK_Q": bq, "BLOCK_K": bk, "num_warps": nw, "num_stages": ns, "tile_config": tc}


get_config = get_preset  # name used in the reference module docstring
