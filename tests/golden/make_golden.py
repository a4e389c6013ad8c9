"""Generate golden fixtures by running the reference's own oracle ``ref_rel_attn``.

Run in a container that has the reference checkout:

    python tests/golden/make_golden.py --reference <reference checkout>

It imports ``src/inkling_fa4/reference.py`` by file path (that file needs only torch), builds
seeded inputs with ``inkling_fa4.workloads.make_case``, and stores, per case, the metadata
needed to rebuild the inputs, float64 checksums of those inputs (to detect generator drift),
and the reference output.  Cases follow the reference test-suite
(tests/test_correctness.py:22-75: prefill_basic S in {64,128}, ragged [64,33,17], long_ctx
512/R=128, sliding_window 128/R=64/W=63, chunked 128x256, decode 1x128, each for head
configurations (4,4) and (8,2)) plus edge cases: fp32 inputs, a non-causal run, a window
without causal masking, a zero-length sequence, a key set shorter than the queries, a
stride-0 per-head bias table and the 1/sqrt(d) scale of the CPU benchmark configuration.

bf16-input cases store the bf16 output bits exactly as the reference returns them
(``out = zeros_like(q)``); fp32-input cases store float32.
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(REPO, "inkling-fa4-relative-attention_b200"))

from inkling_fa4.workloads import make_case  # noqa: E402

HEAD_CONFIGS = [(4, 4), (8, 2)]


def golden_cases():
    """(name, spec) pairs.  spec keys: sq, sk (lists), heads, rel_extent, seed, scale,
    causal, window_left, dtype ('bf16'|'f32'), rel_std, per_head_table."""
    cases = []
    for (hq, hkv) in HEAD_CONFIGS:
        tag = f"h{hq}_{hkv}"
        for s in (64, 128):
            cases.append((f"prefill_basic_s{s}_{tag}", dict(sq=[s], sk=[s], heads=(hq, hkv), rel_extent=1024)))
        cases.append((f"ragged_{tag}", dict(sq=[64, 33, 17], sk=[64, 33, 17], heads=(hq, hkv), rel_extent=1024)))
        cases.append((f"long_ctx_{tag}", dict(sq=[512], sk=[512], heads=(hq, hkv), rel_extent=128)))
        cases.append((f"sliding_window_{tag}", dict(sq=[128], sk=[128], heads=(hq, hkv), rel_extent=64, window_left=63)))
        cases.append((f"chunked_{tag}", dict(sq=[128], sk=[256], heads=(hq, hkv), rel_extent=1024)))
        cases.append((f"decode_{tag}", dict(sq=[1], sk=[128], heads=(hq, hkv), rel_extent=1024)))
    # fp32-input cases pin the restatement more tightly than bf16 output rounding allows
    cases.append(("f32_ragged_h8_2", dict(sq=[70, 1, 129], sk=[70, 1, 129], heads=(8, 2), rel_extent=96, dtype="f32")))
    cases.append(("f32_window_h4_4", dict(sq=[200], sk=[200], heads=(4, 4), rel_extent=32, window_left=40, dtype="f32")))
    cases.append(("f32_chunked_h4_1", dict(sq=[48], sk=[160], heads=(4, 1), rel_extent=200, dtype="f32")))
    # edge cases (bf16)
    cases.append(("noncausal_h4_2", dict(sq=[100], sk=[100], heads=(4, 2), rel_extent=128, causal=False)))
    cases.append(("window_noncausal_h4_2", dict(sq=[130], sk=[130], heads=(4, 2), rel_extent=128, causal=False, window_left=20)))
    cases.append(("zero_len_seq_h4_4", dict(sq=[40, 0, 25], sk=[40, 0, 25], heads=(4, 4), rel_extent=64)))
    cases.append(("sq_gt_sk_h4_4", dict(sq=[96], sk=[64], heads=(4, 4), rel_extent=128)))
    cases.append(("gqa32_8_s160", dict(sq=[160], sk=[160], heads=(32, 8), rel_extent=128, rel_std=0.5)))
    cases.append(("per_head_table_h4_4", dict(sq=[200], sk=[200], heads=(4, 4), rel_extent=128, per_head_table=True, rel_std=0.5)))
    cases.append(("cpu_config1_f32", dict(sq=[128], sk=[128], heads=(4, 4), rel_extent=128, per_head_table=True,
                                          rel_std=0.5, scale=128 ** -0.5, dtype="f32")))
    cases.append(("empty_keys_h4_2", dict(sq=[5, 40, 3], sk=[0, 40, 0], heads=(4, 2), rel_extent=64)))
    for i, (name, spec) in enumerate(cases):
        spec.setdefault("seed", 100 + i)
        spec.setdefault("scale", 1.0 / 128)
        spec.setdefault("causal", True)
        spec.setdefault("window_left", None)
        spec.setdefault("dtype", "bf16")
        spec.setdefault("rel_std", 1.0)
        spec.setdefault("per_head_table", False)
    return cases


def build_inputs(spec):
    """Rebuild a case's inputs from its spec (used by the generator and by the tests)."""
    hq, hkv = spec["heads"]
    c = make_case(spec["sq"], spec["sk"], hq, hkv, spec["rel_extent"], seed=spec["seed"],
                  rel_std=spec["rel_std"], rel_per_head_table=spec["per_head_table"])
    if spec["dtype"] == "f32":
        c.q, c.k, c.v, c.rel = c.q.float(), c.k.float(), c.v.float(), c.rel.float()
    return c


def checksums(c):
    return [float(t.double().sum()) for t in (c.q, c.k, c.v, c.rel)]


def load_reference(path):
    spec = importlib.util.spec_from_file_location("_ifa4_reference_oracle", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod.ref_rel_attn


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="reference checkout (its src/inkling_fa4/reference.py is imported)")
    ap.add_argument("--out", default=HERE)
    args = ap.parse_args()
    ref = load_reference(os.path.join(args.reference, "src", "inkling_fa4", "reference.py"))
    index = {}
    for name, spec in golden_cases():
        c = build_inputs(spec)
        out = ref(c.q, c.k, c.v, c.rel, c.cu_q, c.cu_k, spec["scale"], spec["rel_extent"],
                  causal=spec["causal"], window_left=spec["window_left"])
        if spec["dtype"] == "bf16":
            arr = out.contiguous().view(torch.int16).numpy().view(np.uint16)
        else:
            arr = out.contiguous().numpy().astype(np.float32)
        np.savez_compressed(os.path.join(args.out, f"{name}.npz"), out=arr,
                            checksums=np.array(checksums(c), dtype=np.float64))
        index[name] = spec
        print(f"{name:28s} out{tuple(arr.shape)} {arr.dtype}")
    with open(os.path.join(args.out, "cases.json"), "w") as f:
        json.dump(index, f, indent=1, sort_keys=True)


if __name__ == "__main__":
    main()
