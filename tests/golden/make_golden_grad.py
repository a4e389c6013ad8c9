"""Generate golden GRADIENT fixtures by differentiating the reference's own ``ref_rel_attn``.

The reference has no backward pass; the gradients of its forward (src/inkling_fa4/reference.py
:4-39, plain torch, so autograd differentiates it exactly) are what a backward kernel must
reproduce.  Run in a container that has the reference checkout:

    python tests/golden/make_golden_grad.py --reference <reference checkout>

Inputs are the seeded bf16 values of ``inkling_fa4.workloads.make_case`` taken to float32 (so a
bf16 kernel sees the same numbers), ``dout`` is seeded N(0, 1) rounded to bf16, the loss is
``sum(out * dout)``, and each case stores dq, dk, dv, drel (float32) plus float64 checksums of
the inputs.  No case has a query row without a visible key (the reference's softmax is NaN
there).
"""
from __future__ import annotations

import argparse
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(REPO, "inkling-fa4-relative-attention_b200"))
sys.path.insert(0, HERE)

from inkling_fa4.workloads import make_case  # noqa: E402
from make_golden import load_reference  # noqa: E402


def grad_cases():
    cases = [
        ("grad_ragged_h4_4", dict(sq=[64, 33, 17], sk=[64, 33, 17], heads=(4, 4), rel_extent=64)),
        ("grad_gqa_h8_2", dict(sq=[150], sk=[150], heads=(8, 2), rel_extent=128)),
        ("grad_window_h4_2", dict(sq=[130], sk=[130], heads=(4, 2), rel_extent=32, window_left=40)),
        ("grad_noncausal_h4_1", dict(sq=[90], sk=[90], heads=(4, 1), rel_extent=100, causal=False)),
        ("grad_sk_gt_sq_h4_4", dict(sq=[48], sk=[160], heads=(4, 4), rel_extent=200)),
        ("grad_zero_len_h4_2", dict(sq=[40, 0, 25], sk=[40, 0, 25], heads=(4, 2), rel_extent=16)),
        ("grad_long_h2_1", dict(sq=[300], sk=[300], heads=(2, 1), rel_extent=1024)),
    ]
    for i, (_, spec) in enumerate(cases):
        spec.setdefault("seed", 500 + i)
        spec.setdefault("scale", 1.0 / 128)
        spec.setdefault("causal", True)
        spec.setdefault("window_left", None)
    return cases


def build_grad_inputs(spec):
    """Case (bf16 tensors) and dout (bf16) of a gradient fixture."""
    hq, hkv = spec["heads"]
    c = make_case(spec["sq"], spec["sk"], hq, hkv, spec["rel_extent"], seed=spec["seed"])
    g = torch.Generator(device="cpu")
    g.manual_seed(spec["seed"] * 7 + 5)
    dout = torch.randn(c.q.shape, generator=g).to(torch.bfloat16)
    return c, dout


def checksums(c, dout):
    return [float(t.double().sum()) for t in (c.q, c.k, c.v, c.rel, dout)]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="reference checkout (its src/inkling_fa4/reference.py is imported)")
    ap.add_argument("--out", default=HERE)
    args = ap.parse_args()
    ref = load_reference(os.path.join(args.reference, "src", "inkling_fa4", "reference.py"))
    index = {}
    for name, spec in grad_cases():
        c, dout = build_grad_inputs(spec)
        q, k, v, rel = (t.float().requires_grad_(True) for t in (c.q, c.k, c.v, c.rel))
        out = ref(q, k, v, rel, c.cu_q, c.cu_k, spec["scale"], spec["rel_extent"],
                  causal=spec["causal"], window_left=spec["window_left"])
        (out * dout.float()).sum().backward()
        arrs = {nm: t.grad.numpy().astype(np.float32) for nm, t in
                (("dq", q), ("dk", k), ("dv", v), ("drel", rel))}
        assert all(np.isfinite(a).all() for a in arrs.values()), name
        np.savez_compressed(os.path.join(args.out, f"{name}.npz"),
                            checksums=np.array(checksums(c, dout), dtype=np.float64), **arrs)
        index[name] = spec
        print(f"{name:24s} " + " ".join(f"{k}{tuple(a.shape)}" for k, a in arrs.items()))
    with open(os.path.join(args.out, "grad_cases.json"), "w") as f:
        json.dump(index, f, indent=1, sort_keys=True)


if __name__ == "__main__":
    main()
