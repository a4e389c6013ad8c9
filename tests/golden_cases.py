"""Loader for the committed golden fixtures (outputs of the reference's ``ref_rel_attn``)."""
import json
import os

import numpy as np

from golden.make_golden import build_inputs, checksums  # noqa: F401

GOLDEN_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load_index():
    with open(os.path.join(GOLDEN_DIR, "cases.json")) as f:
        return json.load(f)


def load_case(name):
    """Return (spec, inputs Case, expected float32 output array, stored checksums)."""
    spec = load_index()[name]
    z = np.load(os.path.join(GOLDEN_DIR, f"{name}.npz"))
    out = z["out"]
    if out.dtype == np.uint16:
        out = (out.astype(np.uint32) << 16).view(np.float32)
    return spec, build_inputs(spec), out.astype(np.float32), z["checksums"]


def names():
    return sorted(load_index().keys())
