"""The gradient oracle (torch autograd through the oracle's torch twin) against the golden
gradients of the reference's own ``ref_rel_attn`` (tests/golden/make_golden_grad.py), plus
size-independent properties of the gradients."""
import json
import os

import numpy as np
import pytest
import torch

import oracle
from golden.make_golden_grad import build_grad_inputs, checksums

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def grad_names():
    with open(os.path.join(GOLDEN, "grad_cases.json")) as f:
        return sorted(json.load(f).keys())


def load_grad_case(name):
    with open(os.path.join(GOLDEN, "grad_cases.json")) as f:
        spec = json.load(f)[name]
    c, dout = build_grad_inputs(spec)
    z = np.load(os.path.join(GOLDEN, f"{name}.npz"))
    return spec, c, dout, {k: z[k] for k in ("dq", "dk", "dv", "drel")}, z["checksums"]


@pytest.mark.parametrize("name", grad_names())
def test_grad_oracle_matches_reference_autograd(name):
    spec, c, dout, want, sums = load_grad_case(name)
    np.testing.assert_allclose(checksums(c, dout), sums, rtol=0, atol=0)
    got = oracle.rel_attn_grads_torch(c.q, c.k, c.v, c.rel, dout, c.cu_q, c.cu_k, spec["scale"],
                                      spec["rel_extent"], causal=spec["causal"],
                                      window_left=spec["window_left"])
    for nm, g in zip(("dq", "dk", "dv", "drel"), got):
        w = want[nm]
        np.testing.assert_allclose(g.numpy(), w, rtol=1e-4, atol=1e-5 * max(1.0, np.abs(w).max()),
                                   err_msg=nm)


def test_bias_gradient_is_zero_outside_the_band():
    """d rel[i, h, d] is the logit gradient of the key at distance d, so it vanishes where no
    visible key sits at that distance (d > i for a causal square sequence)."""
    spec, c, dout, want, _ = load_grad_case("grad_ragged_h4_4")
    drel = want["drel"]
    cu = c.cu_q.tolist()
    for b in range(len(cu) - 1):
        for i in range(cu[b + 1] - cu[b]):
            assert np.all(drel[cu[b] + i, :, i + 1:] == 0)


def test_bias_gradient_rows_sum_to_zero():
    """Softmax gradients sum to zero over each row's keys (sum_j dS_ij = 0); with R covering
    every causal distance, the bias gradient of each row is all of dS, so it sums to 0."""
    spec, c, dout, want, _ = load_grad_case("grad_long_h2_1")
    assert spec["rel_extent"] >= 300 and spec["causal"]
    np.testing.assert_allclose(want["drel"].sum(axis=2), 0.0, atol=1e-5)
