"""Backward kernels (dQ, dK, dV, d rel) through the C ABI against the golden gradients of the
reference's forward and against the torch-autograd oracle, over ragged / GQA / mask /
alignment cases; plus determinism, the autograd entry point, and the bias-gradient band."""
import numpy as np
import pytest
import torch

import oracle
from gpu_util import device_status_ok, np32, to_dev
from inkling_fa4 import inkling_fa4_rel_attention, inkling_fa4_rel_attention_backward
from inkling_fa4 import inkling_fa4_rel_attention_triton as prefill
from inkling_fa4.workloads import make_case
from test_oracle_grad import grad_names, load_grad_case

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _status_clean():
    yield
    assert device_status_ok(), "a kernel abandoned a bounded wait"


def assert_grad_close(got, want, what, frac=2.5e-2):
    """bf16 kernels (P and dS are bf16 MMA operands) against fp32 gradients: absolute error
    within frac of the tensor's largest magnitude."""
    got = np.asarray(got, np.float32)
    want = np.asarray(want, np.float32)
    scale = max(float(np.abs(want).max()), 1e-6)
    err = float(np.abs(got - want).max())
    assert np.isfinite(got).all(), f"{what}: non-finite values"
    assert err <= frac * scale, f"{what}: max err {err:.3e} vs scale {scale:.3e}"


def run_backward(c, dout, scale=1 / 128, causal=True, window=None, align="reference"):
    ws = (-1 if window is None else window, 0)
    out, lse = prefill(c.q, c.k, c.v, c.rel, c.cu_q, c.cu_k, c.max_q, c.max_k, c.rel_extent,
                       causal=causal, window_size=ws, softmax_scale=scale, causal_align=align,
                       return_lse=True)
    return inkling_fa4_rel_attention_backward(dout, c.q, c.k, c.v, c.rel, out, lse, c.cu_q,
                                              c.cu_k, c.max_q, c.max_k, c.rel_extent,
                                              causal=causal, window_size=ws,
                                              softmax_scale=scale, causal_align=align)


@pytest.mark.parametrize("name", grad_names())
def test_golden_gradients(name):
    spec, c, dout, want, _ = load_grad_case(name)
    c = to_dev(c)
    got = run_backward(c, dout.cuda(), spec["scale"], spec["causal"], spec["window_left"])
    for nm, g in zip(("dq", "dk", "dv", "drel"), got):
        assert_grad_close(np32(g), want[nm], f"{name}:{nm}")


@pytest.mark.parametrize("heads", [(4, 4), (8, 2), (3, 1)])
@pytest.mark.parametrize("causal,window", [(True, None), (False, None), (True, 70), (False, 33)])
@pytest.mark.parametrize("rel_extent", [128, 1000])
def test_backward_vs_oracle(heads, causal, window, rel_extent):
    hq, hkv = heads
    lens = [1, 127, 128, 129, 300]
    c = make_case(lens, lens, hq, hkv, rel_extent, seed=hq * 7 + rel_extent)
    g = torch.Generator().manual_seed(3)
    dout = torch.randn(c.q.shape, generator=g).to(torch.bfloat16)
    want = oracle.rel_attn_grads_torch(c.q, c.k, c.v, c.rel, dout, c.cu_q, c.cu_k, 1 / 128,
                                       rel_extent, causal=causal, window_left=window)
    got = run_backward(to_dev(c), dout.cuda(), causal=causal, window=window)
    for nm, a, w in zip(("dq", "dk", "dv", "drel"), got, want):
        assert_grad_close(np32(a), w.numpy(), nm)


@pytest.mark.parametrize("window", [None, 100])
def test_chunked_backward_bottom_right(window):
    """Queries of a new chunk against cache + chunk keys (bottom-right alignment)."""
    c = make_case([50, 128, 7], [300, 128, 900], 8, 2, 128, seed=9)
    dout = torch.randn(c.q.shape, generator=torch.Generator().manual_seed(4)).to(torch.bfloat16)
    want = oracle.rel_attn_grads_torch(c.q, c.k, c.v, c.rel, dout, c.cu_q, c.cu_k, 1 / 128, 128,
                                       window_left=window, causal_align="bottom_right")
    got = run_backward(to_dev(c), dout.cuda(), window=window, align="bottom_right")
    for nm, a, w in zip(("dq", "dk", "dv", "drel"), got, want):
        assert_grad_close(np32(a), w.numpy(), nm)


def test_backward_is_deterministic_and_band_limited():
    lens = [700, 64]
    c = to_dev(make_case(lens, lens, 8, 2, 64, seed=2))
    dout = torch.randn(c.q.shape, device="cuda", dtype=torch.bfloat16)
    a = run_backward(c, dout)
    b = run_backward(c, dout)
    for x, y in zip(a, b):
        assert torch.equal(x, y)
    drel = a[3].float()
    # causal, square: row i has no key at distance > i
    for i in (0, 5, 63):
        assert torch.count_nonzero(drel[i, :, i + 1:]) == 0


def test_keys_no_query_sees_get_zero_gradient():
    """Reference alignment with more keys than queries: keys past the last query row are
    masked for every row, so their dK / dV are 0."""
    c = to_dev(make_case([40], [300], 4, 2, 64, seed=3))
    dout = torch.randn(c.q.shape, device="cuda", dtype=torch.bfloat16)
    dq, dk, dv, _ = run_backward(c, dout)
    assert torch.count_nonzero(dk[40:]) == 0 and torch.count_nonzero(dv[40:]) == 0
    assert torch.count_nonzero(dk[:40]) > 0


def test_autograd_entry_point():
    c = to_dev(make_case([200, 31], [200, 31], 8, 2, 128, seed=6))
    q, k, v, rel = (t.clone().requires_grad_(True) for t in (c.q, c.k, c.v, c.rel))
    out = inkling_fa4_rel_attention(q, k, v, rel, c.cu_q, c.cu_k, c.max_q, c.max_k, 128)
    dout = torch.randn_like(out)
    (out.float() * dout.float()).sum().backward()
    ref = run_backward(c, dout)
    for t, r in zip((q, k, v, rel), ref):
        assert torch.equal(t.grad, r)
    assert torch.equal(out.detach(), prefill(c.q, c.k, c.v, c.rel, c.cu_q, c.cu_k, c.max_q,
                                             c.max_k, 128))
