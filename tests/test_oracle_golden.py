"""Pin the CPU oracle (oracle/rel_attn_oracle.py) against the reference's own outputs."""
import numpy as np
import pytest
import torch

import oracle
from golden_cases import checksums, load_case, names


@pytest.mark.parametrize("name", names())
def test_inputs_rebuild_bit_identically(name):
    spec, case, _, stored = load_case(name)
    np.testing.assert_array_equal(np.array(checksums(case)), stored)


@pytest.mark.parametrize("name", names())
def test_oracle_matches_reference_output(name):
    spec, c, expected, _ = load_case(name)
    got = oracle.rel_attn(c.q.float().numpy(), c.k.float().numpy(), c.v.float().numpy(),
                          c.rel.float().numpy(), c.cu_q.numpy(), c.cu_k.numpy(), spec["scale"],
                          spec["rel_extent"], causal=spec["causal"],
                          window_left=spec["window_left"], out_bf16=spec["dtype"] == "bf16")
    nan_exp = np.isnan(expected)
    np.testing.assert_array_equal(np.isnan(got), nan_exp)
    if spec["dtype"] == "bf16":
        # identical algorithm in fp32: the two results may round to neighbouring bf16 values,
        # and values near zero (cancellation) carry fp32 summation-order noise of ~1e-6
        a, b = got[~nan_exp], expected[~nan_exp]
        tol = np.maximum(np.abs(a), np.abs(b)) * 2.0 ** -7 + 1e-5
        assert np.all(np.abs(a - b) <= tol), float(np.abs(a - b).max())
    else:
        np.testing.assert_allclose(got[~nan_exp], expected[~nan_exp], rtol=2e-5, atol=2e-6)


def test_row_blocking_is_exact():
    spec, c, expected, _ = load_case("long_ctx_h8_2")
    args = (c.q.float().numpy(), c.k.float().numpy(), c.v.float().numpy(), c.rel.float().numpy(),
            c.cu_q.numpy(), c.cu_k.numpy(), spec["scale"], spec["rel_extent"])
    a = oracle.rel_attn(*args, row_block=None)
    b = oracle.rel_attn(*args, row_block=37)
    np.testing.assert_allclose(a, b, rtol=1e-6, atol=1e-7)


def test_bottom_right_equals_reference_when_square():
    spec, c, _, _ = load_case("ragged_h4_4")
    args = (c.q.float().numpy(), c.k.float().numpy(), c.v.float().numpy(), c.rel.float().numpy(),
            c.cu_q.numpy(), c.cu_k.numpy(), spec["scale"], spec["rel_extent"])
    np.testing.assert_array_equal(oracle.rel_attn(*args, causal_align="reference"),
                                  oracle.rel_attn(*args, causal_align="bottom_right"))


def test_bottom_right_chunk_equals_full_prefill_rows():
    """Chunked (cache + chunk) in bottom-right alignment equals the last rows of the full
    square prefill, which the reference pins directly."""
    from inkling_fa4.workloads import make_case
    cache, chunk = 150, 70
    full = make_case([cache + chunk], [cache + chunk], 4, 2, 64, seed=5)
    args_full = (full.q.float().numpy(), full.k.float().numpy(), full.v.float().numpy(),
                 full.rel.float().numpy(), full.cu_q.numpy(), full.cu_k.numpy(), 1 / 128, 64)
    ref_rows = oracle.rel_attn(*args_full)[cache:]
    q = full.q.float().numpy()[cache:]
    rel = full.rel.float().numpy()[cache:]
    got = oracle.rel_attn(q, args_full[1], args_full[2], rel, np.array([0, chunk]),
                          np.array([0, cache + chunk]), 1 / 128, 64, causal_align="bottom_right")
    np.testing.assert_allclose(got, ref_rows, rtol=1e-5, atol=1e-6)


def test_reference_decode_is_degenerate():
    """reference alignment with sq=1: the query sees key 0 only (reference.py:36), so the
    output equals v[0] of its kv head and no bias applies."""
    spec, c, expected, _ = load_case("decode_h8_2")
    v0 = c.v[0].float()  # [Hkv, d]
    g = 8 // 2
    want = torch.stack([v0[h // g] for h in range(8)]).to(torch.bfloat16).float().numpy()
    np.testing.assert_array_equal(expected[0], want)


@pytest.mark.parametrize("name", names())
def test_torch_oracle_twin_matches_reference_output(name):
    spec, c, expected, _ = load_case(name)
    got = oracle.rel_attn_torch(c.q, c.k, c.v, c.rel, c.cu_q, c.cu_k, spec["scale"],
                                spec["rel_extent"], causal=spec["causal"],
                                window_left=spec["window_left"], row_block=50).numpy()
    if spec["dtype"] == "bf16":
        got = oracle.round_to_bf16(got)
    nan_exp = np.isnan(expected)
    np.testing.assert_array_equal(np.isnan(got), nan_exp)
    a, b = got[~nan_exp], expected[~nan_exp]
    tol = np.maximum(np.abs(a), np.abs(b)) * 2.0 ** -7 + 1e-5
    assert np.all(np.abs(a - b) <= tol), float(np.abs(a - b).max())


def test_package_ref_rel_attn_matches_reference_output():
    """inkling_fa4.ref_rel_attn (kept for API compatibility) agrees with the reference."""
    from inkling_fa4 import ref_rel_attn
    for name in names():
        spec, c, expected, _ = load_case(name)
        got = ref_rel_attn(c.q, c.k, c.v, c.rel, c.cu_q, c.cu_k, spec["scale"],
                           spec["rel_extent"], causal=spec["causal"],
                           window_left=spec["window_left"]).float().numpy()
        nan_exp = np.isnan(expected)
        np.testing.assert_array_equal(np.isnan(got), nan_exp)
        a, b = got[~nan_exp], expected[~nan_exp]
        tol = np.maximum(np.abs(a), np.abs(b)) * 2.0 ** -7 + 1e-5
        assert np.all(np.abs(a - b) <= tol), (name, float(np.abs(a - b).max()))


def _split_key_case(sq, sk, split, n_heads=4, kv_heads=2, rel_extent=64, seed=31):
    """Non-causal rows whose bias is constant along each row (so the bias of a key does not
    depend on where the key sits), as one full sequence and as the same queries against the
    key ranges [0, split) and [split, sk) (two sequences of one varlen batch)."""
    from inkling_fa4.workloads import make_case
    c = make_case([sq], [sk], n_heads, kv_heads, rel_extent, seed=seed)
    rel = c.rel.float().numpy()
    rel = np.repeat(rel[:, :, :1], rel_extent, axis=2)
    q, k, v = c.q.float().numpy(), c.k.float().numpy(), c.v.float().numpy()
    full = (q, k, v, rel, np.array([0, sq]), np.array([0, sk]))
    parts = (np.concatenate([q, q]), k, v, np.concatenate([rel, rel]),
             np.array([0, sq, 2 * sq]), np.array([0, split, sk]))
    return full, parts


def merge_by_lse(o, lse, sq):
    """Combine two partial attentions over disjoint key ranges: weights exp(lse_i - lse)."""
    l1, l2 = lse[:, :sq], lse[:, sq:]
    lse_all = np.logaddexp(l1, l2)
    w1 = np.exp(l1 - lse_all).T[:, :, None]
    w2 = np.exp(l2 - lse_all).T[:, :, None]
    return w1 * o[:sq] + w2 * o[sq:], lse_all


def test_oracle_lse_is_logsumexp_of_the_scores():
    """The oracle's LSE is log(sum(exp(scores))) of the row's scaled+biased logits."""
    from inkling_fa4.workloads import make_case
    c = make_case([40, 7], [40, 7], 2, 1, 16, seed=3)
    args = (c.q.float().numpy(), c.k.float().numpy(), c.v.float().numpy(), c.rel.float().numpy(),
            c.cu_q.numpy(), c.cu_k.numpy(), 1 / 128, 16)
    out, lse = oracle.rel_attn(*args, return_lse=True)
    np.testing.assert_array_equal(out, oracle.rel_attn(*args))
    q, k, rel = args[0], args[1], args[3]
    for h in range(2):
        for i in range(40):
            s = q[i, h] @ k[:i + 1, 0].T / 128
            d = i - np.arange(i + 1)
            bias = np.where(d < 16, rel[i, h, np.minimum(d, 15)], 0.0)
            want = np.log(np.sum(np.exp((s + bias).astype(np.float64))))
            assert abs(lse[h, i] - want) < 1e-5 * max(1.0, abs(want))


def test_oracle_lse_merges_split_key_ranges():
    full, parts = _split_key_case(50, 300, 123)
    o_full, lse_full = oracle.rel_attn(*full, 1 / 128, 64, causal=False, return_lse=True)
    o_p, lse_p = oracle.rel_attn(*parts, 1 / 128, 64, causal=False, return_lse=True)
    o_m, lse_m = merge_by_lse(o_p, lse_p, 50)
    np.testing.assert_allclose(o_m, o_full, rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(lse_m, lse_full, rtol=1e-6, atol=1e-6)


def test_oracle_lse_of_empty_rows_is_minus_inf():
    from inkling_fa4.workloads import make_case
    c = make_case([3], [0], 2, 2, 8, seed=1)
    _, lse = oracle.rel_attn(c.q.float().numpy(), c.k.float().numpy(), c.v.float().numpy(),
                             c.rel.float().numpy(), c.cu_q.numpy(), c.cu_k.numpy(), 1 / 128, 8,
                             return_lse=True)
    assert np.all(np.isneginf(lse))
