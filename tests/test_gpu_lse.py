"""Log-sum-exp output of the prefill and decode kernels (an extension of the reference call
surface, used to merge attention computed over separate key ranges): against the CPU oracle's
LSE, through the split-key merge identity, across decode split plans, and for rows without
visible keys."""
import numpy as np
import pytest
import torch

from gpu_util import assert_close, device_status_ok, np32, run_decode, run_prefill, to_dev
from inkling_fa4.workloads import Case, cu_from_lens, make_case
from test_oracle_golden import merge_by_lse

import oracle

pytestmark = pytest.mark.gpu

LSE_ATOL = 2e-3  # fp32 statistics of identical bf16 logits; exp2/log2 approximations only


@pytest.fixture(autouse=True)
def _status_clean():
    yield
    assert device_status_ok(), "a kernel abandoned a bounded wait"


def _oracle(c, **kw):
    return oracle.rel_attn(np32(c.q), np32(c.k), np32(c.v), np32(c.rel), c.cu_q.cpu().numpy(),
                           c.cu_k.cpu().numpy(), 1 / 128, c.rel_extent, row_block=512,
                           return_lse=True, **kw)


def _assert_lse(got, want, what=""):
    got, want = np.asarray(got), np.asarray(want)
    ninf = np.isneginf(want)
    assert np.array_equal(np.isneginf(got), ninf), f"{what}: -inf rows differ"
    np.testing.assert_allclose(got[~ninf], want[~ninf], atol=LSE_ATOL, rtol=1e-4, err_msg=what)


@pytest.mark.parametrize("heads", [(4, 4), (8, 2), (3, 1)])
@pytest.mark.parametrize("causal,window", [(True, None), (False, None), (True, 70)])
def test_prefill_lse_vs_oracle(heads, causal, window):
    hq, hkv = heads
    lens = [1, 127, 128, 129, 300, 513]
    c = to_dev(make_case(lens, lens, hq, hkv, 128, seed=hq * 3 + hkv))
    out, lse = run_prefill(c, causal=causal, return_lse=True,
                           window_size=(-1 if window is None else window, 0))
    want_o, want_lse = _oracle(c, causal=causal, window_left=window)
    assert_close(np32(out), want_o)
    _assert_lse(np32(lse), want_lse, "prefill lse")
    plain = run_prefill(c, causal=causal, window_size=(-1 if window is None else window, 0))
    assert torch.equal(plain, out)


def test_prefill_lse_merge_of_split_key_ranges():
    """Attention of the same queries over keys [0, s) and [s, sk), merged through the LSEs,
    equals attention over all keys (bias constant along each row, non-causal)."""
    sq, sk, split = 200, 1500, 611
    base = make_case([sq], [sk], 8, 2, 128, seed=41)
    rel = base.rel[:, :, :1].expand(sq, 8, 128).contiguous()
    full = to_dev(Case(q=base.q, k=base.k, v=base.v, rel=rel, cu_q=base.cu_q, cu_k=base.cu_k,
                       seqlens_q=[sq], seqlens_k=[sk], rel_extent=128))
    parts = to_dev(Case(q=torch.cat([base.q, base.q]), k=base.k, v=base.v,
                        rel=torch.cat([rel, rel]), cu_q=cu_from_lens([sq, sq]),
                        cu_k=torch.tensor([0, split, sk], dtype=torch.int32),
                        seqlens_q=[sq, sq], seqlens_k=[split, sk - split], rel_extent=128))
    o_full, lse_full = run_prefill(full, causal=False, return_lse=True)
    o_p, lse_p = run_prefill(parts, causal=False, return_lse=True)
    o_m, lse_m = merge_by_lse(np32(o_p), np32(lse_p), sq)
    assert_close(o_m, np32(o_full))
    _assert_lse(lse_m, np32(lse_full), "merged lse")


def test_prefill_lse_rows_without_keys():
    c = to_dev(make_case([5, 64], [0, 64], 4, 2, 64, seed=2))
    out, lse = run_prefill(c, return_lse=True)
    lse = np32(lse)
    assert np.all(np.isneginf(lse[:, :5])) and np.all(np.isfinite(lse[:, 5:]))
    # sliding window of 0 keys back from a row that sees only itself stays finite
    out, lse = run_prefill(c, return_lse=True, window_size=(0, 0))
    assert np.all(np.isfinite(np32(lse)[:, 5:]))


def test_prefill_lse_into_strided_buffer():
    lens = [77, 260]
    c = to_dev(make_case(lens, lens, 4, 4, 64, seed=9))
    big = torch.full((4, c.q.shape[0] + 13), 7.0, device="cuda")
    view = big[:, 5:5 + c.q.shape[0]]
    _, lse = run_prefill(c, lse=view)
    assert lse.data_ptr() == view.data_ptr()
    _, ref = run_prefill(c, return_lse=True)
    assert torch.equal(view, ref)
    assert torch.all(big[:, :5] == 7.0) and torch.all(big[:, 5 + c.q.shape[0]:] == 7.0)


@pytest.mark.parametrize("align", ["bottom_right", "reference"])
@pytest.mark.parametrize("window", [None, 300])
def test_decode_lse_vs_oracle(align, window):
    lens = [1, 63, 65, 1000, 4097, 2]
    c = to_dev(make_case([1] * len(lens), lens, 8, 2, 128, seed=12))
    out, lse = run_decode(c, causal_align=align, return_lse=True,
                          window_size=(-1 if window is None else window, 0))
    want_o, want_lse = _oracle(c, window_left=window, causal_align=align)
    assert_close(np32(out), want_o)
    _assert_lse(np32(lse), want_lse, "decode lse")


@pytest.mark.parametrize("splits,chunk", [(1, 0), (3, 128), (0, 0), (64, 64)])
def test_decode_lse_split_invariance(splits, chunk):
    lens = [5000, 17, 3000, 0]
    c = to_dev(make_case([1] * 4, lens, 8, 2, 128, seed=21))
    _, base = run_decode(c, causal_align="bottom_right", num_splits=1, chunk_len=0,
                         return_lse=True)
    _, lse = run_decode(c, causal_align="bottom_right", num_splits=splits, chunk_len=chunk,
                        return_lse=True)
    _assert_lse(np32(lse), np32(base), f"splits={splits}")
    assert np.all(np.isneginf(np32(lse)[:, 3]))


def test_decode_lse_equals_prefill_last_row_lse():
    lens = [300, 1, 1029]
    full = to_dev(make_case(lens, lens, 8, 2, 128, seed=5))
    _, pre_lse = run_prefill(full, return_lse=True)
    last = (full.cu_q[1:] - 1).long()
    dec = Case(q=full.q[last].contiguous(), k=full.k, v=full.v, rel=full.rel[last].contiguous(),
               cu_q=torch.arange(len(lens) + 1, dtype=torch.int32, device="cuda"),
               cu_k=full.cu_k, seqlens_q=[1] * 3, seqlens_k=lens, rel_extent=128)
    _, lse = run_decode(dec, causal_align="bottom_right", return_lse=True)
    _assert_lse(np32(lse), np32(pre_lse[:, last]), "decode vs prefill lse")
