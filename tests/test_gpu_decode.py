"""Decode parity on the B200: split-KV kernel + combine through the drop-in API (C ABI),
against the golden fixtures, the CPU oracle, and the full-prefill kernel."""
import numpy as np
import pytest
import torch

from golden_cases import load_case
from gpu_util import (assert_close, device_status_ok, np32, oracle_full, oracle_rows,
                      run_decode, run_prefill, to_dev)
from inkling_fa4.workloads import Case, config_decode, make_case

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _status_clean():
    yield
    assert device_status_ok(), "a kernel abandoned a bounded wait"


@pytest.mark.parametrize("name", ["decode_h4_4", "decode_h8_2"])
def test_golden_decode(name):
    """tests/test_correctness.py:69-75 (reference alignment: the query sees key 0 only)."""
    spec, c, expected, _ = load_case(name)
    c = to_dev(c)
    out = run_decode(c)
    assert_close(np32(out), expected)


@pytest.mark.parametrize("heads", [(4, 4), (8, 2), (32, 8), (3, 1), (40, 2)])
@pytest.mark.parametrize("window", [None, 300])
@pytest.mark.parametrize("align", ["bottom_right", "reference"])
def test_decode_vs_oracle(heads, window, align):
    hq, hkv = heads
    lens = [1, 63, 64, 65, 1000, 4097, 130, 2]
    c = to_dev(make_case([1] * len(lens), lens, hq, hkv, 128, seed=hq + hkv))
    out = run_decode(c, causal_align=align, window_size=(-1 if window is None else window, 0))
    want = oracle_full(c, 1 / 128, window_left=window, causal_align=align)
    assert_close(np32(out), want)


@pytest.mark.parametrize("splits,chunk", [(1, 0), (2, 64), (3, 128), (7, 256), (0, 0), (64, 64)])
def test_split_count_invariance(splits, chunk):
    lens = [5000, 17, 3000, 640]
    c = to_dev(make_case([1] * 4, lens, 8, 2, 128, seed=21))
    base = run_decode(c, causal_align="bottom_right", num_splits=1, chunk_len=0)
    out = run_decode(c, causal_align="bottom_right", num_splits=splits, chunk_len=chunk)
    assert_close(np32(out), np32(base), atol=5e-3, rtol=5e-3)


def test_decode_equals_last_row_of_full_prefill():
    """north_star: decode results agree with the corresponding full-prefill results."""
    lens = [300, 1, 1029]
    full = to_dev(make_case(lens, lens, 8, 2, 128, seed=5))
    pre = run_prefill(full)
    last = (full.cu_q[1:] - 1).long()
    q = full.q[last].contiguous()
    rel = full.rel[last].contiguous()
    cu_q = torch.arange(len(lens) + 1, dtype=torch.int32, device="cuda")
    from inkling_fa4 import inkling_fa4_rel_attention_decode_triton as dec
    got = dec(q, full.k, full.v, rel, cu_q, full.cu_k, 1, max(lens), 128,
              causal_align="bottom_right")
    assert_close(np32(got), np32(pre[last]), atol=1e-2, rtol=1e-2)


def test_decode_workspace_reuse():
    lens = [9000, 100]
    c = to_dev(make_case([1, 1], lens, 8, 2, 128, seed=7))
    ws = torch.empty(1 << 22, dtype=torch.uint8, device="cuda")
    a = run_decode(c, causal_align="bottom_right", num_splits=8, chunk_len=512, workspace=ws)
    b = run_decode(c, causal_align="bottom_right", num_splits=8, chunk_len=512, workspace=ws)
    torch.testing.assert_close(a, b, atol=0, rtol=0)


def test_config_decode_full_size_sampled():
    c = to_dev(config_decode())
    out = run_decode(c, causal_align="bottom_right")
    heads = [0, 7, 21, 31]
    sub = list(range(0, 128, 9))
    cu_k = c.cu_k.cpu()
    # oracle on the sampled sequences only
    want = []
    for b in sub:
        ks, ke = int(cu_k[b]), int(cu_k[b + 1])
        one = Case(q=c.q[b:b + 1], k=c.k[ks:ke], v=c.v[ks:ke], rel=c.rel[b:b + 1],
                   cu_q=torch.tensor([0, 1], dtype=torch.int32),
                   cu_k=torch.tensor([0, ke - ks], dtype=torch.int32),
                   seqlens_q=[1], seqlens_k=[ke - ks], rel_extent=128)
        _, w = oracle_rows(one, 1, heads, 1 / 128, causal_align="bottom_right")
        want.append(w)
    got = np32(out[sub][:, heads])
    assert_close(got, np.concatenate(want))
