"""Paged KV cache (block tables, as a serving engine's cache) for prefill, chunked prefill and
decode: the paged kernels against the contiguous kernels on the same keys (bit for bit where
the tile boundaries coincide) and against the CPU oracle.  Unused cache slots hold NaN, so any
kernel that let one reach its output fails."""
import numpy as np
import pytest
import torch

from gpu_util import (assert_close, device_status_ok, np32, oracle_full, oracle_rows, run_decode,
                      run_prefill, to_dev)
from inkling_fa4 import inkling_fa4_rel_attention_decode_triton as decode_api
from inkling_fa4 import inkling_fa4_rel_attention_triton as prefill_api
from inkling_fa4.workloads import Case, make_case, page_kv

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _status_clean():
    yield
    assert device_status_ok(), "a kernel abandoned a bounded wait"


def paged_prefill(pc, **kw):
    return prefill_api(pc.q, pc.k, pc.v, pc.rel, pc.cu_q, pc.cu_k, pc.max_q, pc.max_k,
                       pc.rel_extent, block_table=pc.meta["block_table"], **kw)


def paged_decode(pc, **kw):
    return decode_api(pc.q, pc.k, pc.v, pc.rel, pc.cu_q, pc.cu_k, 1, pc.max_k, pc.rel_extent,
                      block_table=pc.meta["block_table"], **kw)


LENS = [1, 15, 16, 17, 127, 128, 129, 300, 1000]


@pytest.mark.parametrize("page_size", [16, 32, 64, 128, 256])
@pytest.mark.parametrize("heads", [(8, 2), (3, 1)])
@pytest.mark.parametrize("causal,window", [(True, None), (False, None), (True, 70)])
def test_paged_prefill_equals_contiguous(page_size, heads, causal, window):
    hq, hkv = heads
    c = to_dev(make_case(LENS, LENS, hq, hkv, 128, seed=page_size + hq))
    pc = page_kv(c, page_size=page_size, seed=page_size)
    kw = dict(causal=causal, window_size=(-1 if window is None else window, 0))
    want = run_prefill(c, **kw)
    got = paged_prefill(pc, **kw)
    assert torch.equal(got, want), float((got.float() - want.float()).abs().max())
    assert not torch.isnan(got.float()).any()


@pytest.mark.parametrize("page_size", [16, 64])
@pytest.mark.parametrize("window", [None, 100])
def test_paged_chunked_prefill_vs_oracle(page_size, window):
    """Chunked prefill: each new chunk's queries attend to the whole cache (cached prefix +
    the chunk's own keys, already written to the cache), bottom-right alignment."""
    cache = [0, 37, 256, 1000]
    new = [50, 128, 1, 301]
    total = [a + b for a, b in zip(cache, new)]
    c = to_dev(make_case(new, total, 8, 2, 128, seed=3 + page_size))
    pc = page_kv(c, page_size=page_size, seed=1)
    kw = dict(causal_align="bottom_right", window_size=(-1 if window is None else window, 0))
    got = paged_prefill(pc, **kw)
    assert torch.equal(got, run_prefill(c, **kw))
    assert_close(np32(got), oracle_full(c, 1 / 128, window_left=window, causal_align="bottom_right"))


def test_long_chunked_prefill_query_slots_first():
    """Chunks over ~14k-key caches with 8 KV heads: the key range of a query tile over all KV
    heads (59 MB) exceeds a third of L2, so both the contiguous and the paged launch use the
    (query slots, head slots, sequences) grid.  Paged equals contiguous bit for bit, and sampled
    rows match the oracle."""
    cache = [16000, 12500]
    new = [300, 64]
    total = [a + b for a, b in zip(cache, new)]
    c = to_dev(make_case(new, total, 32, 8, 128, seed=21))
    pc = page_kv(c, page_size=16, seed=21)
    kw = dict(causal_align="bottom_right")
    want = run_prefill(c, **kw)
    got = paged_prefill(pc, **kw)
    assert torch.equal(got, want), float((got.float() - want.float()).abs().max())
    heads = [0, 13, 31]
    toks, ref = oracle_rows(c, 12, heads, 1 / 128, causal_align="bottom_right", seed=4)
    assert_close(np32(want[torch.from_numpy(toks).cuda()][:, heads]), ref)


@pytest.mark.parametrize("page_size", [16, 32, 64, 128])
@pytest.mark.parametrize("splits,chunk", [(1, 0), (4, 256), (0, 0)])
def test_paged_decode_equals_contiguous(page_size, splits, chunk):
    lens = [1, 15, 16, 17, 63, 64, 65, 1000, 4097, 0]
    c = to_dev(make_case([1] * len(lens), lens, 8, 2, 128, seed=page_size))
    pc = page_kv(c, page_size=page_size, seed=7)
    kw = dict(causal_align="bottom_right", num_splits=splits, chunk_len=chunk)
    want = run_decode(c, **kw)
    got = paged_decode(pc, **kw)
    assert torch.equal(got, want), float((got.float() - want.float()).abs().max())


@pytest.mark.parametrize("page_size", [16, 128])
@pytest.mark.parametrize("window", [5, 300])
@pytest.mark.parametrize("heads", [(8, 2), (40, 2)])
def test_paged_decode_window_vs_oracle(page_size, window, heads):
    """With a window the paged tiles start at the window's first key rounded down to the page
    unit, so the split boundaries differ from the contiguous kernel's: compare to the oracle."""
    hq, hkv = heads
    lens = [1, 17, 300, 301, 1000, 4097]
    c = to_dev(make_case([1] * len(lens), lens, hq, hkv, 128, seed=window))
    pc = page_kv(c, page_size=page_size, seed=2)
    got = paged_decode(pc, causal_align="bottom_right", window_size=(window, 0))
    assert_close(np32(got), oracle_full(c, 1 / 128, window_left=window, causal_align="bottom_right"))


def test_paged_lse_equals_contiguous():
    c = to_dev(make_case(LENS, LENS, 8, 2, 128, seed=11))
    pc = page_kv(c, page_size=16, seed=3)
    o1, l1 = run_prefill(c, return_lse=True)
    o2, l2 = paged_prefill(pc, return_lse=True)
    assert torch.equal(o1, o2) and torch.equal(l1, l2)
    d = to_dev(make_case([1] * 4, [5000, 1, 16, 700], 8, 2, 128, seed=12))
    pd = page_kv(d, page_size=16, seed=4)
    o1, l1 = run_decode(d, causal_align="bottom_right", num_splits=3, chunk_len=512, return_lse=True)
    o2, l2 = paged_decode(pd, causal_align="bottom_right", num_splits=3, chunk_len=512,
                          return_lse=True)
    assert torch.equal(o1, o2) and torch.equal(l1, l2)


def test_invalid_table_entries_read_as_zero_keys():
    """A table entry outside [0, num_pages) gives zero keys and values for its slots (no read);
    the contiguous kernel on the same keys with those rows zeroed gives the same result."""
    lens = [200, 77]
    c = to_dev(make_case(lens, lens, 4, 2, 64, seed=5))
    pc = page_kv(c, page_size=16, seed=5)
    bt = pc.meta["block_table"].clone()
    bt[0, 3] = -1                   # keys 48..63 of sequence 0
    bt[1, 4] = pc.meta["num_pages"]  # keys 64..76 of sequence 1 (its partial last page)
    pc.meta["block_table"] = bt
    k, v = c.k.clone(), c.v.clone()
    k[48:64] = 0
    v[48:64] = 0
    k[200 + 64:200 + 77] = 0
    v[200 + 64:200 + 77] = 0
    zc = Case(q=c.q, k=k, v=v, rel=c.rel, cu_q=c.cu_q, cu_k=c.cu_k, seqlens_q=lens,
              seqlens_k=lens, rel_extent=64)
    assert torch.equal(paged_prefill(pc), run_prefill(zc))


def test_paged_empty_sequences_and_empty_table():
    c = to_dev(make_case([3, 2], [0, 0], 4, 2, 16, seed=1))
    kc = torch.zeros((2, 16, 2, 128), dtype=torch.bfloat16, device="cuda")
    empty = torch.zeros((2, 0), dtype=torch.int32, device="cuda")
    out = prefill_api(c.q, kc, kc, c.rel, c.cu_q, c.cu_k, 3, 0, 16, block_table=empty)
    assert torch.count_nonzero(out) == 0
    d = to_dev(make_case([1, 1], [0, 0], 4, 2, 16, seed=1))
    out = decode_api(d.q, kc, kc, d.rel, d.cu_q, d.cu_k, 1, 0, 16, block_table=empty)
    assert torch.count_nonzero(out) == 0


def test_paged_cache_is_never_copied():
    c = to_dev(make_case([40], [40], 4, 2, 16, seed=1))
    pc = page_kv(c, page_size=16)
    k_bad = pc.k[:, :, :, :64]  # head_dim 64 slice: rejected rather than copied
    with pytest.raises(ValueError):
        prefill_api(pc.q, k_bad, pc.v, pc.rel, pc.cu_q, pc.cu_k, 40, 40, 16,
                    block_table=pc.meta["block_table"])
    k_odd = torch.empty((pc.k.shape[0], 16, 2, 136), dtype=torch.bfloat16, device="cuda")[..., 4:132]
    k_odd.copy_(pc.k)
    with pytest.raises(ValueError, match="paged k cache"):
        prefill_api(pc.q, k_odd, pc.v, pc.rel, pc.cu_q, pc.cu_k, 40, 40, 16,
                    block_table=pc.meta["block_table"])
