"""The package's launch path through the torch operators (csrc/ifa4_torch_ops.cpp) against the
ctypes calls of the same C ABI: identical results, bit for bit, and the same errors."""
import pytest
import torch

from inkling_fa4 import _lib, _ops
from inkling_fa4.workloads import make_case, page_kv

pytestmark = pytest.mark.gpu


def _both(fn):
    assert _lib.torch_ops() is not None, "torch operator library not loaded"
    saved = _ops.USE_TORCH_OPS
    try:
        _ops.USE_TORCH_OPS = True
        a = fn()
        _ops.USE_TORCH_OPS = False
        b = fn()
    finally:
        _ops.USE_TORCH_OPS = saved
    torch.cuda.synchronize()
    return a, b


@pytest.mark.parametrize("lens,heads,kw", [
    ([600, 40, 129], (8, 2), {}),                                  # unsplit
    ([4096], (4, 4), {}),                                          # automatic KV split
    ([300, 257], (4, 2), {"window_size": (100, 0), "kv_splits": 3}),
])
def test_prefill_paths_agree(lens, heads, kw):
    c = make_case(lens, lens, heads[0], heads[1], 1000, seed=len(lens), device="cuda")
    a, b = _both(lambda: _ops.prefill(c.q, c.k, c.v, c.rel, c.cu_q, c.cu_k, c.max_q, c.max_k,
                                      1000, return_lse=True, **kw))
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])


def test_paged_prefill_and_decode_paths_agree():
    c = make_case([64, 200], [900, 1500], 8, 2, 128, seed=2, device="cuda")
    pc = page_kv(c, page_size=16, seed=3)
    a, b = _both(lambda: _ops.prefill(pc.q, pc.k, pc.v, pc.rel, pc.cu_q, pc.cu_k, pc.max_q,
                                      pc.max_k, 128, causal_align="bottom_right",
                                      block_table=pc.meta["block_table"]))
    assert torch.equal(a, b)
    d = make_case([1, 1, 1], [3000, 5, 700], 8, 2, 128, seed=4, device="cuda")
    pd = page_kv(d, page_size=32, seed=5)
    for case, bt in ((d, None), (pd, pd.meta["block_table"])):
        a, b = _both(lambda: _ops.decode(case.q, case.k, case.v, case.rel, case.cu_q, case.cu_k,
                                         1, 3000, 128, causal_align="bottom_right",
                                         return_lse=True, block_table=bt))
        assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])


def test_errors_surface_the_same_way():
    c = make_case([64], [64], 4, 4, 128, seed=1, device="cuda")
    pc = page_kv(c, page_size=16, seed=1)
    for use in (True, False):
        _ops.USE_TORCH_OPS = use
        try:
            with pytest.raises(_lib.Ifa4Error, match="paged-cache variant"):
                _ops.prefill(pc.q, pc.k, pc.v, pc.rel, pc.cu_q, pc.cu_k, 64, 64, 128,
                             tile_config=5, block_table=pc.meta["block_table"])
        finally:
            _ops.USE_TORCH_OPS = True
