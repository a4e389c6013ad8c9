"""Prefill with the KV range of each query tile split over several CTAs (small launches that
would leave SMs idle), merged by a second kernel: parity with the oracle and with the unsplit
kernel, through the C ABI's workspace entry point (ifa4_prefill_launch_ws)."""
import ctypes

import numpy as np
import pytest
import torch

from gpu_util import (assert_close, device_status_ok, np32, oracle_full, oracle_rows,
                      to_dev)
from inkling_fa4 import _lib, _ops
from inkling_fa4.workloads import make_case, page_kv

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _status_clean():
    yield
    assert device_status_ok(), "a kernel abandoned a bounded wait"


def _prefill(c, **kw):
    return _ops.prefill(c.q, c.k, c.v, c.rel, c.cu_q, c.cu_k, c.max_q, c.max_k, c.rel_extent,
                        **kw)


def _workspace_bytes(c, kv_splits=0, **kw):
    q, k, v, rel, out, n_heads, kv_heads, R, wl, scale = _ops._prepare(
        "prefill", c.q, c.k, c.v, c.rel, c.cu_q, c.cu_k, c.rel_extent, True,
        kw.get("window_size", (-1, -1)), None, None, 128, None, "reference", None)
    p = _lib.PrefillParams()
    _ops._fill_lse(p, None)
    _ops._fill_common(p, q, k, v, rel, out, c.cu_q, c.cu_k, n_heads, kv_heads, R, True, wl,
                      "reference")
    p.max_seqlen_q, p.softmax_scale, p.kv_splits = c.max_q, scale, kv_splits
    n = ctypes.c_size_t(0)
    _lib.check(_lib.lib().ifa4_prefill_workspace_size(ctypes.byref(p), ctypes.byref(n)))
    return int(n.value)


def test_reference_benchmark_shape_splits_automatically():
    """S = 4096, Hq = Hkv = 4, R = 1024 (the reference's own benchmark shape): 64 CTAs on a
    148-SM GPU, so the launch splits the KV range; output and log-sum-exp match the oracle and
    the unsplit kernel."""
    c = make_case([4096], [4096], 4, 4, 1024, seed=3, device="cuda", rel_std=0.5)
    assert _workspace_bytes(c) > 0
    out, lse = _prefill(c, return_lse=True)
    ref, ref_lse = _prefill(c, kv_splits=1, return_lse=True)
    torch.cuda.synchronize()
    assert_close(np32(out), np32(ref), what="split vs unsplit")
    np.testing.assert_allclose(lse.cpu().numpy(), ref_lse.cpu().numpy(), atol=2e-3, rtol=1e-4)
    toks, want = oracle_rows(c, 40, [0, 1, 2, 3], 1 / 128, seed=4)
    assert_close(np32(out)[toks], want, what="split vs oracle")


@pytest.mark.parametrize("kv_splits", [2, 5, 16])
@pytest.mark.parametrize("window", [None, 150])
@pytest.mark.parametrize("heads,rext", [((4, 4), 128), ((8, 2), 1000), ((3, 1), 64)])
def test_forced_splits_match_the_oracle(kv_splits, window, heads, rext):
    """Ragged lengths around the tile edges, GQA layouts, windows and rel extents; 16 splits of
    short sequences leave most shares empty (they must weigh nothing in the merge)."""
    hq, hkv = heads
    lens = [1, 130, 700, 257, 1030]
    c = to_dev(make_case(lens, lens, hq, hkv, rext, seed=hq * 11 + kv_splits))
    kw = {} if window is None else {"window_size": (window, 0)}
    out, lse = _prefill(c, kv_splits=kv_splits, return_lse=True, **kw)
    want = oracle_full(c, 1 / 128, window_left=window)
    assert_close(np32(out), want, what=f"{kv_splits} splits")
    ref, ref_lse = _prefill(c, kv_splits=1, return_lse=True, **kw)
    np.testing.assert_allclose(lse.cpu().numpy(), ref_lse.cpu().numpy(), atol=2e-3, rtol=1e-4)


def test_split_chunked_paged_cache():
    """Bottom-right chunked prefill from a 16-token paged cache (NaN in unused slots)."""
    c = to_dev(make_case([256, 100], [1500, 900], 8, 2, 128, seed=9))
    pc = page_kv(c, page_size=16, seed=2)
    out = _ops.prefill(pc.q, pc.k, pc.v, pc.rel, pc.cu_q, pc.cu_k, pc.max_q, pc.max_k, 128,
                       causal_align="bottom_right", block_table=pc.meta["block_table"],
                       kv_splits=4)
    want = oracle_full(c, 1 / 128, causal_align="bottom_right")
    assert_close(np32(out), want, what="paged split")
    assert torch.isfinite(out.float()).all()


def test_rows_without_keys_stay_zero_when_split():
    """A sequence with no keys: every share is empty, so the merge writes 0 and -inf."""
    c = to_dev(make_case([64, 300], [0, 300], 4, 4, 64, seed=13))
    out, lse = _prefill(c, kv_splits=3, return_lse=True)
    want = oracle_full(c, 1 / 128)
    assert_close(np32(out), want)
    assert bool((out[:64].float() == 0).all())
    assert bool(torch.isneginf(lse[:, :64]).all())


def test_no_split_needs_no_workspace():
    c = make_case([4096], [4096], 32, 8, 128, seed=5, device="cuda")  # a full grid
    assert _workspace_bytes(c) == 0
    assert _workspace_bytes(c, kv_splits=1) == 0
    assert _workspace_bytes(c, kv_splits=4) > 0
