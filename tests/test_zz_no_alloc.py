"""The no-allocation decode entry point, for callers that may not call cudaMalloc.

Serving engines that reserve all device memory up front, and plugins reached through a C FFI
with no handle on their host's allocator, cannot pass ``ifa4_decode_launch`` a workspace;
``ifa4_decode_launch_noalloc`` keeps the split-KV partials in a static array inside the library
instead.  This test calls both entry points through the C ABI on the same inputs and checks
that two consecutive no-alloc calls (which reuse the shared array) both match the workspace
version.  It is collected last so that a failure here comes after every other test ran, and it
also passes on its own in a fresh process (the first call performs the per-device set-up).
"""
import ctypes

import pytest
import torch

from gpu_util import ATOL, RTOL
from inkling_fa4 import _lib, _ops
from inkling_fa4.workloads import make_case

pytestmark = pytest.mark.gpu


def _params(c, out, num_splits=0, chunk_len=0):
    return _ops._decode_params(c.q, c.k, c.v, c.rel, out, c.cu_q, c.cu_k, c.q.shape[1],
                               c.k.shape[1], c.rel_extent, True, -1, "bottom_right", c.max_k,
                               1.0 / 128, num_splits, chunk_len)


def test_noalloc_decode_matches_workspace_decode_twice():
    L = _lib.lib()
    c = make_case([1] * 6, [7000, 1, 3000, 129, 12000, 640], 32, 8, 128, seed=31,
                  device="cuda")
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)

    ref = torch.empty_like(c.q)
    p = _params(c, ref)
    nbytes, splits, _ = _ops.decode_plan(p)
    assert splits > 1 and nbytes > 0  # the case exercises the split partials
    ws = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    _lib.check(L.ifa4_decode_launch(ctypes.byref(p), ctypes.c_void_p(ws.data_ptr()),
                                    ctypes.c_size_t(nbytes), stream))

    outs = []
    for _ in range(2):
        out = torch.full_like(c.q, float("nan"))
        _lib.check(L.ifa4_decode_launch_noalloc(ctypes.byref(_params(c, out)), stream))
        outs.append(out)
    torch.cuda.synchronize()
    assert _lib.read_device_status(stream.value or 0) == 0
    for out in outs:
        torch.testing.assert_close(out.float(), ref.float(), atol=ATOL, rtol=RTOL)
    torch.testing.assert_close(outs[0], outs[1], atol=0, rtol=0)


def test_noalloc_rejects_explicit_splits_beyond_the_static_scratch():
    L = _lib.lib()
    c = make_case([1] * 64, [64] * 64, 32, 8, 128, seed=2, device="cuda")
    out = torch.empty_like(c.q)
    # 64 sequences x 32 heads x 64 splits x 129 floats = 67.6 MB > 16 MiB
    p = _params(c, out, num_splits=64, chunk_len=64)
    rc = L.ifa4_decode_launch_noalloc(ctypes.byref(p), None)
    assert rc == _lib.IFA4_ERR_WORKSPACE
    assert b"static scratch" in L.ifa4_last_error_string()


def test_noalloc_caps_the_automatic_plan_when_partials_outgrow_the_scratch():
    """A batch whose automatic split plan needs more partials than the static array holds
    (128 sequences x 32 heads; the longest sequence asks for 10 chunks of 2048 keys, 21 MB of
    partials): the entry point caps the split count so that the partials fit, and CTAs then
    stride over more chunks than there are splits.  Output and log-sum-exp are checked against
    the workspace entry point on the same capped plan (bit for bit) and on its own uncapped
    plan (within the test tolerance)."""
    L = _lib.lib()
    lens = [20000] + [1024 + 97 * i for i in range(127)]
    c = make_case([1] * len(lens), lens, 32, 8, 128, seed=41, device="cuda", rel_std=0.5)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    nbytes, splits, chunk = _ops.decode_plan(_params(c, torch.empty_like(c.q)))
    assert nbytes > _lib.NOALLOC_DECODE_SCRATCH_BYTES  # the automatic plan does not fit
    per_split = len(lens) * 32 * 129 * 4
    capped = _lib.NOALLOC_DECODE_SCRATCH_BYTES // per_split
    assert 2 <= capped < splits and max(lens) > capped * chunk  # CTAs stride over chunks

    def lse_buf():
        return torch.full((32, len(lens)), float("nan"), dtype=torch.float32, device="cuda")

    def with_workspace(num_splits, chunk_len):
        out, lse = torch.full_like(c.q, float("nan")), lse_buf()
        p = _params(c, out, num_splits, chunk_len)
        _ops._fill_lse(p, lse)
        need, _, _ = _ops.decode_plan(p)
        ws = torch.empty(max(need, 16), dtype=torch.uint8, device="cuda")
        _lib.check(L.ifa4_decode_launch(ctypes.byref(p), ctypes.c_void_p(ws.data_ptr()),
                                        ctypes.c_size_t(need), stream))
        torch.cuda.synchronize()
        return out, lse

    ref_out, ref_lse = with_workspace(0, 0)                # uncapped automatic plan
    cap_out, cap_lse = with_workspace(int(capped), chunk)  # the plan the no-alloc call uses
    for _ in range(2):
        out, lse = torch.full_like(c.q, float("nan")), lse_buf()
        p = _params(c, out)
        _ops._fill_lse(p, lse)
        _lib.check(L.ifa4_decode_launch_noalloc(ctypes.byref(p), stream))
        torch.cuda.synchronize()
        assert _lib.read_device_status(stream.value or 0) == 0
        assert torch.equal(out, cap_out) and torch.equal(lse, cap_lse)
        torch.testing.assert_close(out.float(), ref_out.float(), atol=ATOL, rtol=RTOL)
        torch.testing.assert_close(lse, ref_lse, atol=2e-3, rtol=1e-4)
