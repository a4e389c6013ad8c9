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
