"""Failure detection on the GPU without a fault: a kernel's barrier wait that can never complete
runs out after its limit, reports through the status word, makes the other waiter leave through
the abort flag, and leaves the context usable (no trap, no hang, no bad address)."""
import numpy as np
import pytest
import torch

import oracle
from gpu_util import np32, run_prefill, to_dev
from inkling_fa4 import _lib
from inkling_fa4.workloads import make_case

pytestmark = pytest.mark.gpu


def test_bounded_wait_runs_out_and_reports():
    L = _lib.lib()
    stream = torch.cuda.current_stream().cuda_stream
    assert _lib.read_device_status(stream, clear=True) == 0
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    _lib.check(L.ifa4_selftest_bounded_wait(20_000_000, stream))  # 20 ms limit
    e1.record()
    status = _lib.read_device_status(stream, clear=True)  # synchronises
    ms = e0.elapsed_time(e1)
    assert status == 8, f"status {status}: expected the timeout bit only (abort propagated)"
    assert 15.0 <= ms < 150.0, f"kernel took {ms:.1f} ms for a 20 ms limit (the other waiter's own is 200 ms)"
    # the context is intact: a prefill afterwards is correct and reports no abandoned wait
    c = to_dev(make_case([200, 77], [200, 77], 8, 2, 128, seed=9))
    out = run_prefill(c)
    want = oracle.rel_attn(np32(c.q), np32(c.k), np32(c.v), np32(c.rel), c.cu_q.cpu().numpy(),
                           c.cu_k.cpu().numpy(), 1 / 128, 128)
    np.testing.assert_allclose(np32(out), want, atol=2e-2, rtol=2e-2)
    assert _lib.read_device_status(stream, clear=True) == 0


def test_selftest_rejects_bad_limits():
    L = _lib.lib()
    for bad in (0, -5, 2_000_000_000):
        assert L.ifa4_selftest_bounded_wait(bad, None) == _lib.IFA4_ERR_INVALID_ARGUMENT
