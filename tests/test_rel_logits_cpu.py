"""rel_logits producer, the parts that need no GPU: the CPU oracle's formula (positions, tau,
projection), the C ABI's argument validation (rejected before any CUDA call) and the Python
entry point's refusal of CPU tensors.  The reference repository has no code for this step
(only the diagram at outputs/architecture.md:51-64), so these known answers are worked out from
that formula by hand."""
import ctypes
import math

import numpy as np
import pytest
import torch

import oracle
from inkling_fa4 import _lib, inkling_rel_logits


def test_positions_single_sequence():
    assert oracle.token_positions(5).tolist() == [0, 1, 2, 3, 4]


def test_positions_ragged_and_chunked():
    cu_q = [0, 3, 3, 5]          # lengths 3, 0, 2
    assert oracle.token_positions(5, cu_q).tolist() == [0, 1, 2, 0, 1]
    cu_k = [0, 10, 14, 16]       # key lengths 10, 4, 2: queries are the last len_q keys
    assert oracle.token_positions(5, cu_q, cu_k).tolist() == [7, 8, 9, 0, 1]


def test_log_tau_known_values():
    pos = np.array([0, 63, 64, 127, 1023], np.int64)
    tau = oracle.log_tau(pos, 0.1, 64.0)
    assert tau.dtype == np.float32
    # (pos + 1) / nf <= 1 -> tau = 1; otherwise 1 + 0.1 * log((pos + 1) / 64)
    want = [1.0, 1.0, 1 + 0.1 * math.log(65 / 64), 1 + 0.1 * math.log(2.0),
            1 + 0.1 * math.log(16.0)]
    np.testing.assert_allclose(tau, want, rtol=1e-6)


def test_projection_matches_einsum_and_alpha_zero_is_plain():
    rng = np.random.default_rng(0)
    r = rng.standard_normal((7, 3, 16)).astype(np.float32)
    w = rng.standard_normal((16, 24)).astype(np.float32)
    got = oracle.rel_logits_proj(r, w)
    want = np.einsum("thd,de->the", r.astype(np.float64), w.astype(np.float64))
    np.testing.assert_allclose(got, want, rtol=1e-5, atol=1e-5)
    # per-head weights equal to the shared one give the same result
    wh = np.broadcast_to(w, (3, 16, 24))
    np.testing.assert_array_equal(oracle.rel_logits_proj(r, wh), got)


def test_tau_scales_each_token():
    rng = np.random.default_rng(1)
    r = rng.standard_normal((6, 2, 16)).astype(np.float32)
    w = rng.standard_normal((16, 8)).astype(np.float32)
    cu_q = [0, 4, 6]
    base = oracle.rel_logits_proj(r, w, cu_q)
    scaled = oracle.rel_logits_proj(r, w, cu_q, alpha=0.1, nf=2.0)
    tau = oracle.log_tau(oracle.token_positions(6, cu_q), 0.1, 2.0)
    np.testing.assert_allclose(scaled, base * tau[:, None, None], rtol=1e-6)
    assert tau[0] == 1.0 and tau[4] == 1.0 and tau[3] > 1.0


def _params(**kw):
    p = _lib.RelLogitsParams()
    p.total_q, p.batch, p.n_heads, p.d_rel, p.rel_extent = 16, 1, 4, 16, 128
    p.alpha, p.nf = 0.1, 64.0
    for k, v in kw.items():
        setattr(p, k, v)
    return p


_OK_PTRS = dict(r=256, weight=256, rel=256, r_stride_t=64, r_stride_h=16, weight_stride_h=0,
                weight_stride_j=128, rel_stride_t=512, rel_stride_h=128)


@pytest.mark.parametrize("kw,code,msg", [
    (dict(dtype=2), _lib.IFA4_ERR_UNSUPPORTED, b"dtype"),
    (dict(d_rel=32), _lib.IFA4_ERR_UNSUPPORTED, b"d_rel"),
    (dict(rel_extent=100), _lib.IFA4_ERR_UNSUPPORTED, b"multiple of 8"),
    (dict(rel_extent=0), _lib.IFA4_ERR_INVALID_ARGUMENT, b"rel_extent"),
    (dict(n_heads=0), _lib.IFA4_ERR_INVALID_ARGUMENT, b"n_heads"),
    (dict(nf=0.0), _lib.IFA4_ERR_INVALID_ARGUMENT, b"nf"),
    (dict(nf=float("inf")), _lib.IFA4_ERR_INVALID_ARGUMENT, b"nf"),
    (dict(alpha=float("nan")), _lib.IFA4_ERR_INVALID_ARGUMENT, b"alpha"),
    (dict(cu_seqlens_k=64), _lib.IFA4_ERR_INVALID_ARGUMENT, b"without cu_seqlens_q"),
    (dict(cu_seqlens_q=64, batch=0), _lib.IFA4_ERR_INVALID_ARGUMENT, b"batch"),
    (dict(), _lib.IFA4_ERR_INVALID_ARGUMENT, b"null"),
    (dict(_OK_PTRS, r=264), _lib.IFA4_ERR_INVALID_ARGUMENT, b"16-byte"),
    (dict(_OK_PTRS, r_stride_h=12), _lib.IFA4_ERR_INVALID_ARGUMENT, b"multiples of 8"),
    (dict(_OK_PTRS, rel_stride_t=100), _lib.IFA4_ERR_INVALID_ARGUMENT, b"multiples of 8"),
    (dict(_OK_PTRS, weight_stride_j=-1), _lib.IFA4_ERR_INVALID_ARGUMENT, b"weight"),
    (dict(_OK_PTRS, weight_stride_j=100), _lib.IFA4_ERR_INVALID_ARGUMENT, b"weight"),
    (dict(_OK_PTRS, weight=258), _lib.IFA4_ERR_INVALID_ARGUMENT, b"weight"),
])
def test_validation_rejects_before_any_cuda_call(kw, code, msg):
    L = _lib.lib()
    assert L.ifa4_rel_logits_launch(ctypes.byref(_params(**kw)), None) == code
    assert msg in L.ifa4_last_error_string()


def test_null_params_and_empty_input():
    L = _lib.lib()
    assert L.ifa4_rel_logits_launch(None, None) == _lib.IFA4_ERR_INVALID_ARGUMENT
    assert L.ifa4_rel_logits_launch(ctypes.byref(_params(total_q=0)), None) == _lib.IFA4_OK


def test_python_api_refuses_cpu_tensors_and_bad_shapes():
    r = torch.zeros(4, 2, 16, dtype=torch.bfloat16)
    w = torch.zeros(16, 64, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        inkling_rel_logits(r, w)
    with pytest.raises(TypeError):
        inkling_rel_logits(r.float().numpy(), w)
