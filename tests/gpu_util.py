"""Helpers for the GPU parity tests: run the CUDA path through the public API / C ABI and the
CPU oracle on the same seeded inputs."""
import numpy as np
import pytest
import torch

import oracle
from inkling_fa4 import _lib, inkling_fa4_rel_attention_decode_triton, inkling_fa4_rel_attention_triton

ATOL = 2e-2  # bf16 inputs vs the fp32 oracle (north_star tolerance, tests/test_correctness.py:29)
RTOL = 2e-2

requires_cuda = pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU")


def to_dev(case, device="cuda"):
    for nm in ("q", "k", "v", "rel", "cu_q", "cu_k"):
        setattr(case, nm, getattr(case, nm).to(device))
    return case


def np32(t):
    return t.detach().float().cpu().numpy()


def run_prefill(c, **kw):
    return inkling_fa4_rel_attention_triton(c.q, c.k, c.v, c.rel, c.cu_q, c.cu_k, c.max_q,
                                            c.max_k, c.rel_extent, **kw)


def run_decode(c, **kw):
    return inkling_fa4_rel_attention_decode_triton(c.q, c.k, c.v, c.rel, c.cu_q, c.cu_k, 1,
                                                   c.max_k, c.rel_extent, **kw)


def oracle_full(c, scale, causal=True, window_left=None, causal_align="reference"):
    return oracle.rel_attn(np32(c.q), np32(c.k), np32(c.v), np32(c.rel), c.cu_q.cpu().numpy(),
                           c.cu_k.cpu().numpy(), scale, c.rel_extent, causal=causal,
                           window_left=window_left, causal_align=causal_align, row_block=512)


def oracle_rows(c, rows_per_seq, heads, scale, causal=True, window_left=None,
                causal_align="reference", seed=0):
    """Oracle for a sample of rows of every sequence.  Returns (token indices, heads, values
    [n_rows, n_heads, d])."""
    rng = np.random.default_rng(seed)
    cu_q = c.cu_q.cpu().numpy()
    cu_k = c.cu_k.cpu().numpy()
    hq, hkv = c.q.shape[1], c.k.shape[1]
    g = hq // hkv
    toks, vals = [], []
    q = c.q[:, heads].float().cpu().numpy()
    rel = c.rel[:, heads].float().cpu().numpy()
    for b in range(len(cu_q) - 1):
        qs, qe, ks, ke = int(cu_q[b]), int(cu_q[b + 1]), int(cu_k[b]), int(cu_k[b + 1])
        sq, sk = qe - qs, ke - ks
        if sq == 0:
            continue
        n = min(rows_per_seq, sq)
        pos = np.unique(np.concatenate([[0, sq - 1], rng.integers(0, sq, size=n)]))[:max(n, 2)]
        out = np.zeros((len(pos), len(heads), 128), np.float32)
        for j, h in enumerate(heads):
            kh = h // g
            kb = c.k[ks:ke, kh].float().cpu().numpy()
            vb = c.v[ks:ke, kh].float().cpu().numpy()
            out[:, j] = oracle.rel_attn_rows(q[qs + pos, j], kb, vb, rel[qs + pos, j], pos, sq, sk,
                                             scale, c.rel_extent, causal, window_left,
                                             causal_align)
        toks.append(qs + pos)
        vals.append(out)
    return np.concatenate(toks), np.concatenate(vals)


def assert_close(got, want, atol=ATOL, rtol=RTOL, what=""):
    got = np.asarray(got, np.float32)
    want = np.asarray(want, np.float32)
    nan = np.isnan(want)
    if nan.any():  # oracle NaN = row with no visible key; the kernels emit 0 there
        assert np.all(got[nan] == 0), f"{what}: rows without visible keys must be 0"
    np.testing.assert_allclose(got[~nan], want[~nan], atol=atol, rtol=rtol, err_msg=what)


def device_status_ok():
    return _lib.read_device_status(torch.cuda.current_stream().cuda_stream, clear=True) == 0
