"""The entry points launch asynchronously on torch's current stream and never synchronise with
the host, so they can be captured in a CUDA graph: capture prefill (with LSE), split-KV decode
(paged cache) and the backward once, replay with new input values, and compare with eager
calls bit for bit."""
import pytest
import torch

from gpu_util import device_status_ok
from inkling_fa4 import (inkling_fa4_rel_attention_backward,
                         inkling_fa4_rel_attention_decode_triton,
                         inkling_fa4_rel_attention_triton)
from inkling_fa4.workloads import make_case, page_kv

pytestmark = pytest.mark.gpu


def test_capture_and_replay_prefill_decode_backward():
    dev = torch.device("cuda")
    c = make_case([300, 77, 513], [300, 77, 513], 8, 2, 128, seed=3, device=dev)
    d = page_kv(make_case([1] * 3, [4000, 16, 700], 8, 2, 128, seed=4, device=dev), page_size=16)
    dout = torch.randn_like(c.q)
    ws = torch.empty(32 << 20, dtype=torch.uint8, device=dev)
    bws = torch.empty(c.q.shape[1] * c.q.shape[0] * 4, dtype=torch.uint8, device=dev)
    grads = [torch.empty_like(c.q), torch.empty_like(c.k), torch.empty_like(c.v),
             torch.empty_like(c.rel)]

    def step():
        out, lse = inkling_fa4_rel_attention_triton(c.q, c.k, c.v, c.rel, c.cu_q, c.cu_k, 513,
                                                    513, 128, return_lse=True)
        dec = inkling_fa4_rel_attention_decode_triton(
            d.q, d.k, d.v, d.rel, d.cu_q, d.cu_k, 1, 4000, 128, causal_align="bottom_right",
            workspace=ws, block_table=d.meta["block_table"])
        g = inkling_fa4_rel_attention_backward(dout, c.q, c.k, c.v, c.rel, out, lse, c.cu_q,
                                               c.cu_k, 513, 513, 128, dq=grads[0], dk=grads[1],
                                               dv=grads[2], drel=grads[3], workspace=bws)
        return out, lse, dec, g

    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(2):  # warm-up outside capture (per-device attributes, tensor maps)
            step()
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        outs = step()
    # new input values in the same buffers, then replay
    for t in (c.q, c.k, c.v, d.q, dout):
        t.copy_(torch.randn_like(t))
    graph.replay()
    torch.cuda.synchronize()
    replayed = [outs[0].clone(), outs[1].clone(), outs[2].clone()] + [x.clone() for x in outs[3]]
    eager = step()
    torch.cuda.synchronize()
    want = [eager[0], eager[1], eager[2]] + list(eager[3])
    for got, ref in zip(replayed, want):
        assert torch.equal(got, ref)
    assert device_status_ok()
