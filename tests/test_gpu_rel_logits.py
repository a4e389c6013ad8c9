"""rel_logits producer on the GPU (``inkling_rel_logits`` -> ``ifa4_rel_logits_launch``) against
the CPU oracle (oracle/rel_logits_oracle.py).  The kernel's output is the oracle's fp32 value
rounded once to bf16; the tensor-core sums of 16 products may differ from numpy's in the last
fp32 bits, so a result may land on the other side of a bf16 rounding boundary: the bound is one
bf16 step (2^-8 relative) plus 1e-5, and at least 99 % of the elements must be bit-identical to
the oracle rounded to bf16."""
import numpy as np
import pytest
import torch

import oracle
from gpu_util import device_status_ok
from inkling_fa4 import inkling_fa4_rel_attention_triton, inkling_rel_logits
from inkling_fa4.workloads import cu_from_lens

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _status_clean():
    yield
    assert device_status_ok(), "a kernel abandoned a bounded wait"


def _inputs(total, heads, rel_extent, per_head, seed=0):
    g = torch.Generator().manual_seed(seed)
    r = torch.randn(total, heads, 16, generator=g).bfloat16()
    shape = (heads, 16, rel_extent) if per_head else (16, rel_extent)
    w = (0.5 * torch.randn(*shape, generator=g)).bfloat16()
    return r, w


def _check(got, want, what=""):
    got = got.float().cpu().numpy()
    want = np.asarray(want, np.float32)
    assert got.shape == want.shape, what
    err = np.abs(got - want)
    bound = np.abs(want) * 2.0 ** -8 + 1e-5
    assert np.all(err <= bound), f"{what}: max excess {np.max(err - bound)}"
    same = np.mean(got == oracle.round_to_bf16(want))
    assert same >= 0.99, f"{what}: only {same:.4f} bit-identical to the rounded oracle"


def _oracle(r, w, cu_q=None, cu_k=None, alpha=0.0, nf=1.0):
    return oracle.rel_logits_proj(r.float().numpy(), w.float().numpy(),
                                  None if cu_q is None else cu_q.numpy(),
                                  None if cu_k is None else cu_k.numpy(), alpha, nf)


@pytest.mark.parametrize("total,heads,rel_extent,per_head", [
    (1000, 4, 128, False), (1000, 4, 128, True), (300, 3, 1024, True), (257, 2, 64, False),
    (129, 5, 200, True), (64, 1, 8, False), (1, 2, 136, True), (4096, 12, 512, False)])
def test_projection_matches_oracle(total, heads, rel_extent, per_head):
    r, w = _inputs(total, heads, rel_extent, per_head)
    got = inkling_rel_logits(r.cuda(), w.cuda())
    _check(got, _oracle(r, w), f"T={total} H={heads} R={rel_extent} per_head={per_head}")


@pytest.mark.parametrize("chunked", [False, True])
def test_log_tau_over_ragged_sequences(chunked):
    lens_q = [700, 1, 0, 129, 2048]
    lens_k = [900, 5000, 3, 129, 2048] if chunked else None
    cu_q = cu_from_lens(lens_q)
    cu_k = cu_from_lens(lens_k) if chunked else None
    r, w = _inputs(sum(lens_q), 4, 256, True, seed=3)
    got = inkling_rel_logits(r.cuda(), w.cuda(), cu_q.cuda(),
                             None if cu_k is None else cu_k.cuda(), alpha=0.1, nf=64.0)
    _check(got, _oracle(r, w, cu_q, cu_k, 0.1, 64.0), f"chunked={chunked}")


def test_strided_input_and_wider_output():
    """r as a slice of a merged projection output; rel written into a wider buffer whose extra
    columns stay untouched."""
    total, heads, R = 333, 6, 128
    g = torch.Generator().manual_seed(5)
    merged = torch.randn(total, 1000 + heads * 16 + 8, generator=g).bfloat16()
    r = merged[:, 1000:1000 + heads * 16].view(total, heads, 16)
    w = (0.5 * torch.randn(16, R, generator=g)).bfloat16()
    out = torch.full((total, heads, R + 24), 7.0, dtype=torch.bfloat16, device="cuda")
    got = inkling_rel_logits(merged.cuda()[:, 1000:1000 + heads * 16].view(total, heads, 16),
                             w.cuda(), alpha=0.05, nf=16.0, out=out)
    assert got.data_ptr() == out.data_ptr()
    _check(out[:, :, :R], _oracle(r, w, alpha=0.05, nf=16.0), "strided")
    assert torch.all(out[:, :, R:] == 7.0)


def test_alpha_zero_equals_tau_one_and_shared_equals_broadcast():
    r, w = _inputs(777, 4, 128, False, seed=7)
    rd, wd = r.cuda(), w.cuda()
    a = inkling_rel_logits(rd, wd)
    b = inkling_rel_logits(rd, wd, alpha=0.3, nf=1e9)  # (pos + 1) / nf < 1 everywhere: tau = 1
    c = inkling_rel_logits(rd, wd.unsqueeze(0).expand(4, 16, 128).contiguous())
    assert torch.equal(a, b) and torch.equal(a, c)


def test_long_sequence_sampled_rows():
    """32k tokens x 32 heads (the bench's shape): rows sampled across the whole sequence."""
    total, heads, R = 32768, 32, 128
    r, w = _inputs(total, heads, R, True, seed=11)
    got = inkling_rel_logits(r.cuda(), w.cuda(), alpha=0.1, nf=4096.0)
    idx = np.sort(np.random.default_rng(0).choice(total, 512, replace=False))
    idx = np.concatenate([idx, [0, 127, 128, total - 1]])
    tau = oracle.log_tau(oracle.token_positions(total)[idx], 0.1, 4096.0)
    want = np.einsum("thd,hde->the", r[idx].float().numpy(), w.float().numpy(),
                     dtype=np.float32) * tau[:, None, None]
    _check(got[torch.from_numpy(idx).cuda()], want, "32k sampled")


def test_feeds_the_attention():
    """The producer's output is a valid rel_logits argument of the prefill (same result as the
    same values passed from a host-made tensor)."""
    lens = [300, 45]
    cu = cu_from_lens(lens).cuda()
    g = torch.Generator().manual_seed(2)
    q = torch.randn(345, 4, 128, generator=g).bfloat16().cuda()
    k = torch.randn(345, 2, 128, generator=g).bfloat16().cuda()
    v = torch.randn(345, 2, 128, generator=g).bfloat16().cuda()
    r, w = _inputs(345, 4, 128, True, seed=9)
    rel = inkling_rel_logits(r.cuda(), w.cuda(), cu, alpha=0.1, nf=32.0)
    o1 = inkling_fa4_rel_attention_triton(q, k, v, rel, cu, cu, 300, 300, 128)
    o2 = inkling_fa4_rel_attention_triton(q, k, v, rel.cpu().cuda(), cu, cu, 300, 300, 128)
    assert torch.equal(o1, o2)


def test_cuda_graph_capture():
    r, w = _inputs(1024, 8, 128, True, seed=4)
    rd, wd = r.cuda(), w.cuda()
    out = torch.empty(1024, 8, 128, dtype=torch.bfloat16, device="cuda")
    inkling_rel_logits(rd, wd, alpha=0.1, nf=8.0, out=out)  # warm (attributes, tensor maps)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        inkling_rel_logits(rd, wd, alpha=0.1, nf=8.0, out=out)
    out.zero_()
    graph.replay()
    torch.cuda.synchronize()
    _check(out, _oracle(r, w, alpha=0.1, nf=8.0), "graph replay")


def test_weight_slices():
    """A column slice of a wider weight (aligned: used in place) and an unaligned one (copied to
    a contiguous tensor by the wrapper) give the oracle's result."""
    r, _ = _inputs(500, 4, 128, False, seed=13)
    g = torch.Generator().manual_seed(13)
    wide = (0.5 * torch.randn(4, 16, 144, generator=g)).bfloat16()
    for lo in (8, 1):
        w = wide[:, :, lo:lo + 128]
        got = inkling_rel_logits(r.cuda(), wide.cuda()[:, :, lo:lo + 128], alpha=0.1, nf=16.0)
        _check(got, _oracle(r, w, alpha=0.1, nf=16.0), f"slice at {lo}")
