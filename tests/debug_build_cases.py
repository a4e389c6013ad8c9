"""Cases run against both library builds by tests/test_gpu_debug_build.py: every kernel family
(prefill contiguous / paged / split / with LSE, decode contiguous / paged / split, backward,
rel_logits producer) on ragged shapes around the tile edges.  ``python debug_build_cases.py
OUT.pt`` runs them with whichever library ``INKLING_FA4_LIB`` selects and saves the outputs and
the device status word."""
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(os.path.dirname(HERE), "inkling-fa4-relative-attention_b200"))

import torch  # noqa: E402


def run_cases():
    from inkling_fa4 import (_lib, _ops, inkling_fa4_rel_attention_backward,
                             inkling_fa4_rel_attention_decode_triton, inkling_rel_logits)
    from inkling_fa4.workloads import make_case, page_kv

    out = {}
    lens = [1, 129, 300, 17, 1000]
    c = make_case(lens, lens, 8, 2, 1000, seed=1, device="cuda")
    out["prefill"], out["prefill_lse"] = _ops.prefill(
        c.q, c.k, c.v, c.rel, c.cu_q, c.cu_k, c.max_q, c.max_k, 1000, window_size=(200, 0),
        kv_splits=1, return_lse=True)
    out["prefill_split"] = _ops.prefill(c.q, c.k, c.v, c.rel, c.cu_q, c.cu_k, c.max_q, c.max_k,
                                        1000, kv_splits=5)
    ch = make_case([64, 200], [900, 1500], 8, 2, 128, seed=2, device="cuda")
    pc = page_kv(ch, page_size=16, seed=3)
    out["prefill_paged"] = _ops.prefill(pc.q, pc.k, pc.v, pc.rel, pc.cu_q, pc.cu_k, pc.max_q,
                                        pc.max_k, 128, causal_align="bottom_right",
                                        block_table=pc.meta["block_table"], kv_splits=1)
    d = make_case([1, 1, 1], [3000, 5, 700], 8, 2, 128, seed=4, device="cuda")
    out["decode"] = inkling_fa4_rel_attention_decode_triton(
        d.q, d.k, d.v, d.rel, d.cu_q, d.cu_k, 1, 3000, 128, causal_align="bottom_right",
        num_splits=3, chunk_len=256)
    pd = page_kv(d, page_size=32, seed=5)
    out["decode_paged"] = inkling_fa4_rel_attention_decode_triton(
        pd.q, pd.k, pd.v, pd.rel, pd.cu_q, pd.cu_k, 1, 3000, 128, causal_align="bottom_right",
        block_table=pd.meta["block_table"])
    b = make_case([150, 40], [150, 40], 4, 2, 64, seed=6, device="cuda")
    bo, bl = _ops.prefill(b.q, b.k, b.v, b.rel, b.cu_q, b.cu_k, 150, 150, 64, kv_splits=1,
                          return_lse=True)
    g = torch.randn(b.q.shape, generator=torch.Generator().manual_seed(7)).to(torch.bfloat16)
    for name, t in zip(("dq", "dk", "dv", "drel"), inkling_fa4_rel_attention_backward(
            g.cuda(), b.q, b.k, b.v, b.rel, bo, bl, b.cu_q, b.cu_k, 150, 150, 64)):
        out[name] = t
    gen = torch.Generator().manual_seed(8)
    r = torch.randn(300, 4, 16, generator=gen).to(torch.bfloat16).cuda()
    w = (0.5 * torch.randn(4, 16, 128, generator=gen)).to(torch.bfloat16).cuda()
    out["rel_logits"] = inkling_rel_logits(r, w, torch.tensor([0, 200, 300], dtype=torch.int32,
                                                               device="cuda"), alpha=0.1, nf=16.0)
    torch.cuda.synchronize()
    status = _lib.read_device_status(torch.cuda.current_stream().cuda_stream)
    return {k: v.cpu() for k, v in out.items()}, status, _lib.LIB_PATH


if __name__ == "__main__":
    outs, status, path = run_cases()
    torch.save({"outs": outs, "status": status, "lib": path}, sys.argv[1])
