"""KV-head-group sharding on 2 GPUs (one process per GPU, NCCL): each rank runs the prefill and
decode kernels on its head slices (views of the full tensors), the output heads are
all-gathered (or, for the prefill, stored by each rank's kernel into every rank's output
buffer through CUDA IPC mappings), and the result must equal the unsharded single-GPU
computation bit for bit (the per-head computation is identical).  Skipped on boxes with fewer
than 2 GPUs."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank_main(rank, world, port, q_out):
    import datetime

    import torch.distributed as dist

    from inkling_fa4 import (_ops, inkling_fa4_rel_attention_decode_triton,
                             inkling_fa4_rel_attention_triton)
    from inkling_fa4.sharding import (PeerOutputs, gather_heads, head_shard,
                                      prefill_to_all_ranks, shard_tensors)
    from inkling_fa4.workloads import make_case

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        dev = torch.device("cuda", rank)
        c = make_case([700, 129, 1000], [700, 129, 1000], 16, 4, 128, seed=77, device=dev)
        sh = head_shard(16, 4, world, rank)
        q, k, v, rel = shard_tensors(sh, c.q, c.k, c.v, c.rel)
        # The same launch plan on both sides (an unsplit KV range): the automatic plan may split
        # the smaller sharded grid's KV ranges and merge fp32 partials, which rounds differently
        # from the unsharded call; that path is checked against it within the bf16 tolerance.
        part = _ops.prefill(q, k, v, rel, c.cu_q, c.cu_k, 1000, 1000, 128, kv_splits=1)
        full = gather_heads(part, world)
        auto = gather_heads(
            inkling_fa4_rel_attention_triton(q, k, v, rel, c.cu_q, c.cu_k, 1000, 1000, 128), world)
        peers = PeerOutputs(tuple(c.q.shape), device=dev)
        peers.local.fill_(float("nan"))  # every element must come from the kernels' stores
        peers.barrier()
        fused = []
        for _ in range(2):  # the second call overwrites the buffers the first one filled
            fused.append(prefill_to_all_ranks(peers, sh, q, k, v, rel, c.cu_q, c.cu_k, 1000, 1000,
                                              128).clone())
            peers.barrier()
        peers.close()  # collective: no rank frees its buffer while another still maps it
        closed_ok = all(b is None for r, b in enumerate(peers.bases) if r != rank)
        d = make_case([1] * 4, [3000, 70, 5000, 640], 16, 4, 128, seed=78, device=dev)
        dq, dk, dv, drel = shard_tensors(sh, d.q, d.k, d.v, d.rel)
        # a fixed split plan keeps the per-head arithmetic identical to the unsharded call
        dpart = inkling_fa4_rel_attention_decode_triton(dq, dk, dv, drel, d.cu_q, d.cu_k, 1, 5000,
                                                        128, causal_align="bottom_right",
                                                        num_splits=4, chunk_len=512)
        dfull = gather_heads(dpart, world)
        torch.cuda.synchronize()
        if rank == 0:
            ref = _ops.prefill(c.q, c.k, c.v, c.rel, c.cu_q, c.cu_k, 1000, 1000, 128, kv_splits=1)
            dref = inkling_fa4_rel_attention_decode_triton(d.q, d.k, d.v, d.rel, d.cu_q, d.cu_k, 1,
                                                           5000, 128, causal_align="bottom_right",
                                                           num_splits=4, chunk_len=512)
            q_out.put({"prefill": bool(torch.equal(full, ref)),
                       "decode": bool(torch.equal(dfull, dref)),
                       "peer_stores": all(bool(torch.equal(f, ref)) for f in fused),
                       "closed": closed_ok,
                       "auto_max_err": float((auto.float() - ref.float()).abs().max().item())})
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_head_sharded_prefill_and_decode_on_two_gpus():
    ctx = mp.get_context("spawn")
    q_out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q_out)) for r in range(2)]
    for p in procs:
        p.start()
    res = q_out.get(timeout=300)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert res["prefill"], res
    assert res["decode"], res
    assert res["peer_stores"], res
    assert res["closed"], res
    assert res["auto_max_err"] <= 2e-2, res  # bf16 outputs, automatic (possibly split) plan


@pytest.mark.parametrize("world", [2, 4])
def test_head_shards_on_one_gpu_equal_the_unsharded_call(world):
    """The per-rank computation of the split above, every shard on one GPU: with the same launch
    plan (unsplit KV ranges) the shards' outputs, concatenated in rank order, equal the unsharded
    call bit for bit; with the automatic plan (which may split a shard's smaller grid) they agree
    within the bf16 tolerance."""
    from inkling_fa4 import _ops, inkling_fa4_rel_attention_triton
    from inkling_fa4.sharding import head_shard, shard_tensors
    from inkling_fa4.workloads import make_case

    c = make_case([700, 129, 1000], [700, 129, 1000], 16, 4, 128, seed=77, device="cuda")
    ref = _ops.prefill(c.q, c.k, c.v, c.rel, c.cu_q, c.cu_k, 1000, 1000, 128, kv_splits=1)
    pinned, auto = [], []
    for r in range(world):
        q, k, v, rel = shard_tensors(head_shard(16, 4, world, r), c.q, c.k, c.v, c.rel)
        pinned.append(_ops.prefill(q, k, v, rel, c.cu_q, c.cu_k, 1000, 1000, 128, kv_splits=1))
        auto.append(inkling_fa4_rel_attention_triton(q, k, v, rel, c.cu_q, c.cu_k, 1000, 1000,
                                                     128))
    assert torch.equal(torch.cat(pinned, dim=1), ref)
    err = (torch.cat(auto, dim=1).float() - ref.float()).abs().max().item()
    assert err <= 2e-2, err
