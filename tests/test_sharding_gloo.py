"""Multi-rank sharding logic on CPU with the gloo backend (world size 2 and 4).

Each rank computes its KV-head-group shard (with the CPU oracle standing in for the kernel,
which needs a GPU) and the shards are all-gathered; the result must equal the unsharded
computation exactly.  Sequence balancing is checked for coverage and balance."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from inkling_fa4.sharding import balance_sequences, head_shard, select_sequences, shard_tensors


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, result_q):
    import torch.distributed as dist

    import oracle
    from inkling_fa4.sharding import gather_heads, head_shard, shard_tensors
    from inkling_fa4.workloads import make_case

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        c = make_case([70, 33, 129], [70, 33, 129], 16, 4, 64, seed=3)
        sh = head_shard(16, 4, world, rank)
        q, k, v, rel = shard_tensors(sh, c.q, c.k, c.v, c.rel)
        part = torch.from_numpy(oracle.rel_attn(q.float().numpy(), k.float().numpy(),
                                                v.float().numpy(), rel.float().numpy(),
                                                c.cu_q.numpy(), c.cu_k.numpy(), 1 / 128, 64))
        full = gather_heads(part, world)
        if rank == 0:
            result_q.put(full.numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_head_sharded_all_gather_equals_unsharded(world):
    import oracle
    from inkling_fa4.workloads import make_case

    ctx = mp.get_context("spawn")
    q_out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q_out)) for r in range(world)]
    for p in procs:
        p.start()
    got = q_out.get(timeout=180)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    c = make_case([70, 33, 129], [70, 33, 129], 16, 4, 64, seed=3)
    want = oracle.rel_attn(c.q.float().numpy(), c.k.float().numpy(), c.v.float().numpy(),
                           c.rel.float().numpy(), c.cu_q.numpy(), c.cu_k.numpy(), 1 / 128, 64)
    np.testing.assert_array_equal(got, want)


def test_head_shard_arithmetic():
    shards = [head_shard(32, 8, 4, r) for r in range(4)]
    assert [(s.kv_lo, s.kv_hi, s.q_lo, s.q_hi) for s in shards] == [
        (0, 2, 0, 8), (2, 4, 8, 16), (4, 6, 16, 24), (6, 8, 24, 32)]
    assert head_shard(32, 8, 8, 7).n_q == 4
    with pytest.raises(ValueError):
        head_shard(32, 8, 3, 0)
    with pytest.raises(ValueError):
        head_shard(32, 8, 2, 2)


def test_shard_views_share_storage():
    from inkling_fa4.workloads import make_case
    c = make_case([10], [10], 8, 2, 16)
    q, k, v, rel = shard_tensors(head_shard(8, 2, 2, 1), c.q, c.k, c.v, c.rel)
    assert q.data_ptr() == c.q[:, 4].data_ptr() and k.shape[1] == 1
    assert q.stride() == c.q.stride()


def test_balance_sequences_covers_and_balances():
    lens = [4000, 10, 3990, 2000, 2100, 7, 1, 4096, 512, 3000]
    for world in (1, 2, 4, 8):
        groups = balance_sequences(lens, world)
        assert sorted(i for g in groups for i in g) == list(range(len(lens)))
        loads = [sum(lens[i] for i in g) for g in groups]
        assert max(loads) - min(loads) <= max(lens)


def test_select_sequences_packs_subset():
    from inkling_fa4.workloads import make_case
    c = make_case([3, 5, 2], [4, 6, 1], 4, 2, 8)
    q, rel, k, v, cq, ck = select_sequences([0, 2], c.cu_q, c.cu_k, c.q, c.rel, c.k, c.v)
    assert cq.tolist() == [0, 3, 5] and ck.tolist() == [0, 4, 5]
    assert torch.equal(q[3:], c.q[8:10]) and torch.equal(k[4:], c.k[10:11])


def test_peer_ptrs_offsets_follow_the_view():
    """PeerOutputs.peer_ptrs gives, for a view into this rank's buffer, the same byte offset in
    every other rank's buffer (the address arithmetic only; the IPC mapping needs GPUs)."""
    import torch

    from inkling_fa4.sharding import PeerOutputs, head_shard

    po = object.__new__(PeerOutputs)
    po.local = torch.empty((10, 8, 128), dtype=torch.bfloat16)
    po.rank, po.world = 1, 4
    po.bases = [1 << 40, po.local.data_ptr(), 3 << 40, 5 << 40]
    sh = head_shard(8, 4, 4, 1)
    view = po.local[:, sh.q_lo:sh.q_hi]
    off = sh.q_lo * 128 * 2
    assert po.peer_ptrs(view) == [(1 << 40) + off, (3 << 40) + off, (5 << 40) + off]
    with pytest.raises(ValueError):
        po.peer_ptrs(torch.empty(4, dtype=torch.bfloat16))
    po.bases = [None, po.local.data_ptr(), None, None]  # the state close() leaves
    with pytest.raises(RuntimeError):
        po.peer_ptrs(view)
