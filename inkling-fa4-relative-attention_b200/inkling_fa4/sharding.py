"""Multi-GPU sharding of the attention call (one process per GPU, torch.distributed).

The path shards with no exchange during compute:

* by KV-head group: rank r of n owns kv heads [r*Hkv/n, (r+1)*Hkv/n) and their query heads
  [r*Hq/n, (r+1)*Hq/n); it runs the kernels on head slices of q/k/v/rel (views, no copies:
  the kernels take arbitrary head strides) for all sequences.  The full output reaches every
  rank either through the all-gather of the output heads (``gather_heads``, NCCL over
  NVLink, then a head-interleaving copy) or, for the prefill, during the call itself
  (``prefill_to_all_ranks``): each rank's kernel stores its heads' rows into every rank's
  output buffer (``PeerOutputs``, mapped with CUDA IPC) as its tiles finish, and one small
  all-reduce afterwards orders the other ranks' reads after those stores.
* by sequence: ``balance_sequences`` splits a ragged batch into n groups of nearly equal
  token count (for decode, nearly equal KV bytes); each rank runs its sequences.

No kernel reads another GPU's memory; the only remote accesses are the plain 16-byte stores
of finished output rows (no TMA, no multicast).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class HeadShard:
    rank: int
    world: int
    kv_lo: int
    kv_hi: int
    q_lo: int
    q_hi: int

    @property
    def n_q(self) -> int:
        return self.q_hi - self.q_lo

    @property
    def n_kv(self) -> int:
        return self.kv_hi - self.kv_lo


def head_shard(n_heads: int, kv_heads: int, world: int, rank: int) -> HeadShard:
    """KV-head-group shard of rank ``rank`` (GQA groups are never split)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} / world {world}")
    if n_heads % kv_heads:
        raise ValueError("n_heads must be a multiple of kv_heads")
    if kv_heads % world:
        raise ValueError(f"kv_heads {kv_heads} not divisible by world size {world}")
    g = n_heads // kv_heads
    per = kv_heads // world
    kv_lo = rank * per
    return HeadShard(rank, world, kv_lo, kv_lo + per, kv_lo * g, (kv_lo + per) * g)


def shard_tensors(sh: HeadShard, q, k, v, rel):
    """Head-slice views of the inputs for one rank."""
    return (q[:, sh.q_lo:sh.q_hi], k[:, sh.kv_lo:sh.kv_hi], v[:, sh.kv_lo:sh.kv_hi],
            rel[:, sh.q_lo:sh.q_hi])


def gather_heads(out_shard: torch.Tensor, world: int, group=None) -> torch.Tensor:
    """All-gather per-rank outputs [T, Hq/n, d] into the full [T, Hq, d] (rank-ordered head
    blocks).  NCCL uses one all_gather_into_tensor; other backends fall back to all_gather."""
    import torch.distributed as dist

    t, hs, d = out_shard.shape
    src = out_shard.contiguous()
    if dist.get_backend(group) == "nccl":
        buf = torch.empty((world, t, hs, d), dtype=src.dtype, device=src.device)
        dist.all_gather_into_tensor(buf, src, group=group)
    else:
        parts = [torch.empty_like(src) for _ in range(world)]
        dist.all_gather(parts, src, group=group)
        buf = torch.stack(parts)
    return buf.permute(1, 0, 2, 3).reshape(t, world * hs, d)


def balance_sequences(lengths, world: int, weights=None):
    """Greedy longest-first assignment of sequences to ``world`` ranks by weight (default:
    length).  Returns, per rank, the sorted list of sequence indices."""
    w = list(lengths if weights is None else weights)
    order = sorted(range(len(w)), key=lambda i: -w[i])
    load = [0] * world
    groups = [[] for _ in range(world)]
    for i in order:
        r = min(range(world), key=lambda j: (load[j], j))
        groups[r].append(i)
        load[r] += w[i]
    return [sorted(g) for g in groups]


def select_sequences(idx, cu_q, cu_k, *tensors_q_k):
    """Pack the chosen sequences into contiguous varlen tensors.  ``tensors_q_k`` is
    (q, rel, k, v); returns (q, rel, k, v, cu_q, cu_k) for the subset (host-side index
    arithmetic; the copies run on the tensors' device)."""
    q, rel, k, v = tensors_q_k
    cq = [int(x) for x in cu_q.tolist()]
    ck = [int(x) for x in cu_k.tolist()]
    rows_q = torch.cat([torch.arange(cq[i], cq[i + 1]) for i in idx]) if idx else torch.zeros(0, dtype=torch.long)
    rows_k = torch.cat([torch.arange(ck[i], ck[i + 1]) for i in idx]) if idx else torch.zeros(0, dtype=torch.long)
    lq = [cq[i + 1] - cq[i] for i in idx]
    lk = [ck[i + 1] - ck[i] for i in idx]
    new_cq = torch.tensor([0] + list(torch.tensor(lq).cumsum(0).tolist() if lq else []), dtype=torch.int32)
    new_ck = torch.tensor([0] + list(torch.tensor(lk).cumsum(0).tolist() if lk else []), dtype=torch.int32)
    dev = q.device
    rq, rk = rows_q.to(dev), rows_k.to(dev)
    return (q.index_select(0, rq), rel.index_select(0, rq), k.index_select(0, rk),
            v.index_select(0, rk), new_cq.to(dev), new_ck.to(dev))


class PeerOutputs:
    """One output buffer of the same shape on every rank, each rank's buffer mapped into every
    other rank's address space with CUDA IPC (torch's CUDA storage sharing: cudaIpcGetMemHandle
    / cudaIpcOpenMemHandle, a plain peer mapping over NVLink, no multicast object).  Collective:
    every rank of ``group`` constructs it with the same shape.  ``local`` is this rank's buffer;
    ``peer_ptrs(view)`` gives, for a view into ``local``, the addresses of the same elements in
    the other ranks' buffers (valid in this process)."""

    def __init__(self, shape, dtype=torch.bfloat16, device=None, group=None):
        import torch.distributed as dist

        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.local = torch.empty(shape, dtype=dtype, device=device)
        info = self.local.untyped_storage()._share_cuda_()
        infos = [None] * self.world
        dist.all_gather_object(infos, info, group=group)
        self._mapped = []  # keeps the other ranks' mapped storages open
        self.bases = []
        local_dev = self.local.device.index
        for r, (_dev, handle, size, offset, rc_handle, rc_offset, ev_handle, _ev_sync) in \
                enumerate(infos):
            if r == self.rank:
                self.bases.append(self.local.data_ptr())
                continue
            # Opened with this rank's own device current: cudaIpcOpenMemHandle maps the other
            # GPU's allocation into this device's context and enables this device's peer access
            # to it, so this device's kernels can store there.  (Opening it under the owner's
            # device index would map it into a context this device's kernels do not run in.)
            # No IPC event wait: the ranks order their accesses with barriers.
            st = torch.UntypedStorage._new_shared_cuda(local_dev, handle, size, offset,
                                                       rc_handle, rc_offset, ev_handle, False)
            self._mapped.append(st)
            self.bases.append(st.data_ptr())
        self._flag = torch.zeros(1, dtype=torch.int32, device=self.local.device)

    def peer_ptrs(self, view: torch.Tensor):
        """Addresses, in the other ranks' buffers, of the element ``view`` starts at."""
        off = view.data_ptr() - self.local.data_ptr()
        if not 0 <= off < self.local.numel() * self.local.element_size():
            raise ValueError("view does not start inside this rank's buffer")
        peers = [b for r, b in enumerate(self.bases) if r != self.rank]
        if any(b is None for b in peers):
            raise RuntimeError("PeerOutputs is closed: the other ranks' buffers are unmapped")
        return [b + off for b in peers]

    def barrier(self):
        """Stream-ordered barrier over the ranks (a one-element NCCL all-reduce on the current
        stream): once it completes on a rank, every rank's earlier launches on its stream (and
        so their stores into this rank's buffer) have completed."""
        import torch.distributed as dist

        dist.all_reduce(self._flag, group=self.group)

    def close(self):
        """Collective: unmap the other ranks' buffers, then wait until every rank has unmapped
        them, so that no rank frees its buffer (or exits) while another rank still maps it.
        ``local`` stays valid; ``peer_ptrs`` may not be used afterwards."""
        import torch.distributed as dist

        torch.cuda.synchronize(self.local.device)  # no kernel of this rank still stores
        dist.all_reduce(self._flag, group=self.group)  # ... nor of any other rank
        torch.cuda.synchronize(self.local.device)
        self._mapped.clear()
        self.bases = [self.local.data_ptr() if r == self.rank else None
                      for r in range(self.world)]
        dist.all_reduce(self._flag, group=self.group)  # every rank has unmapped
        torch.cuda.synchronize(self.local.device)


def prefill_to_all_ranks(peers: PeerOutputs, sh: HeadShard, q, k, v, rel, cu_seqlens_q,
                         cu_seqlens_k, max_seqlen_q, max_seqlen_k, rel_extent, **kw):
    """Head-sharded prefill whose output assembles itself on every rank: rank ``sh.rank``
    computes its query heads ``[sh.q_lo, sh.q_hi)`` from its slices of the inputs (as
    ``shard_tensors`` gives them) and its kernel stores each finished output row both into its
    own ``peers.local[:, q_lo:q_hi]`` and into the same heads of every other rank's buffer.
    After the stream-ordered barrier every rank's ``peers.local`` holds all heads.  Collective
    (every rank calls it); the caller keeps ranks from reading ``peers.local`` while a later call
    writes it (e.g. by calling the barrier before reusing the buffer)."""
    from . import _ops

    view = peers.local[:, sh.q_lo:sh.q_hi]
    _ops.prefill(q, k, v, rel, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k,
                 rel_extent, out=view, out_peers=peers.peer_ptrs(view), **kw)
    peers.barrier()
    return peers.local
