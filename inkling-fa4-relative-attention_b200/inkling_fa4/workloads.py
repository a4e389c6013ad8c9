"""Seeded synthetic inputs with the shapes and distributions of the benchmark configurations.

All generation happens on the CPU with one ``torch.Generator`` per tensor, so a given seed
gives bit-identical inputs on every machine running this torch build; tensors are then moved
to the requested device.  Distributions follow the benchmark definitions: Q/K/V ~ N(0, 1) and
relative logits ~ N(0, 0.5) (standard deviation 0.5), token-major layouts ``[tokens, heads, d]``
and ``[tokens, Hq, rel_extent]`` as in the reference (reference.py:11-15).
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch

HEAD_DIM = 128


@dataclass
class Case:
    q: torch.Tensor
    k: torch.Tensor
    v: torch.Tensor
    rel: torch.Tensor
    cu_q: torch.Tensor
    cu_k: torch.Tensor
    seqlens_q: list
    seqlens_k: list
    rel_extent: int
    meta: dict = field(default_factory=dict)

    @property
    def max_q(self) -> int:
        return max(self.seqlens_q) if self.seqlens_q else 0

    @property
    def max_k(self) -> int:
        return max(self.seqlens_k) if self.seqlens_k else 0


def _randn(shape, seed, std=1.0, dtype=torch.bfloat16, gen_device="cpu"):
    """N(0, std^2) draws from a generator seeded per tensor.  ``gen_device="cuda"`` draws on
    the GPU (fast for benchmark-size tensors; a different stream of numbers than the CPU)."""
    g = torch.Generator(device=gen_device)
    g.manual_seed(int(seed))
    x = torch.randn(*shape, generator=g, dtype=torch.float32, device=gen_device)
    if std != 1.0:
        x = x * std
    return x.to(dtype)


def cu_from_lens(lens) -> torch.Tensor:
    cu = torch.zeros(len(lens) + 1, dtype=torch.int32)
    if len(lens):
        cu[1:] = torch.cumsum(torch.tensor(lens, dtype=torch.int64), 0).to(torch.int32)
    return cu


def make_case(seqlens_q, seqlens_k, n_heads, kv_heads, rel_extent, seed=0,
              device="cpu", dtype=torch.bfloat16, rel_std=1.0, head_dim=HEAD_DIM,
              rel_per_head_table=False, gen_device="cpu") -> Case:
    """Build one varlen case.  ``rel_std=1.0`` matches the reference tests (``torch.randn``,
    tests/test_correctness.py:11-20); the benchmark configurations use 0.5.

    ``rel_per_head_table`` expresses a per-head distance table ``T[h, 0:R]`` as a
    ``[Tq, Hq, R]`` view with token stride 0.
    """
    tq, tk = int(sum(seqlens_q)), int(sum(seqlens_k))
    gd = gen_device
    q = _randn((tq, n_heads, head_dim), seed * 7 + 1, dtype=dtype, gen_device=gd)
    k = _randn((tk, kv_heads, head_dim), seed * 7 + 2, dtype=dtype, gen_device=gd)
    v = _randn((tk, kv_heads, head_dim), seed * 7 + 3, dtype=dtype, gen_device=gd)
    if rel_per_head_table:
        table = _randn((n_heads, rel_extent), seed * 7 + 4, std=rel_std, dtype=dtype, gen_device=gd)
        rel = table.to(device).unsqueeze(0).expand(tq, n_heads, rel_extent)
    else:
        rel = _randn((tq, n_heads, rel_extent), seed * 7 + 4, std=rel_std, dtype=dtype,
                     gen_device=gd).to(device)
    return Case(q=q.to(device), k=k.to(device), v=v.to(device), rel=rel,
                cu_q=cu_from_lens(seqlens_q).to(device), cu_k=cu_from_lens(seqlens_k).to(device),
                seqlens_q=list(map(int, seqlens_q)), seqlens_k=list(map(int, seqlens_k)),
                rel_extent=rel_extent)


def ragged_lengths(n, lo, hi, seed):
    g = torch.Generator(device="cpu")
    g.manual_seed(int(seed))
    return [int(x) for x in torch.randint(lo, hi + 1, (n,), generator=g)]


# --- benchmark configurations (seeded) --------------------------------------------------

def config_cpu_reference(device="cpu", seed=0) -> Case:
    """Config 1: B=1, S=128, Hq=Hkv=4, d=128, causal, softmax scale 1/sqrt(128), a per-head
    distance table of R=128 entries (token stride 0) ~ N(0, 0.5)."""
    c = make_case([128], [128], 4, 4, 128, seed=seed, device=device, rel_std=0.5,
                  rel_per_head_table=True)
    c.meta.update(name="cpu_reference_s128", softmax_scale=128 ** -0.5, causal=True)
    return c


def ragged_batch_lengths(seed=0, n=16, lo=1, hi=4096) -> list:
    """The sequence lengths of ``config_ragged(seed=seed)``."""
    return ragged_lengths(n, lo, hi, seed + 1000)


def decode_batch_lengths(seed=0, batch=128, lo=1024, hi=32768) -> list:
    """The K/V lengths of ``config_decode(seed=seed, batch=batch)``."""
    return ragged_lengths(batch, lo, hi, seed + 2000)


def config_ragged(device="cpu", seed=0, n=16, lo=1, hi=4096, gen_device="cpu") -> Case:
    """Config 2: 16 sequences with lengths ~ U[1, 4096], GQA 32/8, R=128."""
    lens = ragged_batch_lengths(seed, n, lo, hi)
    c = make_case(lens, lens, 32, 8, 128, seed=seed, device=device, rel_std=0.5,
                  gen_device=gen_device)
    c.meta.update(name="ragged16_u1_4096_gqa32_8", causal=True)
    return c


def config_long(device="cpu", seed=0, seq=32768, window=None, gen_device="cpu") -> Case:
    """Config 3: B=1, S=32768, GQA 32/8, R=128, full causal or window_left=4096."""
    c = make_case([seq], [seq], 32, 8, 128, seed=seed, device=device, rel_std=0.5,
                  gen_device=gen_device)
    c.meta.update(name=f"causal{seq}" + (f"_window{window}" if window is not None else ""),
                  causal=True, window_left=window)
    return c


def config_chunked(device="cpu", seed=0, n=8, cache=16384, chunk=2048, gen_device="cpu") -> Case:
    """Config 4: 8 sequences of 16384 cached K/V tokens plus a 2048-token query chunk
    (bottom-right alignment: query i sits at position cache + i)."""
    c = make_case([chunk] * n, [cache + chunk] * n, 32, 8, 128, seed=seed, device=device,
                  rel_std=0.5, gen_device=gen_device)
    c.meta.update(name=f"chunked{n}x{cache}+{chunk}", causal=True, causal_align="bottom_right")
    return c


def config_decode(device="cpu", seed=0, batch=128, lo=1024, hi=32768, gen_device="cpu") -> Case:
    """Config 5: batch=128 single-token decode, KV lengths ~ U[1024, 32768], GQA 32/8, R=128,
    bottom-right alignment (the query is the last position of its sequence)."""
    lens = decode_batch_lengths(seed, batch, lo, hi)
    c = make_case([1] * batch, lens, 32, 8, 128, seed=seed, device=device, rel_std=0.5,
                  gen_device=gen_device)
    c.meta.update(name=f"decode{batch}_u{lo}_{hi}", causal=True, causal_align="bottom_right")
    return c


def causal_visible_pairs(seqlens_q, seqlens_k, causal=True, window_left=None,
                         causal_align="reference") -> int:
    """Number of (query, key) pairs that survive the masks, summed over sequences (per head).
    The algorithmic FLOP count of one call is ``4 * head_dim * n_heads * pairs``."""
    total = 0
    for sq, sk in zip(seqlens_q, seqlens_k):
        ms = 0 if causal_align == "reference" else sk - sq
        for_all = 0
        # per query row i: visible keys are [lo_i, hi_i)
        # counted in closed form per row to stay O(sq)
        for i in range(sq):
            hi = sk
            if causal:
                hi = min(hi, i + ms + 1)
            lo = 0
            if window_left is not None and window_left >= 0:
                lo = max(0, i + ms - window_left)
            if hi > lo:
                for_all += hi - lo
        total += for_all
    return total


def page_kv(case: Case, page_size: int = 16, seed: int = 0, spare_pages: int = 3,
            extra_cols: int = 2, fill: float = float("nan")) -> Case:
    """The same case with K/V moved into a paged cache, as a serving engine holds them:
    caches [num_pages, page_size, kv_heads, d] whose pages are handed out in a seeded random
    order, a block table [batch, max_pages + extra_cols] (int32, -1 past each sequence's pages),
    and every slot that holds no key set to ``fill`` (NaN by default, so a kernel that let an
    unused slot reach its output would show it).  cu_seqlens_k is unchanged (key counts)."""
    lens = [int(x) for x in case.seqlens_k]
    dev = case.k.device
    n_per = [(n + page_size - 1) // page_size for n in lens]
    used = sum(n_per)
    num_pages = used + spare_pages
    g = torch.Generator(device="cpu")
    g.manual_seed(int(seed))
    perm = torch.randperm(num_pages, generator=g)[:used].to(torch.int32)
    max_pages = max(n_per) if n_per else 0
    table = torch.full((len(lens), max_pages + extra_cols), -1, dtype=torch.int32)
    off = 0
    for b, n in enumerate(n_per):
        table[b, :n] = perm[off:off + n]
        off += n
    hkv, d = case.k.shape[1], case.k.shape[2]
    kc = torch.full((num_pages, page_size, hkv, d), fill, dtype=case.k.dtype, device=dev)
    vc = torch.full_like(kc, fill)
    if sum(lens):
        seq = torch.repeat_interleave(torch.arange(len(lens)), torch.tensor(lens))
        starts = torch.tensor([0] + lens[:-1]).cumsum(0)
        j = torch.arange(sum(lens)) - starts[seq]
        page = table[seq, j // page_size].long().to(dev)
        slot = (j % page_size).to(dev)
        kc[page, slot] = case.k
        vc[page, slot] = case.v
    meta = dict(case.meta)
    meta.update(block_table=table.to(dev), page_size=page_size, num_pages=num_pages)
    return Case(q=case.q, k=kc, v=vc, rel=case.rel, cu_q=case.cu_q, cu_k=case.cu_k,
                seqlens_q=case.seqlens_q, seqlens_k=case.seqlens_k, rel_extent=case.rel_extent,
                meta=meta)
