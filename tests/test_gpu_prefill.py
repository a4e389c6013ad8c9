"""Prefill parity on the B200: the sm_100a kernel, called through the drop-in API (and thus the
C ABI), against the reference's golden outputs and the CPU oracle."""
import numpy as np
import pytest
import torch

from golden_cases import load_case, names
from gpu_util import (assert_close, device_status_ok, np32, oracle_full, oracle_rows,
                      run_prefill, to_dev)
from inkling_fa4 import inkling_fa4_rel_attention_triton
from inkling_fa4.triton_kernel_kv_pruned import inkling_fa4_rel_attention_kv_pruned_triton
from inkling_fa4.workloads import (config_chunked, config_long, config_ragged, make_case)

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _status_clean():
    yield
    assert device_status_ok(), "a kernel abandoned a bounded wait"


@pytest.mark.parametrize("name", names())
def test_golden_prefill(name):
    """All reference test cases (tests/test_correctness.py:22-75) and the edge fixtures."""
    spec, c, expected, _ = load_case(name)
    c = to_dev(c)
    c.q, c.k, c.v, c.rel = (t.to(torch.bfloat16) for t in (c.q, c.k, c.v, c.rel))
    wl = spec["window_left"]
    out = run_prefill(c, causal=spec["causal"], window_size=(-1 if wl is None else wl, 0),
                      softmax_scale=spec["scale"])
    torch.cuda.synchronize()
    assert_close(np32(out), expected, what=name)


def test_kv_pruned_alias_matches():
    spec, c, expected, _ = load_case("sliding_window_h8_2")
    c = to_dev(c)
    out = inkling_fa4_rel_attention_kv_pruned_triton(c.q, c.k, c.v, c.rel, c.cu_q, c.cu_k, 128,
                                                     128, spec["rel_extent"],
                                                     window_size=(spec["window_left"], 0))
    assert_close(np32(out), expected)


EDGE_LENS = [1, 17, 33, 127, 128, 129, 255, 256, 257, 300, 2]


@pytest.mark.parametrize("heads", [(4, 4), (8, 2), (6, 2), (3, 1), (32, 8)])
@pytest.mark.parametrize("causal,window", [(True, None), (False, None), (True, 70), (False, 33)])
@pytest.mark.parametrize("rel_extent", [128, 1000])
def test_ragged_edges_vs_oracle(heads, causal, window, rel_extent):
    hq, hkv = heads
    c = to_dev(make_case(EDGE_LENS, EDGE_LENS, hq, hkv, rel_extent, seed=hq * 7 + hkv))
    out = run_prefill(c, causal=causal, window_size=(-1 if window is None else window, 0))
    want = oracle_full(c, 1 / 128, causal=causal, window_left=window)
    assert_close(np32(out), want)


@pytest.mark.parametrize("align", ["reference", "bottom_right"])
@pytest.mark.parametrize("window", [None, 100])
def test_chunked_vs_oracle(align, window):
    sq, sk = [130, 64, 1, 200], [300, 64, 257, 200]
    c = to_dev(make_case(sq, sk, 8, 2, 128, seed=11))
    out = run_prefill(c, causal_align=align, window_size=(-1 if window is None else window, 0))
    want = oracle_full(c, 1 / 128, window_left=window, causal_align=align)
    assert_close(np32(out), want)


def test_chunked_bottom_right_equals_full_prefill_rows():
    """north_star: chunked results agree with the corresponding full-prefill results."""
    cache, chunk = 700, 333
    full = to_dev(make_case([cache + chunk], [cache + chunk], 8, 2, 128, seed=3))
    ref_rows = run_prefill(full)[cache:]
    q, rel = full.q[cache:].contiguous(), full.rel[cache:].contiguous()
    cu_q = torch.tensor([0, chunk], dtype=torch.int32, device="cuda")
    got = inkling_fa4_rel_attention_triton(q, full.k, full.v, rel, cu_q, full.cu_k, chunk,
                                           cache + chunk, 128, causal_align="bottom_right")
    assert_close(np32(got), np32(ref_rows), atol=1e-2, rtol=1e-2)


def test_stride0_per_head_table_and_sqrt_scale():
    c = make_case([200, 77], [200, 77], 8, 4, 128, seed=4, rel_per_head_table=True, device="cuda")
    assert c.rel.stride(0) == 0
    out = run_prefill(c, softmax_scale=128 ** -0.5)
    assert_close(np32(out), oracle_full(c, 128 ** -0.5))


def test_noncontiguous_inputs_and_out_param():
    base = to_dev(make_case([150], [150], 8, 2, 64, seed=6))
    # q as a head-slice of a wider tensor, k/v as token-strided views
    wide = torch.zeros(150, 16, 128, dtype=torch.bfloat16, device="cuda")
    wide[:, 4:12] = base.q
    kk = torch.zeros(300, 2, 128, dtype=torch.bfloat16, device="cuda")
    kk[::2] = base.k
    vv = torch.zeros(150, 2, 256, dtype=torch.bfloat16, device="cuda")
    vv[:, :, 64:192] = base.v
    q, k, v = wide[:, 4:12], kk[::2], vv[:, :, 64:192]
    out = torch.full((150, 8, 128), 7.0, dtype=torch.bfloat16, device="cuda")
    r = inkling_fa4_rel_attention_triton(q, k, v, base.rel, base.cu_q, base.cu_k, 150, 150, 64,
                                         out=out)
    assert r.data_ptr() == out.data_ptr()
    assert_close(np32(out), oracle_full(base, 1 / 128))


def test_max_seqlen_hint_is_not_trusted_for_correctness():
    """Wrong max_seqlen hints change only the grid shape (and, with the automatic KV split of
    small launches, the split count, i.e. the rounding of the merge), never the result."""
    from inkling_fa4 import _ops
    c = to_dev(make_case([600, 40], [600, 40], 4, 2, 128, seed=8))
    good = _ops.prefill(c.q, c.k, c.v, c.rel, c.cu_q, c.cu_k, 600, 600, 128, kv_splits=1)
    bad = _ops.prefill(c.q, c.k, c.v, c.rel, c.cu_q, c.cu_k, 1, 1, 128, kv_splits=1)
    torch.testing.assert_close(bad, good, atol=0, rtol=0)
    auto_bad = inkling_fa4_rel_attention_triton(c.q, c.k, c.v, c.rel, c.cu_q, c.cu_k, 1, 1, 128)
    assert_close(np32(auto_bad), oracle_full(c, 1 / 128))


def test_empty_keys_give_zero_rows():
    c = to_dev(make_case([5, 40], [0, 40], 4, 4, 64, seed=9))
    out = run_prefill(c)
    assert torch.all(out[:5] == 0)
    assert_close(np32(out[5:]), oracle_full(c, 1 / 128)[5:])


def test_deterministic_across_calls():
    c = to_dev(make_case([1000, 333], [1000, 333], 8, 2, 128, seed=10))
    a, b = run_prefill(c), run_prefill(c)
    torch.testing.assert_close(a, b, atol=0, rtol=0)


# ---- benchmark configurations, checked on sampled rows (full-size) ---------------------

def test_config_ragged_spot_rows():
    c = to_dev(config_ragged())
    out = run_prefill(c)
    toks, want = oracle_rows(c, 6, list(range(0, 32, 5)), 1 / 128, seed=1)
    got = np32(out[torch.as_tensor(toks, device="cuda")][:, list(range(0, 32, 5))])
    assert_close(got, want)


@pytest.mark.parametrize("window", [None, 4096])
def test_config_32k_spot_rows(window):
    c = to_dev(config_long(window=window))
    out = run_prefill(c, window_size=(-1 if window is None else window, 0))
    heads = [0, 13, 31]
    toks, want = oracle_rows(c, 24, heads, 1 / 128, window_left=window, seed=2)
    got = np32(out[torch.as_tensor(toks, device="cuda")][:, heads])
    assert_close(got, want)
    assert torch.isfinite(out.float()).all()


def test_config_chunked_spot_rows():
    c = to_dev(config_chunked())
    out = run_prefill(c, causal_align="bottom_right")
    heads = [1, 30]
    toks, want = oracle_rows(c, 5, heads, 1 / 128, causal_align="bottom_right", seed=3)
    got = np32(out[torch.as_tensor(toks, device="cuda")][:, heads])
    assert_close(got, want)


@pytest.mark.parametrize("tile_config", [1, 2, 3, 4, 5, 6, 7, 8])
def test_tile_config_variants_match_oracle(tile_config):
    """Every kernel variant (fraction of exponentials computed on the FMA pipe) is correct,
    including rows that see no key (must be 0, not the ~2^-125 of an emulated exp2(-inf))."""
    from inkling_fa4 import _ops
    c = to_dev(make_case([300, 17, 129, 5], [300, 17, 129, 0], 8, 2, 128, seed=12))
    for causal, window in ((True, None), (True, 40), (False, None)):
        out = _ops.prefill(c.q, c.k, c.v, c.rel, c.cu_q, c.cu_k, 300, 300, 128, causal=causal,
                           window_size=(-1 if window is None else window, 0),
                           tile_config=tile_config)
        want = oracle_full(c, 1 / 128, causal=causal, window_left=window)
        assert_close(np32(out), want)
        assert torch.all(out[-5:] == 0)
    ref = _ops.prefill(c.q, c.k, c.v, c.rel, c.cu_q, c.cu_k, 300, 300, 128, tile_config=1)
    got = _ops.prefill(c.q, c.k, c.v, c.rel, c.cu_q, c.cu_k, 300, 300, 128,
                       tile_config=tile_config)
    # variants differ only in the last bits of some p values: at most one bf16 ulp of the output
    assert_close(np32(got), np32(ref), atol=1e-2, rtol=1e-2)


@pytest.mark.parametrize("scale", [60.0, 400.0, 3000.0])
@pytest.mark.parametrize("tile_config", [1, 3, 6])
def test_scores_far_above_the_running_max(scale, tile_config):
    """Interior tiles take their exponentials against the running max without a row-max pass
    and keep the tile only if its sum of p stays <= 2^32.  Keys scaled up from position 1000 on
    push scores 2^30 (x60) to far beyond 2^128 (x400, x3000) above that max: the tile must then
    be redone with its true max (SFU, FMA-pipe polynomial and fp16 SFU exponentials alike)."""
    from inkling_fa4.workloads import Case
    c = make_case([2048, 1500], [2048, 1500], 4, 2, 128, seed=int(scale))
    k = c.k.float()
    k[1000:2048] *= scale
    k[2048 + 700:] *= scale
    c = Case(q=c.q, k=k.to(torch.bfloat16), v=c.v, rel=c.rel, cu_q=c.cu_q, cu_k=c.cu_k,
             seqlens_q=c.seqlens_q, seqlens_k=c.seqlens_k, rel_extent=128)
    c = to_dev(c)
    toks, want = oracle_rows(c, 48, list(range(4)), 1 / 128, seed=int(scale) + 1)
    from inkling_fa4 import _ops
    out, lse = _ops.prefill(c.q, c.k, c.v, c.rel, c.cu_q, c.cu_k, c.max_q, c.max_k, 128,
                            tile_config=tile_config, return_lse=True)
    assert_close(np32(out)[toks], want, what=f"tile_config {tile_config}")
    assert torch.isfinite(lse).all() and torch.isfinite(out.float()).all()


def test_window_row_without_keys_is_zero_in_default_config():
    # bottom-right chunk shorter than a window gap: early query rows see no key at all
    c = to_dev(make_case([64], [64], 4, 4, 64, seed=13))
    out = run_prefill(c, causal_align="bottom_right", window_size=(0, 0))
    want = oracle_full(c, 1 / 128, window_left=0, causal_align="bottom_right")
    assert_close(np32(out), want)


@pytest.mark.parametrize("jump", [1000, 1024, 1056, 1090, 1130])
def test_running_max_growth_inside_interior_tiles(jump):
    """Keys from `jump` on are scaled 60x, so for rows far past them the scores jump by much
    more than the rescale threshold inside an interior (unmasked, unbiased) KV tile, at the 32-
    column chunk position the offset selects: the single-pass softmax must correct its running
    max, sum, stored P and O there."""
    from inkling_fa4.workloads import Case
    c = make_case([2048, 1500], [2048, 1500], 4, 2, 128, seed=jump)
    k = c.k.float()
    k[jump:2048] *= 60.0
    k[2048 + jump // 2:] *= 60.0
    c = Case(q=c.q, k=k.to(torch.bfloat16), v=c.v, rel=c.rel, cu_q=c.cu_q, cu_k=c.cu_k,
             seqlens_q=c.seqlens_q, seqlens_k=c.seqlens_k, rel_extent=128)
    c = to_dev(c)
    toks, want = oracle_rows(c, 48, list(range(4)), 1 / 128, seed=jump)
    from inkling_fa4 import _ops
    for tc in (1, 3):  # all-SFU and FMA-pipe exponential variants
        out = _ops.prefill(c.q, c.k, c.v, c.rel, c.cu_q, c.cu_k, c.max_q, c.max_k, 128,
                           tile_config=tc)
        assert_close(np32(out)[toks], want, what=f"tile_config {tc}")


@pytest.mark.parametrize("scale", [60.0, 3000.0])
@pytest.mark.parametrize("tile_config", [0, 1, 3])
@pytest.mark.parametrize("window", [None, 511])
def test_band_tiles_with_scores_far_above_the_running_max(scale, tile_config, window):
    """Band tiles (relative bias on every one of them at R = 1024) and window-boundary tiles
    also take the single pass against the running max; keys scaled up near each row's diagonal
    push their scores far above it, so those tiles must be redone with their true max."""
    from inkling_fa4.workloads import Case
    c = make_case([2048, 1500], [2048, 1500], 8, 2, 1024, seed=int(scale) + 7, rel_std=2.0)
    k = c.k.float()
    k[1500:1700] *= scale
    k[2048 + 900:2048 + 1000] *= scale
    c = Case(q=c.q, k=k.to(torch.bfloat16), v=c.v, rel=c.rel, cu_q=c.cu_q, cu_k=c.cu_k,
             seqlens_q=c.seqlens_q, seqlens_k=c.seqlens_k, rel_extent=1024)
    c = to_dev(c)
    toks, want = oracle_rows(c, 48, [0, 3, 5], 1 / 128, window_left=window, seed=int(scale) + 2)
    from inkling_fa4 import _ops
    out = _ops.prefill(c.q, c.k, c.v, c.rel, c.cu_q, c.cu_k, c.max_q, c.max_k, 1024,
                       window_size=(-1 if window is None else window, 0), tile_config=tile_config)
    assert_close(np32(out)[:, [0, 3, 5]][toks], want, what=f"tile_config {tile_config}")
    assert torch.isfinite(out.float()).all()


def test_window_rows_whose_first_keys_are_far_below_zero():
    """Rows whose first visible KV tile (the window's left edge) comes after a tile they see
    nothing of enter the single pass with no running max yet; if all their scores in that tile
    are far below 0 (about -185 in log2 units), every p underflows, and the tile must be redone
    with its true max rather than kept as zero."""
    from inkling_fa4.workloads import Case
    c = make_case([1024], [1024], 4, 2, 512, seed=21)
    u = torch.randn(128, generator=torch.Generator().manual_seed(5))
    q, k = c.q.float(), c.k.float()
    q[450:700] = u           # every head of these rows
    k[200:330] = -128.0 * u  # q.k / 128 = -|u|^2, about -128 (-185 in log2 units)
    c = Case(q=q.to(torch.bfloat16), k=k.to(torch.bfloat16), v=c.v, rel=c.rel, cu_q=c.cu_q,
             cu_k=c.cu_k, seqlens_q=c.seqlens_q, seqlens_k=c.seqlens_k, rel_extent=512)
    c = to_dev(c)
    for window in (300, 250):
        out = run_prefill(c, window_size=(window, 0))
        want = oracle_full(c, 1 / 128, window_left=window)
        assert_close(np32(out), want, what=f"window {window}")
