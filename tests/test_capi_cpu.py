"""C ABI checks that need no GPU: the library loads, exports every function declared in
include/inkling_fa4.h, the ctypes mirrors match the C struct layouts, argument validation
rejects bad input with the documented codes, and the Python API refuses CPU tensors (there is
no CPU fallback)."""
import ctypes
import os
import re
import subprocess
import tempfile

import pytest
import torch

from conftest import REPO
from inkling_fa4 import _lib

HEADER = os.path.join(REPO, "include", "inkling_fa4.h")


def header_functions():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\*?\s+\*?(ifa4_\w+)\s*\(", text, re.M)))


def test_library_exports_every_declared_symbol():
    L = _lib.lib()
    declared = header_functions()
    assert declared, "no declarations parsed"
    assert set(declared) == set(_lib.EXPORTED_SYMBOLS)
    for name in declared:
        assert hasattr(L, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True,
                         text=True).stdout
    for name in declared:
        assert re.search(rf"\bT {name}\b", out), name


def test_abi_version_and_tile_name():
    L = _lib.lib()
    assert L.ifa4_abi_version() == _lib.ABI_VERSION
    from inkling_fa4.autotune_configs import TILE_CONFIGS
    names = [L.ifa4_prefill_tile_config_name(i) for i in range(len(TILE_CONFIGS))]
    assert all(n is not None and n.startswith(b"sm100") for n in names), names
    assert len(set(names)) == len(names)
    assert L.ifa4_prefill_tile_config_name(len(TILE_CONFIGS)) == b""
    assert L.ifa4_prefill_tile_config_name(99) == b""


@pytest.mark.parametrize("cls,cname", [(_lib.PrefillParams, "IFA4PrefillParams"),
                                       (_lib.DecodeParams, "IFA4DecodeParams"),
                                       (_lib.BackwardParams, "IFA4BackwardParams"),
                                       (_lib.RelLogitsParams, "IFA4RelLogitsParams")])
def test_struct_layout_matches_header(cls, cname):
    fields = [f[0] for f in cls._fields_]
    src = "#include <stdio.h>\n#include <stddef.h>\n#include \"inkling_fa4.h\"\nint main(){\n"
    src += f'printf("%zu\\n", sizeof({cname}));\n'
    for f in fields:
        src += f'printf("%zu\\n", offsetof({cname}, {f}));\n'
    src += "return 0;}\n"
    with tempfile.TemporaryDirectory() as d:
        c = os.path.join(d, "t.c")
        exe = os.path.join(d, "t")
        open(c, "w").write(src)
        subprocess.run(["gcc", "-I", os.path.dirname(HEADER), c, "-o", exe], check=True)
        vals = [int(x) for x in subprocess.run([exe], capture_output=True, text=True,
                                               check=True).stdout.split()]
    assert vals[0] == ctypes.sizeof(cls)
    assert vals[1:] == [getattr(cls, f).offset for f in fields]


def _params(**kw):
    p = _lib.PrefillParams()
    p.batch, p.n_heads, p.kv_heads, p.head_dim, p.rel_extent = 1, 4, 4, 128, 128
    p.total_q = p.total_k = 16
    p.softmax_scale = 1.0 / 128
    for k, v in kw.items():
        setattr(p, k, v)
    return p


@pytest.mark.parametrize("kw,code", [
    (dict(head_dim=64), _lib.IFA4_ERR_UNSUPPORTED),
    (dict(dtype=3), _lib.IFA4_ERR_UNSUPPORTED),
    (dict(n_heads=6, kv_heads=4), _lib.IFA4_ERR_INVALID_ARGUMENT),
    (dict(rel_extent=0), _lib.IFA4_ERR_INVALID_ARGUMENT),
    (dict(softmax_scale=0.0), _lib.IFA4_ERR_INVALID_ARGUMENT),
    (dict(causal_align=7), _lib.IFA4_ERR_INVALID_ARGUMENT),
    (dict(), _lib.IFA4_ERR_INVALID_ARGUMENT),  # null tensor pointers
])
def test_prefill_validation_rejects_before_any_cuda_call(kw, code):
    L = _lib.lib()
    rc = L.ifa4_prefill_launch(ctypes.byref(_params(**kw)), None)
    assert rc == code
    assert L.ifa4_last_error_string()


def test_prefill_null_params():
    assert _lib.lib().ifa4_prefill_launch(None, None) == _lib.IFA4_ERR_INVALID_ARGUMENT


def test_empty_batch_is_a_no_op():
    p = _params(batch=0)
    assert _lib.lib().ifa4_prefill_launch(ctypes.byref(p), None) == _lib.IFA4_OK


def test_misaligned_strides_rejected():
    p = _params(q=16, k=16, v=16, rel=16, out=16, cu_seqlens_q=16, cu_seqlens_k=16,
                q_stride_t=4 * 128 + 4, q_stride_h=128, k_stride_t=512, k_stride_h=128,
                v_stride_t=512, v_stride_h=128, rel_stride_t=512, rel_stride_h=128,
                out_stride_t=512, out_stride_h=128)
    assert _lib.lib().ifa4_prefill_launch(ctypes.byref(p), None) == _lib.IFA4_ERR_INVALID_ARGUMENT
    assert b"multiples of 8" in _lib.lib().ifa4_last_error_string()


def test_python_api_refuses_cpu_tensors():
    from inkling_fa4 import inkling_fa4_rel_attention_triton as f
    from inkling_fa4.workloads import make_case
    c = make_case([8], [8], 4, 4, 16)
    with pytest.raises(ValueError, match="CUDA"):
        f(c.q, c.k, c.v, c.rel, c.cu_q, c.cu_k, 8, 8, 16)


def test_decode_requires_workspace_when_split():
    p = _lib.DecodeParams()
    p.batch, p.n_heads, p.kv_heads, p.head_dim, p.rel_extent = 2, 8, 2, 128, 128
    p.total_q, p.total_k = 2, 70000
    p.softmax_scale = 1 / 128
    p.q = p.k = p.v = p.rel = p.out = p.cu_seqlens_q = p.cu_seqlens_k = 256
    for nm in ("q", "k", "v", "rel", "out"):
        setattr(p, nm + "_stride_t", 1024)
        setattr(p, nm + "_stride_h", 128)
    p.num_splits, p.chunk_len = 4, 512
    nbytes = ctypes.c_size_t(0)
    ns, cl = ctypes.c_int32(0), ctypes.c_int32(0)
    L = _lib.lib()
    assert L.ifa4_decode_workspace_size(ctypes.byref(p), ctypes.byref(nbytes), ctypes.byref(ns),
                                        ctypes.byref(cl)) == 0
    assert (ns.value, cl.value) == (4, 512)
    assert nbytes.value == 2 * 8 * 4 * (128 + 1) * 4
    assert L.ifa4_decode_launch(ctypes.byref(p), None, 0, None) == _lib.IFA4_ERR_WORKSPACE
    p.chunk_len = 100
    assert L.ifa4_decode_workspace_size(ctypes.byref(p), ctypes.byref(nbytes), None,
                                        None) == _lib.IFA4_ERR_INVALID_ARGUMENT


def _paged_params(**kw):
    base = dict(q=16, k=16, v=16, rel=16, out=16, cu_seqlens_q=16, cu_seqlens_k=16,
                q_stride_t=512, q_stride_h=128, k_stride_t=512, k_stride_h=128,
                v_stride_t=512, v_stride_h=128, rel_stride_t=512, rel_stride_h=128,
                out_stride_t=512, out_stride_h=128, block_table=16, block_table_stride=4,
                page_size=16, num_pages=8, k_stride_page=16 * 512, v_stride_page=16 * 512)
    base.update(kw)
    return _params(**base)


@pytest.mark.parametrize("kw,code,msg", [
    (dict(page_size=8), _lib.IFA4_ERR_INVALID_ARGUMENT, b"page_size"),
    (dict(page_size=48), _lib.IFA4_ERR_INVALID_ARGUMENT, b"page_size"),
    (dict(num_pages=0), _lib.IFA4_ERR_INVALID_ARGUMENT, b"num_pages"),
    (dict(block_table_stride=-1), _lib.IFA4_ERR_INVALID_ARGUMENT, b"block_table_stride"),
    (dict(k_stride_page=4), _lib.IFA4_ERR_INVALID_ARGUMENT, b"page strides"),
    (dict(v_stride_page=0), _lib.IFA4_ERR_INVALID_ARGUMENT, b"page strides"),
    (dict(tile_config=4), _lib.IFA4_ERR_UNSUPPORTED, b"paged"),
])
def test_paged_cache_validation(kw, code, msg):
    L = _lib.lib()
    assert L.ifa4_prefill_launch(ctypes.byref(_paged_params(**kw)), None) == code
    assert msg in L.ifa4_last_error_string()


def test_page_kv_roundtrip():
    """The paged test/bench layout holds exactly the contiguous keys, in shuffled pages, with
    NaN in every unused slot and -1 past each sequence's pages."""
    import numpy as np
    from inkling_fa4.workloads import make_case, page_kv
    lens = [0, 1, 15, 16, 17, 100]
    c = make_case(lens, lens, 4, 2, 16, seed=4)
    pc = page_kv(c, page_size=16, seed=9)
    bt = pc.meta["block_table"]
    cu = c.cu_k.tolist()
    for b, n in enumerate(lens):
        npg = (n + 15) // 16
        assert bool((bt[b, npg:] == -1).all()) and bool((bt[b, :npg] >= 0).all())
        for j in range(n):
            pg, sl = int(bt[b, j // 16]), j % 16
            assert torch.equal(pc.k[pg, sl], c.k[cu[b] + j]) and torch.equal(pc.v[pg, sl], c.v[cu[b] + j])
    used = bt[bt >= 0]
    assert len(set(used.tolist())) == used.numel()
    mask = torch.zeros(pc.k.shape[:2], dtype=torch.bool)
    for b, n in enumerate(lens):
        for j in range(n):
            mask[int(bt[b, j // 16]), j % 16] = True
    assert bool(torch.isnan(pc.k[~mask].float()).all()) and bool(torch.isnan(pc.v[~mask].float()).all())
    assert np.isfinite(pc.k[mask].float().numpy()).all()


def test_selftest_limit_validated_before_any_cuda_call():
    L = _lib.lib()
    assert L.ifa4_selftest_bounded_wait(0, None) == _lib.IFA4_ERR_INVALID_ARGUMENT
    assert b"timeout_ns" in L.ifa4_last_error_string()


def test_read_stream_hook_validates_before_any_cuda_call():
    L = _lib.lib()
    assert L.ifa4_measure_read_stream(None, 16, None, None) == _lib.IFA4_ERR_INVALID_ARGUMENT
    # misaligned size, with non-null (never dereferenced) pointers
    assert L.ifa4_measure_read_stream(16, 24, 16, None) == _lib.IFA4_ERR_INVALID_ARGUMENT
    assert b"16-byte" in L.ifa4_last_error_string()


def _valid_prefill(**kw):
    base = dict(q=256, k=256, v=256, rel=256, out=256, cu_seqlens_q=256, cu_seqlens_k=256,
                q_stride_t=512, q_stride_h=128, k_stride_t=512, k_stride_h=128, v_stride_t=512,
                v_stride_h=128, rel_stride_t=512, rel_stride_h=128, out_stride_t=512,
                out_stride_h=128)
    base.update(kw)
    return _params(**base)


@pytest.mark.parametrize("kw,entry,code", [
    (dict(kv_splits=2), "launch", _lib.IFA4_ERR_INVALID_ARGUMENT),  # a split needs a workspace
    (dict(kv_splits=-1), "ws", _lib.IFA4_ERR_INVALID_ARGUMENT),
    (dict(kv_splits=_lib.MAX_KV_SPLITS + 1), "ws", _lib.IFA4_ERR_INVALID_ARGUMENT),
    (dict(kv_splits=2, tile_config=1), "ws", _lib.IFA4_ERR_UNSUPPORTED),
])
def test_prefill_kv_split_validation_before_any_cuda_call(kw, entry, code):
    L = _lib.lib()
    p = _valid_prefill(**kw)
    if entry == "launch":
        rc = L.ifa4_prefill_launch(ctypes.byref(p), None)
    else:
        rc = L.ifa4_prefill_launch_ws(ctypes.byref(p), None, 0, None)
        nbytes = ctypes.c_size_t(123)
        assert L.ifa4_prefill_workspace_size(ctypes.byref(p), ctypes.byref(nbytes)) == code
    assert rc == code
    assert b"kv_splits" in L.ifa4_last_error_string()


def test_prefill_workspace_size_of_an_empty_batch_is_zero():
    L = _lib.lib()
    nbytes = ctypes.c_size_t(123)
    assert L.ifa4_prefill_workspace_size(ctypes.byref(_valid_prefill(batch=0)),
                                         ctypes.byref(nbytes)) == _lib.IFA4_OK
    assert nbytes.value == 0
    assert L.ifa4_prefill_workspace_size(ctypes.byref(_valid_prefill()), None) == \
        _lib.IFA4_ERR_INVALID_ARGUMENT


def test_torch_operator_library_registers_its_schemas():
    """The operator library loads without a GPU and declares prefill_ / decode_ (the package's
    launch path); its CUDA kernels run only in the GPU tests."""
    import torch
    ops = _lib.torch_ops()
    assert ops is not None, "libifa4_torch_ops.so not built"
    for name in ("prefill_", "decode_"):
        schema = str(getattr(ops, name).default._schema)
        assert schema.startswith(f"inkling_fa4::{name}(Tensor q")
    assert torch.ops.inkling_fa4 is ops
