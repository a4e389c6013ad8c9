"""ctypes binding of the C ABI declared in include/inkling_fa4.h.

The shared library ``_lib/libinkling_fa4.so`` is built in-tree by ``inkling_fa4.build``.  There
is no fallback: if the library is missing or fails to load, every kernel entry point raises.
"""
from __future__ import annotations

import ctypes
import os

_LIB_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_lib")
# INKLING_FA4_LIB=debug loads the index-checking debug build (python -m inkling_fa4.build --debug)
LIB_PATH = os.path.join(_LIB_DIR, "libinkling_fa4_debug.so"
                        if os.environ.get("INKLING_FA4_LIB") == "debug" else "libinkling_fa4.so")

IFA4_OK = 0
IFA4_ERR_INVALID_ARGUMENT = -1
IFA4_ERR_UNSUPPORTED = -2
IFA4_ERR_CUDA = -3
IFA4_ERR_WORKSPACE = -4
IFA4_ERR_DEVICE_TIMEOUT = -5
STATUS_DEBUG_BOUNDS = 64
IFA4_ALIGN_REFERENCE = 0
IFA4_ALIGN_BOTTOM_RIGHT = 1
IFA4_DTYPE_BF16 = 0
ABI_VERSION = 7
MAX_OUT_PEERS = 7
MAX_KV_SPLITS = 16
NOALLOC_DECODE_SCRATCH_BYTES = 16 * 1024 * 1024

EXPORTED_SYMBOLS = (
    "ifa4_prefill_launch",
    "ifa4_prefill_launch_ws",
    "ifa4_prefill_workspace_size",
    "ifa4_decode_launch",
    "ifa4_decode_launch_noalloc",
    "ifa4_decode_workspace_size",
    "ifa4_backward_launch",
    "ifa4_backward_workspace_size",
    "ifa4_rel_logits_launch",
    "ifa4_read_device_status",
    "ifa4_selftest_bounded_wait",
    "ifa4_measure_read_stream",
    "ifa4_prefill_tile_config_name",
    "ifa4_last_error_string",
    "ifa4_abi_version",
)

_COMMON = [
    ("q", ctypes.c_void_p), ("k", ctypes.c_void_p), ("v", ctypes.c_void_p),
    ("rel", ctypes.c_void_p), ("out", ctypes.c_void_p),
    ("cu_seqlens_q", ctypes.c_void_p), ("cu_seqlens_k", ctypes.c_void_p),
    ("q_stride_t", ctypes.c_int64), ("q_stride_h", ctypes.c_int64),
    ("k_stride_t", ctypes.c_int64), ("k_stride_h", ctypes.c_int64),
    ("v_stride_t", ctypes.c_int64), ("v_stride_h", ctypes.c_int64),
    ("rel_stride_t", ctypes.c_int64), ("rel_stride_h", ctypes.c_int64),
    ("out_stride_t", ctypes.c_int64), ("out_stride_h", ctypes.c_int64),
    ("total_q", ctypes.c_int64), ("total_k", ctypes.c_int64),
    ("batch", ctypes.c_int32), ("n_heads", ctypes.c_int32), ("kv_heads", ctypes.c_int32),
    ("head_dim", ctypes.c_int32), ("rel_extent", ctypes.c_int32), ("causal", ctypes.c_int32),
    ("window_left", ctypes.c_int32), ("causal_align", ctypes.c_int32),
]


class PrefillParams(ctypes.Structure):
    """Mirror of ``IFA4PrefillParams``."""
    _fields_ = _COMMON + [
        ("max_seqlen_q", ctypes.c_int32), ("dtype", ctypes.c_int32),
        ("softmax_scale", ctypes.c_float), ("tile_config", ctypes.c_int32),
        ("lse", ctypes.c_void_p), ("lse_stride_h", ctypes.c_int64), ("lse_stride_t", ctypes.c_int64),
        ("block_table", ctypes.c_void_p), ("block_table_stride", ctypes.c_int64),
        ("k_stride_page", ctypes.c_int64), ("v_stride_page", ctypes.c_int64),
        ("page_size", ctypes.c_int32), ("num_pages", ctypes.c_int32),
        ("out_peers", ctypes.POINTER(ctypes.c_void_p)), ("n_out_peers", ctypes.c_int32),
        ("kv_splits", ctypes.c_int32), ("max_seqlen_k", ctypes.c_int32),
    ]


class DecodeParams(ctypes.Structure):
    """Mirror of ``IFA4DecodeParams``."""
    _fields_ = _COMMON + [
        ("max_seqlen_k", ctypes.c_int32), ("dtype", ctypes.c_int32),
        ("softmax_scale", ctypes.c_float), ("num_splits", ctypes.c_int32),
        ("chunk_len", ctypes.c_int32),
        ("lse", ctypes.c_void_p), ("lse_stride_h", ctypes.c_int64), ("lse_stride_t", ctypes.c_int64),
        ("block_table", ctypes.c_void_p), ("block_table_stride", ctypes.c_int64),
        ("k_stride_page", ctypes.c_int64), ("v_stride_page", ctypes.c_int64),
        ("page_size", ctypes.c_int32), ("num_pages", ctypes.c_int32),
    ]


def _pairs(*names):
    return [(f"{n}_stride_{x}", ctypes.c_int64) for n in names for x in ("t", "h")]


class BackwardParams(ctypes.Structure):
    """Mirror of ``IFA4BackwardParams``."""
    _fields_ = [(n, ctypes.c_void_p) for n in ("q", "k", "v", "rel", "out", "dout", "lse", "dq",
                                               "dk", "dv", "drel", "cu_seqlens_q",
                                               "cu_seqlens_k")] + \
        _pairs("q", "k", "v", "rel", "out", "dout") + \
        [("lse_stride_h", ctypes.c_int64), ("lse_stride_t", ctypes.c_int64)] + \
        _pairs("dq", "dk", "dv", "drel") + \
        [("total_q", ctypes.c_int64), ("total_k", ctypes.c_int64)] + \
        [(n, ctypes.c_int32) for n in ("batch", "n_heads", "kv_heads", "head_dim", "rel_extent",
                                       "causal", "window_left", "causal_align", "max_seqlen_q",
                                       "max_seqlen_k", "dtype")] + \
        [("softmax_scale", ctypes.c_float)]


class RelLogitsParams(ctypes.Structure):
    """Mirror of ``IFA4RelLogitsParams``."""
    _fields_ = [(n, ctypes.c_void_p) for n in ("r", "weight", "rel", "cu_seqlens_q",
                                               "cu_seqlens_k")] + \
        [("r_stride_t", ctypes.c_int64), ("r_stride_h", ctypes.c_int64),
         ("weight_stride_h", ctypes.c_int64), ("weight_stride_j", ctypes.c_int64),
         ("rel_stride_t", ctypes.c_int64), ("rel_stride_h", ctypes.c_int64),
         ("total_q", ctypes.c_int64)] + \
        [(n, ctypes.c_int32) for n in ("batch", "n_heads", "d_rel", "rel_extent", "dtype")] + \
        [("alpha", ctypes.c_float), ("nf", ctypes.c_float)]


class Ifa4Error(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(f"inkling_fa4 error {code}: {message}")
        self.code = code


_lib = None
_torch_ops = None
TORCH_OPS_PATH = os.path.join(_LIB_DIR, "libifa4_torch_ops.so")


def torch_ops():
    """The torch operators ``torch.ops.inkling_fa4`` over the C ABI (``prefill_``, ``decode_``),
    or None when they are not built or the debug library is selected (they link the release
    library).  The package then calls the C ABI through ctypes instead: the same entry points,
    with more host work per call."""
    global _torch_ops
    if _torch_ops is not None:
        return _torch_ops or None
    _torch_ops = False
    if os.environ.get("INKLING_FA4_LIB") == "debug" or not os.path.exists(TORCH_OPS_PATH):
        return None
    import torch

    lib()  # load the C ABI first (one shared instance: status word, last-error message)
    torch.ops.load_library(TORCH_OPS_PATH)
    _torch_ops = torch.ops.inkling_fa4
    return _torch_ops


def lib() -> ctypes.CDLL:
    """Load the CUDA library (once).  Raises if it is absent: no CPU fallback exists."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(
            f"inkling_fa4 CUDA library not found at {LIB_PATH}; build it with "
            "`python -m inkling_fa4.build` (nvcc, sm_100a)")
    L = ctypes.CDLL(LIB_PATH)
    vp, i32, sz = ctypes.c_void_p, ctypes.c_int32, ctypes.c_size_t
    L.ifa4_prefill_launch.argtypes = [ctypes.POINTER(PrefillParams), vp]
    L.ifa4_prefill_launch.restype = ctypes.c_int
    L.ifa4_prefill_launch_ws.argtypes = [ctypes.POINTER(PrefillParams), vp, sz, vp]
    L.ifa4_prefill_launch_ws.restype = ctypes.c_int
    L.ifa4_prefill_workspace_size.argtypes = [ctypes.POINTER(PrefillParams), ctypes.POINTER(sz)]
    L.ifa4_prefill_workspace_size.restype = ctypes.c_int
    L.ifa4_decode_launch.argtypes = [ctypes.POINTER(DecodeParams), vp, sz, vp]
    L.ifa4_decode_launch.restype = ctypes.c_int
    L.ifa4_decode_launch_noalloc.argtypes = [ctypes.POINTER(DecodeParams), vp]
    L.ifa4_decode_launch_noalloc.restype = ctypes.c_int
    L.ifa4_decode_workspace_size.argtypes = [ctypes.POINTER(DecodeParams), ctypes.POINTER(sz),
                                             ctypes.POINTER(i32), ctypes.POINTER(i32)]
    L.ifa4_decode_workspace_size.restype = ctypes.c_int
    L.ifa4_backward_launch.argtypes = [ctypes.POINTER(BackwardParams), vp, sz, vp]
    L.ifa4_backward_launch.restype = ctypes.c_int
    L.ifa4_backward_workspace_size.argtypes = [ctypes.POINTER(BackwardParams), ctypes.POINTER(sz)]
    L.ifa4_backward_workspace_size.restype = ctypes.c_int
    L.ifa4_rel_logits_launch.argtypes = [ctypes.POINTER(RelLogitsParams), vp]
    L.ifa4_rel_logits_launch.restype = ctypes.c_int
    L.ifa4_selftest_bounded_wait.argtypes = [ctypes.c_int64, vp]
    L.ifa4_selftest_bounded_wait.restype = ctypes.c_int
    L.ifa4_measure_read_stream.argtypes = [vp, sz, vp, vp]
    L.ifa4_measure_read_stream.restype = ctypes.c_int
    L.ifa4_read_device_status.argtypes = [vp, i32, ctypes.POINTER(i32)]
    L.ifa4_read_device_status.restype = ctypes.c_int
    L.ifa4_prefill_tile_config_name.argtypes = [i32]
    L.ifa4_prefill_tile_config_name.restype = ctypes.c_char_p
    L.ifa4_last_error_string.argtypes = []
    L.ifa4_last_error_string.restype = ctypes.c_char_p
    L.ifa4_abi_version.argtypes = []
    L.ifa4_abi_version.restype = i32
    if L.ifa4_abi_version() != ABI_VERSION:
        raise RuntimeError(f"libinkling_fa4 ABI {L.ifa4_abi_version()} != {ABI_VERSION}")
    _lib = L
    return L


def check(rc: int) -> None:
    if rc != IFA4_OK:
        msg = lib().ifa4_last_error_string().decode(errors="replace")
        raise Ifa4Error(rc, msg)


def read_device_status(stream_handle: int = 0, clear: bool = True) -> int:
    """Synchronising read of the kernels' bounded-wait status word (0 = healthy)."""
    out = ctypes.c_int32(0)
    check(lib().ifa4_read_device_status(ctypes.c_void_p(stream_handle), int(clear),
                                        ctypes.byref(out)))
    return int(out.value)
