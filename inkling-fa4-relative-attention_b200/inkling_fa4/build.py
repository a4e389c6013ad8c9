"""Build the in-tree CUDA library ``inkling_fa4/_lib/libinkling_fa4.so`` for sm_100a.

    python -m inkling_fa4.build [--verbose] [--debug]

``--debug`` builds ``_lib/libinkling_fa4_debug.so`` with ``-DIFA4_DEBUG``: the kernels then
check their computed row, head, split and page indices before the global accesses that use them
and report a failed check in the status word (bit ``kStatusDebugBounds``) instead of touching
memory out of range (the accesses are skipped).  ``INKLING_FA4_LIB=debug`` makes the package
load it.

nvcc cross-compiles without a GPU.  The library links the CUDA runtime statically and reaches
the driver's ``cuTensorMapEncodeTiled`` through ``cudaGetDriverEntryPoint``, so it needs no
``-lcuda`` at link time.
"""
from __future__ import annotations

import argparse
import os
import re
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG_DIR)
CSRC = os.path.join(ROOT, "csrc")
OUT = os.path.join(PKG_DIR, "_lib", "libinkling_fa4.so")
OUT_DEBUG = os.path.join(PKG_DIR, "_lib", "libinkling_fa4_debug.so")
OUT_TORCH_OPS = os.path.join(PKG_DIR, "_lib", "libifa4_torch_ops.so")
SOURCES = ["ifa4_capi.cu", "ifa4_prefill_sm100.cu", "ifa4_decode_sm100.cu", "ifa4_backward_sm100.cu",
           "ifa4_rel_logits_sm100.cu"]
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    p = shutil.which("nvcc")
    if p:
        return p
    cand = "/usr/local/cuda/bin/nvcc"
    if os.path.exists(cand):
        return cand
    raise RuntimeError("nvcc not found")


def build(verbose: bool = False, force: bool = False, debug: bool = False) -> str:
    out = OUT_DEBUG if debug else OUT
    srcs = [os.path.join(CSRC, s) for s in SOURCES]
    headers = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".h", ".cuh"))]
    headers.append(os.path.join(os.path.dirname(ROOT), "include", "inkling_fa4.h"))
    if not force and os.path.exists(out):
        newest = max(os.path.getmtime(f) for f in srcs + headers if os.path.exists(f))
        if os.path.getmtime(out) >= newest:
            return out
    os.makedirs(os.path.dirname(out), exist_ok=True)
    tmp = out + ".tmp"
    cmd = [nvcc_path(), *ARCH_FLAGS, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
           "-Xptxas=-v", "-shared", "-o", tmp, *srcs]
    if debug:
        cmd.insert(1, "-DIFA4_DEBUG=1")
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if verbose or r.returncode != 0:
        sys.stdout.write(r.stdout)
        sys.stderr.write(r.stderr)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed ({r.returncode})")
    os.replace(tmp, out)
    return out


def build_torch_ops(verbose: bool = False, force: bool = False) -> str:
    """Compile ``csrc/ifa4_torch_ops.cpp`` (the torch operators inkling_fa4::prefill_ and
    inkling_fa4::decode_ over the C ABI) with g++ against torch's headers and libraries, linked
    to the in-tree ``libinkling_fa4.so`` (found next to it at run time)."""
    import torch
    from torch.utils import cpp_extension

    src = os.path.join(CSRC, "ifa4_torch_ops.cpp")
    header = os.path.join(os.path.dirname(ROOT), "include", "inkling_fa4.h")
    if not force and os.path.exists(OUT_TORCH_OPS):
        newest = max(os.path.getmtime(f) for f in (src, header, OUT))
        if os.path.getmtime(OUT_TORCH_OPS) >= newest:
            return OUT_TORCH_OPS
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    incs = cpp_extension.include_paths() + [os.path.join(cuda_home, "include")]
    libdir = cpp_extension.library_paths()[0]
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    tmp = OUT_TORCH_OPS + ".tmp"
    cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           *[f"-I{i}" for i in incs], src, "-o", tmp, f"-L{libdir}", f"-L{os.path.dirname(OUT)}",
           "-linkling_fa4", "-lc10", "-lc10_cuda", "-ltorch_cpu", "-ltorch",
           "-Wl,-rpath,$ORIGIN", f"-Wl,-rpath,{libdir}"]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if verbose or r.returncode != 0:
        sys.stdout.write(r.stdout)
        sys.stderr.write(r.stderr)
    if r.returncode != 0:
        raise RuntimeError(f"g++ failed ({r.returncode})")
    os.replace(tmp, OUT_TORCH_OPS)
    return OUT_TORCH_OPS


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--debug", action="store_true")
    a = ap.parse_args()
    print(build(verbose=a.verbose, force=a.force, debug=a.debug))
    if not a.debug:
        print(build_torch_ops(verbose=a.verbose, force=a.force))
