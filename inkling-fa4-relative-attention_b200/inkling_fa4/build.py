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


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--debug", action="store_true")
    a = ap.parse_args()
    print(build(verbose=a.verbose, force=a.force, debug=a.debug))
