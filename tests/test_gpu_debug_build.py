"""The index-checking debug build (python -m inkling_fa4.build --debug, loaded with
INKLING_FA4_LIB=debug; compute-sanitizer is closed on this pool, so the kernels check their own
computed row, head, split and page indices): on every kernel family it reports no failed check
and produces the release build's outputs."""
import os
import subprocess
import sys

import pytest
import torch

from inkling_fa4 import _lib

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
DEBUG_LIB = os.path.join(os.path.dirname(_lib.LIB_PATH), "libinkling_fa4_debug.so")


@pytest.mark.skipif(not os.path.exists(DEBUG_LIB), reason="debug build not built")
def test_debug_build_reports_no_failed_check_and_matches_release(tmp_path):
    dst = str(tmp_path / "debug.pt")
    env = dict(os.environ, INKLING_FA4_LIB="debug")
    r = subprocess.run([sys.executable, os.path.join(HERE, "debug_build_cases.py"), dst],
                       env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    dbg = torch.load(dst)
    assert dbg["lib"].endswith("libinkling_fa4_debug.so")
    assert dbg["status"] == 0, f"debug build status word {dbg['status']}"
    sys.path.insert(0, HERE)
    from debug_build_cases import run_cases
    rel, status, path = run_cases()
    assert status == 0 and path.endswith("libinkling_fa4.so")
    for k, v in rel.items():
        torch.testing.assert_close(dbg["outs"][k], v, atol=0, rtol=0, msg=k)
