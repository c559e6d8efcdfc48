"""The index-checked build (libseedvr2_cuda_checked.so, compiled with S2_DEBUG_BOUNDS).

Its table-driven kernels -- the q/k/v gather (prepare_qkv, row_src), the attention scatter
(video_indices, the window text partial rows) and the text pool (partial rows) -- test every index
they read from a schedule table before it addresses memory, record a bad one in the status word
and skip the access.  This is the stand-in for a memory checker while compute-sanitizer is not
available: a schedule corrupted on the CPU must end in s2_status = -1 with the GPU untouched.

GPU: tests/checked_bounds_case.py runs in a process of its own against the checked library (one
process loads one build of the library) and reports four corrupted-table forwards plus a clean
run before and after them.  CPU: the normal build refuses to corrupt a schedule at all.
"""
import json
import os
import subprocess
import sys

import pytest

from tests.conftest import ROOT


@pytest.mark.gpu
def test_checked_build_turns_bad_table_indices_into_an_error():
    lib = os.path.join(ROOT, "seedvr2_ncnn_b200", "libseedvr2_cuda_checked.so")
    assert os.path.exists(lib), "build it: python -c 'from seedvr2_ncnn_b200 import build; build.build_checked()'"
    env = dict(os.environ, S2_CUDA_LIB=lib)
    r = subprocess.run([sys.executable, os.path.join(ROOT, "tests", "checked_bounds_case.py")], env=env, cwd=ROOT,
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-3000:]
    out = json.loads(r.stdout.strip().splitlines()[-1])
    assert out["clean_status"] == 0 and out["clean_finite"], out
    for name in ("gather_video", "gather_text", "scatter_row", "scatter_peer"):
        # the poke took (0) and the forward over it reported the bad index (-1)
        assert out[name] == [0, -1], (name, out)
    # the same context afterwards: clean, and bit-identical to the first run
    assert out["after_status"] == 0 and out["after_equal"], out


def test_unchecked_build_refuses_to_corrupt_a_schedule(s2lib):
    p = s2lib.Plan([[3, 7, 11]], [2, 3, 4], s2lib.S2_WINDOW_EXTENT, True)

    class _NoContext:
        handle = None

    assert p.debug_poke(_NoContext(), 0, 0, 1 << 27) == s2lib.S2_ERR_INVALID
