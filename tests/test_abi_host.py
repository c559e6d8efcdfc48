"""CPU: the C-ABI library loads without a GPU, exports every symbol the
header declares, and its host-side window planner is bit-exact with the
reference (golden fixtures) and the oracle."""
import ctypes
import hashlib
import os
import re

import numpy as np
import pytest

from tests.conftest import ROOT


def _declared_symbols():
    names = set()
    for f in os.listdir(os.path.join(ROOT, "include")):
        if f.endswith(".h"):
            text = open(os.path.join(ROOT, "include", f)).read()
            text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
            names |= set(re.findall(r"\b(s2_[a-z0-9_]+)\s*\(", text))
    return names


def test_library_exports_every_declared_symbol(s2lib):
    declared = _declared_symbols()
    assert declared == set(s2lib.EXPORTED), declared ^ set(s2lib.EXPORTED)
    lib = ctypes.CDLL(s2lib.LIB_PATH)
    for name in sorted(declared):
        assert hasattr(lib, name), name


def test_error_strings(s2lib):
    lib = s2lib.lib()
    for code in (0, -1, -2, -3, -4, -5, -100):
        assert lib.s2_error_string(code)
    assert lib.s2_version() >= 1


def test_init_without_gpu_fails_cleanly(s2lib):
    import torch

    if torch.cuda.is_available():
        pytest.skip("GPU present")
    h = ctypes.c_void_p()
    r = s2lib.lib().s2_init(0, None, ctypes.byref(h))
    assert r == s2lib.S2_ERR_DEVICE and not h.value


def test_host_plan_matches_golden(s2lib, golden):
    g = golden["plans"]
    cases = sorted({k.split("__")[0] for k in g.files})
    for case in cases:
        shapes = g[f"{case}__shapes"].tolist()
        target = g[f"{case}__target"].tolist()
        shifted = case.endswith("_s1")
        a = s2lib.Plan(shapes, target, s2lib.S2_WINDOW_TARGET, shifted).arrays()
        np.testing.assert_array_equal(a["windows"], g[f"{case}__windows"], err_msg=case)
        np.testing.assert_array_equal(a["sample_window_count"], g[f"{case}__sample_window_count"], err_msg=case)
        for name in ("video_indices", "inverse_video_indices", "local_positions"):
            digest = hashlib.sha256(np.ascontiguousarray(a[name], np.int32).tobytes()).hexdigest()
            assert digest == bytes(g[f"{case}__sha_{name}"]).decode(), (case, name)


def test_host_plan_matches_oracle_both_modes(s2lib, port):
    rng = np.random.default_rng(21)
    for _ in range(300):
        shapes = rng.integers(1, 50, size=(int(rng.integers(1, 3)), 3)).tolist()
        win = rng.integers(1, 12, size=3).tolist()
        mode = int(rng.integers(0, 2))
        shifted = bool(rng.integers(0, 2))
        a = s2lib.Plan(shapes, win, mode, shifted).arrays()
        b = port.plan(shapes, win, int(shifted), mode=mode).as_dict()
        for k in b:
            np.testing.assert_array_equal(a[k], b[k], err_msg=f"{k} {shapes} {win} {mode} {shifted}")


def test_baseline_window_counts(s2lib):
    """Window counts of the BASELINE configurations (explicit extents)."""
    E = s2lib.S2_WINDOW_EXTENT
    cases = [([1, 32, 32], [1, 16, 16], 4, 9), ([1, 64, 64], [1, 16, 16], 16, 25),
             ([6, 45, 80], [2, 15, 20], 36, 80), ([12, 68, 120], [4, 17, 30], 48, 100)]
    for shape, win, n0, n1 in cases:
        assert len(s2lib.Plan([shape], win, E, False).arrays()["windows"]) == n0
        assert len(s2lib.Plan([shape], win, E, True).arrays()["windows"]) == n1
    # the reference's own target mode reaches the 720p extents with target (4,3,4)
    w = s2lib.Plan([[6, 45, 80]], [4, 3, 4], s2lib.S2_WINDOW_TARGET, False).arrays()["windows"]
    assert len(w) == 36 and (w[0, 2] - w[0, 1], w[0, 4] - w[0, 3], w[0, 6] - w[0, 5]) == (2, 15, 20)


def test_plan_errors(s2lib):
    with pytest.raises(s2lib.S2Error) as e:
        s2lib.Plan([[0, 4, 4]], [1, 1, 1])
    assert e.value.code == s2lib.S2_ERR_INVALID
    with pytest.raises(s2lib.S2Error):
        s2lib.Plan([[1, 4, 4]], [1, 0, 1])
