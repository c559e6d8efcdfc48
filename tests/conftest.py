import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) GPU")


@pytest.fixture(scope="session")
def port():
    from oracle import oracle

    oracle.build()
    return oracle.Port()


@pytest.fixture(scope="session")
def ref():
    """The reference's own layer code (built only where its tree is present)."""
    from oracle import oracle

    if not os.path.exists(oracle.REF_SO):
        pytest.skip("oracle/_ref/libs2_ref.so not built (reference tree absent)")
    return oracle.Ref()


@pytest.fixture(scope="session")
def golden():
    return {name: np.load(os.path.join(GOLDEN, f"{name}.npz")) for name in ("plans", "awa", "linear", "dit_io", "vae_conv")}


@pytest.fixture(scope="session")
def refio():
    """The reference's own patchify / timestep / unpatchify (built only where its tree is present)."""
    from oracle import oracle

    if not os.path.exists(oracle.REF_IO_SO):
        pytest.skip("oracle/_ref/libs2_ref_dit_io.so not built (reference tree absent)")
    return oracle.RefIO()


@pytest.fixture(scope="session")
def s2lib():
    from seedvr2_ncnn_b200 import abi, build

    build.build()
    return abi


@pytest.fixture(scope="session")
def gpu_ctx(s2lib):
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    ctx = s2lib.Context(0)
    yield ctx
    assert ctx.status() == 0, "a kernel recorded a device error"
    ctx.close()


def cosine(a, b) -> float:
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b) + 1e-300))


def rel_maxabs(a, b) -> float:
    """max |a - b| / max |b|  (b = fp32 reference)."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))
