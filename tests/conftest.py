"""Shared fixtures: markers, the reference oracle import, seeded RNG."""

import os
import sys
import tempfile

import numpy as np
import pytest
import torch

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)

# The oracle is the reference package: TGCM_REFERENCE_DIR when set, else the
# unmodified copy that the benchmark's reference arm installs under
# baseline/_ref; the oracle tests skip when neither exists.
REFERENCE_DIR = os.environ.get("TGCM_REFERENCE_DIR") or os.path.join(REPO, "baseline", "_ref", "tornado_gcm")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200)")
    config.addinivalue_line("markers", "oracle: compares against the reference implementation")
    config.addinivalue_line("markers", "slow: long-running CPU test")


def _reference_importable() -> bool:
    return os.path.isdir(os.path.join(REFERENCE_DIR, "core"))


@pytest.fixture(scope="session")
def ref():
    """Import the reference package read-only under the name ``tornado_gcm``."""
    if not _reference_importable():
        pytest.skip("reference implementation not available on this machine")
    root = tempfile.mkdtemp(prefix="tgcm_ref_")
    link = os.path.join(root, "tornado_gcm")
    os.symlink(REFERENCE_DIR, link)
    sys.path.insert(0, root)
    import importlib

    mods = {}
    for name in ["core.spherical_harmonic", "core.primitive_equations", "core.sigma_coordinates",
                 "core.time_integration", "core.filtering", "core.coordinate_systems",
                 "core.associated_legendre", "core.fourier"]:
        mods[name.split(".")[-1]] = importlib.import_module("tornado_gcm." + name)

    class _Ref:
        pass

    r = _Ref()
    r.__dict__.update(mods)
    r.import_module = importlib.import_module
    return r


@pytest.fixture
def rng():
    return np.random.default_rng(0)


def requires_cuda():
    return pytest.mark.skipif(not torch.cuda.is_available(), reason="needs CUDA")


@pytest.fixture(autouse=True)
def _restore_matmul_precision():
    """Tests that apply a precision policy switch TF32 on process-wide; undo it after each test so that
    fp32 oracles computed by later tests stay fp32."""
    saved = (torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32,
             torch.get_float32_matmul_precision())
    yield
    torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32 = saved[:2]
    torch.set_float32_matmul_precision(saved[2])
