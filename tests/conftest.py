"""pytest configuration: the `gpu` marker and import paths for the host package."""

from __future__ import annotations

import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
PKG = REPO / "cd-cuda-course-project_b200"
for p in (str(REPO), str(PKG), str(PKG / "src")):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = Path(__file__).resolve().parent / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def _cuda_available() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:  # pragma: no cover
        return False


@pytest.fixture(scope="session")
def dev():
    import torch
    if not _cuda_available():
        pytest.skip("no CUDA device")
    torch.cuda.set_device(0)
    return torch.device("cuda", 0)


@pytest.fixture(scope="session")
def lib():
    """The default kernel library; it must exist (no fallback)."""
    import kt_lib
    import build as kt_build
    if kt_build.default_library_stale():
        kt_build.build_default()
    return kt_lib.load()


@pytest.fixture(scope="session")
def golden():
    import numpy as np
    return dict(np.load(GOLDEN / "reference_kat.npz"))
