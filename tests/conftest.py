import os
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]
PKG = REPO / "lava.jl_b200"
for p in (str(REPO), str(PKG)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")
    config.addinivalue_line("markers", "slow: full-size benchmark-config parity cases")


def _has_gpu() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    if _has_gpu():
        return
    skip = pytest.mark.skip(reason="no CUDA device visible (GPU tier runs on the B200 box)")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)


@pytest.fixture(scope="session")
def lvb():
    # Build on demand so a fresh checkout can run the CPU tier.
    import importlib.util
    spec = importlib.util.spec_from_file_location("lvb_build", PKG / "build.py")
    b = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(b)
    b.build()
    import lvb as mod
    return mod


@pytest.fixture(scope="session")
def torch_cuda():
    import torch
    assert torch.cuda.is_available()
    torch.cuda.init()
    return torch
