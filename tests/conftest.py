import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200); run with -m gpu")
    config.addinivalue_line("markers", "slow: longer CPU test")


@pytest.fixture(scope="session")
def golden_dir():
    return ROOT / "tests" / "golden"


def _cuda_ok():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    if _cuda_ok():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


def reference_path():
    """The reference package to test the drop-in against: NS_REFERENCE_PATH, else baseline/_ref."""
    p = os.environ.get("NS_REFERENCE_PATH") or str(ROOT / "baseline" / "_ref")
    return p if os.path.isdir(os.path.join(p, "neurostream")) else None


@pytest.fixture
def reference(monkeypatch):
    """Puts the reference package on sys.path (skips when it is not installed on this machine)."""
    p = reference_path()
    if p is None:
        pytest.skip("reference package not installed (baseline/_ref or NS_REFERENCE_PATH)")
    monkeypatch.syspath_prepend(p)
    sys.dont_write_bytecode = True
    return p
