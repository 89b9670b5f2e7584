import importlib
import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

PKG_NAME = "2026_ai_pilot_challenge-1st_solution_b200"
GOLDEN = Path(__file__).resolve().parent / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); run with -m gpu")


def pkg_module(name=None):
    mod = PKG_NAME if name is None else f"{PKG_NAME}.{name}"
    return importlib.import_module(mod)


@pytest.fixture(scope="session")
def pkg():
    return pkg_module()


def has_cuda():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def cuda():
    if not has_cuda():
        pytest.fail("gpu test requested but no CUDA device is visible")
    import torch
    return torch.device("cuda", 0)


def reference_tree():
    """The reference checkout ($F16_REFERENCE, else a "reference" directory beside this
    repository), or None where it is absent (tests that need it skip with that message)."""
    p = Path(os.environ.get("F16_REFERENCE") or ROOT.parent / "reference")
    return p if (p / "cuda_fdm").exists() else None
