import importlib
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))

PKG_NAME = "cupilot-kernels_b200"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


def import_pkg(sub: str | None = None):
    """Import the package (its directory name has a hyphen) or a submodule."""
    return importlib.import_module(PKG_NAME if sub is None else f"{PKG_NAME}.{sub}")


@pytest.fixture(scope="session")
def pkg():
    return import_pkg()


@pytest.fixture(scope="session")
def capi():
    return import_pkg("capi")


@pytest.fixture(scope="session")
def ops():
    import torch

    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return import_pkg("ops")
