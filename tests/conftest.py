"""Test configuration: the `gpu` marker and import paths.

The package directory is named `ryzenai-npu-lab_b200` (not a Python
identifier), so tests import it with importlib through the `pkg` fixture or
`load_pkg()`; the repository root is put on sys.path for that and for the
CPU oracle under oracle/.
"""
import importlib
import pathlib
import sys

import pytest

ROOT = pathlib.Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

PKG_NAME = "ryzenai-npu-lab_b200"


def load_pkg(sub: str | None = None):
    return importlib.import_module(PKG_NAME + ("." + sub if sub else ""))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (run with -m gpu)")


@pytest.fixture(scope="session")
def pkg():
    return load_pkg()


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test collected without a CUDA device")
    return torch.device("cuda:0")
