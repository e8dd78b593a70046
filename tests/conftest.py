"""Shared test fixtures.

Markers: ``gpu`` tests need a B200 (sm_100a); everything else runs on CPU.
The package directory name is not a Python identifier, so it is imported
from its path under the module name ``b2g``.
"""
from __future__ import annotations

import importlib.util
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG_DIR = ROOT / "llama-3.2-3b-instruct-gemm-optimization_b200"
GOLDEN = ROOT / "tests" / "golden"


def _load(name: str, path: Path, package: bool = False):
    if name in sys.modules:
        return sys.modules[name]
    kw = {"submodule_search_locations": [str(path.parent)]} if package else {}
    spec = importlib.util.spec_from_file_location(name, path, **kw)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def load_b2g():
    return _load("b2g", PKG_DIR / "__init__.py", package=True)


def load_synthetic():
    return _load("b2g_synthetic", PKG_DIR / "synthetic.py")


def load_oracle():
    return _load("oracle", ROOT / "oracle" / "oracle.py")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU (sm_100a)")


@pytest.fixture(scope="session")
def b2g():
    return load_b2g()


@pytest.fixture(scope="session")
def syn():
    return load_synthetic()


@pytest.fixture(scope="session")
def orc():
    return load_oracle()


@pytest.fixture(scope="session")
def cuda():
    import torch
    assert torch.cuda.is_available(), "GPU test run without a CUDA device"
    major, minor = torch.cuda.get_device_capability()
    assert (major, minor) == (10, 0), f"expected sm_100 (B200), got sm_{major}{minor}"
    return torch.device("cuda:0")
