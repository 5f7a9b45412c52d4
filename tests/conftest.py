"""Shared fixtures: the package under test, the CPU oracle, the gpu marker."""
from __future__ import annotations

import importlib.util
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG_DIR = ROOT / "gemv-q4_k-optimization_b200"
sys.path.insert(0, str(ROOT / "oracle"))


def load_package():
    """Import gemv-q4_k-optimization_b200/ (not an identifier) as module q4k_b200."""
    if "q4k_b200" in sys.modules:
        return sys.modules["q4k_b200"]
    spec = importlib.util.spec_from_file_location("q4k_b200", PKG_DIR / "__init__.py",
                                                  submodule_search_locations=[str(PKG_DIR)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["q4k_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def pytest_collection_modifyitems(config, items):
    try:
        import torch
        has_gpu = torch.cuda.is_available()
    except Exception:
        has_gpu = False
    if has_gpu:
        return
    skip = pytest.mark.skip(reason="no CUDA device in this environment")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def q4k():
    return load_package()


@pytest.fixture(scope="session")
def oracle():
    import oracle as O
    O.build()
    return O
