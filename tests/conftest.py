"""Shared test setup.

Markers: ``gpu`` -- needs a B200 (run with ``-m gpu``); everything else runs on
CPU (``-m "not gpu"``).  The package directory has a hyphen in its name
(tensor-bridge_b200/), so it is loaded by path as module ``tensor_bridge_b200``.
"""
import importlib.util
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))


def load_package():
    name = "tensor_bridge_b200"
    if name in sys.modules:
        return sys.modules[name]
    pkg_dir = os.path.join(ROOT, "tensor-bridge_b200")
    spec = importlib.util.spec_from_file_location(name, os.path.join(pkg_dir, "__init__.py"),
                                                  submodule_search_locations=[pkg_dir])
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 GPU (B200)")


@pytest.fixture(scope="session")
def tb():
    return load_package()


@pytest.fixture(scope="session")
def golden():
    return np.load(os.path.join(ROOT, "tests", "golden", "golden.npz"))


@pytest.fixture(scope="session")
def cuda():
    """torch with a CUDA device; skips when there is none (CPU containers)."""
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch
