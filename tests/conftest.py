"""Shared fixtures.  GPU tests are marked ``gpu``; everything else runs on CPU."""
from __future__ import annotations

import importlib.util
import os
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_DIR = os.path.join(REPO, "qwen2.5-jetson-inference_b200")
if REPO not in sys.path:
    sys.path.insert(0, REPO)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200)")


def load_package():
    """Import the product package (its directory name is not an identifier)."""
    name = "qwen25_b200"
    if name in sys.modules:
        return sys.modules[name]
    spec = importlib.util.spec_from_file_location(
        name, os.path.join(PKG_DIR, "__init__.py"),
        submodule_search_locations=[PKG_DIR])
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


@pytest.fixture(scope="session")
def b200():
    lib = os.path.join(PKG_DIR, "libb200linear.so")
    if not os.path.exists(lib):
        spec = importlib.util.spec_from_file_location(
            "b200_build", os.path.join(PKG_DIR, "build.py"))
        m = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(m)
        m.build()
    return load_package()


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as O
    O.lib()
    return O


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")


def golden(name):
    return np.load(os.path.join(REPO, "tests", "golden", name))


# ------------------------------------------------------- torch <-> BF16 bits
def to_bits(t) -> np.ndarray:
    """BF16 torch tensor -> numpy uint16 bit patterns (host)."""
    import torch
    return t.detach().contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def from_bits(bits: np.ndarray, device):
    """numpy uint16 BF16 bits -> torch.bfloat16 tensor on device."""
    import torch
    a = np.ascontiguousarray(bits, dtype=np.uint16).view(np.int16)
    return torch.from_numpy(a.copy()).to(device).view(torch.bfloat16)
