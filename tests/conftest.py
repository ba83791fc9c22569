"""Shared fixtures: the B200 package (loaded from its in-tree directory), the CPU oracle,
and the `gpu` marker (tests that need a B200; the CPU suite runs with -m "not gpu")."""
from __future__ import annotations

import importlib.util
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG_DIR = ROOT / "qwen3-asr-wgpu_b200"
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tests"))


def load_package():
    """Import qwen3-asr-wgpu_b200/ as module `qasr_b200` (the directory name has dashes)."""
    if "qasr_b200" in sys.modules:
        return sys.modules["qasr_b200"]
    spec = importlib.util.spec_from_file_location("qasr_b200", PKG_DIR / "__init__.py",
                                                  submodule_search_locations=[str(PKG_DIR)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["qasr_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU (sm_100a)")
    config.addinivalue_line("markers", "slow: long-running parity case")


@pytest.fixture(scope="session")
def qasr():
    return load_package()


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as o
    return o


@pytest.fixture(scope="session")
def cuda_device():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test collected on a machine without CUDA")
    major, _ = torch.cuda.get_device_capability(0)
    if major != 10:
        pytest.fail("the B200 kernels need an sm_100 device")
    return 0
