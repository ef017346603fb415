"""Shared test plumbing.

Tests marked ``gpu`` need a CUDA device (a B200) and call the kernels through
the C-ABI; everything else runs on the CPU (oracle, reference CPU path, host
logic, library exports).
"""
from __future__ import annotations

import importlib.util
import json
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = ROOT / "tests" / "golden"
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU; calls the sm_100a kernels through the C-ABI")


def import_package(name: str = "lis_b200"):
    """Imports the llm-inference-server_b200 directory as package `name`."""
    if name in sys.modules:
        return sys.modules[name]
    pkg = ROOT / "llm-inference-server_b200"
    spec = importlib.util.spec_from_file_location(name, pkg / "__init__.py", submodule_search_locations=[str(pkg)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


@pytest.fixture(scope="session")
def b2():
    return import_package()


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as O
    O.load()
    return O


@pytest.fixture(scope="session")
def golden():
    def _load(name: str):
        return json.loads((GOLDEN / name).read_text())
    return _load


@pytest.fixture(scope="session")
def cuda():
    import torch
    assert torch.cuda.is_available(), "GPU test run without a CUDA device"
    torch.cuda.init()
    return torch.device("cuda:0")


@pytest.fixture
def rng():
    return np.random.Generator(np.random.PCG64(1234))
