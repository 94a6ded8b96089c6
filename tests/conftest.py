"""Shared fixtures.  Markers: `gpu` = needs a CUDA device (run on the B200 box with -m gpu)."""
from __future__ import annotations

import importlib.util
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200); run with -m gpu")
    config.addinivalue_line("markers", "slow: long-running case")


def load_pkg():
    """The product package (directory name has dots) under the module name iq4xs_b200."""
    spec = importlib.util.spec_from_file_location("_iq4xs_loader", ROOT / "qwen_3.8_27b_optimizations_b200" / "loader.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod.load()


@pytest.fixture(scope="session")
def pkg():
    return load_pkg()


@pytest.fixture(scope="session")
def O():
    from oracle import oracle
    return oracle


@pytest.fixture(scope="session")
def golden():
    return np.load(ROOT / "tests" / "golden" / "golden_v1.npz")
