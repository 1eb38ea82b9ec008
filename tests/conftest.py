"""Shared test setup.

Markers: `gpu` tests need a B200 and call the product library through its C
ABI; everything else runs on the CPU (oracle pinning, host logic, ABI
exports, multi-process gloo tests).

The CPU oracles are built on demand (oracle/Makefile): the C++ restatement
(oracle/_build/libmg_oracle.so) always, and the reference build
(oracle/_ref/libmg_ref.so) when the reference source tree is available or the
library was prebuilt and shipped with the repository.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tests"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU (runs on the GPU box)")
    config.addinivalue_line("markers", "slow: longer CPU test")


@pytest.fixture(scope="session")
def oracle():
    from orc import load_oracle

    return load_oracle()


@pytest.fixture(scope="session")
def refimpl():
    from orc import load_ref

    r = load_ref()
    if r is None:
        pytest.skip("reference build oracle/_ref/libmg_ref.so unavailable (no reference tree to build it from)")
    return r


@pytest.fixture(scope="session")
def hostenv():
    from orc import load_hostenv

    return load_hostenv()


@pytest.fixture(scope="session")
def mg():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("GPU test run without a CUDA device")
    import metalgym_b200

    return metalgym_b200.lib()
