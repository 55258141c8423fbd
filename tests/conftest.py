"""Shared test set-up.

Markers: ``gpu`` = needs a B200 (compute capability 10.0). The CPU suite
(``-m "not gpu"``) covers the oracle against the reference's golden vectors,
host logic and the C-ABI surface without launching kernels.
"""
from __future__ import annotations

import importlib
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "best-matmul_b200")
ORACLE_DIR = os.path.join(ROOT, "oracle")
for p in (ROOT, PKG, ORACLE_DIR):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: test needs a B200 GPU (sm_100a)")


def _ensure_built():
    lib = os.path.join(PKG, "lib", "libbmgemm.so")
    orc = os.path.join(ORACLE_DIR, "lib", "libbm_oracle.so")
    if not (os.path.exists(lib) and os.path.exists(orc)):
        importlib.import_module("__graft_entry__").build()


_ensure_built()


@pytest.fixture(scope="session")
def orc():
    from oracle import Oracle
    return Oracle()


@pytest.fixture(scope="session")
def reflib():
    from oracle import REF_LIB, RefLib
    if not os.path.exists(REF_LIB):
        pytest.skip("reference shim (oracle/_ref) not built here")
    return RefLib()


@pytest.fixture(scope="session")
def bm():
    return importlib.import_module("bmgemm")


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test needs CUDA")
    major, minor = torch.cuda.get_device_capability(0)
    if (major, minor) != (10, 0):
        pytest.fail(f"GPU test needs compute capability 10.0, found {major}.{minor}")
    torch.cuda.set_device(0)
    return torch
