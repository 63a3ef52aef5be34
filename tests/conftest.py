"""Shared pytest setup.

Markers: `gpu` tests need a B200 and run the product kernels through the C
ABI (libgemm.so); everything else runs on a CPU-only host.
"""
from __future__ import annotations

import json
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "fp8-mlp-metal41-bench_b200")
GOLDEN = os.path.join(ROOT, "tests", "golden")
for p in (ROOT, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU (runs libgemm.so kernels)")


def golden(name: str):
    with open(os.path.join(GOLDEN, name), encoding="utf-8") as f:
        return json.load(f)


@pytest.fixture(scope="session")
def gemm():
    """libgemm.so initialised on device 0 (GPU tests only)."""
    from mlpgemm import lib as G
    G.init(0)
    return G
