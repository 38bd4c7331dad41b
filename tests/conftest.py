"""pytest configuration: markers, import paths, shared fixtures.

``-m "not gpu"`` runs on any host (oracle vs golden vectors, host logic, C-ABI exports,
gloo multi-rank logic). ``-m gpu`` runs the parity tests through the C ABI on a B200.
"""
from __future__ import annotations

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SRC = os.path.join(ROOT, "dcr-attention_v3_b200")
for p in (ROOT, SRC, os.path.join(ROOT, "tests", "golden")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and libdcr_b200.so")
    config.addinivalue_line("markers", "slow: long-running (full-size) case")


@pytest.fixture(scope="session")
def oracle_mod():
    from oracle import oracle as O
    O.build()
    return O


@pytest.fixture(scope="session")
def cuda_lib():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from dcr_b200 import _lib
    return _lib.load()
