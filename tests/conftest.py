"""Test configuration: import paths, the ``gpu`` marker and shared fixtures.

CPU tests (``-m "not gpu"``) check the numpy oracle against the reference's
golden fixtures, the host-side logic and the C-ABI library's exports.  GPU
tests (``-m gpu``) check the CUDA path against the oracle and the fixtures,
always through ``libsdl_b200.so``.
"""

from __future__ import annotations

import json
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "speculative-decoding-lab_b200")
GOLDEN = os.path.join(ROOT, "tests", "golden")
for p in (PKG, ROOT):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (runs the sm_100a kernels)")


def pytest_collection_modifyitems(config, items):
    try:
        import torch

        has_gpu = torch.cuda.is_available()
    except Exception:  # pragma: no cover
        has_gpu = False
    if has_gpu:
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


def load_json(name: str):
    with open(os.path.join(GOLDEN, name)) as f:
        return json.load(f)


def load_npz(name: str):
    return np.load(os.path.join(GOLDEN, name))


@pytest.fixture(scope="session")
def golden():
    return {"json": load_json, "npz": load_npz}


@pytest.fixture(scope="session")
def cuda():
    import torch

    from engine import _lib

    _lib.load()
    return torch.device("cuda", 0)
