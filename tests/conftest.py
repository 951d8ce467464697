"""Shared test set-up: the ``gpu`` marker, import paths and golden fixtures.

Tests marked ``gpu`` need a B200 and the built CUDA library; everything else
runs on a CPU-only host."""

from __future__ import annotations

import json
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_ROOT = os.path.join(ROOT, "mlx-lean-moe_b200")
GOLDEN_DIR = os.path.join(ROOT, "tests", "golden")
for p in (ROOT, PKG_ROOT, GOLDEN_DIR):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200) and the built library")


@pytest.fixture(scope="session")
def golden():
    with np.load(os.path.join(GOLDEN_DIR, "golden.npz")) as data:
        return {k: data[k] for k in data.files}


@pytest.fixture(scope="session")
def manifest():
    with open(os.path.join(GOLDEN_DIR, "golden_manifest.json")) as f:
        return json.load(f)
