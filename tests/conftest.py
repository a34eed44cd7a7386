"""Shared test setup.

Markers
  gpu : needs a CUDA device (run on a B200 with `pytest -m gpu`); everything
        else runs on CPU.
"""
from __future__ import annotations

import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "s2.cpp_b200")
ORACLE = os.path.join(ROOT, "oracle")
for p in (PKG, ORACLE):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: test needs a CUDA device (B200)")


@pytest.fixture(scope="session")
def golden():
    return dict(np.load(os.path.join(ROOT, "tests", "golden", "quants.npz")))


@pytest.fixture(scope="session")
def small_model_data():
    import synthetic
    hp = synthetic.preset("small")
    tensors = list(synthetic.make_model(hp, seed=11, norm_std=0.1))
    return hp, tensors


@pytest.fixture(scope="session")
def small_oracle(small_model_data):
    import oracle
    hp, tensors = small_model_data
    om = oracle.OracleModel(hp)
    om.load_tensors(tensors)
    return om
