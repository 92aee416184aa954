"""Shared pytest setup.

* Registers the ``gpu`` marker: tests that need a B200.  ``-m "not gpu"`` runs
  the CPU suite (oracle pins, layout, ABI exports, host logic, gloo ranks).
* Builds the in-tree libraries when they are missing (nvcc cross-compiles for
  sm_100a without a GPU), so the suite is self-contained.
"""
from __future__ import annotations

import importlib.util
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
GOLDEN = os.path.join(ROOT, "tests", "golden")


def _ensure_built() -> None:
    spec = importlib.util.spec_from_file_location("_oracle_b200_build", os.path.join(ROOT, "oracle_b200", "build.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    mod.build_all()


_ensure_built()


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 GPU (sm_100a)")


def golden(name: str):
    return np.load(os.path.join(GOLDEN, name))


@pytest.fixture(scope="session")
def port():
    import oracle
    return oracle.port()


@pytest.fixture(scope="session")
def ref():
    import oracle
    if not os.path.exists(oracle.REF_PATH):
        pytest.skip("reference checker library not built (reference tree absent)")
    return oracle.ref()


@pytest.fixture(scope="session")
def ctx():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import oracle_b200 as ob
    c = ob.Context(0)
    yield c
    c.close()
