"""GPU: the C++20 adapter (include/oracle_cuda.hpp) as Oracle's C++ host would
use it, checked inside a C++ program against the reference's own compiled
functions (tests/cpp/adapter_test.cpp): known answers of the reference's tests,
bit-identical outputs for every type the reference decodes, and the same
exception class and message for invalid input."""
from __future__ import annotations

import os
import subprocess

import pytest

from conftest import ROOT

pytestmark = pytest.mark.gpu
BINARY = os.path.join(ROOT, "tests", "cpp", "adapter_test")


def test_cpp_adapter_against_reference():
    if not os.path.exists(BINARY):
        pytest.skip("adapter_test is built only where the reference headers exist")
    r = subprocess.run([BINARY], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "all checks passed" in r.stdout
