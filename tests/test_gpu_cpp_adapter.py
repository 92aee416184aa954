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


def test_mapped_gguf_views_through_cpp_adapter(tmp_path):
    """A GGUF file mapped by Oracle's own MappedGgufModel; every tensor view goes through the
    C++ adapter and must match the reference's compiled functions (or the restatement for Q4_K)."""
    import subprocess
    import sys

    binary = os.path.join(ROOT, "tests", "cpp", "gguf_test")
    if not os.path.exists(binary):
        pytest.skip("tests/cpp/gguf_test is built only where the reference tree exists")
    sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))
    import make_gguf
    path = str(tmp_path / "synthetic.gguf")
    tensors = make_gguf.write(path)
    r = subprocess.run([binary, path], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert f"{len(tensors) + 1} tensors, 0 failures" in r.stdout, r.stdout
