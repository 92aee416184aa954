"""CPU: the C-ABI library loads, exports every declared entry point, and its
host-only layout registry answers exactly like the reference's
(src/model/ggml_type.cpp:12-94), errors included.  No GPU calls here."""
from __future__ import annotations

import ctypes
import os
import re

import pytest

import oracle_b200 as ob
from conftest import ROOT


def declared_functions():
    names = []
    for header in sorted(os.listdir(os.path.join(ROOT, "include"))):
        if not header.endswith(".h"):
            continue
        text = open(os.path.join(ROOT, "include", header)).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names += re.findall(r"\b(oracle_[a-z0-9_]+)\s*\(", text)
    return sorted(set(names))


def test_header_declares_entry_points():
    names = declared_functions()
    for must in ["oracle_cuda_create", "oracle_cuda_storage_matvec", "oracle_cuda_quantize_q8_k",
                 "oracle_cuda_decode_rows", "oracle_cuda_host_storage_matvec", "oracle_ggml_row_byte_size"]:
        assert must in names


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(ob.LIB_PATH)
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing
    assert ob.abi_version() == 1


def test_layout_table_matches_reference(ref):
    for t in range(0, 50):
        want = ref.type_layout(t)
        got = ob.type_layout(t)
        assert got == want, t


def test_layout_sizes_of_the_path():
    # test_phase1c.cpp:139-173 and the layout contract of this path
    assert ob.type_layout(12) == ("q4_K", 256, 144, True)
    assert ob.type_layout(14) == ("q6_K", 256, 210, True)
    assert ob.type_layout(8) == ("q8_0", 32, 34, True)
    assert ob.type_layout(15) == ("q8_K", 256, 292, True)
    assert ob.type_layout(4) is None and ob.type_layout(999) is None
    assert ob.row_byte_size(4096, 12) == 2304
    assert ob.row_byte_size(12288, 12) == 6912
    assert ob.row_byte_size(4096, 14) == 3360
    assert ob.row_byte_size(4096, 8) == 4352
    assert ob.row_byte_size(4096, 15) == 4672


@pytest.mark.parametrize("cols,qtype", [(17, 8), (0, 8), (256, 999), (256, 4), (2**63, 0), (31, 2), (255, 12)])
def test_row_byte_size_errors_match_reference(ref, cols, qtype):
    import oracle
    try:
        want = ref.row_byte_size(cols, qtype)
        want_err = None
    except oracle.ReferenceError_ as e:
        want, want_err = None, e
    if want_err is None:
        assert ob.row_byte_size(cols, qtype) == want
        return
    with pytest.raises(ob.OracleCudaError) as got:
        ob.row_byte_size(cols, qtype)
    assert got.value.status == want_err.code
    assert str(got.value) == want_err.message


def test_context_without_gpu_fails_loudly():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    with pytest.raises(ob.OracleCudaError):
        ob.Context(0)


def test_argmax_key_decode_without_gpu():
    """oracle_cuda_argmax_decode is host code: keys built by hand decode to the token, and the
    NaN / non-finite keys fail with the messages of Oracle's sampler (sampler.cpp:33-43)."""
    import struct

    def key(value, index):
        b = struct.unpack("<I", struct.pack("<f", value))[0]
        b = (~b & 0xFFFFFFFF) if b & 0x80000000 else (b | 0x80000000)
        return (b << 32) | (~index & 0xFFFFFFFF)

    assert ob.argmax_decode(key(1.5, 7)) == 7
    assert ob.argmax_decode(max(key(1.5, 7), key(1.5, 3), key(-2.0, 1))) == 3
    with pytest.raises(ob.InvalidArgument, match="logits contain NaN"):
        ob.argmax_decode(0xFFFFFFFFFFFFFFFF)
    with pytest.raises(ob.InvalidArgument, match="no finite candidates"):
        ob.argmax_decode(key(float("inf"), 0))
