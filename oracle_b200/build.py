"""Build recipe for the in-tree native libraries.

* ``oracle_b200/liboracle_cuda.so`` -- the product: CUDA kernels for sm_100a
  plus the C ABI of ``include/oracle_cuda.h``, built by nvcc with
  ``-gencode arch=compute_100a,code=sm_100a`` (cudart linked statically).
* ``oracle/liboracle_port.so`` and ``oracle/_ref/liboracle_ref.so`` -- the CPU
  checkers used by the tests (``oracle/Makefile``); the second one only when
  the environment variable ``ORACLE_REFERENCE_TREE`` names Oracle's source
  tree (there is no default).  Without it the build says so and keeps the
  checker libraries already built, if any.

This file is loaded by path (``__graft_entry__.build``, ``tests/conftest.py``)
so that it runs before the package's library exists.
"""
from __future__ import annotations

import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
LIB = os.path.join(HERE, "liboracle_cuda.so")
CSRC = os.path.join(HERE, "csrc")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
# Oracle's source tree (the checker and the C++ tests compile its files);
# no default: a machine without it uses the checker libraries built elsewhere.
REFERENCE_TREE = os.environ.get("ORACLE_REFERENCE_TREE", "")


def _reference_tree() -> str | None:
    if REFERENCE_TREE and os.path.isdir(os.path.join(REFERENCE_TREE, "src")):
        return REFERENCE_TREE
    return None


def _say(msg: str) -> None:
    print(f"[oracle_b200.build] {msg}", file=sys.stderr, flush=True)


def _sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu"))) + sorted(glob.glob(os.path.join(CSRC, "*.cuh"))) + \
        sorted(glob.glob(os.path.join(CSRC, "*.hpp"))) + [os.path.join(ROOT, "include", "oracle_cuda.h")]


def _stale(target: str, deps) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


BUILD_DIR = os.path.join(HERE, "_build")
LIBM_GEN_SRC = os.path.join(CSRC, "libm_tables.c")
LIBM_TABLES = os.path.join(BUILD_DIR, "libm_tables.bin")
LIBM_OBJ = os.path.join(BUILD_DIR, "libm_blob.o")


def build_libm_tables() -> str:
    """The host C library's expf / log1pf correction tables (csrc/libm_tables.c:
    runs the library on every float input of the decoder's domains, ~1 min on 8
    cores), assembled into an object that is linked into liboracle_cuda.so."""
    os.makedirs(BUILD_DIR, exist_ok=True)
    gen = os.path.join(BUILD_DIR, "libm_tables")
    if _stale(gen, [LIBM_GEN_SRC]):
        subprocess.run(["gcc", "-O2", "-pthread", "-o", gen, LIBM_GEN_SRC, "-lm"], check=True)
    if _stale(LIBM_TABLES, [gen]):
        _say("generating the expf/log1pf tables from the host C library (about a minute)")
        subprocess.run([gen, LIBM_TABLES], check=True)
    if _stale(LIBM_OBJ, [LIBM_TABLES]):
        asm = os.path.join(BUILD_DIR, "libm_blob.S")
        with open(asm, "w") as f:
            f.write("\t.section .rodata\n\t.balign 16\n\t.globl oracle_libm_blob\noracle_libm_blob:\n"
                    f"\t.incbin \"{LIBM_TABLES}\"\n\t.globl oracle_libm_blob_end\noracle_libm_blob_end:\n"
                    "\t.section .note.GNU-stack,\"\",@progbits\n")
        subprocess.run(["gcc", "-c", "-fPIC", "-o", LIBM_OBJ, asm], check=True)
    return LIBM_OBJ


def build_cuda(force: bool = False, verbose: bool = False) -> str:
    obj = build_libm_tables()
    if force or _stale(LIB, _sources() + [obj]):
        cmd = [NVCC, *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-shared",
               "-o", LIB, os.path.join(CSRC, "oracle_cuda.cu"), obj]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
        subprocess.run(cmd, check=True)
    return LIB


def build_oracle() -> None:
    targets = ["port"]
    tree = _reference_tree()
    if tree:
        targets += ["ref", "ref_q8k", "ref_gate"]
    else:
        have = [p for p in ("liboracle_ref.so", "liboracle_ref_q8k.so", "liboracle_ref_gate.so")
                if os.path.exists(os.path.join(ROOT, "oracle", "_ref", p))]
        _say("ORACLE_REFERENCE_TREE is not set to Oracle's source tree: the reference checker "
             f"(oracle/_ref) is NOT rebuilt; prebuilt libraries present: {have or 'none'}")
    subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "oracle"), f"REF={tree or ''}", *targets],
                   check=True)


CPP_TEST = os.path.join(ROOT, "tests", "cpp", "adapter_test")
CPP_GGUF_TEST = os.path.join(ROOT, "tests", "cpp", "gguf_test")


def build_cpp_tests() -> None:
    """The C++ tests (tests/cpp/adapter_test.cpp, gguf_test.cpp): compiled
    against Oracle's headers, so only where the reference tree exists; the
    binaries travel with the repository snapshot."""
    tree = _reference_tree()
    if not tree:
        _say("ORACLE_REFERENCE_TREE is not set: the C++ adapter tests (tests/cpp) are NOT rebuilt")
        return
    inc = os.path.join(tree, "include")
    ref_dir = os.path.join(ROOT, "oracle", "_ref")
    port_dir = os.path.join(ROOT, "oracle")
    for binary, name in ((CPP_TEST, "adapter_test.cpp"), (CPP_GGUF_TEST, "gguf_test.cpp")):
        src = os.path.join(ROOT, "tests", "cpp", name)
        deps = [src, os.path.join(ROOT, "include", "oracle_cuda.hpp"), os.path.join(ROOT, "include", "oracle_cuda.h"),
                LIB]
        if not _stale(binary, deps):
            continue
        subprocess.run(["g++", "-std=c++20", "-O2", "-I", os.path.join(ROOT, "include"), "-I", inc, src, "-o", binary,
                        "-L", HERE, "-loracle_cuda", "-L", ref_dir, "-loracle_ref", "-L", port_dir, "-loracle_port",
                        "-Wl,-rpath,$ORIGIN/../../oracle_b200", "-Wl,-rpath,$ORIGIN/../../oracle/_ref",
                        "-Wl,-rpath,$ORIGIN/../../oracle"], check=True)


def build_all(force: bool = False) -> None:
    build_cuda(force=force)
    build_oracle()
    build_cpp_tests()


if __name__ == "__main__":
    build_all(force="--force" in sys.argv)
