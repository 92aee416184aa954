"""B200 (sm_100a) quantized-weight path of Oracle, behind a C ABI.

This package is the Python host mirror of ``include/oracle_cuda.h``.  It loads
``liboracle_cuda.so`` (built in-tree by ``oracle_b200.build``) with ctypes and
exposes the reference's entry points under the reference's names:

=========================================  ==============================================
reference (Oracle repository)              here
=========================================  ==============================================
ggml_type_layout / ggml_row_byte_size      :func:`type_layout` / :func:`row_byte_size`
 (src/model/ggml_type.cpp:69-94)
decode_storage_row,                        :meth:`Context.decode_rows` (device),
 reference_decode_mapped_tensor             :meth:`Context.host_decode_rows` (host)
 (storage_decode.cpp:244-294,
  quantized_reference.cpp:85-105)
reference_storage_dot (:24-82)             :meth:`Context.host_storage_dot`
reference_storage_matvec (:128-162)        :meth:`Context.storage_matvec` (device),
                                           :meth:`Context.host_storage_matvec` (host)
(no counterpart) Q8_K quantizer            :meth:`Context.quantize_q8_k`
=========================================  ==============================================

Errors raise the subclass of :class:`OracleCudaError` that names the C++
exception the reference throws for the same input, with the reference's
message.  There is no CPU fallback: importing this package without the built
library raises ``ImportError``.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

from . import synth  # noqa: F401  (re-exported helper module)

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle_cuda.so")

TYPE_F32, TYPE_F16, TYPE_Q8_0, TYPE_Q4_K, TYPE_Q5_K, TYPE_Q6_K, TYPE_Q8_K, TYPE_BF16 = (
    0, 1, 8, 12, 13, 14, 15, 30)
CONTRACT_F32, CONTRACT_Q8K = 0, 1
FLAG_PDL = 1
FLAG_BUILD_IN_KERNEL = 2
Q8K_BLOCK_BYTES = 292

if not os.path.exists(LIB_PATH):
    raise ImportError(
        f"{LIB_PATH} is missing: build it with `python -c 'import __graft_entry__ as g; g.build()'` "
        "(there is no CPU fallback for this path)")


class _Library:
    """liboracle_cuda.so, mapped on the first call through it.

    Importing the package (its seeded generators, the model description)
    maps nothing, so a process that only uses those -- the CPU checkers and
    ``bench.py --impl reference`` -- never loads the CUDA library.  The first
    attribute access loads it and applies every prototype declared with
    :func:`_proto`."""

    def __init__(self, path: str):
        self._path = path
        self._cdll = None
        self._protos = {}

    def _load(self):
        if self._cdll is None:
            lib = C.CDLL(self._path)
            for name, (args, res) in self._protos.items():
                fn = getattr(lib, name)
                fn.argtypes = args
                fn.restype = res
            self._cdll = lib
        return self._cdll

    def __getattr__(self, name):
        if name.startswith("_"):
            raise AttributeError(name)
        return getattr(self._load(), name)


_lib = _Library(LIB_PATH)

_vp, _u32, _u64, _i32 = C.c_void_p, C.c_uint32, C.c_uint64, C.c_int
_u64p = C.POINTER(C.c_uint64)


def _proto(name, args, res=C.c_int):
    """Declare an entry point's argument and result types (applied on load)."""
    _lib._protos[name] = (args, res)


def loaded() -> bool:
    """Whether this process has mapped liboracle_cuda.so yet."""
    return _lib._cdll is not None


_proto("oracle_cuda_abi_version", [])
_proto("oracle_cuda_status_name", [_i32], C.c_char_p)
_proto("oracle_cuda_last_error", [_vp], C.c_char_p)
_proto("oracle_ggml_type_layout", [_u32, _u64p, _u64p, C.POINTER(C.c_int), C.POINTER(C.c_char_p)])
_proto("oracle_ggml_row_byte_size", [_u64, _u32, _u64p])
_proto("oracle_cuda_create", [_i32, C.POINTER(_vp)])
_proto("oracle_cuda_destroy", [_vp])
_proto("oracle_cuda_set_flags", [_vp, _u32])
_proto("oracle_cuda_device_status", [_vp])
_proto("oracle_cuda_launch_count", [_vp], C.c_uint64)
_proto("oracle_cuda_selftest_bounded_wait", [_vp, _u64])
_proto("oracle_cuda_decode_rows", [_vp, _u32, _u64, _u64, _vp, _u64, _vp, _u64, _vp])
_proto("oracle_cuda_quantize_q8_k", [_vp, _vp, _u64, _u64, _vp, _u64, _vp])
_proto("oracle_cuda_storage_matvec", [_vp, _i32, _u32, _u64, _u64, _vp, _u64, _vp, _u64, _vp, _u64, _vp])
_proto("oracle_cuda_matvec_q8k_prequantized", [_vp, _u32, _u64, _u64, _vp, _u64, _vp, _u64, _vp, _u64, _vp])
_proto("oracle_cuda_batch_image_bytes", [_u64], C.c_uint64)
_proto("oracle_cuda_batch_quantize", [_vp, _vp, _u64, _u32, _vp, _u64, _vp])
_proto("oracle_cuda_batch_norm_quantize", [_vp, _vp, _vp, _vp, _vp, C.c_float, _u64, _u32, _vp, _u64, _vp])
_proto("oracle_cuda_batch_matvec", [_vp, _u32, _u64, _u64, _vp, _u64, _vp, _u64, _u32, _vp, _u64, _vp])


class MatvecOp(C.Structure):
    """oracle_cuda_matvec_op of include/oracle_cuda.h."""
    _fields_ = [("type", C.c_uint32), ("after_previous", C.c_uint32), ("rows", C.c_uint64),
                ("cols", C.c_uint64), ("w_dev", C.c_void_p), ("w_nbytes", C.c_uint64),
                ("x_dev", C.c_void_p), ("y_dev", C.c_void_p)]


class MatvecOpEx(C.Structure):
    """oracle_cuda_matvec_op_ex of include/oracle_cuda.h."""
    _fields_ = [("base", MatvecOp), ("xform", C.c_uint32), ("eps", C.c_float), ("x2_dev", C.c_void_p),
                ("norm_dev", C.c_void_p), ("residual_dev", C.c_void_p), ("act_dev", C.c_void_p)]


XFORM_NONE, XFORM_RMS, XFORM_SWIGLU, XFORM_COMBINE_RMS = 0, 1, 2, 3
PROGRAM_MAX_OPS = 16


class ShardedOp(C.Structure):
    """oracle_cuda_sharded_op of include/oracle_cuda.h."""
    _fields_ = [("ex", MatvecOpEx), ("push", C.c_uint32), ("wait", C.c_uint32), ("announce", C.c_uint32),
                ("segments", C.c_uint32), ("swiglu_gate", C.c_void_p), ("combined_dev", C.c_void_p)]


class ShardedStep(C.Structure):
    """oracle_cuda_sharded_step of include/oracle_cuda.h."""
    _fields_ = [("first_dep", C.c_uint32), ("deps_per_step", C.c_uint32), ("end_of_step", C.c_uint32),
                ("tail_wait", C.c_uint32)]
_proto("oracle_cuda_matvec_program", [_vp, C.POINTER(MatvecOp), _u32, _vp])
_proto("oracle_cuda_matvec_program_ex", [_vp, C.POINTER(MatvecOpEx), _u32, _vp])
_proto("oracle_cuda_matvec_program_ex_allgather", [_vp, _vp, C.POINTER(MatvecOpEx), _u32, _vp])
_proto("oracle_cuda_matvec_program_sharded", [_vp, _vp, C.POINTER(ShardedOp), _u32, C.POINTER(ShardedStep), _vp])
_proto("oracle_cuda_set_program_trace", [_vp, _vp, _u32])
TRACE_WORDS = 50
_proto("oracle_cuda_matvec_program_noalloc", [C.POINTER(MatvecOp), _u32, _vp])
_proto("oracle_cuda_noalloc_status", [_i32])
_proto("oracle_cuda_noalloc_selftest_bounded_wait", [_u64, _vp])
NOALLOC_IMAGE_BYTES = 65536


def _matvec_ops(ops):
    arr = (MatvecOp * len(ops))()
    for i, (qtype, rows, cols, w, x, y, after) in enumerate(ops):
        arr[i] = MatvecOp(qtype, 1 if after else 0, rows, cols, _addr(w), _nbytes(w), _addr(x), _addr(y))
    return arr


def matvec_program_noalloc(ops, stream=None) -> None:
    """oracle_cuda_matvec_program_noalloc: the matvec program without any
    device allocation (no context; scratch is a static device array), for
    callers that cannot allocate device memory.  Runs on the current device;
    ops as for :meth:`Context.matvec_program`."""
    arr = _matvec_ops(ops)
    _raise(_lib.oracle_cuda_matvec_program_noalloc(arr, len(ops), _stream(stream)), None)


def noalloc_status(device: int = 0) -> None:
    """oracle_cuda_noalloc_status: raise DeviceTimeout if a bounded device-side
    wait of the last no-allocation call on ``device`` expired (waits for the
    device's work; allocates nothing)."""
    _raise(_lib.oracle_cuda_noalloc_status(device), None)


def noalloc_selftest_bounded_wait(limit_ns: int, stream=None) -> None:
    """oracle_cuda_noalloc_selftest_bounded_wait: a wait nothing completes,
    given up after limit_ns, recorded in the no-allocation status word."""
    _raise(_lib.oracle_cuda_noalloc_selftest_bounded_wait(limit_ns, _stream(stream)), None)
_proto("oracle_cuda_weight_upload", [_vp, _u32, _u64, _u64, _vp, _u64, _u64, _u64, C.POINTER(_vp)])
_proto("oracle_cuda_weight_free", [_vp])
_proto("oracle_cuda_weight_info", [_vp, C.POINTER(_u32), _u64p, _u64p, _u64p, C.POINTER(_vp), _u64p])
_proto("oracle_cuda_host_storage_matvec", [_vp, _i32, _u32, _u64, _u64, _vp, _u64, _vp, _u64, _vp, _u64])
_proto("oracle_cuda_host_storage_dot", [_vp, _i32, _u32, _u64, _vp, _u64, _vp, _u64, _vp])
_proto("oracle_cuda_host_decode_rows", [_vp, _u32, _u64, _u64, _vp, _u64, _vp, _u64])
_proto("oracle_cuda_evict_resident", [_vp])
_proto("oracle_cuda_register_host_weight", [_vp, _u32, _u64, _u64, _vp, _u64])
_proto("oracle_cuda_unregister_host_weight", [_vp, _vp, _u64])


class HostMatvecOp(C.Structure):
    """oracle_cuda_host_matvec_op of include/oracle_cuda.h."""
    _fields_ = [("type", C.c_uint32), ("rows", C.c_uint64), ("cols", C.c_uint64), ("w_host", C.c_void_p),
                ("w_nbytes", C.c_uint64), ("x_host", C.c_void_p), ("y_host", C.c_void_p)]


_proto("oracle_cuda_host_matvec_program", [_vp, C.POINTER(HostMatvecOp), _u32])
_proto("oracle_cuda_host_program_create", [_vp, C.POINTER(HostMatvecOp), _u32, C.POINTER(_vp)])
_proto("oracle_cuda_host_program_run", [_vp])
_proto("oracle_cuda_host_program_destroy", [_vp])
_proto("oracle_cuda_prefill_gemm", [_vp, _u32, _u64, _u64, _vp, _u64, _vp, _u64, _vp, _vp])
_proto("oracle_cuda_peer_group_create", [_vp, _u32, _u32, _u64, C.POINTER(_vp), _vp])
_proto("oracle_cuda_peer_group_connect", [_vp, _vp])
_proto("oracle_cuda_peer_group_data", [_vp, C.POINTER(_vp)])
_proto("oracle_cuda_peer_group_destroy", [_vp])
_proto("oracle_cuda_matvec_program_allgather", [_vp, _vp, C.POINTER(MatvecOp), _u32, _vp])
_proto("oracle_cuda_gather_rows", [_vp, _u32, _u64, _u64, _vp, _u64, _vp, _u64, _vp, _vp])
_proto("oracle_cuda_argmax", [_vp, _vp, _u64, _u32, _vp, _vp])
_proto("oracle_cuda_argmax_decode", [C.c_uint64, C.POINTER(_u32), C.POINTER(C.c_float)])
_proto("oracle_cuda_greedy_token", [_vp, _vp, _u64, C.POINTER(_u32)])
_proto("oracle_cuda_rms_norm_rows", [_vp, _vp, _vp, _u64, _u64, C.c_float, _vp, _vp])
_proto("oracle_cuda_rope", [_vp, _vp, _u64, _u64, _u64, C.POINTER(C.c_int32), C.c_float, _u64, _u64, _u64, _vp])
_proto("oracle_cuda_attention_step", [_vp, _vp, _vp, _vp, _vp, _vp, _u64, _u64, _u32, _u32, _u32, _u32, _vp, _vp,
                                      _vp])
_proto("oracle_cuda_conv_step", [_vp, _vp, _vp, _vp, _u64, _u32, _i32, _vp, _vp])
_proto("oracle_cuda_gated_delta_step", [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _u32, _u32, _u32, _u32, C.c_float, _vp,
                                        _vp])
_proto("oracle_cuda_rope_table", [_vp, _u64, C.POINTER(C.c_int32), C.c_float, _u64, _vp])
_proto("oracle_cuda_rope_at", [_vp, _vp, _u64, _u64, _u64, _vp, _u64, _vp, _vp])
_proto("oracle_cuda_attention_step_at", [_vp, _vp, _vp, _vp, _vp, _vp, _u64, _vp, _u32, _u32, _u32, _u32, _vp, _vp,
                                         _vp])
_proto("oracle_cuda_position_advance", [_vp, _vp, _vp])
_proto("oracle_cuda_split_query_gate", [_vp, _vp, _u32, _u32, _vp, _vp, _vp])
_proto("oracle_cuda_gate_sigmoid_mul", [_vp, _vp, _vp, _u64, _vp])
_proto("oracle_cuda_mul_silu", [_vp, _vp, _vp, _u64, _vp])
_proto("oracle_cuda_gdn_gates", [_vp, _vp, _vp, _vp, _vp, _u32, _vp, _vp, _vp])
_proto("oracle_cuda_token_commit", [_vp, _vp, _vp, _u32, _vp, _vp, _vp, _u32, _vp])
_proto("oracle_cuda_argmax_rows", [_vp, _vp, _u32, _u64, _vp, _vp])
_proto("oracle_cuda_token_commit_rows", [_vp, _vp, _u32, _vp, _u32, _vp, _vp, _vp, _u32, _vp])
_proto("oracle_cuda_gdn_core_seqs", [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _u32, _u32, _u32, _u32,
                                     C.c_float, _vp, _u32, _vp, _vp])
_proto("oracle_cuda_gdn_core", [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _u32, _u32, _u32, _u32,
                                C.c_float, _vp, _vp, _vp])
_proto("oracle_cuda_attention_prep_at", [_vp, _vp, _vp, _vp, _vp, _vp, C.c_float, _vp, _u64, _u32, _u32, _u32, _vp,
                                         _vp, _u64, _vp, _vp, _vp])
_proto("oracle_cuda_attention_core_at", [_vp, _vp, _vp, _vp, _u64, _vp, _u32, _u32, _u32, _u32, _vp, _u32, _vp, _vp,
                                         _vp])
_proto("oracle_cuda_swiglu", [_vp, _vp, _vp, _u64, _vp, _vp])
_proto("oracle_cuda_add", [_vp, _vp, _vp, _u64, _vp, _vp])
IPC_HANDLE_BYTES = 64
MAX_PEERS = 8


def argmax_decode(key: int) -> int:
    """oracle_cuda_argmax_decode: token id of an argmax key (raises like Oracle's sampler)."""
    t = _u32()
    _raise(_lib.oracle_cuda_argmax_decode(key, C.byref(t), None), None)
    return int(t.value)


class _CudaArray:
    """A raw device float32 array exposed through __cuda_array_interface__."""

    def __init__(self, ptr: int, n: int):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": "<f4", "data": (ptr, False), "version": 2}


class PeerGroup:
    """oracle_cuda_peer_group: this rank's gather buffer plus the mapped
    buffers of the other ranks (CUDA IPC), for row-sharded matvec programs
    whose outputs are all-gathered inside the kernel.  Publish ``handle`` to
    the other ranks, then :meth:`connect` with every rank's handle in rank
    order."""

    def __init__(self, ctx: "Context", rank: int, world: int, data_bytes: int):
        self._ctx = ctx
        self._h = C.c_void_p()
        buf = (C.c_ubyte * IPC_HANDLE_BYTES)()
        ctx._check(_lib.oracle_cuda_peer_group_create(ctx._h, rank, world, data_bytes, C.byref(self._h), buf))
        self.handle = bytes(buf)
        self.rank, self.world, self.data_bytes = rank, world, data_bytes
        p = C.c_void_p()
        ctx._check(_lib.oracle_cuda_peer_group_data(self._h, C.byref(p)))
        self.data_ptr = p.value

    def connect(self, handles) -> None:
        blob = b"".join(handles)
        if len(blob) != self.world * IPC_HANDLE_BYTES:
            raise InvalidArgument("one IPC handle per rank expected")
        self._ctx._check(_lib.oracle_cuda_peer_group_connect(self._h, blob))

    def tensor(self):
        """The gather data region as a float32 CUDA tensor (no copy)."""
        import torch
        return torch.as_tensor(_CudaArray(self.data_ptr, self.data_bytes // 4), device="cuda")

    def close(self) -> None:
        if self._h:
            _lib.oracle_cuda_peer_group_destroy(self._h)
            self._h = None


class OracleCudaError(Exception):
    """A non-OK status from the C ABI; ``status`` is the integer code."""

    status = -1
    reference_exception = "std::exception"

    def __init__(self, message: str, status: int | None = None):
        super().__init__(message)
        if status is not None:
            self.status = status


class InvalidArgument(OracleCudaError, ValueError):
    status, reference_exception = 1, "std::invalid_argument"


class OutOfRange(OracleCudaError, IndexError):
    status, reference_exception = 2, "std::out_of_range"


class Overflow(OracleCudaError, OverflowError):
    status, reference_exception = 3, "std::overflow_error"


class RuntimeError_(OracleCudaError, RuntimeError):
    status, reference_exception = 4, "std::runtime_error"


class LogicError(OracleCudaError):
    status, reference_exception = 5, "std::logic_error"


class CudaError(OracleCudaError):
    status = 6


class OutOfMemory(OracleCudaError, MemoryError):
    status = 7


class DeviceTimeout(OracleCudaError):
    status = 8


class Unsupported(OracleCudaError):
    status = 9


_ERRORS = {c.status: c for c in (InvalidArgument, OutOfRange, Overflow, RuntimeError_, LogicError,
                                 CudaError, OutOfMemory, DeviceTimeout, Unsupported)}


def _raise(status: int, ctx) -> None:
    if status == 0:
        return
    msg = _lib.oracle_cuda_last_error(ctx)
    msg = msg.decode() if msg else ""
    cls = _ERRORS.get(status, OracleCudaError)
    raise cls(msg, status)


def abi_version() -> int:
    return int(_lib.oracle_cuda_abi_version())


def type_layout(qtype: int):
    """(name, block_elements, bytes_per_block, quantized) or None for an unknown id."""
    be, bb, q, name = C.c_uint64(), C.c_uint64(), C.c_int(), C.c_char_p()
    st = _lib.oracle_ggml_type_layout(qtype, C.byref(be), C.byref(bb), C.byref(q), C.byref(name))
    if st:
        return None
    return name.value.decode(), be.value, bb.value, bool(q.value)


def row_byte_size(cols: int, qtype: int) -> int:
    out = C.c_uint64()
    _raise(_lib.oracle_ggml_row_byte_size(cols, qtype, C.byref(out)), None)
    return out.value


def _addr(t) -> int:
    """Device or host address of a torch tensor, numpy array or raw int."""
    if t is None:
        return 0
    if isinstance(t, int):
        return t
    if isinstance(t, np.ndarray):
        return t.ctypes.data
    return t.data_ptr()


def _nbytes(t) -> int:
    if isinstance(t, np.ndarray):
        return t.nbytes
    return t.numel() * t.element_size()


def _numel(t) -> int:
    return t.size if isinstance(t, np.ndarray) else t.numel()


def _stream(stream) -> int:
    if stream is None:
        try:
            import torch
            return torch.cuda.current_stream().cuda_stream
        except Exception:  # pragma: no cover - torch without CUDA
            return 0
    if isinstance(stream, int):
        return stream
    return stream.cuda_stream


class Weight:
    """A weight (or a row shard of one) resident in HBM."""

    def __init__(self, ctx: "Context", handle: int):
        self._ctx = ctx
        self._h = handle
        t, r, c, rb, dev, nb = C.c_uint32(), C.c_uint64(), C.c_uint64(), C.c_uint64(), C.c_void_p(), C.c_uint64()
        _raise(_lib.oracle_cuda_weight_info(handle, C.byref(t), C.byref(r), C.byref(c), C.byref(rb),
                                            C.byref(dev), C.byref(nb)), None)
        self.type, self.rows, self.cols = t.value, r.value, c.value
        self.row_begin, self.dev, self.nbytes = rb.value, dev.value, nb.value

    def free(self) -> None:
        if self._h:
            _lib.oracle_cuda_weight_free(self._h)
            self._h = 0

    def __del__(self):  # pragma: no cover - best effort
        try:
            self.free()
        except Exception:
            pass


class Context:
    """One library context on one CUDA device (oracle_cuda_create)."""

    def __init__(self, device: int = 0, flags: int = 0):
        h = C.c_void_p()
        _raise(_lib.oracle_cuda_create(device, C.byref(h)), None)
        self._h = h.value
        self.device = device
        self.flags = 0
        if flags:
            self.set_flags(flags)

    # -------------------------------------------------------------- lifecycle
    def close(self) -> None:
        if self._h:
            _lib.oracle_cuda_destroy(self._h)
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def _check(self, status: int) -> None:
        _raise(status, self._h)

    def set_flags(self, flags: int) -> None:
        self._check(_lib.oracle_cuda_set_flags(self._h, flags))
        self.flags = flags

    def device_status(self) -> None:
        """Raise DeviceTimeout if any kernel's bounded wait expired."""
        self._check(_lib.oracle_cuda_device_status(self._h))

    def selftest_bounded_wait(self, limit_ns: int) -> None:
        self._check(_lib.oracle_cuda_selftest_bounded_wait(self._h, limit_ns))

    def launch_count(self) -> int:
        return int(_lib.oracle_cuda_launch_count(self._h))

    # -------------------------------------------------------------- device-pointer path
    def decode_rows(self, qtype, rows, cols, w, out, stream=None) -> None:
        self._check(_lib.oracle_cuda_decode_rows(self._h, qtype, rows, cols, _addr(w), _nbytes(w), _addr(out),
                                                 _numel(out), _stream(stream)))

    def quantize_q8_k(self, x, cols, batch, q8k, stream=None) -> None:
        self._check(_lib.oracle_cuda_quantize_q8_k(self._h, _addr(x), cols, batch, _addr(q8k), _nbytes(q8k),
                                                   _stream(stream)))

    def storage_matvec(self, contract, qtype, rows, cols, w, x, y, stream=None, w_nbytes=None) -> None:
        self._check(_lib.oracle_cuda_storage_matvec(
            self._h, contract, qtype, rows, cols, _addr(w), _nbytes(w) if w_nbytes is None else w_nbytes,
            _addr(x), _numel(x), _addr(y), _numel(y), _stream(stream)))

    @staticmethod
    def batch_image_bytes(cols: int) -> int:
        """oracle_cuda_batch_image_bytes: size of the batch image of cols-wide vectors."""
        return int(_lib.oracle_cuda_batch_image_bytes(cols))

    def batch_quantize(self, x, cols, batch, image, stream=None) -> None:
        """oracle_cuda_batch_quantize: x[batch][cols] (device f32) -> batch image (device uint8)."""
        self._check(_lib.oracle_cuda_batch_quantize(self._h, _addr(x), cols, batch, _addr(image), _nbytes(image),
                                                    _stream(stream)))

    def batch_norm_quantize(self, a, b, sum_out, weight, eps, cols, batch, image, stream=None) -> None:
        """oracle_cuda_batch_norm_quantize: rms_norm(a (+ b)) into a batch image; the
        sum a + b is also written to sum_out when given."""
        self._check(_lib.oracle_cuda_batch_norm_quantize(self._h, _addr(a), _addr(b), _addr(sum_out), _addr(weight),
                                                         eps, cols, batch, _addr(image), _nbytes(image),
                                                         _stream(stream)))

    def batch_matvec(self, qtype, rows, cols, w, image, batch, y, stream=None, w_nbytes=None) -> None:
        """oracle_cuda_batch_matvec: y[b][rows] = W (q4_K / q6_K) x vector b of a batch image."""
        self._check(_lib.oracle_cuda_batch_matvec(self._h, qtype, rows, cols, _addr(w),
                                                  _nbytes(w) if w_nbytes is None else w_nbytes, _addr(image),
                                                  _nbytes(image), batch, _addr(y), _numel(y), _stream(stream)))

    def matvec_q8k_prequantized(self, qtype, rows, cols, w, q8k, y, stream=None) -> None:
        self._check(_lib.oracle_cuda_matvec_q8k_prequantized(
            self._h, qtype, rows, cols, _addr(w), _nbytes(w), _addr(q8k), _nbytes(q8k), _addr(y), _numel(y),
            _stream(stream)))

    def matvec_program(self, ops, stream=None) -> None:
        """ops: sequence of (qtype, rows, cols, w, x, y, after_previous) with
        device tensors (or addresses); one persistent launch (Q8_K contract)."""
        arr = (MatvecOp * len(ops))()
        for i, (qtype, rows, cols, w, x, y, after) in enumerate(ops):
            arr[i] = MatvecOp(qtype, 1 if after else 0, rows, cols, _addr(w), _nbytes(w), _addr(x), _addr(y))
        self._check(_lib.oracle_cuda_matvec_program(self._h, arr, len(ops), _stream(stream)))

    @staticmethod
    def _ops_ex(ops):
        arr = (MatvecOpEx * len(ops))()
        for i, o in enumerate(ops):
            arr[i].base = MatvecOp(o["qtype"], 1 if o.get("after") else 0, o["rows"], o["cols"], _addr(o["w"]),
                                   _nbytes(o["w"]), _addr(o["x"]), _addr(o["y"]))
            arr[i].xform = o.get("xform", XFORM_NONE)
            arr[i].eps = o.get("eps", 0.0)
            arr[i].x2_dev = _addr(o.get("x2"))
            arr[i].norm_dev = _addr(o.get("norm"))
            arr[i].residual_dev = _addr(o.get("residual"))
            arr[i].act_dev = _addr(o.get("act"))
        return arr

    def matvec_program_ex_allgather(self, group: "PeerGroup", ops, stream=None) -> None:
        """oracle_cuda_matvec_program_ex_allgather: ops as for matvec_program_ex,
        rows this rank's shard, outputs inside the group's gather buffer."""
        self._check(_lib.oracle_cuda_matvec_program_ex_allgather(self._h, group._h, self._ops_ex(ops), len(ops),
                                                                 _stream(stream)))

    def matvec_program_sharded(self, group: "PeerGroup", ops, first_dep: int, deps_per_step: int,
                               end_of_step: bool = False, tail_wait: bool = False, stream=None) -> None:
        """oracle_cuda_matvec_program_sharded: ops as for matvec_program_ex plus
        push (bool), wait (0-3), announce (bool), segments and combined
        (combine ops) and swiglu_gate (epilogue, into act); xform
        XFORM_COMBINE_RMS takes the residual as x and the partial sums as x2."""
        ex = self._ops_ex(ops)
        arr = (ShardedOp * len(ops))()
        for i, o in enumerate(ops):
            arr[i].ex = ex[i]
            arr[i].push = 1 if o.get("push") else 0
            arr[i].wait = int(o.get("wait", 0))
            arr[i].announce = 1 if o.get("announce") else 0
            arr[i].segments = int(o.get("segments", 0))
            arr[i].swiglu_gate = _addr(o.get("swiglu_gate"))
            arr[i].combined_dev = _addr(o.get("combined"))
        st = ShardedStep(first_dep, deps_per_step, 1 if end_of_step else 0, 1 if tail_wait else 0)
        self._check(_lib.oracle_cuda_matvec_program_sharded(self._h, group._h, arr, len(ops), C.byref(st),
                                                            _stream(stream)))

    def set_program_trace(self, trace, records: int) -> None:
        """oracle_cuda_set_program_trace: trace = int64 CUDA tensor of at least
        1 + records * TRACE_WORDS words (word 0 zero), or None / records 0 to stop."""
        if records and (trace is None or trace.numel() < 1 + records * TRACE_WORDS):
            raise InvalidArgument("trace buffer too small")
        self._check(_lib.oracle_cuda_set_program_trace(self._h, _addr(trace), records))

    def matvec_program_ex(self, ops, stream=None) -> None:
        """ops: sequence of dicts with keys qtype, rows, cols, w, x, y and
        optional after (bool), xform (XFORM_*), eps, x2, norm, residual, act."""
        self._check(_lib.oracle_cuda_matvec_program_ex(self._h, self._ops_ex(ops), len(ops), _stream(stream)))

    def gather_rows(self, qtype, rows, cols, w, ids, out, stream=None, w_nbytes=None) -> None:
        """oracle_cuda_gather_rows: out[t] = decode(row ids[t]) (device uint32 ids, f32 out)."""
        self._check(_lib.oracle_cuda_gather_rows(self._h, qtype, rows, cols, _addr(w),
                                                 _nbytes(w) if w_nbytes is None else w_nbytes, _addr(ids),
                                                 _numel(ids), _addr(out), _stream(stream)))

    def argmax(self, x, key, index_base=0, stream=None) -> None:
        """oracle_cuda_argmax: the argmax key of device f32 x into device key (uint64 / int64 tensor)."""
        self._check(_lib.oracle_cuda_argmax(self._h, _addr(x), _numel(x), index_base, _addr(key), _stream(stream)))

    def greedy_token(self, logits) -> int:
        """oracle_cuda_greedy_token: Oracle's greedy sampler on device logits."""
        t = _u32()
        self._check(_lib.oracle_cuda_greedy_token(self._h, _addr(logits), _numel(logits), C.byref(t)))
        return int(t.value)

    # -------------------------------------------------------------- decoder glue
    def rms_norm_rows(self, x, weight, rows, width, eps, out, stream=None) -> None:
        self._check(_lib.oracle_cuda_rms_norm_rows(self._h, _addr(x), _addr(weight), rows, width, eps, _addr(out),
                                                   _stream(stream)))

    def rope(self, heads, n_heads, head_dim, rotary_dim, sections, base, position, stream=None) -> None:
        sec = (C.c_int32 * 4)(*sections)
        pt, ph, pw = position
        self._check(_lib.oracle_cuda_rope(self._h, _addr(heads), n_heads, head_dim, rotary_dim, sec, base, pt, ph, pw,
                                          _stream(stream)))

    def attention_step(self, q, k_new, v_new, keys, values, capacity, length, q_heads, kv_heads, key_dim, value_dim,
                       scores, out, stream=None) -> None:
        self._check(_lib.oracle_cuda_attention_step(self._h, _addr(q), _addr(k_new), _addr(v_new), _addr(keys),
                                                    _addr(values), capacity, length, q_heads, kv_heads, key_dim,
                                                    value_dim, _addr(scores), _addr(out), _stream(stream)))

    def conv_step(self, x, weights, history, channels, kernel, apply_silu, out, stream=None) -> None:
        self._check(_lib.oracle_cuda_conv_step(self._h, _addr(x), _addr(weights), _addr(history), channels, kernel,
                                               1 if apply_silu else 0, _addr(out), _stream(stream)))

    def gated_delta_step(self, q, k, v, beta, log_decay, state, heads, key_dim, value_dim, eps, out,
                         stream=None, qk_heads=None) -> None:
        """oracle_cuda_gated_delta_step; q and k hold qk_heads rows (default: heads)."""
        self._check(_lib.oracle_cuda_gated_delta_step(self._h, _addr(q), _addr(k), _addr(v), _addr(beta),
                                                      _addr(log_decay), _addr(state), heads,
                                                      heads if qk_heads is None else qk_heads, key_dim, value_dim,
                                                      eps, _addr(out), _stream(stream)))

    # -------------------------------------------------------------- graph-replayable step
    def rope_table(self, rotary_dim, sections, base, positions, table) -> None:
        sec = (C.c_int32 * 4)(*sections)
        self._check(_lib.oracle_cuda_rope_table(self._h, rotary_dim, sec, base, positions, _addr(table)))

    def rope_at(self, heads, n_heads, head_dim, rotary_dim, table, positions, pos, stream=None) -> None:
        self._check(_lib.oracle_cuda_rope_at(self._h, _addr(heads), n_heads, head_dim, rotary_dim, _addr(table),
                                             positions, _addr(pos), _stream(stream)))

    def attention_step_at(self, q, k_new, v_new, keys, values, capacity, pos, q_heads, kv_heads, key_dim, value_dim,
                          scores, out, stream=None) -> None:
        self._check(_lib.oracle_cuda_attention_step_at(self._h, _addr(q), _addr(k_new), _addr(v_new), _addr(keys),
                                                       _addr(values), capacity, _addr(pos), q_heads, kv_heads,
                                                       key_dim, value_dim, _addr(scores), _addr(out),
                                                       _stream(stream)))

    def position_advance(self, pos, stream=None) -> None:
        self._check(_lib.oracle_cuda_position_advance(self._h, _addr(pos), _stream(stream)))

    def split_query_gate(self, full, heads, width, query, gate, stream=None) -> None:
        self._check(_lib.oracle_cuda_split_query_gate(self._h, _addr(full), heads, width, _addr(query), _addr(gate),
                                                      _stream(stream)))

    def gate_sigmoid_mul(self, x, gate, n, stream=None) -> None:
        self._check(_lib.oracle_cuda_gate_sigmoid_mul(self._h, _addr(x), _addr(gate), n, _stream(stream)))

    def mul_silu(self, x, z, n, stream=None) -> None:
        self._check(_lib.oracle_cuda_mul_silu(self._h, _addr(x), _addr(z), n, _stream(stream)))

    def token_commit(self, key, prompt, n_prompt, pos, next_id, tokens, tokens_capacity, stream=None) -> None:
        self._check(_lib.oracle_cuda_token_commit(self._h, _addr(key), _addr(prompt), n_prompt, _addr(pos),
                                                  _addr(next_id), _addr(tokens), tokens_capacity, _stream(stream)))

    def argmax_rows(self, x, rows, n, keys, stream=None) -> None:
        """oracle_cuda_argmax_rows: keys[b] = argmax key of logits row x[b][n]."""
        self._check(_lib.oracle_cuda_argmax_rows(self._h, _addr(x), rows, n, _addr(keys), _stream(stream)))

    def token_commit_rows(self, keys, rows, prompt, n_prompt, pos, next_id, tokens, tokens_capacity,
                          stream=None) -> None:
        self._check(_lib.oracle_cuda_token_commit_rows(self._h, _addr(keys), rows, _addr(prompt), n_prompt,
                                                       _addr(pos), _addr(next_id), _addr(tokens), tokens_capacity,
                                                       _stream(stream)))

    def gdn_core_seqs(self, qkv, z, beta, alpha, time_step_bias, decay, conv_weights, history, state, norm,
                      key_heads, value_heads, head_dim, conv_kernel, eps, pos, seqs, out, stream=None) -> None:
        self._check(_lib.oracle_cuda_gdn_core_seqs(self._h, _addr(qkv), _addr(z), _addr(beta), _addr(alpha),
                                                   _addr(time_step_bias), _addr(decay), _addr(conv_weights),
                                                   _addr(history), _addr(state), _addr(norm), key_heads,
                                                   value_heads, head_dim, conv_kernel, eps, _addr(pos), seqs,
                                                   _addr(out), _stream(stream)))

    def gdn_core(self, qkv, z, beta, alpha, time_step_bias, decay, conv_weights, history, state, norm, key_heads,
                 value_heads, head_dim, conv_kernel, eps, pos, out, stream=None) -> None:
        self._check(_lib.oracle_cuda_gdn_core(self._h, _addr(qkv), _addr(z), _addr(beta), _addr(alpha),
                                              _addr(time_step_bias), _addr(decay), _addr(conv_weights),
                                              _addr(history), _addr(state), _addr(norm), key_heads, value_heads,
                                              head_dim, conv_kernel, eps, _addr(pos), _addr(out), _stream(stream)))

    def attention_prep_at(self, q_full, k, v, q_norm, k_norm, eps, table, rotary_dim, q_heads, kv_heads, head_dim,
                          keys, values, capacity, pos, q_out, stream=None) -> None:
        self._check(_lib.oracle_cuda_attention_prep_at(self._h, _addr(q_full), _addr(k), _addr(v), _addr(q_norm),
                                                       _addr(k_norm), eps, _addr(table), rotary_dim, q_heads,
                                                       kv_heads, head_dim, _addr(keys), _addr(values), capacity,
                                                       _addr(pos), _addr(q_out), _stream(stream)))

    def attention_core_at(self, q, keys, values, capacity, pos, q_heads, kv_heads, key_dim, value_dim, gate,
                          gate_stride, scores, out, stream=None) -> None:
        self._check(_lib.oracle_cuda_attention_core_at(self._h, _addr(q), _addr(keys), _addr(values), capacity,
                                                       _addr(pos), q_heads, kv_heads, key_dim, value_dim, _addr(gate),
                                                       gate_stride, _addr(scores), _addr(out), _stream(stream)))

    def gdn_gates(self, beta, alpha, time_step_bias, decay, heads, beta_out, log_decay, stream=None) -> None:
        self._check(_lib.oracle_cuda_gdn_gates(self._h, _addr(beta), _addr(alpha), _addr(time_step_bias),
                                               _addr(decay), heads, _addr(beta_out), _addr(log_decay),
                                               _stream(stream)))

    def swiglu(self, gate, up, n, out, stream=None) -> None:
        self._check(_lib.oracle_cuda_swiglu(self._h, _addr(gate), _addr(up), n, _addr(out), _stream(stream)))

    def add(self, a, b, n, out, stream=None) -> None:
        self._check(_lib.oracle_cuda_add(self._h, _addr(a), _addr(b), n, _addr(out), _stream(stream)))

    def matvec_program_allgather(self, group: "PeerGroup", ops, stream=None) -> None:
        """oracle_cuda_matvec_program_allgather: the program on this rank's
        rows, every output row also stored into every peer's gather buffer;
        ops as for :meth:`matvec_program`, y inside the group's data region."""
        arr = _matvec_ops(ops)
        self._check(_lib.oracle_cuda_matvec_program_allgather(self._h, group._h, arr, len(ops), _stream(stream)))

    def prefill_gemm(self, qtype, rows, cols, w, x, m, y, stream=None, w_nbytes=None) -> None:
        """oracle_cuda_prefill_gemm: y[m][n] = sum_k x[m][k] * W[n][k] on the
        tensor cores (bf16 operands, f32 accumulation); x is m x cols f32,
        y is m x rows f32, all device memory."""
        self._check(_lib.oracle_cuda_prefill_gemm(
            self._h, qtype, rows, cols, _addr(w), _nbytes(w) if w_nbytes is None else w_nbytes, _addr(x), m,
            _addr(y), _stream(stream)))

    # -------------------------------------------------------------- resident weights
    def upload(self, qtype, rows, cols, host: np.ndarray, row_begin=0, row_end=None) -> Weight:
        host = np.ascontiguousarray(host, np.uint8)
        h = C.c_void_p()
        self._check(_lib.oracle_cuda_weight_upload(self._h, qtype, rows, cols, host.ctypes.data, host.nbytes,
                                                   row_begin, rows if row_end is None else row_end, C.byref(h)))
        return Weight(self, h.value)

    def matvec_weight(self, contract, weight: Weight, x, y, stream=None) -> None:
        self.storage_matvec(contract, weight.type, weight.rows, weight.cols, weight.dev, x, y, stream,
                            w_nbytes=weight.nbytes)

    # -------------------------------------------------------------- host drop-ins
    def host_storage_matvec(self, contract, qtype, rows, cols, w: np.ndarray, x: np.ndarray,
                            y: np.ndarray | None = None) -> np.ndarray:
        w = np.ascontiguousarray(w, np.uint8)
        x = np.ascontiguousarray(x, np.float32)
        batch = max(1, x.size // cols) if cols else 1
        if y is None:
            y = np.empty(rows * batch, np.float32)
        self._check(_lib.oracle_cuda_host_storage_matvec(self._h, contract, qtype, rows, cols, w.ctypes.data,
                                                         w.nbytes, x.ctypes.data, x.size, y.ctypes.data, y.size))
        return y

    def host_storage_dot(self, contract, qtype, cols, row: np.ndarray, x: np.ndarray) -> float:
        row = np.ascontiguousarray(row, np.uint8)
        x = np.ascontiguousarray(x, np.float32)
        out = C.c_float()
        self._check(_lib.oracle_cuda_host_storage_dot(self._h, contract, qtype, cols, row.ctypes.data, row.nbytes,
                                                      x.ctypes.data, x.size, C.byref(out)))
        return out.value

    def host_decode_rows(self, qtype, rows, cols, w: np.ndarray, out: np.ndarray | None = None) -> np.ndarray:
        w = np.ascontiguousarray(w, np.uint8)
        if out is None:
            out = np.empty(rows * cols, np.float32)
        self._check(_lib.oracle_cuda_host_decode_rows(self._h, qtype, rows, cols, w.ctypes.data, w.nbytes,
                                                      out.ctypes.data, out.size))
        return out

    def evict_resident(self) -> None:
        """oracle_cuda_evict_resident: unregister every registered weight span."""
        self._check(_lib.oracle_cuda_evict_resident(self._h))

    def register_host_weight(self, qtype, rows, cols, w: np.ndarray) -> None:
        """oracle_cuda_register_host_weight: the bytes of ``w`` (which must not
        change while registered) become resident; host calls given the same
        array then read the resident copy."""
        if not (w.flags.c_contiguous and w.dtype == np.uint8):
            raise InvalidArgument("register a C-contiguous uint8 array (the host calls must see the same address)")
        self._check(_lib.oracle_cuda_register_host_weight(self._h, qtype, rows, cols, w.ctypes.data, w.nbytes))

    def unregister_host_weight(self, w: np.ndarray) -> None:
        self._check(_lib.oracle_cuda_unregister_host_weight(self._h, w.ctypes.data, w.nbytes))

    def host_matvec_program(self, ops) -> None:
        """oracle_cuda_host_matvec_program: ops = [(qtype, rows, cols, w, x, y)]
        with host numpy arrays (uint8 weights, f32 x and y); an op whose x is
        an earlier op's y (the same array) reads that result on the device.
        One launch, one synchronize; y arrays are filled in place."""
        self.host_program(ops)()

    def prepare_host_program(self, ops) -> "PreparedHostProgram":
        """oracle_cuda_host_program_create: the op list of
        :meth:`host_matvec_program` planned and captured once (every weight
        registered); call the result to run it on the arrays' contents."""
        return PreparedHostProgram(self, ops)

    def host_program(self, ops) -> "HostProgram":
        """The op list of :meth:`host_matvec_program` marshalled once; calling
        the result runs oracle_cuda_host_matvec_program on the arrays' current
        contents (a caller that repeats a step pays only the C call)."""
        return HostProgram(self, ops)


def _host_ops(ops):
    arr = (HostMatvecOp * len(ops))()
    for i, (qtype, rows, cols, w, x, y) in enumerate(ops):
        for a, dt in ((w, np.uint8), (x, np.float32), (y, np.float32)):
            if not (a.flags.c_contiguous and a.dtype == dt):
                raise InvalidArgument(f"op {i}: host arrays must be C-contiguous {np.dtype(dt).name}")
        arr[i] = HostMatvecOp(qtype, rows, cols, w.ctypes.data, w.nbytes, x.ctypes.data, y.ctypes.data)
    return arr


class HostProgram:
    """An oracle_cuda_host_matvec_program op list marshalled once (see
    :meth:`Context.host_program`).  Keeps the arrays alive."""

    def __init__(self, ctx: "Context", ops):
        self._ctx = ctx
        self._keep = list(ops)
        self._arr = _host_ops(ops)
        self._n = len(ops)
        self._fn = _lib.oracle_cuda_host_matvec_program

    def __call__(self) -> None:
        self._ctx._check(self._fn(self._ctx._h, self._arr, self._n))


class PreparedHostProgram:
    """oracle_cuda_host_program_create / _run / _destroy: the host program
    planned and captured once (every weight registered); each call copies
    the arrays' current x in and y out around one graph replay."""

    def __init__(self, ctx: "Context", ops):
        self._ctx = ctx
        self._keep = list(ops)
        arr = _host_ops(ops)
        h = C.c_void_p()
        ctx._check(_lib.oracle_cuda_host_program_create(ctx._h, arr, len(ops), C.byref(h)))
        self._h = h.value
        self._run = _lib.oracle_cuda_host_program_run

    def __call__(self) -> None:
        self._ctx._check(self._run(self._h))

    def close(self) -> None:
        if self._h:
            _lib.oracle_cuda_host_program_destroy(self._h)
            self._h = None

    def __del__(self):  # pragma: no cover - best effort
        try:
            self.close()
        except Exception:
            pass
