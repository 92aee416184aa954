"""CPU checkers for the quantized-weight path -- TEST INFRASTRUCTURE ONLY.

Two libraries, loaded with ctypes:

* ``port`` -- ``liboracle_port.so``, the C restatement in ``quant_oracle.c``
  (Oracle's decoders and f32 contract, plus GGML's Q8_K quantizer and integer
  dots restated; provenance in ``quant_oracle.h``).
* ``ref``  -- ``_ref/liboracle_ref.so``, the reference's own hot-path sources
  compiled unmodified (``Makefile``), reached through ``ref_shim.cpp``.
* ``Qwen35Reference`` -- the reference's own Qwen3.5 decode step and greedy
  loop (``ref_qwen35.cpp``), from ``liboracle_ref.so`` (Oracle's f32 contract)
  or ``_ref/liboracle_ref_q8k.so`` (the same sources with GGML's Q8_K
  contract for Q4_K/Q6_K projections, ``ref_q8k_projection.cpp``).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
and reference legs may import this package.  The product library never does.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
PORT_PATH = os.path.join(HERE, "liboracle_port.so")
REF_PATH = os.path.join(HERE, "_ref", "liboracle_ref.so")
REF_Q8K_PATH = os.path.join(HERE, "_ref", "liboracle_ref_q8k.so")
REF_GATE_PATH = os.path.join(HERE, "_ref", "liboracle_ref_gate.so")
# Oracle's source tree, for (re)building the reference checker; no default.
REFERENCE_TREE = os.environ.get("ORACLE_REFERENCE_TREE", "")

TYPE_F32, TYPE_F16, TYPE_Q8_0, TYPE_Q4_K, TYPE_Q5_K, TYPE_Q6_K, TYPE_Q8_K, TYPE_BF16 = (
    0, 1, 8, 12, 13, 14, 15, 30)
Q8K_BLOCK_BYTES = 292

_u8p = C.POINTER(C.c_uint8)
_f32p = C.POINTER(C.c_float)
_f64p = C.POINTER(C.c_double)
_u64p = C.POINTER(C.c_uint64)


def build(reference_tree: str | None = REFERENCE_TREE) -> None:
    """Compile the restatement, and the reference checker when its tree exists."""
    targets = ["port"]
    if reference_tree and os.path.isdir(reference_tree):
        targets += ["ref", "ref_q8k", "ref_gate"]
    subprocess.run(["make", "-s", "-C", HERE, f"REF={reference_tree or ''}", *targets], check=True)


def _ptr(a: np.ndarray, t):
    return a.ctypes.data_as(t)


class _Port:
    def __init__(self, path: str = PORT_PATH):
        if not os.path.exists(path):
            build()
        lib = C.CDLL(path)
        lib.oq_f16_to_f32.argtypes = [C.c_uint16]
        lib.oq_f16_to_f32.restype = C.c_float
        lib.oq_bf16_to_f32.argtypes = [C.c_uint16]
        lib.oq_bf16_to_f32.restype = C.c_float
        lib.oq_f32_to_bf16_rne.argtypes = [C.c_float]
        lib.oq_f32_to_bf16_rne.restype = C.c_uint16
        lib.oq_row_bytes.argtypes = [C.c_uint32, C.c_uint64]
        lib.oq_row_bytes.restype = C.c_uint64
        lib.oq_decode_row.argtypes = [C.c_uint32, C.c_uint64, _u8p, _f32p]
        lib.oq_quantize_row_q8_k.argtypes = [_f32p, C.c_uint64, _u8p]
        lib.oq_block_sums_q4_k.argtypes = [_u8p, _u8p, C.POINTER(C.c_int32), C.POINTER(C.c_int32)]
        lib.oq_block_sums_q6_k.argtypes = [_u8p, _u8p, C.POINTER(C.c_int32), C.POINTER(C.c_int32)]
        lib.oq_vec_dot_q8_k.argtypes = [C.c_uint32, C.c_uint64, _u8p, _u8p]
        lib.oq_vec_dot_q8_k.restype = C.c_float
        lib.oq_vec_dot_q8_k_ggml_order.argtypes = [C.c_uint32, C.c_uint64, _u8p, _u8p]
        lib.oq_vec_dot_q8_k_ggml_order.restype = C.c_float
        lib.oq_matvec_q8_k.argtypes = [C.c_uint32, C.c_uint64, C.c_uint64, _u8p, _u8p,
                                       C.c_uint64, _f32p]
        lib.oq_storage_dot_f32.argtypes = [C.c_uint32, C.c_uint64, _u8p, _f32p]
        lib.oq_storage_dot_f32.restype = C.c_float
        lib.oq_storage_matvec_f32.argtypes = [C.c_uint32, C.c_uint64, C.c_uint64, _u8p, _f32p,
                                              C.c_uint64, _f32p]
        lib.oq_storage_matvec_f64.argtypes = [C.c_uint32, C.c_uint64, C.c_uint64, _u8p, _f32p,
                                              C.c_uint64, _f64p]
        lib.oq_gemm_sampled.argtypes = [C.c_uint32, C.c_uint64, C.c_uint64, _u8p, C.c_uint64,
                                        _f32p, C.c_uint64, _u64p, _u64p, C.c_int, _f64p]
        lib.oq_rms_norm_rows.argtypes = [_f32p, _f32p, C.c_uint64, C.c_uint64, C.c_float, _f32p]
        lib.oq_swiglu.argtypes = [_f32p, _f32p, C.c_uint64, _f32p]
        lib.oq_swiglu.restype = None
        self.lib = lib

    def row_bytes(self, qtype: int, k: int) -> int:
        return int(self.lib.oq_row_bytes(qtype, k))

    def f16_to_f32(self, bits: int) -> float:
        return float(self.lib.oq_f16_to_f32(bits))

    def decode_rows(self, qtype: int, rows: int, k: int, w: np.ndarray) -> np.ndarray:
        w = np.ascontiguousarray(w, dtype=np.uint8).reshape(-1)
        rb = self.row_bytes(qtype, k)
        out = np.empty((rows, k), np.float32)
        for r in range(rows):
            seg = w[r * rb:(r + 1) * rb]
            rc = self.lib.oq_decode_row(qtype, k, _ptr(seg, _u8p), _ptr(out[r], _f32p))
            if rc:
                raise ValueError(f"oq_decode_row failed with {rc}")
        return out

    def quantize_q8_k(self, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        if x.ndim == 1:
            x = x[None]
        batch, k = x.shape
        out = np.empty((batch, (k // 256) * Q8K_BLOCK_BYTES), np.uint8)
        for b in range(batch):
            if self.lib.oq_quantize_row_q8_k(_ptr(x[b], _f32p), k, _ptr(out[b], _u8p)):
                raise ValueError("k must be a positive multiple of 256")
        return out

    def block_sums(self, qtype: int, wblock: np.ndarray, q8block: np.ndarray):
        i, m = C.c_int32(), C.c_int32()
        wb = np.ascontiguousarray(wblock, np.uint8)
        qb = np.ascontiguousarray(q8block, np.uint8)
        fn = self.lib.oq_block_sums_q4_k if qtype == TYPE_Q4_K else self.lib.oq_block_sums_q6_k
        fn(_ptr(wb, _u8p), _ptr(qb, _u8p), C.byref(i), C.byref(m))
        return i.value, m.value

    def matvec_q8_k(self, qtype: int, rows: int, k: int, w: np.ndarray, q8k: np.ndarray) -> np.ndarray:
        w = np.ascontiguousarray(w, np.uint8).reshape(-1)
        q8k = np.ascontiguousarray(q8k, np.uint8)
        batch = q8k.size // ((k // 256) * Q8K_BLOCK_BYTES)
        y = np.empty((batch, rows), np.float32)
        rc = self.lib.oq_matvec_q8_k(qtype, rows, k, _ptr(w, _u8p), _ptr(q8k, _u8p), batch,
                                     _ptr(y, _f32p))
        if rc:
            raise ValueError(f"oq_matvec_q8_k failed with {rc}")
        return y

    def vec_dot_q8_k_ggml_order(self, qtype: int, k: int, wrow: np.ndarray, q8row: np.ndarray) -> float:
        wr = np.ascontiguousarray(wrow, np.uint8)
        qr = np.ascontiguousarray(q8row, np.uint8)
        return float(self.lib.oq_vec_dot_q8_k_ggml_order(qtype, k, _ptr(wr, _u8p), _ptr(qr, _u8p)))

    def storage_matvec_f32(self, qtype: int, rows: int, k: int, w: np.ndarray, x: np.ndarray) -> np.ndarray:
        w = np.ascontiguousarray(w, np.uint8).reshape(-1)
        x = np.ascontiguousarray(x, np.float32)
        batch = x.size // k
        y = np.empty((batch, rows), np.float32)
        rc = self.lib.oq_storage_matvec_f32(qtype, rows, k, _ptr(w, _u8p), _ptr(x, _f32p), batch,
                                            _ptr(y, _f32p))
        if rc:
            raise ValueError(f"oq_storage_matvec_f32 failed with {rc}")
        return y

    def storage_matvec_f64(self, qtype: int, rows: int, k: int, w: np.ndarray, x: np.ndarray) -> np.ndarray:
        w = np.ascontiguousarray(w, np.uint8).reshape(-1)
        x = np.ascontiguousarray(x, np.float32)
        batch = x.size // k
        y = np.empty((batch, rows), np.float64)
        rc = self.lib.oq_storage_matvec_f64(qtype, rows, k, _ptr(w, _u8p), _ptr(x, _f32p), batch,
                                            _ptr(y, _f64p))
        if rc:
            raise ValueError(f"oq_storage_matvec_f64 failed with {rc}")
        return y

    def gemm_sampled(self, qtype: int, n: int, k: int, w: np.ndarray, x: np.ndarray,
                     m_index: np.ndarray, n_index: np.ndarray, mode: int) -> np.ndarray:
        w = np.ascontiguousarray(w, np.uint8).reshape(-1)
        x = np.ascontiguousarray(x, np.float32)
        m = x.size // k
        order = np.lexsort((m_index, n_index))  # group by weight row for decode reuse
        mi = np.ascontiguousarray(np.asarray(m_index, np.uint64)[order])
        ni = np.ascontiguousarray(np.asarray(n_index, np.uint64)[order])
        y = np.empty(len(mi), np.float64)
        rc = self.lib.oq_gemm_sampled(qtype, n, k, _ptr(w, _u8p), m, _ptr(x, _f32p), len(mi),
                                      _ptr(mi, _u64p), _ptr(ni, _u64p), mode, _ptr(y, _f64p))
        if rc:
            raise ValueError(f"oq_gemm_sampled failed with {rc}")
        out = np.empty_like(y)
        out[order] = y
        return out


    def rms_norm_rows(self, x: np.ndarray, weight: np.ndarray, eps: float) -> np.ndarray:
        """Oracle's rms_norm_rows (qwen35_block.cpp:161-188); x is rows x width."""
        x = np.ascontiguousarray(x, np.float32)
        w = np.ascontiguousarray(weight, np.float32).reshape(-1)
        out = np.empty_like(x)
        rc = self.lib.oq_rms_norm_rows(_ptr(x, _f32p), _ptr(w, _f32p), x.size // w.size, w.size, eps, _ptr(out, _f32p))
        if rc:
            raise ValueError(f"oq_rms_norm_rows failed with {rc}")
        return out

    def swiglu(self, gate: np.ndarray, up: np.ndarray) -> np.ndarray:
        """silu(gate) * up as Oracle's FFN computes it (qwen35_block.cpp:315-318)."""
        g = np.ascontiguousarray(gate, np.float32).reshape(-1)
        u = np.ascontiguousarray(up, np.float32).reshape(-1)
        out = np.empty_like(g)
        self.lib.oq_swiglu(_ptr(g, _f32p), _ptr(u, _f32p), g.size, _ptr(out, _f32p))
        return out


class ReferenceError_(Exception):
    """An exception the reference raised, carried across the C shim."""

    KINDS = {1: "invalid_argument", 2: "out_of_range", 3: "overflow_error",
             4: "runtime_error", 5: "logic_error", 9: "exception"}

    def __init__(self, code: int, message: str):
        super().__init__(f"{self.KINDS.get(code, code)}: {message}")
        self.code = code
        self.kind = self.KINDS.get(code, str(code))
        self.message = message


class _Ref:
    def __init__(self, path: str = REF_PATH):
        if not os.path.exists(path):
            build()
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} is not built and the reference tree is absent")
        lib = C.CDLL(path)
        cp, sz = C.c_char_p, C.c_size_t
        lib.oref_f16_to_f32.argtypes = [C.c_uint16]
        lib.oref_f16_to_f32.restype = C.c_float
        lib.oref_bf16_to_f32.argtypes = [C.c_uint16]
        lib.oref_bf16_to_f32.restype = C.c_float
        lib.oref_type_layout.argtypes = [C.c_uint32, _u64p, _u64p, C.POINTER(C.c_int), cp, sz]
        lib.oref_row_byte_size.argtypes = [C.c_uint64, C.c_uint32, _u64p, cp, sz]
        lib.oref_decode_row.argtypes = [C.c_uint32, C.c_uint64, C.c_void_p, C.c_uint64, _f32p,
                                        C.c_uint64, cp, sz]
        lib.oref_storage_dot.argtypes = [C.c_uint32, C.c_uint64, C.c_void_p, C.c_uint64, _f32p,
                                         C.c_uint64, _f32p, cp, sz]
        lib.oref_storage_matvec.argtypes = [C.c_uint32, C.c_uint64, C.c_uint64, C.c_void_p,
                                            C.c_uint64, _f32p, C.c_uint64, _f32p, C.c_uint64, cp, sz]
        lib.oref_mapped_tensor_matvec.argtypes = [C.c_uint32, _u64p, C.c_uint64, C.c_void_p,
                                                  C.c_uint64, _f32p, C.c_uint64, _f32p,
                                                  C.c_uint64, cp, sz]
        lib.oref_decode_mapped_tensor.argtypes = [C.c_uint32, _u64p, C.c_uint64, C.c_void_p,
                                                  C.c_uint64, _f32p, C.c_uint64, cp, sz]
        lib.oref_greedy_token.argtypes = [_f32p, C.c_uint64, C.POINTER(C.c_uint32), cp, sz]
        u64 = C.c_uint64
        lib.oref_rope.argtypes = [_f32p, u64, u64, u64, C.POINTER(C.c_int32), C.c_float, u64, u64, u64, cp, sz]
        lib.oref_attention_step.argtypes = [_f32p, _f32p, _f32p, _f32p, _f32p, u64, u64, u64, u64, u64, u64, _f32p,
                                            cp, sz]
        lib.oref_conv_step.argtypes = [_f32p, _f32p, _f32p, u64, u64, C.c_int, _f32p, cp, sz]
        lib.oref_gated_delta_step.argtypes = [_f32p, _f32p, _f32p, _f32p, _f32p, _f32p, u64, u64, u64, C.c_float,
                                              _f32p, cp, sz]
        self.lib = lib

    @staticmethod
    def _check(rc: int, err) -> None:
        if rc:
            raise ReferenceError_(rc, err.value.decode())

    def type_layout(self, qtype: int):
        be, bb, q = C.c_uint64(), C.c_uint64(), C.c_int()
        name = C.create_string_buffer(64)
        if not self.lib.oref_type_layout(qtype, C.byref(be), C.byref(bb), C.byref(q), name, 64):
            return None
        return name.value.decode(), be.value, bb.value, bool(q.value)

    def row_byte_size(self, k: int, qtype: int) -> int:
        out, err = C.c_uint64(), C.create_string_buffer(512)
        self._check(self.lib.oref_row_byte_size(k, qtype, C.byref(out), err, 512), err)
        return out.value

    def f16_to_f32(self, bits: int) -> float:
        return float(self.lib.oref_f16_to_f32(bits))

    def decode_row(self, qtype: int, k: int, row: np.ndarray, out_len: int | None = None) -> np.ndarray:
        row = np.ascontiguousarray(row, np.uint8)
        out = np.empty(k if out_len is None else out_len, np.float32)
        err = C.create_string_buffer(512)
        self._check(self.lib.oref_decode_row(qtype, k, row.ctypes.data, row.size,
                                             _ptr(out, _f32p), out.size, err, 512), err)
        return out

    def rope(self, heads: np.ndarray, rotary_dim: int, sections, base: float, position) -> np.ndarray:
        """apply_qwen35_rope (reference_kernels.cpp:74-123) on a copy of heads [n x head_dim]."""
        h = np.array(heads, np.float32, copy=True)
        sec = (C.c_int32 * 4)(*sections)
        err = C.create_string_buffer(512)
        pt, ph, pw = position
        self._check(self.lib.oref_rope(_ptr(h, _f32p), h.shape[0], h.shape[1], rotary_dim, sec, base, pt, ph, pw,
                                       err, 512), err)
        return h

    def attention_step(self, q, k_new, v_new, keys, values, capacity) -> np.ndarray:
        """causal_attention_step (reference_kernels.cpp:125-190) after `len(keys)` cached tokens."""
        q, k_new, v_new = (np.ascontiguousarray(a, np.float32) for a in (q, k_new, v_new))
        keys = np.ascontiguousarray(keys, np.float32)
        values = np.ascontiguousarray(values, np.float32)
        hq, dk = q.shape
        hkv, dv = v_new.shape
        out = np.empty((hq, dv), np.float32)
        err = C.create_string_buffer(512)
        self._check(self.lib.oref_attention_step(_ptr(q, _f32p), _ptr(k_new, _f32p), _ptr(v_new, _f32p),
                                                 _ptr(keys, _f32p), _ptr(values, _f32p), keys.shape[0], capacity,
                                                 hq, hkv, dk, dv, _ptr(out, _f32p), err, 512), err)
        return out

    def conv_step(self, x, weights, history, apply_silu=True):
        """causal_depthwise_convolution_step (reference_kernels.cpp:192-219): (out, new history)."""
        x = np.ascontiguousarray(x, np.float32).reshape(-1)
        w = np.ascontiguousarray(weights, np.float32)
        hist = np.array(history, np.float32, copy=True)
        out = np.empty_like(x)
        err = C.create_string_buffer(512)
        self._check(self.lib.oref_conv_step(_ptr(x, _f32p), _ptr(w, _f32p), _ptr(hist, _f32p), x.size,
                                            hist.size // x.size, 1 if apply_silu else 0, _ptr(out, _f32p), err, 512),
                    err)
        return out, hist

    def gated_delta_step(self, q, k, v, beta, log_decay, state, eps=1e-6):
        """gated_delta_step (reference_kernels.cpp:221-335): (out, new state)."""
        q, k, v = (np.ascontiguousarray(a, np.float32) for a in (q, k, v))
        b = np.ascontiguousarray(beta, np.float32)
        g = np.ascontiguousarray(log_decay, np.float32)
        st = np.array(state, np.float32, copy=True)
        heads, dk = q.shape
        dv = v.shape[1]
        out = np.empty((heads, dv), np.float32)
        err = C.create_string_buffer(512)
        self._check(self.lib.oref_gated_delta_step(_ptr(q, _f32p), _ptr(k, _f32p), _ptr(v, _f32p), _ptr(b, _f32p),
                                                   _ptr(g, _f32p), _ptr(st, _f32p), heads, dk, dv, eps,
                                                   _ptr(out, _f32p), err, 512), err)
        return out, st

    def greedy_token(self, logits: np.ndarray) -> int:
        """Oracle's Sampler::sample at temperature 0 (sampler.cpp:22-46)."""
        logits = np.ascontiguousarray(logits, np.float32).reshape(-1)
        out, err = C.c_uint32(), C.create_string_buffer(512)
        self._check(self.lib.oref_greedy_token(_ptr(logits, _f32p), logits.size, C.byref(out), err, 512), err)
        return int(out.value)

    def storage_dot(self, qtype: int, k: int, row: np.ndarray, x: np.ndarray) -> float:
        row = np.ascontiguousarray(row, np.uint8)
        x = np.ascontiguousarray(x, np.float32)
        out, err = C.c_float(), C.create_string_buffer(512)
        self._check(self.lib.oref_storage_dot(qtype, k, row.ctypes.data, row.size,
                                              _ptr(x, _f32p), x.size, C.byref(out), err, 512), err)
        return out.value

    def storage_matvec(self, qtype: int, rows: int, cols: int, w: np.ndarray, x: np.ndarray,
                       y_len: int | None = None) -> np.ndarray:
        w = np.ascontiguousarray(w, np.uint8).reshape(-1)
        x = np.ascontiguousarray(x, np.float32).reshape(-1)
        y = np.empty(rows if y_len is None else y_len, np.float32)
        err = C.create_string_buffer(512)
        self._check(self.lib.oref_storage_matvec(qtype, rows, cols, w.ctypes.data, w.size,
                                                 _ptr(x, _f32p), x.size, _ptr(y, _f32p), y.size,
                                                 err, 512), err)
        return y

    def mapped_tensor_matvec(self, qtype: int, dims, w: np.ndarray, x: np.ndarray,
                             y_len: int) -> np.ndarray:
        d = np.asarray(dims, np.uint64)
        w = np.ascontiguousarray(w, np.uint8).reshape(-1)
        x = np.ascontiguousarray(x, np.float32)
        y = np.empty(y_len, np.float32)
        err = C.create_string_buffer(512)
        self._check(self.lib.oref_mapped_tensor_matvec(qtype, _ptr(d, _u64p), d.size, w.ctypes.data,
                                                       w.size, _ptr(x, _f32p), x.size,
                                                       _ptr(y, _f32p), y.size, err, 512), err)
        return y

    def decode_mapped_tensor(self, qtype: int, dims, w: np.ndarray, out_len: int) -> np.ndarray:
        d = np.asarray(dims, np.uint64)
        w = np.ascontiguousarray(w, np.uint8).reshape(-1)
        out = np.empty(out_len, np.float32)
        err = C.create_string_buffer(512)
        self._check(self.lib.oref_decode_mapped_tensor(qtype, _ptr(d, _u64p), d.size,
                                                       w.ctypes.data, w.size, _ptr(out, _f32p),
                                                       out.size, err, 512), err)
        return out


class _Qwen35Manifest(C.Structure):
    """oref_qwen35_manifest (ref_qwen35.cpp): the Qwen35Manifest fields of a
    model held in host buffers."""
    _fields_ = [(n, C.c_uint32) for n in ("block_count", "context_length", "embedding_length",
                                          "feed_forward_length", "head_count", "head_count_kv", "key_length",
                                          "value_length")] + [
        ("rms_epsilon", C.c_float), ("rope_dimension_count", C.c_uint32), ("rope_sections", C.c_int32 * 4),
        ("rope_frequency_base", C.c_float)] + [
        (n, C.c_uint32) for n in ("conv_kernel", "state_size", "group_count", "time_step_rank", "inner_size",
                                  "full_attention_interval", "vocabulary_size")]


_qwen35_libs = {}


def _qwen35_lib(contract: str):
    path = {"f32": REF_PATH, "q8k": REF_Q8K_PATH, "gate": REF_GATE_PATH}[contract]
    if contract not in _qwen35_libs:
        if not os.path.exists(path):
            build()
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} is not built and the reference tree is absent")
        lib = C.CDLL(path)
        cp, sz, vp, u32, u64 = C.c_char_p, C.c_size_t, C.c_void_p, C.c_uint32, C.c_uint64
        lib.oref_qwen35_open_gguf.argtypes = [cp, C.c_int, u64, C.POINTER(vp), cp, sz]
        lib.oref_qwen35_open_buffers.argtypes = [C.POINTER(_Qwen35Manifest), u32, C.POINTER(cp),
                                                 C.POINTER(u32), C.POINTER(u32), C.POINTER(u64), C.POINTER(vp),
                                                 C.POINTER(u64), C.c_int, u64, C.POINTER(vp), cp, sz]
        lib.oref_qwen35_vocab.argtypes = [vp]
        lib.oref_qwen35_vocab.restype = u32
        lib.oref_qwen35_reset.argtypes = [vp]
        lib.oref_qwen35_forward.argtypes = [vp, u32, _f32p, cp, sz]
        lib.oref_qwen35_greedy.argtypes = [vp, C.POINTER(u32), u64, u64, C.POINTER(u32), cp, sz]
        lib.oref_qwen35_close.argtypes = [vp]
        _qwen35_libs[contract] = lib
    return _qwen35_libs[contract]


class Qwen35Reference:
    """Oracle's own Qwen3.5 decode (execute_qwen35_reference_token on its
    HybridCache, greedy Sampler) over one model.

    contract "f32": the reference compiled unmodified (its f32 contract; its
    binder admits Q5_K/Q6_K/Q8_0/float matrices).  contract "q8k": the same
    sources with Q4_K/Q6_K projections on GGML's Q8_K contract and Q4_K
    admitted (``admit_q4k``) by this checker's own binding.  contract
    "gate": the "q8k" build whose binder is the reference's own
    ``bind_qwen35_weights`` compiled with the one-line type-gate change
    (Q4_K admitted in ``allowed_storage_type``'s matrix branch,
    qwen35_weights.cpp:49-59; ``oracle/Makefile`` target ``ref_gate``).  The model is a GGUF file (``gguf_path``) or
    host buffers: ``tensors`` = [(name, ggml_type, dims, uint8 array)], dims
    GGUF-ordered (dims[0] = columns), with ``manifest`` a dict of
    ``_Qwen35Manifest`` fields."""

    def __init__(self, contract: str, gguf_path: str | None = None, tensors=None, manifest: dict | None = None,
                 admit_q4k: bool = False, max_tokens: int = 4096):
        self.lib = _qwen35_lib(contract)
        self._h = C.c_void_p()
        err = C.create_string_buffer(512)
        if gguf_path is not None:
            rc = self.lib.oref_qwen35_open_gguf(gguf_path.encode(), int(admit_q4k), max_tokens, C.byref(self._h),
                                                err, 512)
        else:
            mf = _Qwen35Manifest()
            for k, v in manifest.items():
                if k == "rope_sections":
                    mf.rope_sections = (C.c_int32 * 4)(*v)
                else:
                    setattr(mf, k, v)
            n = len(tensors)
            self._keep = [np.ascontiguousarray(t[3]).view(np.uint8) for t in tensors]
            names = (C.c_char_p * n)(*[t[0].encode() for t in tensors])
            types = (C.c_uint32 * n)(*[t[1] for t in tensors])
            ndims = (C.c_uint32 * n)(*[len(t[2]) for t in tensors])
            dims = (C.c_uint64 * (4 * n))()
            for i, t in enumerate(tensors):
                for j, d in enumerate(t[2]):
                    dims[4 * i + j] = d
            data = (C.c_void_p * n)(*[a.ctypes.data for a in self._keep])
            sizes = (C.c_uint64 * n)(*[a.nbytes for a in self._keep])
            rc = self.lib.oref_qwen35_open_buffers(C.byref(mf), n, names, types, ndims, dims, data, sizes,
                                                   int(admit_q4k), max_tokens, C.byref(self._h), err, 512)
        if rc:
            raise ReferenceError_(rc, err.value.decode())
        self.vocab = int(self.lib.oref_qwen35_vocab(self._h))

    def reset(self) -> None:
        self.lib.oref_qwen35_reset(self._h)

    def forward(self, token: int) -> np.ndarray:
        """One token at the cache's current length; returns the logits."""
        out = np.empty(self.vocab, np.float32)
        err = C.create_string_buffer(512)
        rc = self.lib.oref_qwen35_forward(self._h, token, _ptr(out, _f32p), err, 512)
        if rc:
            raise ReferenceError_(rc, err.value.decode())
        return out

    def greedy(self, prompt, n_new: int) -> np.ndarray:
        """Fresh greedy generation of n_new tokens after the prompt."""
        p = np.ascontiguousarray(prompt, np.uint32)
        out = np.zeros(n_new, np.uint32)
        err = C.create_string_buffer(512)
        rc = self.lib.oref_qwen35_greedy(self._h, p.ctypes.data_as(C.POINTER(C.c_uint32)), p.size, n_new,
                                         out.ctypes.data_as(C.POINTER(C.c_uint32)), err, 512)
        if rc:
            raise ReferenceError_(rc, err.value.decode())
        return out

    def close(self) -> None:
        if self._h:
            self.lib.oref_qwen35_close(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


_port = None
_ref = None


def port() -> _Port:
    global _port
    if _port is None:
        _port = _Port()
    return _port


def ref() -> _Ref:
    global _ref
    if _ref is None:
        _ref = _Ref()
    return _ref


def ref_available() -> bool:
    return os.path.exists(REF_PATH) or bool(REFERENCE_TREE and os.path.isdir(REFERENCE_TREE))
