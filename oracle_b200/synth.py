"""Seeded synthetic GGML tensors with the distributions of the benchmark configs.

Every tensor is generated from one 64-bit seed derived from (config, tensor
name) with BLAKE2b, fed to numpy's PCG64.  The same call therefore yields the
same bytes on every machine, so CPU checkers and the GPU run see identical
inputs.  Distributions (per block / super-block):

* Q8_0  -- d = f16(U[1e-3, 1e-2]), 32 int8 quants U{-127..127}.
* Q4_K  -- d = f16(U[1e-3, 2e-2]), dmin = f16(U[0, 1e-2]), 8 scales and 8 mins
  U{0..63} packed into 12 bytes (inverse of Oracle's unpack_scale_min_k4,
  src/model/storage_decode.cpp:44-61), 256 nibbles U{0..15}.
* Q5_K  -- as Q4_K plus a uniform fifth bit per element.
* Q6_K  -- 6-bit quants U{0..63} (ql/qh bytes uniform), 16 int8 scales
  U{-127..127}, d = f16(U[1e-4, 5e-3]).
* activations -- f32 N(0, 1).

A uniform 6-bit quant is the same as independent uniform bits, so nibble and
high-bit planes are drawn as uniform bytes, which keeps 500 MB tensors cheap.
"""
from __future__ import annotations

import hashlib

import numpy as np

TYPE_F32, TYPE_F16, TYPE_Q8_0, TYPE_Q4_K, TYPE_Q5_K, TYPE_Q6_K, TYPE_Q8_K, TYPE_BF16 = (
    0, 1, 8, 12, 13, 14, 15, 30)

BLOCK = {TYPE_Q8_0: (32, 34), TYPE_Q4_K: (256, 144), TYPE_Q5_K: (256, 176),
         TYPE_Q6_K: (256, 210), TYPE_F32: (1, 4), TYPE_F16: (1, 2), TYPE_BF16: (1, 2)}


def seed_for(config: str, name: str) -> int:
    digest = hashlib.blake2b(f"{config}/{name}".encode(), digest_size=8).digest()
    return int.from_bytes(digest, "little")


def rng_for(config: str, name: str) -> np.random.Generator:
    return np.random.Generator(np.random.PCG64(seed_for(config, name)))


def row_bytes(qtype: int, k: int) -> int:
    be, bb = BLOCK[qtype]
    if k % be:
        raise ValueError(f"row length {k} is not divisible by block size {be}")
    return (k // be) * bb


def _f16_bytes(values: np.ndarray) -> np.ndarray:
    return values.astype(np.float16).view(np.uint8).reshape(values.shape[0], 2)


def pack_scale_min_k4(sc: np.ndarray, mn: np.ndarray) -> np.ndarray:
    """Pack (n, 8) 6-bit scales and mins into (n, 12) bytes; the inverse of
    Oracle's unpack_scale_min_k4 (storage_decode.cpp:44-61)."""
    sc = sc.astype(np.uint8)
    mn = mn.astype(np.uint8)
    out = np.empty((sc.shape[0], 12), np.uint8)
    out[:, 0:4] = (sc[:, 0:4] & 63) | ((sc[:, 4:8] >> 4) << 6)
    out[:, 4:8] = (mn[:, 0:4] & 63) | ((mn[:, 4:8] >> 4) << 6)
    out[:, 8:12] = (sc[:, 4:8] & 15) | ((mn[:, 4:8] & 15) << 4)
    return out


def q8_0_blocks(rng: np.random.Generator, n: int) -> np.ndarray:
    out = np.empty((n, 34), np.uint8)
    out[:, 0:2] = _f16_bytes(rng.uniform(1e-3, 1e-2, n))
    out[:, 2:] = rng.integers(-127, 128, (n, 32), dtype=np.int8).view(np.uint8)
    return out


def q4_k_blocks(rng: np.random.Generator, n: int) -> np.ndarray:
    out = np.empty((n, 144), np.uint8)
    out[:, 0:2] = _f16_bytes(rng.uniform(1e-3, 2e-2, n))
    out[:, 2:4] = _f16_bytes(rng.uniform(0.0, 1e-2, n))
    sc = rng.integers(0, 64, (n, 8), dtype=np.uint8)
    mn = rng.integers(0, 64, (n, 8), dtype=np.uint8)
    out[:, 4:16] = pack_scale_min_k4(sc, mn)
    out[:, 16:] = rng.integers(0, 256, (n, 128), dtype=np.uint8)
    return out


def q5_k_blocks(rng: np.random.Generator, n: int) -> np.ndarray:
    out = np.empty((n, 176), np.uint8)
    out[:, 0:2] = _f16_bytes(rng.uniform(1e-3, 2e-2, n))
    out[:, 2:4] = _f16_bytes(rng.uniform(0.0, 1e-2, n))
    sc = rng.integers(0, 64, (n, 8), dtype=np.uint8)
    mn = rng.integers(0, 64, (n, 8), dtype=np.uint8)
    out[:, 4:16] = pack_scale_min_k4(sc, mn)
    out[:, 16:] = rng.integers(0, 256, (n, 160), dtype=np.uint8)
    return out


def q6_k_blocks(rng: np.random.Generator, n: int) -> np.ndarray:
    out = np.empty((n, 210), np.uint8)
    out[:, 0:192] = rng.integers(0, 256, (n, 192), dtype=np.uint8)
    out[:, 192:208] = rng.integers(-127, 128, (n, 16), dtype=np.int8).view(np.uint8)
    out[:, 208:210] = _f16_bytes(rng.uniform(1e-4, 5e-3, n))
    return out


_BLOCK_GEN = {TYPE_Q8_0: q8_0_blocks, TYPE_Q4_K: q4_k_blocks, TYPE_Q5_K: q5_k_blocks,
              TYPE_Q6_K: q6_k_blocks}


def weight(qtype: int, rows: int, k: int, config: str, name: str = "W") -> np.ndarray:
    """A (rows, row_bytes) uint8 matrix of GGML blocks, row-major."""
    rng = rng_for(config, name)
    be, bb = BLOCK[qtype]
    if qtype in (TYPE_F32, TYPE_F16, TYPE_BF16):
        vals = rng.standard_normal((rows, k), dtype=np.float32)
        if qtype == TYPE_F32:
            return vals.view(np.uint8).reshape(rows, 4 * k)
        if qtype == TYPE_F16:
            return vals.astype(np.float16).view(np.uint8).reshape(rows, 2 * k)
        return (vals.view(np.uint32) >> 16).astype(np.uint16).view(np.uint8).reshape(rows, 2 * k)
    blocks = _BLOCK_GEN[qtype](rng, rows * (k // be))
    return blocks.reshape(rows, (k // be) * bb)


def activations(k: int, batch: int, config: str, name: str = "x") -> np.ndarray:
    rng = rng_for(config, name)
    return rng.standard_normal((batch, k), dtype=np.float32)
