"""Generate the committed golden fixtures under tests/golden/.

Run from the repository root in a container that has the reference tree and
gguf-py installed:

    python tests/golden/make_golden.py

Fixtures (numpy .npz, small):

* ``decode_ggufpy.npz`` -- seeded and hand-made blocks of Q8_0, Q4_K, Q5_K and
  Q6_K with their f32 decode by gguf-py 0.19.0 (``gguf.quants.dequantize``),
  an implementation independent of both Oracle and this repository.  Q4_K has
  no decoder in Oracle, so this is its outside pin.
* ``reference.npz`` -- outputs of the reference's own compiled code
  (oracle/_ref, i.e. Oracle's decode_storage_row and reference_storage_matvec)
  on seeded rows of every type Oracle decodes.
* ``q8k.npz`` -- this repository's Q8_K quantization and integer dots on crafted
  activations (ties, zeros, extremes).  GGML is not vendored anywhere here, so
  these are a regression lock on the restatement, not an outside pin.
"""
from __future__ import annotations

import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

import oracle  # noqa: E402
from oracle_b200 import synth  # noqa: E402

OUT = os.path.dirname(os.path.abspath(__file__))
CFG = "golden"


def crafted_blocks(qtype: int) -> np.ndarray:
    """Blocks with edge values in the f16 scale fields: subnormal, negative,
    zero, largest normal, and all-ones / all-zero quant planes."""
    bb = synth.BLOCK[qtype][1]
    out = []
    for d_bits, fill in [(0x0001, 0xFF), (0x8400, 0x00), (0x0000, 0x5A), (0x7BFF, 0x0F), (0x3C00, 0xF0),
                         (0x83FF, 0xA5)]:
        b = np.full(bb, fill, np.uint8)
        if qtype == synth.TYPE_Q6_K:
            b[208:210] = np.frombuffer(np.uint16(d_bits).tobytes(), np.uint8)
        else:
            b[0:2] = np.frombuffer(np.uint16(d_bits).tobytes(), np.uint8)
            if qtype in (synth.TYPE_Q4_K, synth.TYPE_Q5_K):
                b[2:4] = np.frombuffer(np.uint16(d_bits ^ 0x8000).tobytes(), np.uint8)
        out.append(b)
    return np.stack(out)


def make_decode_ggufpy() -> None:
    import gguf.quants as gq
    from gguf import GGMLQuantizationType as G

    data = {}
    for qtype, name in [(synth.TYPE_Q8_0, "Q8_0"), (synth.TYPE_Q4_K, "Q4_K"), (synth.TYPE_Q5_K, "Q5_K"),
                        (synth.TYPE_Q6_K, "Q6_K")]:
        be, bb = synth.BLOCK[qtype]
        seeded = synth.weight(qtype, 16, be, CFG, f"ggufpy_{name}").reshape(16, bb)
        blocks = np.concatenate([seeded, crafted_blocks(qtype)])
        dec = gq.dequantize(blocks, getattr(G, name)).astype(np.float32).reshape(len(blocks), be)
        data[f"{name}_blocks"] = blocks
        data[f"{name}_decoded"] = dec
    np.savez_compressed(os.path.join(OUT, "decode_ggufpy.npz"), **data)


def make_reference() -> None:
    ref = oracle.ref()
    data = {}
    for qtype, name, k in [(synth.TYPE_Q8_0, "Q8_0", 96), (synth.TYPE_Q5_K, "Q5_K", 512),
                           (synth.TYPE_Q6_K, "Q6_K", 512), (synth.TYPE_F16, "F16", 37),
                           (synth.TYPE_BF16, "BF16", 37), (synth.TYPE_F32, "F32", 37)]:
        rows = 5
        w = synth.weight(qtype, rows, k, CFG, f"ref_{name}")
        x = synth.activations(k, 1, CFG, f"ref_x_{name}")[0]
        data[f"{name}_w"] = w
        data[f"{name}_x"] = x
        data[f"{name}_decoded"] = np.stack([ref.decode_row(qtype, k, w[r]) for r in range(rows)])
        data[f"{name}_matvec"] = ref.storage_matvec(qtype, rows, k, w, x)
    np.savez_compressed(os.path.join(OUT, "reference.npz"), **data)


def crafted_activations() -> np.ndarray:
    rng = synth.rng_for(CFG, "q8k_crafted")
    xs = []
    xs.append(np.zeros(256, np.float32))                      # all-zero block
    t = rng.standard_normal(256).astype(np.float32)
    t[7], t[200] = 3.0, -3.0                                   # tie: first (+) wins
    xs.append(t)
    t = rng.standard_normal(256).astype(np.float32)
    t[5], t[9] = -4.0, 4.0                                     # tie: first (-) wins
    xs.append(t)
    xs.append(np.full(256, -1e-30, np.float32))                # tiny, constant
    t = np.linspace(-1, 1, 256, dtype=np.float32)
    xs.append(t)                                               # halves -> ties-to-even in rounding
    xs.append(rng.standard_normal(256).astype(np.float32) * 1e4)
    t = np.zeros(256, np.float32)
    t[255] = 1.0
    xs.append(t)                                               # single non-zero at the end
    return np.concatenate(xs)


def make_q8k() -> None:
    port = oracle.port()
    x = crafted_activations()
    q = port.quantize_q8_k(x)[0]
    k = x.size
    w4 = synth.weight(synth.TYPE_Q4_K, 3, k, CFG, "q8k_w4")
    w6 = synth.weight(synth.TYPE_Q6_K, 3, k, CFG, "q8k_w6")
    nb = k // 256
    sums4 = np.array([[port.block_sums(synth.TYPE_Q4_K, w4[r, 144 * i:144 * (i + 1)], q[292 * i:292 * (i + 1)])
                       for i in range(nb)] for r in range(3)], np.int32)
    sums6 = np.array([[port.block_sums(synth.TYPE_Q6_K, w6[r, 210 * i:210 * (i + 1)], q[292 * i:292 * (i + 1)])
                       for i in range(nb)] for r in range(3)], np.int32)
    np.savez_compressed(os.path.join(OUT, "q8k.npz"), x=x, q8k=q, w4=w4, w6=w6, sums4=sums4, sums6=sums6,
                        y4=port.matvec_q8_k(synth.TYPE_Q4_K, 3, k, w4, q)[0],
                        y6=port.matvec_q8_k(synth.TYPE_Q6_K, 3, k, w6, q)[0])


if __name__ == "__main__":
    make_decode_ggufpy()
    make_reference()
    make_q8k()
    print("golden fixtures written to", OUT)
