"""Write a small synthetic GGUF file of GGML-quantized tensors (test fixture).

Run at test time (the file is not committed): every 2-D weight type the path
handles (Q8_0, Q4_K, Q5_K, Q6_K, F16, BF16, F32) plus a 1-D F32 norm vector,
with bytes from oracle_b200.synth, written by gguf-py's GGUFWriter so that
Oracle's own MappedGgufModel (src/model/mapped_gguf.cpp) maps it.
GGUF dims are [columns, rows] (dims[0] = K), as Oracle reads them.
"""
from __future__ import annotations

import sys

import numpy as np

TENSORS = [  # (name, ggml type, rows, cols)
    ("blk.0.ffn_up.weight", 12, 96, 1024),
    ("blk.0.ffn_down.weight", 14, 64, 512),
    ("blk.0.attn_v.weight", 13, 40, 768),
    ("blk.0.eh_proj.weight", 8, 48, 256),
    ("blk.0.attn_q.weight", 1, 33, 160),
    ("blk.0.attn_k.weight", 30, 17, 96),
    ("blk.0.ssm_out.weight", 0, 9, 64),
]


def write(path: str) -> list:
    import gguf

    from oracle_b200 import synth

    w = gguf.GGUFWriter(path, "qwen35")
    for name, t, rows, cols in TENSORS:
        data = synth.weight(t, rows, cols, "gguf", name).reshape(-1)
        if t in (0, 1, 30):
            dt = {0: np.float32, 1: np.float16, 30: np.uint16}[t]
            arr = data.view(dt).reshape(rows, cols)
            if t == 30:
                w.add_tensor(name, arr, raw_dtype=gguf.GGMLQuantizationType.BF16)
            else:
                w.add_tensor(name, arr)
        else:
            w.add_tensor(name, data.reshape(rows, -1), raw_dtype=gguf.GGMLQuantizationType(t))
    norm = np.random.default_rng(3).standard_normal(1024).astype(np.float32)
    w.add_tensor("blk.0.ffn_norm.weight", norm)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    return TENSORS


if __name__ == "__main__":
    write(sys.argv[1] if len(sys.argv) > 1 else "synthetic.gguf")
