"""Qwen3.5-style hybrid decoder: shapes, tensor names and seeded synthetic weights.

The model is Oracle's Qwen3.5 backbone (src/model/qwen35_manifest.cpp,
src/model/qwen35_weights.cpp, src/runtime/qwen35_block.cpp): blocks whose
index i has (i + 1) % full_attention_interval == 0 are gated full-attention
blocks, the others Gated DeltaNet (recurrent) blocks, each followed by a
SwiGLU MLP.  Tensor names and GGUF dims (dims[0] = columns) are those the
reference's binder requires.

``Qwen35Config`` mirrors the manifest fields; ``CONFIG5`` is the benchmark's
full model (32 blocks, hidden 4096, FFN 12288, 32 query / 4 KV heads of 128,
partial RoPE over 64 dimensions, 32 Gated DeltaNet value heads with 128 x 128
states fed by 16 key heads, conv width 4, vocabulary 151936, RMS eps 1e-6).

Storage recipes:

* ``q4_k_m`` -- llama.cpp's published Q4_K_M mix: Q4_K everywhere except the
  output projection (Q6_K) and ``ffn_down`` / ``attn_v`` of the layers its
  ``use_more_bits`` rule selects (Q6_K); vectors and the depthwise conv
  kernel stay F32.  Oracle's binder rejects Q4_K matrices, so this model
  runs on the CPU only through the Q8_K checker build.
* ``oracle`` -- only types Oracle's binder and storage decoder admit (Q5_K,
  Q6_K, Q8_0 matrices, F32 vectors), so the unmodified reference can decode
  it; used to check the GPU decoder on Oracle's own f32 contract.

Synthetic values are zero-mean with a standard deviation of gain/sqrt(fan-in)
per projection (so activations keep unit scale through the stack): Q4_K /
Q5_K blocks take dmin = 8 d (16 d for Q5_K) and each sub-block's min
m = round(sc * 15/16) (Q5_K: round(sc * 31/32), halves up), which cancels the
mean of the uniform quants.  Every tensor's bytes come from a PCG64 stream seeded by
BLAKE2b(config, tensor name), so CPU and GPU see identical models.
"""
from __future__ import annotations

import dataclasses
import hashlib

import numpy as np

TYPE_F32, TYPE_Q8_0, TYPE_Q4_K, TYPE_Q5_K, TYPE_Q6_K = 0, 8, 12, 13, 14
BLOCK = {TYPE_Q8_0: (32, 34), TYPE_Q4_K: (256, 144), TYPE_Q5_K: (256, 176), TYPE_Q6_K: (256, 210), TYPE_F32: (1, 4)}


@dataclasses.dataclass(frozen=True)
class Qwen35Config:
    hidden: int
    ffn: int
    layers: int
    heads: int
    kv_heads: int
    head_dim: int
    rope_dim: int
    rope_sections: tuple
    rope_base: float
    conv_kernel: int
    state_size: int
    key_heads: int       # ssm.group_count
    value_heads: int     # ssm.time_step_rank
    vocab: int
    eps: float           # an f32 value (the manifest field is f32)
    interval: int        # full_attention_interval
    context: int         # KV cache capacity (tokens)

    # qwen35_ssm_layout (src/runtime/hybrid_cache.cpp)
    @property
    def key_width(self) -> int:
        return self.key_heads * self.state_size

    @property
    def value_width(self) -> int:
        return self.value_heads * self.state_size

    @property
    def conv_channels(self) -> int:
        return 2 * self.key_width + self.value_width

    @property
    def q_width(self) -> int:
        return self.heads * self.head_dim

    @property
    def kv_width(self) -> int:
        return self.kv_heads * self.head_dim

    def is_attention(self, i: int) -> bool:
        """Qwen35Manifest::is_full_attention_block (qwen35_manifest.cpp:146-149)."""
        return (i + 1) % self.interval == 0

    def manifest(self) -> dict:
        """Fields of the reference's Qwen35Manifest (oracle.Qwen35Reference)."""
        return dict(block_count=self.layers, context_length=self.context, embedding_length=self.hidden,
                    feed_forward_length=self.ffn, head_count=self.heads, head_count_kv=self.kv_heads,
                    key_length=self.head_dim, value_length=self.head_dim, rms_epsilon=self.eps,
                    rope_dimension_count=self.rope_dim, rope_sections=tuple(self.rope_sections),
                    rope_frequency_base=self.rope_base, conv_kernel=self.conv_kernel, state_size=self.state_size,
                    group_count=self.key_heads, time_step_rank=self.value_heads,
                    inner_size=self.value_width, full_attention_interval=self.interval,
                    vocabulary_size=self.vocab)


CONFIG5 = Qwen35Config(hidden=4096, ffn=12288, layers=32, heads=32, kv_heads=4, head_dim=128, rope_dim=64,
                       rope_sections=(11, 11, 10, 0), rope_base=1.0e7, conv_kernel=4, state_size=128, key_heads=16,
                       value_heads=32, vocab=151936, eps=float(np.float32(1e-6)), interval=4,
                       context=4096)

# The same architecture at test scale: every shape rule of CONFIG5 (head dims,
# RoPE sections, GQA ratio, key-head repetition) on a model the CPU reference
# decodes in seconds.
SMALL = Qwen35Config(hidden=512, ffn=1536, layers=4, heads=4, kv_heads=2, head_dim=128, rope_dim=64,
                     rope_sections=(11, 11, 10, 0), rope_base=1.0e7, conv_kernel=4, state_size=128, key_heads=2,
                     value_heads=4, vocab=2048, eps=float(np.float32(1e-6)), interval=4,
                     context=512)


def use_more_bits(i: int, n: int) -> bool:
    """llama.cpp's Q4_K_M layer selector for the Q6_K tensors."""
    return i < n // 8 or i >= 7 * n // 8 or (i - n // 8) % 3 == 2


def tensor_specs(cfg: Qwen35Config, recipe: str = "q4_k_m") -> list:
    """[(name, ggml type, gguf dims, kind, gain)]; kind is "matrix",
    "embedding", "norm", "conv", "decay" or "dt_bias"."""
    H, F = cfg.hidden, cfg.ffn
    q4 = recipe == "q4_k_m"
    proj = TYPE_Q4_K if q4 else TYPE_Q5_K
    small = TYPE_Q4_K if q4 else TYPE_Q8_0
    specs = [("token_embd.weight", TYPE_Q4_K if q4 else TYPE_Q6_K, (H, cfg.vocab), "embedding", 1.0),
             ("output_norm.weight", TYPE_F32, (H,), "norm", 1.0),
             ("output.weight", TYPE_Q6_K, (H, cfg.vocab), "matrix", 1.0)]
    n_attn = sum(cfg.is_attention(i) for i in range(cfg.layers))
    i_attn = 0
    for i in range(cfg.layers):
        p = f"blk.{i}."
        specs += [(p + "attn_norm.weight", TYPE_F32, (H,), "norm", 1.0),
                  (p + "post_attention_norm.weight", TYPE_F32, (H,), "norm", 1.0)]
        if cfg.is_attention(i):
            v_type = (TYPE_Q6_K if use_more_bits(i_attn, n_attn) else TYPE_Q4_K) if q4 else TYPE_Q8_0
            i_attn += 1
            specs += [(p + "attn_q.weight", proj, (H, 2 * cfg.q_width), "matrix", 1.0),
                      (p + "attn_k.weight", proj, (H, cfg.kv_width), "matrix", 1.0),
                      (p + "attn_v.weight", v_type, (H, cfg.kv_width), "matrix", 1.0),
                      (p + "attn_output.weight", proj, (cfg.q_width, H), "matrix", 1.0),
                      (p + "attn_q_norm.weight", TYPE_F32, (cfg.head_dim,), "norm", 1.0),
                      (p + "attn_k_norm.weight", TYPE_F32, (cfg.head_dim,), "norm", 1.0)]
        else:
            specs += [(p + "attn_qkv.weight", proj, (H, cfg.conv_channels), "matrix", 1.0),
                      (p + "attn_gate.weight", proj, (H, cfg.value_width), "matrix", 1.0),
                      (p + "ssm_conv1d.weight", TYPE_F32, (cfg.conv_kernel, cfg.conv_channels), "conv", 1.0),
                      (p + "ssm_dt.bias", TYPE_F32, (cfg.value_heads,), "dt_bias", 1.0),
                      (p + "ssm_a", TYPE_F32, (cfg.value_heads,), "decay", 1.0),
                      (p + "ssm_beta.weight", small, (H, cfg.value_heads), "matrix", 1.0),
                      (p + "ssm_alpha.weight", small, (H, cfg.value_heads), "matrix", 1.0),
                      (p + "ssm_norm.weight", TYPE_F32, (cfg.state_size,), "norm", 1.0),
                      (p + "ssm_out.weight", proj, (cfg.value_width, H), "matrix", 1.0)]
        down = (TYPE_Q6_K if use_more_bits(i, cfg.layers) else TYPE_Q4_K) if q4 else TYPE_Q6_K
        specs += [(p + "ffn_gate.weight", proj, (H, F), "matrix", 1.0),
                  (p + "ffn_up.weight", proj, (H, F), "matrix", 1.0),
                  (p + "ffn_down.weight", down, (F, H), "matrix", 1.0)]
    return specs


def _rng(config: str, name: str) -> np.random.Generator:
    digest = hashlib.blake2b(f"{config}/{name}".encode(), digest_size=8).digest()
    return np.random.Generator(np.random.PCG64(int.from_bytes(digest, "little")))


def _f16(values: np.ndarray) -> np.ndarray:
    return values.astype(np.float16).view(np.uint8).reshape(-1, 2)


def _pack_scale_min_k4(sc: np.ndarray, mn: np.ndarray) -> np.ndarray:
    out = np.empty((sc.shape[0], 12), np.uint8)
    out[:, 0:4] = (sc[:, 0:4] & 63) | ((sc[:, 4:8] >> 4) << 6)
    out[:, 4:8] = (mn[:, 0:4] & 63) | ((mn[:, 4:8] >> 4) << 6)
    out[:, 8:12] = (sc[:, 4:8] & 15) | ((mn[:, 4:8] & 15) << 4)
    return out


def _random_bytes(rng: np.random.Generator, n: int, width: int) -> np.ndarray:
    """(n, width) uniform bytes straight from the bit generator's 64-bit words."""
    words = rng.bit_generator.random_raw((n * width + 7) // 8)
    return words.view(np.uint8)[:n * width].reshape(n, width)


def _blocks(rng: np.random.Generator, qtype: int, n: int, std: float) -> np.ndarray:
    """n zero-mean GGML blocks whose values have standard deviation ~std."""
    u = rng.uniform(0.5, 1.5, n)
    if qtype == TYPE_Q8_0:
        out = np.empty((n, 34), np.uint8)
        out[:, 0:2] = _f16(u * std / 73.5)
        out[:, 2:] = rng.integers(-127, 128, (n, 32), dtype=np.int8).view(np.uint8)
        return out
    if qtype == TYPE_Q6_K:
        out = np.empty((n, 210), np.uint8)
        out[:, 0:192] = _random_bytes(rng, n, 192)
        out[:, 192:208] = rng.integers(-127, 128, (n, 16), dtype=np.int8).view(np.uint8)
        out[:, 208:210] = _f16(u * std / 1360.0)
        return out
    q5 = qtype == TYPE_Q5_K
    nb = 176 if q5 else 144
    out = np.empty((n, nb), np.uint8)
    d = (u * std / (337.0 if q5 else 168.0)).astype(np.float16)
    out[:, 0:2] = d.view(np.uint8).reshape(n, 2)
    out[:, 2:4] = _f16(d.astype(np.float32) * (16.0 if q5 else 8.0))
    sc = rng.integers(1, 64, (n, 8), dtype=np.uint8)
    mn = ((sc.astype(np.uint16) * 31 + 16) // 32 if q5 else (sc.astype(np.uint16) * 15 + 8) // 16).astype(np.uint8)
    out[:, 4:16] = _pack_scale_min_k4(sc, mn)
    out[:, 16:] = _random_bytes(rng, n, nb - 16)
    return out


def tensor_bytes(spec, config: str = "qwen35") -> np.ndarray:
    """The seeded bytes of one tensor (uint8, GGML row-major)."""
    name, qtype, dims, kind, gain = spec
    rng = _rng(config, name)
    n = int(np.prod(dims))
    if qtype == TYPE_F32:
        if kind == "norm":
            v = 1.0 + 0.1 * rng.standard_normal(n)
        elif kind == "conv":
            v = rng.standard_normal(n) / np.sqrt(dims[0])
        elif kind == "decay":  # ssm_a = -exp(A_log), A in [1, 16]
            v = -rng.uniform(1.0, 16.0, n)
        elif kind == "dt_bias":  # softplus^-1 of a time step in [1e-3, 1e-1]
            dt = np.exp(rng.uniform(np.log(1e-3), np.log(1e-1), n))
            v = np.log(np.expm1(dt))
        else:
            v = rng.standard_normal(n) * gain / np.sqrt(dims[0])
        return v.astype(np.float32).view(np.uint8)
    cols = dims[0]
    std = gain if kind == "embedding" else gain / np.sqrt(cols)
    be = BLOCK[qtype][0]
    return _blocks(rng, qtype, n // be, std).reshape(-1)


def synthetic_model(cfg: Qwen35Config, recipe: str = "q4_k_m", config: str = "qwen35") -> list:
    """[(name, ggml type, gguf dims, uint8 bytes)] for every tensor."""
    return [(s[0], s[1], s[2], tensor_bytes(s, config)) for s in tensor_specs(cfg, recipe)]


def model_bytes(cfg: Qwen35Config, recipe: str = "q4_k_m") -> int:
    total = 0
    for _, qtype, dims, _, _ in tensor_specs(cfg, recipe):
        be, bb = BLOCK[qtype]
        total += int(np.prod(dims)) // be * bb
    return total


def write_gguf(path: str, cfg: Qwen35Config, tensors) -> None:
    """Write the model as a GGUF file Oracle's MappedGgufModel and
    load_qwen35_manifest accept (gguf-py's writer; synthetic token strings)."""
    import gguf

    w = gguf.GGUFWriter(path, "qwen35")
    w.add_uint32("qwen35.block_count", cfg.layers)
    w.add_uint32("qwen35.context_length", cfg.context)
    w.add_uint32("qwen35.embedding_length", cfg.hidden)
    w.add_uint32("qwen35.feed_forward_length", cfg.ffn)
    w.add_uint32("qwen35.attention.head_count", cfg.heads)
    w.add_uint32("qwen35.attention.head_count_kv", cfg.kv_heads)
    w.add_uint32("qwen35.attention.key_length", cfg.head_dim)
    w.add_uint32("qwen35.attention.value_length", cfg.head_dim)
    w.add_float32("qwen35.attention.layer_norm_rms_epsilon", cfg.eps)
    w.add_uint32("qwen35.rope.dimension_count", cfg.rope_dim)
    w.add_float32("qwen35.rope.freq_base", cfg.rope_base)
    w.add_array("qwen35.rope.dimension_sections", [int(s) for s in cfg.rope_sections])
    w.add_uint32("qwen35.ssm.conv_kernel", cfg.conv_kernel)
    w.add_uint32("qwen35.ssm.state_size", cfg.state_size)
    w.add_uint32("qwen35.ssm.group_count", cfg.key_heads)
    w.add_uint32("qwen35.ssm.time_step_rank", cfg.value_heads)
    w.add_uint32("qwen35.ssm.inner_size", cfg.value_width)
    w.add_uint32("qwen35.full_attention_interval", cfg.interval)
    w.add_token_list([f"t{i}" for i in range(cfg.vocab)])
    w.add_token_types([1] * cfg.vocab)
    for name, qtype, dims, data in tensors:
        if qtype == TYPE_F32:
            arr = np.asarray(data).view(np.float32).reshape(tuple(reversed(dims)))
            w.add_tensor(name, arr)
        else:
            be, bb = BLOCK[qtype]
            rows = int(np.prod(dims[1:]))
            w.add_tensor(name, np.asarray(data).reshape(rows, dims[0] // be * bb),
                         raw_dtype=gguf.GGMLQuantizationType(qtype))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
