"""CPU: the Qwen3.5 model description and the reference decode harness.

* The synthetic model's tensor names and shapes are the ones Oracle's own
  binder requires: the unmodified reference binds the ``oracle`` recipe from a
  GGUF file this package writes, and decodes it.
* The GGUF writer and the product's GGUF reader round-trip every tensor and
  every manifest field.
* The reference decode harness gives the same tokens from a mapped GGUF file
  and from host buffers, for both checker builds.
* The Q8_K checker build routes Q4_K / Q6_K projections to GGML's contract
  and leaves the others to the reference.
* With the one-line type-gate change compiled in, the reference's own binder
  binds the Q4_K_M model.
"""
from __future__ import annotations

import os

import numpy as np
import pytest

from oracle_b200 import qwen35

pytest.importorskip("gguf")


@pytest.fixture(scope="module")
def models(tmp_path_factory):
    import oracle
    if not oracle.ref_available():
        pytest.skip("reference checker library not built")
    d = tmp_path_factory.mktemp("qwen35")
    out = {}
    for recipe in ("oracle", "q4_k_m"):
        tensors = qwen35.synthetic_model(qwen35.SMALL, recipe)
        path = str(d / f"{recipe}.gguf")
        qwen35.write_gguf(path, qwen35.SMALL, tensors)
        out[recipe] = (path, tensors)
    return out


def test_config5_shapes():
    cfg = qwen35.CONFIG5
    assert cfg.conv_channels == 8192 and cfg.value_width == 4096 and cfg.key_width == 2048
    assert [i for i in range(cfg.layers) if cfg.is_attention(i)] == [3, 7, 11, 15, 19, 23, 27, 31]
    specs = qwen35.tensor_specs(cfg)
    types = {name: t for name, t, *_ in specs}
    assert types["output.weight"] == qwen35.TYPE_Q6_K and types["token_embd.weight"] == qwen35.TYPE_Q4_K
    six = [i for i in range(32) if types[f"blk.{i}.ffn_down.weight"] == qwen35.TYPE_Q6_K]
    assert six == [i for i in range(32) if qwen35.use_more_bits(i, 32)]
    assert 4.0e9 < qwen35.model_bytes(cfg) < 5.0e9


def test_gguf_round_trip(models):
    from oracle_b200.decoder import tensors_from_gguf
    for recipe, (path, tensors) in models.items():
        cfg, read = tensors_from_gguf(path)
        assert cfg == qwen35.SMALL
        assert [(n, t, d) for n, t, d, _ in read] == [(n, t, d) for n, t, d, _ in tensors]
        for (_, _, _, a), (_, _, _, b) in zip(read, tensors):
            assert np.array_equal(a, b)


def test_reference_binder_accepts_oracle_recipe(models):
    import oracle
    path, tensors = models["oracle"]
    prompt = np.arange(5, 13, dtype=np.uint32) * 37 % qwen35.SMALL.vocab
    from_file = oracle.Qwen35Reference("f32", gguf_path=path, max_tokens=64).greedy(prompt, 8)
    from_buffers = oracle.Qwen35Reference("f32", tensors=tensors, manifest=qwen35.SMALL.manifest(),
                                          max_tokens=64).greedy(prompt, 8)
    assert np.array_equal(from_file, from_buffers)
    assert len(set(from_file.tolist())) > 1


def test_reference_binder_rejects_q4k(models):
    import oracle
    path, _ = models["q4_k_m"]
    with pytest.raises(oracle.ReferenceError_, match="unsupported storage type"):
        oracle.Qwen35Reference("f32", gguf_path=path, max_tokens=64)


def test_q8k_checker_routes_q6k_projections(models):
    """The two checker builds on the same Oracle-admissible model: the f32
    build decodes every projection with Oracle's f32 contract, the Q8_K build
    sends its Q6_K projections (ffn_down, output) through GGML's Q8_K
    contract, so the logits differ, slightly; file and buffer models agree."""
    import oracle
    path, tensors = models["oracle"]
    f32 = oracle.Qwen35Reference("f32", gguf_path=path, max_tokens=64).forward(7)
    q8k = oracle.Qwen35Reference("q8k", gguf_path=path, max_tokens=64)
    a = q8k.forward(7)
    q8k.reset()
    assert np.array_equal(q8k.forward(7), a)
    assert not np.array_equal(a, f32)
    assert np.abs(a - f32).max() < 0.25 * f32.std()  # 8-bit activations: ~1% per projection
    rb = oracle.Qwen35Reference("q8k", tensors=tensors, manifest=qwen35.SMALL.manifest(), max_tokens=64)
    assert np.array_equal(rb.forward(7), a)


def _gate_checker_or_skip():
    import oracle
    if not os.path.exists(oracle.REF_GATE_PATH):
        pytest.skip("gate-patched reference checker (oracle/_ref/liboracle_ref_gate.so) not built")
    return oracle


def test_patched_type_gate_binds_q4k_m_through_reference_binder(models):
    """The type gate with the one-line change of the integration notes
    (Q4_K admitted in allowed_storage_type's matrix branch,
    src/model/qwen35_weights.cpp:49-59), compiled into the reference's own
    bind_qwen35_weights (oracle/Makefile, target ref_gate): the Q4_K_M model
    binds through the reference's binder -- names, shapes, byte sizes and
    roles checked by the reference itself -- from a mapped GGUF file and from
    host buffers, and decodes to the same greedy tokens as the checker build
    that binds with its own gate-free binding.  The unmodified binder still
    rejects the same file (test_reference_binder_rejects_q4k)."""
    oracle = _gate_checker_or_skip()
    path, tensors = models["q4_k_m"]
    prompt = np.arange(3, 15, dtype=np.uint32) * 53 % qwen35.SMALL.vocab
    gated = oracle.Qwen35Reference("gate", gguf_path=path, max_tokens=64).greedy(prompt, 10)
    gated_buffers = oracle.Qwen35Reference("gate", tensors=tensors, manifest=qwen35.SMALL.manifest(),
                                           max_tokens=64).greedy(prompt, 10)
    own = oracle.Qwen35Reference("q8k", gguf_path=path, admit_q4k=True, max_tokens=64).greedy(prompt, 10)
    assert np.array_equal(gated, own)
    assert np.array_equal(gated_buffers, own)
    assert len(set(gated.tolist())) > 1


def test_patched_type_gate_still_checks_geometry(models):
    """The patched gate admits Q4_K but the reference binder's other checks
    stay: a Q4_K matrix with the wrong shape is still rejected with the
    reference's message."""
    oracle = _gate_checker_or_skip()
    _, tensors = models["q4_k_m"]
    bad = []
    for name, qtype, dims, data in tensors:
        if name == "blk.0.ffn_gate.weight":
            dims = (dims[0], dims[1] - 1)
            data = data[: len(data) - dims[0] // 256 * 144]
        bad.append((name, qtype, dims, data))
    with pytest.raises(oracle.ReferenceError_, match="blk.0.ffn_gate.weight: expected dimensions"):
        oracle.Qwen35Reference("gate", tensors=bad, manifest=qwen35.SMALL.manifest(), max_tokens=64)
