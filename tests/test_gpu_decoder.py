"""GPU: greedy decoding of the Qwen3.5 hybrid model against Oracle's own decode loop.

The checker is the reference's execute_qwen35_reference_token and greedy
Sampler compiled from its sources (oracle/ref_qwen35.cpp):

* ``q8k``: the Q4_K_M model, projections on GGML's Q8_K contract in both
  (the checker build routes Q4_K / Q6_K projections to the restatement of
  GGML's quantizer and integer dots; the GPU runs the matvec program);
* ``f32``: a model of the storage types Oracle admits, decoded by the
  UNMODIFIED reference from a GGUF file, and by the GPU with Oracle's f32
  contract from the same file.

Criterion: identical greedy tokens (the north star's decoder bar).  Logits of
the first steps are also compared: the matvecs are bit-identical and exp /
log1p reproduce the host C library's results bit for bit (the decoder's
correction tables), so the only remaining freedom is the order of double sums
inside RMSNorm / attention / gated delta, which changes a float result only
when a double sum straddles a float rounding boundary; the bound kept here is
1e-3 of the logits' standard deviation (measured: 0 on the q8k model).
"""
from __future__ import annotations

import numpy as np
import pytest

from oracle_b200 import qwen35

pytestmark = pytest.mark.gpu
pytest.importorskip("gguf")

PROMPT = (np.arange(16, dtype=np.uint64) * 2654435761 % qwen35.SMALL.vocab).astype(np.uint32)


@pytest.fixture(scope="module")
def gguf_models(tmp_path_factory):
    d = tmp_path_factory.mktemp("qwen35gpu")
    out = {}
    for recipe in ("oracle", "q4_k_m"):
        tensors = qwen35.synthetic_model(qwen35.SMALL, recipe)
        path = str(d / f"{recipe}.gguf")
        qwen35.write_gguf(path, qwen35.SMALL, tensors)
        out[recipe] = path
    return out


def _checker(contract, path):
    import oracle
    if not oracle.ref_available():
        pytest.skip("reference checker library not built")
    return oracle.Qwen35Reference(contract, gguf_path=path, admit_q4k=contract == "q8k", max_tokens=512)


def _decoder(ctx, path, contract, **kw):
    from oracle_b200.decoder import Qwen35Decoder, tensors_from_gguf
    cfg, tensors = tensors_from_gguf(path)
    return Qwen35Decoder(ctx, cfg, tensors, contract=contract, **kw)


@pytest.mark.parametrize("contract,recipe", [("q8k", "q4_k_m"), ("f32", "oracle")])
def test_greedy_tokens_match_reference(ctx, gguf_models, contract, recipe):
    path = gguf_models[recipe]
    want = _checker(contract, path).greedy(PROMPT, 48)
    dec = _decoder(ctx, path, contract, capacity=512, max_new=64)
    got = dec.generate(PROMPT, 48)
    assert np.array_equal(got, want), (got.tolist(), want.tolist())
    # a second generation from the same decoder (state reset, graph reused)
    assert np.array_equal(dec.generate(PROMPT, 48), want)


@pytest.mark.parametrize("contract,recipe", [("q8k", "q4_k_m"), ("f32", "oracle")])
def test_step_logits_close_to_reference(ctx, gguf_models, contract, recipe):
    path = gguf_models[recipe]
    ref = _checker(contract, path)
    dec = _decoder(ctx, path, contract, capacity=512, max_new=64)
    dec.start(PROMPT)
    for t in PROMPT[:6]:
        want = ref.forward(int(t))
        got = dec.forward(int(t))
        assert int(np.argmax(got)) == int(np.argmax(want))
        assert np.abs(got - want).max() <= 1e-3 * want.std(), np.abs(got - want).max()


def test_kv_capacity_overflow_reported(ctx, gguf_models):
    import oracle_b200 as ob
    dec = _decoder(ctx, gguf_models["q4_k_m"], "q8k", capacity=8, max_new=8)
    with pytest.raises(ob.Overflow, match="KV cache capacity exceeded"):
        dec.generate(PROMPT[:6], 4)
    ctx.device_status()  # cleared: the context stays usable
    assert len(dec.generate(PROMPT[:4], 4)) == 4


def test_fused_step_matches_unfused(ctx, gguf_models):
    """The fused step (one matvec program per block boundary with norms, SwiGLU
    and residual adds inside; one kernel per block core) against the step of
    separate kernels: same tokens, logits equal up to the order of the double
    sums inside RMSNorm (float results differ in rare last-bit cases)."""
    path = gguf_models["q4_k_m"]
    fused = _decoder(ctx, path, "q8k", capacity=512, max_new=64, fused=True)
    plain = _decoder(ctx, path, "q8k", capacity=512, max_new=64, fused=False)
    assert np.array_equal(fused.generate(PROMPT, 32), plain.generate(PROMPT, 32))
    fused.start(PROMPT)
    plain.start(PROMPT)
    for t in PROMPT[:4]:
        a, b = fused.forward(int(t)), plain.forward(int(t))
        assert np.abs(a - b).max() <= 1e-4 * b.std()
    assert 4 * fused.launches_per_step() <= plain.launches_per_step()
