"""GPU: batched greedy decoding (``BatchDecoder``, several sequences in lockstep).

Bars:
* every sequence's greedy tokens equal Oracle's own decode loop on that
  sequence's prompt (the reference's execute_qwen35_reference_token with the
  greedy Sampler, compiled from its sources, Q8_K contract) -- the decoder
  bar of the single-sequence decoder;
* batching changes nothing: sequence b of a batch gets the logits, bit for
  bit, and the tokens that a batch of one gives it alone (every operation of
  the step is per sequence; the batched matvec is bit-identical per vector).
"""
from __future__ import annotations

import numpy as np
import pytest

from oracle_b200 import qwen35

pytestmark = pytest.mark.gpu
pytest.importorskip("gguf")

N_PROMPT = 16


def prompts(batch: int, seed: int = 7) -> np.ndarray:
    return np.random.default_rng(seed).integers(0, qwen35.SMALL.vocab, (batch, N_PROMPT)).astype(np.uint32)


@pytest.fixture(scope="module")
def model(tmp_path_factory):
    from oracle_b200.decoder import tensors_from_gguf
    path = str(tmp_path_factory.mktemp("qwen35batch") / "q4_k_m.gguf")
    qwen35.write_gguf(path, qwen35.SMALL, qwen35.synthetic_model(qwen35.SMALL, "q4_k_m"))
    cfg, tensors = tensors_from_gguf(path)
    return path, cfg, tensors


def _decoder(ctx, model, batch, **kw):
    from oracle_b200.batch_decoder import BatchDecoder
    _, cfg, tensors = model
    return BatchDecoder(ctx, cfg, tensors, batch, capacity=256, max_new=64, **kw)


def test_batch_tokens_match_reference(ctx, model):
    import oracle
    if not oracle.ref_available():
        pytest.skip("reference checker library not built")
    path = model[0]
    ps = prompts(4)
    dec = _decoder(ctx, model, 4)
    got = dec.generate(ps, 40)
    for b in range(4):
        ref = oracle.Qwen35Reference("q8k", gguf_path=path, admit_q4k=True, max_tokens=512)
        want = ref.greedy(ps[b], 40)
        assert np.array_equal(got[b], want), (b, got[b].tolist(), want.tolist())
    # the graph is reused for a second generation from a clean state
    assert np.array_equal(dec.generate(ps, 40), got)


def test_batch_logits_equal_single_sequence(ctx, model):
    ps = prompts(3, seed=11)
    many = _decoder(ctx, model, 3)
    ones = [_decoder(ctx, model, 1) for _ in range(3)]
    many.start(ps)
    for one, p in zip(ones, ps):
        one.start(p[None, :])
    for step in range(6):
        a = many.forward(ps[:, step])
        for b, one in enumerate(ones):
            lb = one.forward(ps[b:b + 1, step])[0]
            assert np.array_equal(a[b].view(np.uint32), lb.view(np.uint32)), (step, b)


def test_batch16_tokens_equal_single_sequence(ctx, model):
    ps = prompts(16, seed=3)
    got = _decoder(ctx, model, 16).generate(ps, 24)
    one = _decoder(ctx, model, 1)
    for b in range(16):
        assert np.array_equal(one.generate(ps[b:b + 1], 24)[0], got[b]), b


def test_batch_decoder_rejects_bad_shapes(ctx, model):
    from oracle_b200.batch_decoder import BatchDecoder
    _, cfg, tensors = model
    with pytest.raises(ValueError):
        BatchDecoder(ctx, cfg, tensors, 17)
    dec = _decoder(ctx, model, 2)
    with pytest.raises(ValueError):
        dec.generate(prompts(3), 4)
