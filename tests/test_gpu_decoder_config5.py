"""GPU: the full config-5 decoder against Oracle's own greedy tokens.

The fixture ``tests/golden/config5_tokens.npz`` holds the 256 greedy tokens
Oracle's decode loop produced (``execute_qwen35_reference_token`` on its
``HybridCache`` with the greedy ``Sampler``, src/runtime/qwen35_generation.cpp:
718-1380 and src/runtime/sampler.cpp:22, compiled from its sources with the
Q8_K projection contract) for the seeded 128-token prompt over the full
32-block Qwen3.5-style model of ``oracle_b200.qwen35.CONFIG5`` with the Q4_K_M
recipe -- the model ``bench.py --workload config5`` decodes.  The script that
made it is ``tests/golden/make_config5_tokens.py`` (about half an hour of one
CPU core).

The GPU decoder must produce the same 256 tokens, token for token (the north
star's decoder bar).  The smallest top-2 logit margin on Oracle's side is
8.9e-5 (step 172), so this holds only if the logits are the reference's bit
for bit: Q8_K quantization turns any last-bit difference of an activation
into a jump of one quantization step.  The fixture also records each step's
margin, so a mismatch is reported with it.
"""
from __future__ import annotations

import os

import numpy as np
import pytest

from conftest import GOLDEN

pytestmark = pytest.mark.gpu
FIXTURE = os.path.join(GOLDEN, "config5_tokens.npz")


@pytest.mark.skipif(not os.path.exists(FIXTURE), reason="config-5 token fixture not generated")
def test_config5_greedy_tokens_equal_oracle(ctx):
    import torch

    from oracle_b200 import qwen35
    from oracle_b200.decoder import Qwen35Decoder

    g = np.load(FIXTURE)
    prompt, want, margins = g["prompt"], g["tokens"], g["margins"]
    cfg = qwen35.CONFIG5
    # the fixture's prompt is the bench's (numpy default_rng(5150) over the vocabulary)
    assert np.array_equal(prompt, np.random.default_rng(5150).integers(0, cfg.vocab, 128).astype(np.uint32))
    tensors = qwen35.synthetic_model(cfg, "q4_k_m", "config5")
    dec = Qwen35Decoder(ctx, cfg, tensors, contract="q8k", capacity=cfg.context, max_new=len(want))
    del tensors
    got = dec.generate(prompt, len(want))
    torch.cuda.synchronize()
    bad = np.nonzero(got != want)[0]
    assert bad.size == 0, (f"first mismatch at step {int(bad[0])} (Oracle's top-2 margin there "
                           f"{float(margins[bad[0]]):.3g}): got {got[:int(bad[0]) + 1].tolist()}, "
                           f"want {want[:int(bad[0]) + 1].tolist()}")
