"""Oracle's greedy tokens for the full config-5 decoder (test fixture generator).

The checker is Oracle's own decode loop compiled from its sources
(``oracle.Qwen35Reference``, ``oracle/ref_qwen35.cpp``: the reference's
``execute_qwen35_reference_token`` on its ``HybridCache`` with the greedy
``Sampler``, src/runtime/qwen35_generation.cpp:718-1380 and
src/runtime/sampler.cpp:22) over the full 32-block Qwen3.5-style model of
``oracle_b200.qwen35.CONFIG5`` with the Q4_K_M recipe -- the same seeded bytes
``bench.py --workload config5`` decodes -- in the Q8_K checker build (Q4_K /
Q6_K projections on GGML's Q8_K contract, Q4_K admitted by the binder).

Prompt: 128 tokens from ``numpy.random.default_rng(5150)`` over the
vocabulary (bench.py's prompt).  256 new tokens, greedy.

Two workers run side by side (spawned processes, one core each):

* ``greedy`` -- ``Qwen35Reference.greedy(prompt, 256)``: the fixture's tokens;
* ``margins`` -- the same decode token by token through
  ``Qwen35Reference.forward`` with the first-maximum argmax the greedy
  ``Sampler`` uses, recording each step's top-2 logit margin so that a
  near-tie flip on the GPU is diagnosable.  Its tokens must equal the
  greedy worker's.

Output: ``config5_tokens.npz`` beside this file (prompt, tokens, margins,
the top logit per step).  About 25 minutes on one 2.7 GHz core per worker:

    python tests/golden/make_config5_tokens.py
"""
from __future__ import annotations

import multiprocessing as mp
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
OUT = os.path.join(HERE, "config5_tokens.npz")
PROMPT_LEN, N_NEW, PROMPT_SEED = 128, 256, 5150


def prompt(vocab: int) -> np.ndarray:
    return np.random.default_rng(PROMPT_SEED).integers(0, vocab, PROMPT_LEN).astype(np.uint32)


def _model():
    sys.path.insert(0, ROOT)
    from oracle_b200 import qwen35
    cfg = qwen35.CONFIG5
    return cfg, qwen35.synthetic_model(cfg, "q4_k_m", "config5")


def _worker(mode: str, q) -> None:
    sys.path.insert(0, ROOT)
    import oracle
    cfg, tensors = _model()
    p = prompt(cfg.vocab)
    ref = oracle.Qwen35Reference("q8k", tensors=tensors, manifest=cfg.manifest(), admit_q4k=True,
                                 max_tokens=PROMPT_LEN + N_NEW + 1)
    t0 = time.perf_counter()
    if mode == "greedy":
        toks = ref.greedy(p, N_NEW)
        np.save(OUT + ".greedy.npy", toks)  # kept until the fixture is written
        q.put((mode, toks, None, None, time.perf_counter() - t0))
        return
    tokens = np.zeros(N_NEW, np.uint32)
    margins = np.zeros(N_NEW, np.float32)
    top = np.zeros(N_NEW, np.float32)
    logits = None
    for t in p:
        logits = ref.forward(int(t))
    for g in range(N_NEW):
        tok = int(np.argmax(logits))           # first maximum, as Sampler::sample's strict '>'
        tokens[g] = tok
        two = np.partition(logits, -2)[-2:]
        top[g], margins[g] = logits[tok], float(two[1]) - float(two[0])
        if g + 1 < N_NEW:
            logits = ref.forward(tok)
    np.savez(OUT + ".margins.npz", tokens=tokens, margins=margins, top_logit=top)
    q.put((mode, tokens, margins, top, time.perf_counter() - t0))


def main() -> None:
    sys.path.insert(0, ROOT)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(m, q)) for m in ("greedy", "margins")]
    for pr in procs:
        pr.start()
    res = {}
    for _ in procs:
        mode, toks, margins, top, secs = q.get()
        res[mode] = (toks, margins, top)
        print(f"{mode}: {secs:.0f} s", flush=True)
    for pr in procs:
        pr.join()
    greedy, (tokens, margins, top) = res["greedy"][0], res["margins"]
    if not np.array_equal(greedy, tokens):
        raise SystemExit(f"greedy and token-by-token decodes disagree: {greedy.tolist()} vs {tokens.tolist()}")
    from oracle_b200 import qwen35
    np.savez_compressed(OUT, prompt=prompt(qwen35.CONFIG5.vocab), tokens=greedy, margins=margins, top_logit=top)
    for part in (OUT + ".greedy.npy", OUT + ".margins.npz"):
        os.remove(part)
    print(f"wrote {OUT}: min top-2 margin {margins.min():.3g} at step {int(margins.argmin())}")


if __name__ == "__main__":
    main()
