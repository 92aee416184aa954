"""Embedding gather and greedy argmax on the GPU against Oracle's own code.

Gather: every output row must equal the reference's decode of the token's
row (decode_storage_row, via the C restatement pinned to it) bit for bit; an
out-of-range id must be reported as OUT_OF_RANGE without touching memory.
Argmax: the token must equal Oracle's compiled Sampler::sample at temperature 0
(oracle/_ref), including ties, signed zeros and the NaN / non-finite errors.
"""
import numpy as np
import pytest
import torch

import oracle_b200 as ob
from oracle_b200 import synth

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


@pytest.mark.parametrize("qtype,rows,cols", [(ob.TYPE_Q4_K, 1000, 4096), (ob.TYPE_Q6_K, 777, 1024),
                                             (ob.TYPE_Q8_0, 500, 96), (ob.TYPE_F16, 300, 37),
                                             (ob.TYPE_BF16, 64, 130), (ob.TYPE_Q5_K, 33, 512)])
def test_gather_rows(ctx, port, qtype, rows, cols):
    w = synth.weight(qtype, rows, cols, "gather", f"emb_{qtype}_{cols}")
    rng = np.random.default_rng(qtype + cols)
    ids = np.concatenate([rng.integers(0, rows, 200), [0, rows - 1, 0]]).astype(np.uint32)
    out = torch.full((ids.size * cols,), float("nan"), device=DEV)
    ctx.gather_rows(qtype, rows, cols, torch.from_numpy(w.reshape(-1)).to(DEV), torch.from_numpy(ids).to(DEV), out)
    ctx.device_status()
    want = port.decode_rows(qtype, rows, cols, w)[ids]
    assert np.array_equal(out.cpu().numpy().reshape(ids.size, cols).view(np.uint32), want.view(np.uint32))


def test_gather_rows_out_of_range(ctx, port):
    rows, cols = 64, 256
    w = synth.weight(ob.TYPE_Q4_K, rows, cols, "gather", "oor")
    ids = np.array([3, 64, 5], np.uint32)
    out = torch.zeros(ids.size * cols, device=DEV)
    ctx.gather_rows(ob.TYPE_Q4_K, rows, cols, torch.from_numpy(w.reshape(-1)).to(DEV),
                    torch.from_numpy(ids).to(DEV), out)
    with pytest.raises(ob.OutOfRange, match="token id 64 exceeds the embedding row count"):
        ctx.device_status()
    got = out.cpu().numpy().reshape(3, cols)
    dec = port.decode_rows(ob.TYPE_Q4_K, rows, cols, w)
    assert np.array_equal(got[0], dec[3]) and np.array_equal(got[2], dec[5]) and not got[1].any()
    ctx.device_status()  # reported once


def _logit_cases():
    rng = np.random.default_rng(5)
    big = rng.standard_normal(151936).astype(np.float32)
    tie = big.copy()
    tie[[100, 90000, 151935]] = tie.max() + 1.0  # first of three equal maxima wins
    zeros = np.zeros(1000, np.float32)
    zeros[:500] = -0.0
    neg = -np.abs(rng.standard_normal(4097)).astype(np.float32)
    neg[17] = -np.inf
    return [big, tie, zeros, neg, np.array([2.5], np.float32), np.array([-np.inf, 1.0, -np.inf], np.float32)]


@pytest.mark.parametrize("case", range(6))
def test_greedy_token_matches_reference(ctx, ref, case):
    logits = _logit_cases()[case]
    assert ctx.greedy_token(torch.from_numpy(logits).to(DEV)) == ref.greedy_token(logits)


@pytest.mark.parametrize("bad,message", [([1.0, float("nan"), 3.0], "logits contain NaN"),
                                         ([1.0, float("inf")], "logits contain no finite candidates"),
                                         ([float("-inf")] * 5, "logits contain no finite candidates")])
def test_greedy_token_errors(ctx, ref, bad, message):
    logits = np.array(bad, np.float32)
    with pytest.raises(ob.InvalidArgument, match=message):
        ctx.greedy_token(torch.from_numpy(logits).to(DEV))
    with pytest.raises(Exception, match=message):
        ref.greedy_token(logits)


def test_argmax_keys_combine_over_shards(ctx, ref):
    """Row-sharded logits: one key per shard (with its token-id base); the largest key is the answer."""
    logits = _logit_cases()[1]
    parts = np.array_split(np.arange(logits.size), 8)
    keys = torch.zeros(8, dtype=torch.int64, device=DEV)
    x = torch.from_numpy(logits).to(DEV)
    for i, p in enumerate(parts):
        ctx.argmax(x[p[0]:p[-1] + 1], keys[i:i + 1], index_base=int(p[0]))
    torch.cuda.synchronize()
    best = max(int(k) & 0xFFFFFFFFFFFFFFFF for k in keys.cpu().tolist())
    assert ob.argmax_decode(best) == ref.greedy_token(logits)
