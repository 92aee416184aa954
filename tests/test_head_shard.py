"""Head sharding of the decoder, checked on CPU.

* The shard plan of the full config-5 model at 1, 2, 4 and 8 ranks (and of
  the test-scale model at 1 and 2): every head, FFN block and vocabulary row is
  owned by exactly one rank, and the local heads map to their local key / KV
  heads by the rules the block-core kernels use.
* The partial-sum identity the sharded projections rest on: rank q computes,
  with the C restatement of the Q8_K dot, each row over its own 256-column
  blocks of every 16-block segment (a column shard of the matrix and of the
  Q8_K activation); folding the ranks' partials by the remaining strides of
  the canonical order, adding the segments and then the residual gives
  residual + (the unsharded row dot) bit for bit -- for Q4_K and Q6_K rows of
  one and of three segments.
* The same with two gloo ranks exchanging their partials (all_gather).
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle_b200 import qwen35
from oracle_b200.tp_decoder import BLOCK, SEGMENT, ShardPlan, owned_blocks, take_blocks, take_rows

TYPE_Q4_K, TYPE_Q6_K = 12, 14
Q8K_BYTES = 292


@pytest.mark.parametrize("cfg,worlds", [(qwen35.CONFIG5, (1, 2, 4, 8)), (qwen35.SMALL, (1, 2))])
def test_plan_covers_every_head_once(cfg, worlds):
    for world in worlds:
        plans = [ShardPlan.make(cfg, world, r) for r in range(world)]
        for field, total in (("value_heads", cfg.value_heads), ("q_heads", cfg.heads),
                             ("ffn_blocks", cfg.ffn // BLOCK)):
            got = sorted(h for p in plans for h in getattr(p, field))
            assert got == list(range(total)), (field, world)
        assert [(p.vocab_lo, p.vocab_hi) for p in plans] == [(r * cfg.vocab // world, (r + 1) * cfg.vocab // world)
                                                              for r in range(world)]
        for p in plans:
            for l, h in enumerate(p.value_heads):
                assert p.key_heads[l % len(p.key_heads)] == h % cfg.key_heads
            lg = len(p.q_heads) // len(p.kv_heads)
            for l, g in enumerate(p.q_heads):
                assert p.kv_heads[l // lg] == g // (cfg.heads // cfg.kv_heads)
            # a rank's heads fill whole Q8_K blocks of the output projection's input
            assert len(p.value_heads) * cfg.state_size % BLOCK == 0


def test_plan_rejects_unsplittable():
    with pytest.raises(ValueError):
        ShardPlan.make(qwen35.SMALL, 4, 0)   # 2 blocks per segment over 4 ranks
    with pytest.raises(ValueError):
        ShardPlan.make(qwen35.CONFIG5, 3, 0)
    assert owned_blocks(48, 4, 1) == [g * SEGMENT + j for g in range(3) for j in (1, 5, 9, 13)]


def fold(partials: np.ndarray, base: np.ndarray) -> np.ndarray:
    """base + the canonical fold of partials [world][segments][rows] (f32)."""
    world, segments, _ = partials.shape
    total = np.zeros(partials.shape[2], np.float32)
    for g in range(segments):
        s = [partials[q, g].astype(np.float32) for q in range(world)]
        h = world // 2
        while h >= 1:
            for q in range(h):
                s[q] = s[q] + s[q + h]
            h //= 2
        total = total + s[0]
    return base + total


def rank_partials(o, qtype, rows, k, w, q8, world, rank) -> np.ndarray:
    """[segments][rows]: this rank's partial sums, one column shard per segment."""
    nb = k // BLOCK
    blocks = owned_blocks(nb, world, rank)
    q8b = q8.reshape(nb, Q8K_BYTES)
    out = []
    for g in range((nb + SEGMENT - 1) // SEGMENT):
        seg = [b for b in blocks if b // SEGMENT == g]
        wl = take_blocks(w, qtype, (k, rows), seg)
        out.append(o.matvec_q8_k(qtype, rows, len(seg) * BLOCK, wl, np.ascontiguousarray(q8b[seg]).reshape(-1))[0])
    return np.stack(out)


@pytest.mark.parametrize("qtype,k", [(TYPE_Q4_K, 4096), (TYPE_Q4_K, 12288), (TYPE_Q6_K, 4096), (TYPE_Q6_K, 12288)])
def test_partial_fold_equals_unsharded_row(qtype, k):
    import oracle
    from oracle_b200 import synth
    o = oracle.port()
    rows = 96
    w = synth.weight(qtype, rows, k, "heads", f"w{qtype}_{k}")
    q8 = o.quantize_q8_k(synth.activations(k, 1, "heads", f"x{k}"))
    base = synth.activations(rows, 1, "heads", "base").reshape(-1)
    want = base + o.matvec_q8_k(qtype, rows, k, w, q8)[0]
    for world in (1, 2, 4, 8):
        parts = np.stack([rank_partials(o, qtype, rows, k, w, q8, world, r) for r in range(world)])
        got = fold(parts, base)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), world


def test_take_rows_and_blocks():
    from oracle_b200 import synth
    w = synth.weight(TYPE_Q4_K, 8, 1024, "heads", "small").reshape(-1)
    rb = 4 * 144
    rows = take_rows(w, TYPE_Q4_K, (1024, 8), np.array([5, 1]))
    assert np.array_equal(rows, np.concatenate([w[5 * rb:6 * rb], w[rb:2 * rb]]))
    cols = take_blocks(w, TYPE_Q4_K, (1024, 8), [3, 0]).reshape(8, 2, 144)
    full = w.reshape(8, 4, 144)
    assert np.array_equal(cols[:, 0], full[:, 3]) and np.array_equal(cols[:, 1], full[:, 0])


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, q):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        import oracle
        from oracle_b200 import synth
        o = oracle.port()
        ok = True
        for qtype, k, rows in ((TYPE_Q4_K, 12288, 64), (TYPE_Q6_K, 4096, 64)):
            w = synth.weight(qtype, rows, k, "heads-gloo", f"w{qtype}_{k}")
            q8 = o.quantize_q8_k(synth.activations(k, 1, "heads-gloo", f"x{k}"))
            base = synth.activations(rows, 1, "heads-gloo", "base").reshape(-1)
            mine = torch.from_numpy(rank_partials(o, qtype, rows, k, w, q8, world, rank).copy())
            parts = [torch.empty_like(mine) for _ in range(world)]
            dist.all_gather(parts, mine)
            got = fold(torch.stack(parts).numpy(), base)
            want = base + o.matvec_q8_k(qtype, rows, k, w, q8)[0]
            ok = ok and np.array_equal(got.view(np.uint32), want.view(np.uint32))
        dist.destroy_process_group()
        q.put((rank, ok, ""))
    except Exception as e:  # reported to the parent, which fails the test
        q.put((rank, False, repr(e)))


def test_partial_fold_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, ok, err in results:
        assert ok, f"rank {rank}: {err}"


def test_trace_step_breakdown():
    """oracle_b200.trace.step_breakdown on a hand-made trace of two steps of
    two programs (one op, then two ops)."""
    from oracle_b200 import TRACE_WORDS
    from oracle_b200.trace import step_breakdown
    recs = np.zeros((5, TRACE_WORDS), np.int64)
    t = 0
    for i in range(5):
        recs[i, 0] = t                                # consumers start
        ops = 1 if i % 2 == 0 else 2
        for k in range(ops):
            recs[i, 1 + 3 * k:4 + 3 * k] = (t + 1000, t + 3000, t + 7000)  # wait 1, build 2, rows 4 us
            t += 7000
        recs[i, -1] = t + 500                         # CTA 0 done
        t += 500 + 2000                               # 2 us to the next program
    words = np.concatenate([[5], recs.reshape(-1)])
    got = step_breakdown(words, 2, [0, 1], lambda p: f"p{p}")
    assert got["p0"] == {"total": 7.5, "gap_to_next": 2.0, "op0_wait": 1.0, "op0_build": 2.0, "op0_rows": 4.0}
    assert got["p1"]["op1_wait"] == 1.0 and got["p1"]["total"] == 14.5


@pytest.mark.parametrize("world", [2, 4, 8])
def test_announcement_counter_protocol(world):
    """The sharded programs' cross-rank protocol, modelled on the host with
    random interleavings: each rank announces dependency j of step s (adds 1
    to every peer's counter) and then waits until its own counter reaches
    (s * D + j + 1) * (world - 1) before going on (to announce j + 1, or the
    next step's first).  Whenever a wait passes, every peer has announced
    (s, j) -- the counter never fills early with later announcements -- and
    no rank deadlocks."""
    rng = np.random.default_rng(world)
    D, steps = 5, 6
    total = D * steps
    counter = [0] * world
    announced = [0] * world          # dependencies announced so far, per rank
    state = ["announce"] * world     # next action
    for _ in range(200_000):  # a deadlock runs out of moves and fails below
        if all(st == "done" for st in state):
            break
        runnable = [r for r in range(world) if state[r] != "done"]
        r = int(rng.choice(runnable))
        g = announced[r]             # the rank's current dependency (s * D + j)
        if state[r] == "announce":
            for p in range(world):
                if p != r:
                    counter[p] += 1
            announced[r] += 1
            state[r] = "wait"
        elif state[r] == "wait":
            target = g * (world - 1)  # (s * D + j + 1) * (world - 1) for the dependency just announced
            if counter[r] >= target:
                assert all(a >= g for a in announced), (r, g, announced)
                state[r] = "announce" if g < total else "done"
    assert all(st == "done" for st in state)
    assert counter == [total * (world - 1)] * world
