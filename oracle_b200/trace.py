"""Matvec-program launch trace: where a decode step's time goes.

``Context.set_program_trace`` makes every matvec program launched (or
captured) afterwards record global-timer stamps as its CTA 0 sees them
(include/oracle_cuda.h, oracle_cuda_set_program_trace).  ``step_breakdown``
turns the records of consecutive decode steps into per-block averages: for
each op of a program its wait for earlier ops (the in-kernel dependency, the
cross-rank one in a sharded program), its activation-image build and its rows;
the program's total; and the gap to the next program (the block core kernel
between them plus the launch handover).  Multi-rank runs cannot be profiled
with ncu, so this is how a head-sharded step is broken down.

Run as a module for the config-5 decoder (synthetic model, 32-token prompt,
40 warm-up and 20 traced graph replays), one JSON line per rank:

    python -m oracle_b200.trace single        # Qwen35Decoder, one GPU
    python -m oracle_b200.trace sharded       # HeadShardedDecoder, world 1
    python -m torch.distributed.run --nproc-per-node 2 --master-addr 127.0.0.1 \\
        -m oracle_b200.trace sharded          # HeadShardedDecoder, 2 GPUs
"""
from __future__ import annotations

import json
import os
import sys

import numpy as np

from . import TRACE_WORDS


def step_breakdown(words: np.ndarray, programs_per_step: int, steps, kind_of) -> dict:
    """words: the trace buffer (int64, word 0 = launches recorded).  steps:
    the step indices to average over (each followed by another recorded
    step).  kind_of(p) -> a label for program p of a step.  Returns
    {label: {"total", "gap_to_next", "op<k>_wait", "op<k>_build", "op<k>_rows"}}
    in microseconds."""
    n = int(words[0])
    recs = words[1:1 + n * TRACE_WORDS].reshape(n, TRACE_WORDS)
    ops_words = TRACE_WORDS - 2
    out: dict = {}
    for st in steps:
        base = st * programs_per_step
        for p in range(programs_per_step):
            r = recs[base + p]
            nxt = recs[base + p + 1]
            stamps = r[1:1 + ops_words].reshape(-1, 3)
            nops = int(np.count_nonzero(stamps[:, 2]))
            row = {"total": (r[-1] - r[0]) / 1e3, "gap_to_next": (nxt[0] - r[-1]) / 1e3}
            prev = r[0]
            for k, (w, b, e) in enumerate(stamps[:nops]):
                row[f"op{k}_wait"] = (w - prev) / 1e3
                row[f"op{k}_build"] = (b - w) / 1e3
                row[f"op{k}_rows"] = (e - b) / 1e3
                prev = e
            out.setdefault(kind_of(p), []).append(row)
    return {kind: {k: round(float(np.mean([r.get(k, 0.0) for r in rows])), 2) for k in rows[0]}
            for kind, rows in out.items()}


def _main(mode: str) -> None:
    import torch

    import oracle_b200 as ob
    from oracle_b200 import qwen35
    from oracle_b200.decoder import Qwen35Decoder
    from oracle_b200.tp_decoder import HeadShardedDecoder

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    torch.cuda.set_device(rank)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=300))

    def exchange(h):
        if world == 1:
            return [h]
        hs = [None] * world
        dist.all_gather_object(hs, h)
        return hs

    cfg = qwen35.CONFIG5
    tensors = qwen35.synthetic_model(cfg, "q4_k_m", "config5")
    ctx = ob.Context(rank)
    if mode == "single":
        dec = Qwen35Decoder(ctx, cfg, tensors, contract="q8k", capacity=1024, max_new=128, device=rank)
    else:
        dec = HeadShardedDecoder(ctx, cfg, tensors, rank, world, exchange, capacity=1024, max_new=128, device=rank)
    per_step = 1 + cfg.layers  # matvec programs per step
    records = per_step * 64
    trace = torch.zeros(1 + records * TRACE_WORDS, dtype=torch.int64, device=f"cuda:{rank}")
    ctx.set_program_trace(trace, records)
    prompt = np.random.default_rng(5150).integers(0, cfg.vocab, 32).astype(np.uint32)
    if dist:
        dist.barrier()
    dec.start(prompt)  # captures the step (its warm-up step is traced too)
    trace.zero_()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(dec.stream):
        for _ in range(40):
            dec.graph.replay()
        start.record(dec.stream)
        for _ in range(20):
            dec.graph.replay()
        end.record(dec.stream)
    dec.stream.synchronize()
    ctx.device_status()
    ms = start.elapsed_time(end) / 20

    def kind_of(p):
        if p == 0:
            return "first"
        return ("attention" if cfg.is_attention(p - 1) else "recurrent") + (" (last)" if p == cfg.layers else "")

    res = {"rank": rank, "world": world, "mode": mode, "ms_per_step": ms,
           "blocks": step_breakdown(trace.cpu().numpy(), per_step, range(30, 59), kind_of)}
    print(json.dumps(res), flush=True)
    if dist:
        dist.barrier()
    dec.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    _main(sys.argv[1] if len(sys.argv) > 1 else "sharded")
