"""GPU: the head-sharded decoder (oracle_b200/tp_decoder.py).

* One GPU (world 1): the sharded step -- partial sums, the combine transform,
  announcements -- gives logits bit-identical to the single-GPU decoder's and
  the same greedy tokens, on the test-scale model.
* Two GPUs (skipped with fewer): each rank holds and computes only its own
  heads, FFN columns and vocabulary rows; the logits every rank holds after
  each step are bit-identical to the single-GPU decoder's, and both ranks'
  greedy tokens equal it (and so Oracle's decode loop, which the single-GPU
  decoder matches).  Child processes (spawned), gloo for the handle exchange,
  NVLS off.
* Argument checks of oracle_cuda_matvec_program_sharded.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

import oracle_b200 as ob
from oracle_b200 import qwen35

pytestmark = pytest.mark.gpu

PROMPT = (np.arange(12, dtype=np.uint64) * 2654435761 % qwen35.SMALL.vocab).astype(np.uint32)


def _single(ctx, cfg, tensors):
    from oracle_b200.decoder import Qwen35Decoder
    return Qwen35Decoder(ctx, cfg, tensors, capacity=256, max_new=64, device=0)


def test_world_one_matches_single_gpu_decoder():
    from oracle_b200.tp_decoder import HeadShardedDecoder
    cfg = qwen35.SMALL
    tensors = qwen35.synthetic_model(cfg, "q4_k_m")
    ctx = ob.Context(0)
    dec = HeadShardedDecoder(ctx, cfg, tensors, 0, 1, lambda h: [h], capacity=256, max_new=64, device=0)
    single = _single(ob.Context(0), cfg, tensors)
    dec.start(PROMPT)
    single.start(PROMPT)
    for t in PROMPT[:4]:
        a, b = dec.forward(int(t)), single.forward(int(t))
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    assert np.array_equal(dec.generate(PROMPT, 24), single.generate(PROMPT, 24))
    assert dec.launches_per_step() == single.launches_per_step()
    dec.close()


def test_sharded_program_argument_checks():
    ctx = ob.Context(0)
    group = ob.PeerGroup(ctx, 0, 1, 1 << 16)
    group.connect([group.handle])
    data = group.tensor()
    from oracle_b200 import synth
    w = torch.from_numpy(synth.weight(ob.TYPE_Q4_K, 64, 512, "heads", "w").reshape(-1)).cuda()
    x = torch.zeros(512, device="cuda")
    norm = torch.ones(512, device="cuda")
    base = dict(qtype=ob.TYPE_Q4_K, rows=64, cols=512, w=w, x=x, y=data[:64])
    bad = [
        [dict(base), dict(base, wait=2)],                                      # the op before does not announce
        [dict(base, wait=1)],                                                  # the first op cannot wait
        [dict(base, announce=True), dict(base, wait=2, xform=ob.XFORM_COMBINE_RMS, x2=data[1024:1536],
                                         segments=0, norm=norm, eps=1e-6)],    # no segments
        [dict(base, announce=True), dict(base, wait=1, xform=ob.XFORM_COMBINE_RMS, x2=data[1024:1536],
                                         segments=1, norm=norm, eps=1e-6)],    # a combine must wait for every rank
        [dict(base, announce=True), dict(base, wait=2, xform=ob.XFORM_COMBINE_RMS, x2=x, segments=1, norm=norm,
                                         eps=1e-6)],                           # partials outside the gather buffer
        [dict(base, wait=0, swiglu_gate=x)],                                   # SwiGLU epilogue without act
    ]
    for ops in bad:
        with pytest.raises(ob.InvalidArgument):
            ctx.matvec_program_sharded(group, ops, 0, 4)
    with pytest.raises(ob.InvalidArgument):   # more announcements than the step holds
        ctx.matvec_program_sharded(group, [dict(base, announce=True, push=True)], 3, 3)
    with pytest.raises(ob.InvalidArgument):   # tail wait without an announcement
        ctx.matvec_program_sharded(group, [dict(base)], 0, 4, tail_wait=True)
    torch.cuda.synchronize()
    group.close()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, q):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        os.environ["NCCL_NVLS_ENABLE"] = "0"
        import datetime

        import torch.distributed as dist
        torch.cuda.set_device(rank)
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
        from oracle_b200.tp_decoder import HeadShardedDecoder

        def exchange(handle):
            hs = [None] * world
            dist.all_gather_object(hs, handle)
            return hs

        cfg = qwen35.SMALL
        tensors = qwen35.synthetic_model(cfg, "q4_k_m")
        ctx = ob.Context(rank)
        dec = HeadShardedDecoder(ctx, cfg, tensors, rank, world, exchange, capacity=256, max_new=64, device=rank)
        tokens = dec.generate(PROMPT, 32)
        dec.start(PROMPT)
        logits = [dec.forward(int(t)) for t in PROMPT[:3]]
        result = {"tokens": tokens.tolist(), "logits_same": None, "want": None}
        if rank == 0:
            single = _single(ob.Context(0), cfg, tensors)
            single.start(PROMPT)
            ref_logits = [single.forward(int(t)) for t in PROMPT[:3]]
            result["logits_same"] = all(np.array_equal(a.view(np.uint32), b.view(np.uint32))
                                        for a, b in zip(logits, ref_logits))
            result["want"] = single.generate(PROMPT, 32).tolist()
        dist.barrier()
        dec.close()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, result))
    except Exception as e:  # pragma: no cover - reported to the parent
        q.put((rank, repr(e)))


def test_two_gpus_match_one_gpu():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=600) for _ in procs)
    for p in procs:
        p.join(timeout=120)
    for rank in (0, 1):
        assert isinstance(results[rank], dict), f"rank {rank}: {results[rank]}"
    assert results[0]["logits_same"]
    assert results[0]["tokens"] == results[0]["want"]
    assert results[1]["tokens"] == results[0]["want"]
