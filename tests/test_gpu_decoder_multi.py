"""GPU x2: the hybrid decoder split over two GPUs (tensor parallel).

Every projection's rows are split between the ranks; the matvec programs fill
a peer group's gather buffer on both GPUs over NVLink and their in-kernel
dependencies wait for both ranks (oracle_cuda_matvec_program_ex_allgather).
Checked: the logits of a step on each rank are bit-identical to the
single-GPU decoder's, and both ranks' greedy tokens equal Oracle's own decode
loop (the Q8_K checker build).  Two child processes (spawned), gloo for the
handle exchange, NVLS off.  Needs two GPUs; skipped otherwise.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


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
        import oracle_b200 as ob
        from oracle_b200 import qwen35
        from oracle_b200.decoder import Qwen35Decoder

        def exchange(handle):
            hs = [None] * world
            dist.all_gather_object(hs, handle)
            return hs

        cfg = qwen35.SMALL
        tensors = qwen35.synthetic_model(cfg, "q4_k_m")
        prompt = (np.arange(16, dtype=np.uint64) * 2654435761 % cfg.vocab).astype(np.uint32)
        ctx = ob.Context(rank)
        dec = Qwen35Decoder(ctx, cfg, tensors, capacity=256, max_new=64, device=rank, rank=rank, world=world,
                            exchange=exchange)
        tokens = dec.generate(prompt, 32)
        dec.start(prompt)
        logits = [dec.forward(int(t)) for t in prompt[:3]]
        result = {"tokens": tokens.tolist(), "logits_same": None, "want": None}
        if rank == 0:
            single = Qwen35Decoder(ctx, cfg, tensors, capacity=256, max_new=64, device=0)
            single.start(prompt)
            ref_logits = [single.forward(int(t)) for t in prompt[:3]]
            result["logits_same"] = all(np.array_equal(a.view(np.uint32), b.view(np.uint32))
                                        for a, b in zip(logits, ref_logits))
            import oracle
            result["want"] = oracle.Qwen35Reference("q8k", tensors=tensors, manifest=cfg.manifest(),
                                                    admit_q4k=True, max_tokens=256).greedy(prompt, 32).tolist()
        dist.barrier()
        dec.close()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, result))
    except Exception as e:  # pragma: no cover - reported to the parent
        q.put((rank, repr(e)))


def test_decoder_two_gpus_matches_one_gpu_and_reference():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    pytest.importorskip("gguf")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = dict(q.get(timeout=600) for _ in procs)
    for p in procs:
        p.join(timeout=120)
    for r in range(2):
        assert isinstance(out[r], dict), out[r]
    assert out[0]["logits_same"] is True
    assert out[0]["tokens"] == out[0]["want"]
    assert out[1]["tokens"] == out[0]["want"]
