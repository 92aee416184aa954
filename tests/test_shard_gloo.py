"""Row sharding + all-gather, checked on CPU with two gloo ranks.

Each rank computes its rows of several matvecs with the CPU restatement, packs
them, all-gathers over gloo and unpacks; the result must equal the unsharded
matvec bit for bit (rows are independent, so sharding cannot change a value).
The GPU benchmark uses the same plan with NCCL.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle_b200.shard import PackPlan, RowShard

TYPE_Q4_K, TYPE_Q6_K = 12, 14
MATS = [(TYPE_Q4_K, 512, 96), (TYPE_Q4_K, 768, 32), (TYPE_Q6_K, 256, 64)]  # (type, K, N)


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
        plan = PackPlan([n for _, _, n in MATS], world, rank)
        pack = np.empty(plan.pack_len, np.float32)
        fulls, wants = [], []
        for (t, k, n), shard, off in zip(MATS, plan.shards, plan.offsets):
            w = synth.weight(t, n, k, "shard", f"w_{t}_{k}_{n}")
            x = synth.activations(k, 1, "shard", f"x_{k}")
            q8 = o.quantize_q8_k(x)
            pack[off:off + shard.local_rows] = o.matvec_q8_k(t, shard.local_rows, k, shard.weight_slice(w), q8)[0]
            wants.append(o.matvec_q8_k(t, n, k, w, q8)[0])
        parts = [torch.empty(plan.pack_len) for _ in range(world)]
        dist.all_gather(parts, torch.from_numpy(pack))
        got = plan.unpack(torch.stack(parts).numpy())
        ok = all(np.array_equal(g.view(np.uint32), w_.view(np.uint32)) for g, w_ in zip(got, wants))
        dist.destroy_process_group()
        q.put((rank, ok, ""))
    except Exception as e:  # reported to the parent, which fails the test
        q.put((rank, False, repr(e)))


@pytest.mark.parametrize("world", [2])
def test_sharded_matvec_all_gather_gloo(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    assert all(ok for _, ok, _ in results), results


def test_row_shard_plan():
    s = RowShard(151936, 8, 3)
    assert (s.local_rows, s.begin, s.end) == (18992, 56976, 75968)
    with pytest.raises(ValueError):
        RowShard(100, 8, 0)
    with pytest.raises(ValueError):
        RowShard(128, 2, 2)
    plan = PackPlan([12288, 4096, 4096], 4, 1)
    assert plan.offsets == [0, 3072, 4096] and plan.pack_len == 5120
    g = np.arange(4 * 5120, dtype=np.float32).reshape(4, 5120)
    y0, y1, _ = plan.unpack(g)
    assert y0[3072] == g[1, 0] and y1[1023] == g[0, 3072 + 1023] and y1.size == 4096
