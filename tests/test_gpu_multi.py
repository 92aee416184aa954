"""Row-sharded matvec programs over two GPUs with the all-gather inside the
kernel (oracle_cuda_matvec_program_allgather).

Two child processes (one per GPU, spawned) exchange CUDA IPC handles over a
gloo group, run the program on their halves of every matrix and must each end
up with every row, bit-identical to the unsharded CPU restatement.  The last
case has rank 1 skip one launch: rank 0's kernel must give up after its
bounded wait and report a device timeout, and the context must stay usable.
Needs two GPUs; skipped otherwise.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

MATS = [(12, 1024, 256), (14, 512, 128), (12, 2048, 64), (12, 4096, 512)]  # (type, K, N)


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
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
        import oracle
        import oracle_b200 as ob
        from oracle_b200 import synth
        from oracle_b200.shard import PackPlan
        o = oracle.port()
        dev = torch.device("cuda", rank)
        plan = PackPlan([n for _, _, n in MATS], world, rank)
        ctx = ob.Context(rank)
        group = ob.PeerGroup(ctx, rank, world, world * plan.pack_len * 4)
        handles = [None] * world
        dist.all_gather_object(handles, group.handle)
        group.connect(handles)
        gathered = group.tensor()[:world * plan.pack_len]
        mine = gathered[rank * plan.pack_len:(rank + 1) * plan.pack_len]
        ops, wants, keep = [], [], []
        for (t, k, n), sh, off in zip(MATS, plan.shards, plan.offsets):
            w = synth.weight(t, n, k, "multi", f"w_{t}_{k}_{n}")
            x = synth.activations(k, 1, "multi", f"x_{k}")
            wd = torch.from_numpy(np.ascontiguousarray(sh.weight_slice(w)).reshape(-1)).to(dev)
            xd = torch.from_numpy(x.reshape(-1)).to(dev)
            keep += [wd, xd]
            ops.append((t, sh.local_rows, k, wd, xd, mine[off:off + sh.local_rows], 0))
            wants.append(o.matvec_q8_k(t, n, k, w, o.quantize_q8_k(x))[0])
        ok = True
        for it in range(3):
            gathered.fill_(float("nan"))
            torch.cuda.synchronize()
            dist.barrier()
            ctx.matvec_program_allgather(group, ops)
            torch.cuda.synchronize()
            ctx.device_status()
            got = plan.unpack(gathered.cpu().numpy())
            ok = ok and all(np.array_equal(g.view(np.uint32), w_.view(np.uint32)) for g, w_ in zip(got, wants))
            dist.barrier()
        # failure detection: rank 1 does not launch; rank 0 must time out (bounded) and report it
        timed_out = None
        if rank == 0:
            ctx.matvec_program_allgather(group, ops)
            torch.cuda.synchronize()
            try:
                ctx.device_status()
                timed_out = False
            except ob.DeviceTimeout:
                timed_out = True
            ctx.selftest_bounded_wait(1_000_000)  # the context still runs kernels
            try:
                ctx.device_status()
            except ob.DeviceTimeout:
                pass
        dist.barrier()
        group.close()
        ctx.close()
        dist.destroy_process_group()
        q.put((rank, ok, timed_out, ""))
    except Exception as e:  # reported to the parent, which fails the test
        q.put((rank, False, None, repr(e)))


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_program_allgather_two_gpus():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = sorted(q.get(timeout=600) for _ in range(2))
    for p in procs:
        p.join(timeout=120)
    assert all(ok for _, ok, _, _ in results), results
    assert results[0][2] is True, results  # rank 0 saw the bounded peer wait expire
