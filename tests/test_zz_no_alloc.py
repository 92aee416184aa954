"""GPU: the matvec program entry point that allocates nothing.

oracle_cuda_matvec_program_noalloc serves callers that cannot allocate device
memory -- an engine that has already reserved nearly all of HBM for its own
pools, or a latency-critical path where cudaMalloc (which can synchronise the
device) is not allowed.  Its scratch is one static device array instead of a
context's buffers.  These tests call it through the C ABI and check that two
calls in a row give exactly what the context-based oracle_cuda_matvec_program
gives (the bar for this path is bit equality), including a dependent chain
whose completion counters live in that array, that a program too large for
the array is refused, and that a device-side wait that expired is reported by
oracle_cuda_noalloc_status.  The file is collected last and also passes when
run alone in a fresh process.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle_b200 as ob
from oracle_b200 import synth

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def _dev(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a).reshape(-1)).to(DEV)


def _program(specs, cfg):
    ops_a, ops_b = [], []
    prev = None
    for i, (qtype, rows, cols, after) in enumerate(specs):
        w = _dev(synth.weight(qtype, rows, cols, cfg, f"w{i}"))
        ya = torch.full((rows,), float("nan"), dtype=torch.float32, device=DEV)
        yb = torch.full((rows,), float("nan"), dtype=torch.float32, device=DEV)
        if after:
            xa, xb = prev
        else:
            xa = xb = _dev(synth.activations(cols, 1, cfg, f"x{i}")[0])
        ops_a.append((qtype, rows, cols, w, xa, ya, after))
        ops_b.append((qtype, rows, cols, w, xb, yb, after))
        prev = (ya, yb)
    return ops_a, ops_b


SPECS = [(ob.TYPE_Q4_K, 12288, 4096, 0), (ob.TYPE_Q4_K, 4096, 12288, 1), (ob.TYPE_Q6_K, 4099, 4096, 1),
         (ob.TYPE_Q4_K, 777, 4096, 0)]


def test_noalloc_program_matches_context_program_twice():
    torch.cuda.set_device(0)
    ops_ref, ops_na = _program(SPECS, "noalloc")
    with ob.Context(0) as ctx:
        ctx.matvec_program(ops_ref)
        ctx.device_status()
    want = [op[5].cpu().numpy() for op in ops_ref]
    for _ in range(2):  # the static array keeps the previous call's contents
        for op in ops_na:
            op[5].fill_(float("nan"))
        ob.matvec_program_noalloc(ops_na)
        torch.cuda.synchronize()
        for op, y in zip(ops_na, want):
            got = op[5].cpu().numpy()
            assert np.array_equal(got.view(np.uint32), y.view(np.uint32))


def test_noalloc_program_rejects_oversize_images():
    torch.cuda.set_device(0)
    # 12 independent ops of 8192 columns: 12 * 11392 B = 136704 B of activation images > 65536
    w = _dev(synth.weight(ob.TYPE_Q4_K, 2, 8192, "noalloc", "big"))
    x = torch.zeros(8192, dtype=torch.float32, device=DEV)
    y = torch.empty(2, dtype=torch.float32, device=DEV)
    with pytest.raises(ob.InvalidArgument, match="no-allocation entry point holds at most 65536"):
        ob.matvec_program_noalloc([(ob.TYPE_Q4_K, 2, 8192, w, x, y, 0)] * 12)


def test_noalloc_status_reports_an_expired_wait():
    """A call's outputs are only complete when none of its bounded waits
    expired; oracle_cuda_noalloc_status says which.  A wait that nothing
    completes (the self-test kernel, on the array's status word) gives up
    after 2 ms and is reported; the next call clears the word."""
    torch.cuda.set_device(0)
    ob.noalloc_status(0)  # the previous calls' waits all completed
    ob.noalloc_selftest_bounded_wait(2_000_000)
    with pytest.raises(ob.DeviceTimeout, match="site 99"):
        ob.noalloc_status(0)
    ops_ref, ops_na = _program(SPECS[:2], "noalloc_status")
    with ob.Context(0) as ctx:
        ctx.matvec_program(ops_ref)
        ctx.device_status()
    ob.matvec_program_noalloc(ops_na)
    ob.noalloc_status(0)
    for a, b in zip(ops_ref, ops_na):
        assert np.array_equal(a[5].cpu().numpy().view(np.uint32), b[5].cpu().numpy().view(np.uint32))
