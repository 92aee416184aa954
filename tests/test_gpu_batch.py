"""GPU: the batched Q8_K matvec (2..16 vectors per launch, matvec_batch.cuh).

Bar: bit-exact, vector by vector, with the restatement's Q8_K dot
(``oq_vec_dot_q8_k``, canonical order) -- the same bar as the batch-1 kernels.
The shapes cover one and several 16-super-block segments (the multi-segment
path combines per-tile partial sums in a second step), a ragged last segment,
Q6_K rows whose starts are not 16-byte aligned (odd super-block counts), row
counts that leave a partial 8-row tile, and batches that are not a multiple
of 16 (a remainder of one goes through the batch-1 kernel).
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle_b200 as ob
from oracle_b200 import synth

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def to_dev(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a).reshape(-1)).to(DEV)


def bits_equal(a, b) -> bool:
    a = np.asarray(a, np.float32).reshape(-1)
    b = np.asarray(b, np.float32).reshape(-1)
    return bool(np.all((a.view(np.uint32) == b.view(np.uint32)) | (np.isnan(a) & np.isnan(b))))


SHAPES = [(1, 256), (8, 256), (13, 768), (37, 4096), (300, 4096), (64, 4352), (77, 8192), (40, 12288),
          (9, 12800), (2000, 2048)]


@pytest.mark.parametrize("qtype", [ob.TYPE_Q4_K, ob.TYPE_Q6_K])
@pytest.mark.parametrize("rows,k", SHAPES)
@pytest.mark.parametrize("batch", [2, 16])
def test_batch_matvec_bit_exact(ctx, port, qtype, rows, k, batch):
    w = synth.weight(qtype, rows, k, "gpu", f"bmv_{qtype}_{rows}_{k}")
    x = synth.activations(k, batch, "gpu", f"bmv_x_{k}_{batch}")
    want = port.matvec_q8_k(qtype, rows, k, w, port.quantize_q8_k(x))
    y = torch.full((batch * rows,), float("nan"), dtype=torch.float32, device=DEV)
    wd, xd = to_dev(w), to_dev(x)
    ctx.storage_matvec(ob.CONTRACT_Q8K, qtype, rows, k, wd, xd, y)
    ctx.device_status()
    got = y.cpu().numpy().reshape(batch, rows)
    for b in range(batch):
        assert bits_equal(got[b], want[b]), (b, int(np.argmax(got[b].view(np.uint32) != want[b].view(np.uint32))))
    # a second call reuses the per-tile counters (reset by the last arrival)
    y.fill_(float("nan"))
    ctx.storage_matvec(ob.CONTRACT_Q8K, qtype, rows, k, wd, xd, y)
    ctx.device_status()
    assert bits_equal(y.cpu().numpy(), want)


@pytest.mark.parametrize("batch", [3, 7, 15, 17, 33])
def test_batch_sizes(ctx, port, batch):
    """Batches below 16 (zero vectors fill the MMA's rows) and above (chunks of
    16, a remainder of one on the batch-1 kernel)."""
    rows, k = 123, 4608
    for qtype in (ob.TYPE_Q4_K, ob.TYPE_Q6_K):
        w = synth.weight(qtype, rows, k, "gpu", f"bsz_{qtype}")
        x = synth.activations(k, batch, "gpu", f"bsz_x_{batch}")
        want = port.matvec_q8_k(qtype, rows, k, w, port.quantize_q8_k(x))
        y = torch.empty(batch * rows, dtype=torch.float32, device=DEV)
        ctx.storage_matvec(ob.CONTRACT_Q8K, qtype, rows, k, to_dev(w), to_dev(x), y)
        ctx.device_status()
        assert bits_equal(y.cpu().numpy(), want), (qtype, batch)


def test_batch_equals_single_vector_calls(ctx):
    """Each vector of a batch gets the bits a batch-1 call gives it."""
    rows, k, batch = 4096, 12288, 16
    w = to_dev(synth.weight(ob.TYPE_Q4_K, rows, k, "gpu", "bsingle"))
    x = synth.activations(k, batch, "gpu", "bsingle_x")
    yb = torch.empty(batch * rows, dtype=torch.float32, device=DEV)
    ctx.storage_matvec(ob.CONTRACT_Q8K, ob.TYPE_Q4_K, rows, k, w, to_dev(x), yb)
    for b in range(batch):
        y1 = torch.empty(rows, dtype=torch.float32, device=DEV)
        ctx.storage_matvec(ob.CONTRACT_Q8K, ob.TYPE_Q4_K, rows, k, w, to_dev(x[b]), y1)
        assert torch.equal(y1.view(torch.int32), yb[b * rows:(b + 1) * rows].view(torch.int32)), b
    ctx.device_status()


def test_batch_special_values(ctx, port):
    """Zero vectors (d_x = 0), a zero weight row, and huge activations."""
    rows, k, batch = 24, 4096, 4
    for qtype in (ob.TYPE_Q4_K, ob.TYPE_Q6_K):
        w = synth.weight(qtype, rows, k, "gpu", f"bspec_{qtype}")
        w = w.copy()
        w[3] = 0
        x = synth.activations(k, batch, "gpu", "bspec_x").reshape(batch, k).copy()
        x[1] = 0.0
        x[2, 7] = 3.0e38
        want = port.matvec_q8_k(qtype, rows, k, w, port.quantize_q8_k(x))
        y = torch.empty(batch * rows, dtype=torch.float32, device=DEV)
        ctx.storage_matvec(ob.CONTRACT_Q8K, qtype, rows, k, to_dev(w), to_dev(x), y)
        ctx.device_status()
        assert bits_equal(y.cpu().numpy(), want), qtype


@pytest.mark.parametrize("batch,cols", [(16, 4096), (5, 512), (1, 8192)])
def test_fused_norm_quantize_equals_separate_kernels(ctx, batch, cols):
    """oracle_cuda_batch_norm_quantize gives the image (and the residual sum)
    of the separate add, rms_norm_rows and batch_quantize launches, byte for
    byte."""
    a = to_dev(synth.activations(cols, batch, "glue", "a"))
    b = to_dev(synth.activations(cols, batch, "glue", "b"))
    w = to_dev(synth.activations(cols, 1, "glue", "w"))
    eps = float(np.float32(1e-6))
    nbytes = ob.Context.batch_image_bytes(cols)
    want, got = (torch.zeros(nbytes, dtype=torch.uint8, device=DEV) for _ in range(2))
    s_want, normed = (torch.zeros(batch * cols, device=DEV) for _ in range(2))
    s_got = torch.full((batch * cols,), 7.0, device=DEV)
    ctx.add(a, b, batch * cols, s_want)
    ctx.rms_norm_rows(s_want, w, batch, cols, eps, normed)
    ctx.batch_quantize(normed, cols, batch, want)
    ctx.batch_norm_quantize(a, b, s_got, w, eps, cols, batch, got)
    torch.cuda.synchronize()
    assert torch.equal(want, got) and bits_equal(s_want.cpu(), s_got.cpu())
    ctx.rms_norm_rows(a, w, batch, cols, eps, normed)            # no residual add, no sum written
    ctx.batch_quantize(normed, cols, batch, want)
    ctx.batch_norm_quantize(a, None, None, w, eps, cols, batch, got)
    torch.cuda.synchronize()
    ctx.device_status()
    assert torch.equal(want, got)
    with pytest.raises(ob.InvalidArgument):
        ctx.batch_norm_quantize(a, b, a, w, eps, cols, batch, got)   # the sum would overwrite an input
