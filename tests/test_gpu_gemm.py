"""Prefill dequant-GEMM on the tensor cores (oracle_cuda_prefill_gemm).

Expected values come from the C restatement (oracle/quant_oracle.c,
oq_gemm_sampled), evaluated in double at sampled (m, n) pairs:
  * mode 1 (both operands rounded to bf16, as the kernel multiplies them): the
    kernel may differ only by its f32 accumulation, |got - ref| <= 1e-4 *
    sum|x*w| per element;
  * mode 0 (f32 operands): the north star's bf16-GEMM tolerance, 1e-2
    relative, taken normwise over the sampled elements.
"""
import numpy as np
import pytest
import torch

import oracle_b200 as ob
from oracle_b200 import synth

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def run_gemm(ctx, w, x, n, k, m):
    wd = torch.from_numpy(np.ascontiguousarray(w).reshape(-1)).to(DEV)
    xd = torch.from_numpy(np.ascontiguousarray(x, np.float32).reshape(-1)).to(DEV)
    y = torch.full((m * n,), float("nan"), dtype=torch.float32, device=DEV)
    ctx.prefill_gemm(ob.TYPE_Q4_K, n, k, wd, xd, m, y)
    ctx.device_status()
    return y.cpu().numpy().reshape(m, n)


def check(port, w, x, n, k, m, got, mi, ni):
    ref1 = port.gemm_sampled(ob.TYPE_Q4_K, n, k, w, x, mi, ni, 1)
    scale = port.gemm_sampled(ob.TYPE_Q4_K, n, k, w, x, mi, ni, 2)
    ref0 = port.gemm_sampled(ob.TYPE_Q4_K, n, k, w, x, mi, ni, 0)
    g = got[mi, ni].astype(np.float64)
    assert np.all(np.isfinite(g))
    err = np.abs(g - ref1)
    bad = err > 1e-4 * scale + 1e-6
    assert not bad.any(), (int(bad.sum()), float((err / (scale + 1e-30)).max()))
    rel = np.linalg.norm(g - ref0) / max(np.linalg.norm(ref0), 1e-30)
    assert rel <= 1e-2, rel


def sample(rng, m, n, count):
    mi = np.concatenate([rng.integers(0, m, count), [0, m - 1, 0, m - 1]])
    ni = np.concatenate([rng.integers(0, n, count), [0, n - 1, n - 1, 0]])
    return mi, ni


@pytest.mark.parametrize("n,k,m", [(128, 256, 256), (256, 1024, 64), (200, 512, 300), (384, 2048, 512),
                                   (128, 256, 1)])
def test_gemm_every_element(ctx, port, n, k, m):
    w = synth.weight(ob.TYPE_Q4_K, n, k, "gemm", f"w_{n}_{k}")
    x = synth.activations(k, m, "gemm", f"x_{k}_{m}")
    got = run_gemm(ctx, w, x, n, k, m)
    mi, ni = np.meshgrid(np.arange(m), np.arange(n), indexing="ij")
    check(port, w, x, n, k, m, got, mi.reshape(-1), ni.reshape(-1))


@pytest.mark.parametrize("n,k,m", [(12288, 4096, 512), (4096, 12288, 512), (12288, 4096, 2048)])
def test_gemm_config4(ctx, port, n, k, m):
    """BASELINE config 4 shapes; weights generated as in config 2."""
    w = synth.weight(ob.TYPE_Q4_K, n, k, "config4", f"W_{k}_{n}")
    x = synth.activations(k, m, "config4", f"X_{k}_{m}")
    got = run_gemm(ctx, w, x, n, k, m)
    assert np.all(np.isfinite(got))
    rng = np.random.default_rng(n + k + m)
    mi, ni = sample(rng, m, n, 3000)
    check(port, w, x, n, k, m, got, mi, ni)


def test_gemm_wave_tail_split(ctx, port):
    """More tiles than SMs: whole waves of whole tiles, then the leftover weight-row
    tiles split along K (zeroed output columns, accumulation) in a second launch.
    150 tiles of 128 rows x 256 tokens: 148 whole, the last weight-row tile split in two."""
    import torch
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    n, k, m = 128 * ((sms + 2) // 2), 2048, 512
    w = synth.weight(ob.TYPE_Q4_K, n, k, "gemm", f"tail_w_{n}")
    x = synth.activations(k, m, "gemm", "tail_x")
    got = run_gemm(ctx, w, x, n, k, m)
    rng = np.random.default_rng(5)
    mi, ni = sample(rng, m, n, 1500)
    tail_rows = rng.integers(n - 256, n, 1500)  # the K-split tiles
    check(port, w, x, n, k, m, got, np.concatenate([mi, rng.integers(0, m, 1500)]), np.concatenate([ni, tail_rows]))


def test_gemm_repeatable(ctx):
    """Without a K split the result does not depend on timing: two calls agree bit for bit."""
    n, k, m = 12288, 1024, 512  # 192 tiles: no K split
    w = synth.weight(ob.TYPE_Q4_K, n, k, "gemm", "rep_w")
    x = synth.activations(k, m, "gemm", "rep_x")
    a = run_gemm(ctx, w, x, n, k, m)
    b = run_gemm(ctx, w, x, n, k, m)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_gemm_validation(ctx):
    n, k, m = 128, 256, 4
    w = torch.from_numpy(synth.weight(ob.TYPE_Q4_K, n, k, "gemm", "val").reshape(-1)).to(DEV)
    x = torch.zeros(m * k + 4, dtype=torch.float32, device=DEV)
    y = torch.empty(m * n, dtype=torch.float32, device=DEV)
    with pytest.raises(ob.Unsupported):
        ctx.prefill_gemm(ob.TYPE_Q6_K, n, k, w, x, m, y, w_nbytes=n * 210)
    with pytest.raises(ob.InvalidArgument, match="byte size mismatch"):
        ctx.prefill_gemm(ob.TYPE_Q4_K, n, k, w, x, m, y, w_nbytes=n * 144 - 1)
    with pytest.raises(ob.InvalidArgument, match="16-byte aligned"):
        ctx.prefill_gemm(ob.TYPE_Q4_K, n, k, w, x[1:], m, y)
    with pytest.raises(ob.RuntimeError_, match="not divisible by block size"):
        ctx.prefill_gemm(ob.TYPE_Q4_K, n, 200, w, x, m, y)
    ctx.device_status()


def test_gemm_cta_pair_mode(port, monkeypatch):
    """The CTA-pair kernel (tcgen05.mma cta_group::2, ORACLE_CUDA_GEMM_PAIR=1) gives the same products."""
    monkeypatch.setenv("ORACLE_CUDA_GEMM_PAIR", "1")
    with ob.Context(0) as ctx2:
        for n, k, m in [(256, 512, 300), (384, 1024, 64), (1024, 4096, 512)]:
            w = synth.weight(ob.TYPE_Q4_K, n, k, "gemm", f"pair_w_{n}_{k}")
            x = synth.activations(k, m, "gemm", f"pair_x_{k}_{m}")
            got = run_gemm(ctx2, w, x, n, k, m)
            rng = np.random.default_rng(n + k)
            mi, ni = sample(rng, m, n, 2000)
            check(port, w, x, n, k, m, got, mi, ni)
