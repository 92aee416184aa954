"""Decoder glue kernels against Oracle's own compiled CPU functions.

RoPE, attention, depthwise convolution and gated-delta are compared with the
reference's reference_kernels.cpp compiled into oracle/_ref; RMSNorm and
SwiGLU (anonymous-namespace helpers of qwen35_block.cpp) with their C
restatement.  Bit-exact where the kernel keeps the reference's operations and
order (RoPE, RMSNorm, residual add); elsewhere the differences are CUDA's
expf (within 2 ulp of glibc's) and the order of double sums, and the bound is
1e-5 relative / 1e-6 absolute, the north star's matvec tolerance.  Shapes are
config 5's: 32 query / 4 KV heads of 128, partial RoPE over 64 dimensions,
32 gated-delta heads with 128 x 128 state, conv width 4.
"""
import numpy as np
import pytest
import torch

import oracle_b200 as ob

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
RNG = np.random.default_rng(35)


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(DEV)


def close(got, want, rel=1e-5, ab=1e-6):
    got, want = np.asarray(got, np.float64), np.asarray(want, np.float64)
    bad = np.abs(got - want) > ab + rel * np.abs(want)
    assert not bad.any(), (int(bad.sum()), float(np.abs(got - want).max()))


def bits(a, b):
    return np.array_equal(np.asarray(a, np.float32).view(np.uint32), np.asarray(b, np.float32).view(np.uint32))


@pytest.mark.parametrize("rows,width", [(1, 4096), (16, 4096), (3, 128), (7, 1000)])
def test_rms_norm_rows(ctx, port, rows, width):
    x = (RNG.standard_normal((rows, width)) * 3).astype(np.float32)
    w = RNG.standard_normal(width).astype(np.float32)
    out = torch.empty(rows * width, device=DEV)
    ctx.rms_norm_rows(dev(x), dev(w), rows, width, 1e-6, out)
    ctx.device_status()
    assert bits(out.cpu().numpy().reshape(rows, width), port.rms_norm_rows(x, w, 1e-6))


@pytest.mark.parametrize("heads,position,sections", [(32, (0, 0, 0), (11, 11, 10, 0)), (4, (127, 127, 127), (11, 11, 10, 0)),
                                                     (32, (4095, 4095, 4095), (32, 0, 0, 0)),
                                                     (8, (300, 17, 5), (11, 11, 10, 0))])
def test_rope(ctx, ref, heads, position, sections):
    h = RNG.standard_normal((heads, 128)).astype(np.float32)
    d = dev(h)
    ctx.rope(d, heads, 128, 64, sections, 1.0e7, position)
    ctx.device_status()
    assert bits(d.cpu().numpy(), ref.rope(h, 64, sections, 1.0e7, position))


def test_rope_validation(ctx):
    d = torch.zeros(128, device=DEV)
    with pytest.raises(ob.InvalidArgument, match="sections must sum to half"):
        ctx.rope(d, 1, 128, 64, (10, 10, 10, 0), 1.0e7, (0, 0, 0))
    with pytest.raises(ob.InvalidArgument, match="non-zero, even"):
        ctx.rope(d, 1, 128, 63, (11, 11, 10, 0), 1.0e7, (0, 0, 0))


@pytest.mark.parametrize("length", [0, 1, 127, 1000])
def test_attention_step(ctx, ref, length):
    hq, hkv, dk, dv, cap = 32, 4, 128, 128, 1024
    keys = RNG.standard_normal((length, hkv, dk)).astype(np.float32)
    values = RNG.standard_normal((length, hkv, dv)).astype(np.float32)
    q = RNG.standard_normal((hq, dk)).astype(np.float32)
    kn = RNG.standard_normal((hkv, dk)).astype(np.float32)
    vn = RNG.standard_normal((hkv, dv)).astype(np.float32)
    kc = torch.zeros(cap * hkv * dk, device=DEV)
    vc = torch.zeros(cap * hkv * dv, device=DEV)
    kc[:length * hkv * dk] = dev(keys.reshape(-1))
    vc[:length * hkv * dv] = dev(values.reshape(-1))
    scores = torch.empty(hq * (length + 1), device=DEV)
    out = torch.empty(hq * dv, device=DEV)
    ctx.attention_step(dev(q), dev(kn), dev(vn), kc, vc, cap, length, hq, hkv, dk, dv, scores, out)
    ctx.device_status()
    want = ref.attention_step(q, kn, vn, keys.reshape(length, hkv * dk), values.reshape(length, hkv * dv), cap)
    close(out.cpu().numpy().reshape(hq, dv), want)
    # the new token landed in the cache
    assert bits(kc[length * hkv * dk:(length + 1) * hkv * dk].cpu().numpy(), kn.reshape(-1))
    assert bits(vc[length * hkv * dv:(length + 1) * hkv * dv].cpu().numpy(), vn.reshape(-1))


def test_attention_capacity(ctx):
    z = torch.zeros(4 * 128, device=DEV)
    with pytest.raises(ob.Overflow, match="KV cache capacity exceeded"):
        ctx.attention_step(z, z, z, z, z, 1, 1, 4, 1, 128, 128, z, z)


@pytest.mark.parametrize("silu", [True, False])
def test_conv_step(ctx, ref, silu):
    ch, kw = 8192, 4
    w = RNG.standard_normal((ch, kw)).astype(np.float32)
    hist = RNG.standard_normal((ch, kw)).astype(np.float32)
    hist_d = dev(hist)
    want_hist = hist
    for step in range(3):
        x = RNG.standard_normal(ch).astype(np.float32)
        out = torch.empty(ch, device=DEV)
        ctx.conv_step(dev(x), dev(w), hist_d, ch, kw, silu, out)
        ctx.device_status()
        want, want_hist = ref.conv_step(x, w, want_hist, silu)
        close(out.cpu().numpy(), want)
        assert bits(hist_d.cpu().numpy().reshape(ch, kw), want_hist)


def test_gated_delta_steps(ctx, ref):
    heads, dk, dv = 32, 128, 128
    state = (RNG.standard_normal((heads, dk, dv)) * 0.1).astype(np.float32)
    sd = dev(state)
    want_state = state
    for step in range(4):
        q = RNG.standard_normal((heads, dk)).astype(np.float32)
        k = RNG.standard_normal((heads, dk)).astype(np.float32)
        v = RNG.standard_normal((heads, dv)).astype(np.float32)
        beta = RNG.uniform(0, 1, heads).astype(np.float32)
        g = -RNG.uniform(0, 2, heads).astype(np.float32)
        out = torch.empty(heads * dv, device=DEV)
        ctx.gated_delta_step(dev(q), dev(k), dev(v), dev(beta), dev(g), sd, heads, dk, dv, 1e-6, out)
        ctx.device_status()
        want, want_state = ref.gated_delta_step(q, k, v, beta, g, want_state)
        close(out.cpu().numpy().reshape(heads, dv), want)
        close(sd.cpu().numpy().reshape(heads, dk, dv), want_state)


def test_swiglu_and_add(ctx, port):
    n = 12288
    g = (RNG.standard_normal(n) * 4).astype(np.float32)
    u = RNG.standard_normal(n).astype(np.float32)
    out = torch.empty(n, device=DEV)
    ctx.swiglu(dev(g), dev(u), n, out)
    close(out.cpu().numpy(), port.swiglu(g, u), rel=4e-7, ab=1e-30)
    ctx.add(dev(g), dev(u), n, out)
    assert bits(out.cpu().numpy(), g + u)
