"""GPU: the decode-step fusions, against the restatement and the unfused kernels.

* Matvec programs with activation transforms (RMSNorm, SwiGLU) and residual
  outputs, built in the prebuilt quantizer (first op) and in-kernel (dependent
  ops), with image sharing: bit-exact against the restatement computing the
  same chain unfused on the CPU (rms_norm_rows / swiglu / quantize_row_q8_K /
  integer dots / add, each as Oracle's or GGML's code does it).
* The fused Gated DeltaNet core and the fused attention kernels against the
  separate kernels they replace (themselves checked against Oracle's compiled
  functions) over several steps: attention bit-identical; the recurrent core
  within 1e-5 relative / 1e-6 absolute (its key-index sums are split four
  ways), conv histories bit-identical.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle_b200 as ob

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
RNG = np.random.default_rng(77)
EPS = float(np.float32(1e-6))


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def close(got, want, rel=1e-5, ab=1e-6):
    got, want = np.asarray(got, np.float64), np.asarray(want, np.float64)
    bad = np.abs(got - want) > ab + rel * np.abs(want)
    assert not bad.any(), (int(bad.sum()), float(np.abs(got - want).max()))


def same(a, b):
    return np.array_equal(np.asarray(a, np.float32).view(np.uint32), np.asarray(b, np.float32).view(np.uint32))


def weight(qtype, rows, cols, name):
    from oracle_b200 import synth
    return synth.weight(qtype, rows, cols, "program_ex", name)


def cpu_mv(port, qtype, w, x):
    rows = w.shape[0]
    return port.matvec_q8_k(qtype, rows, x.size, w, port.quantize_q8_k(x))[0]


def test_rms_transform_prebuilt(ctx, port):
    h = (RNG.standard_normal(4096) * 5).astype(np.float32)
    nw = (1 + 0.1 * RNG.standard_normal(4096)).astype(np.float32)
    w = weight(12, 1024, 4096, "rms")
    y = torch.empty(1024, device=DEV)
    ctx.matvec_program_ex([dict(qtype=12, rows=1024, cols=4096, w=dev(w), x=dev(h), y=y, xform=ob.XFORM_RMS,
                                eps=EPS, norm=dev(nw))])
    ctx.device_status()
    want = cpu_mv(port, 12, w, port.rms_norm_rows(h[None], nw, EPS)[0])
    assert same(y.cpu().numpy(), want)


@pytest.mark.parametrize("in_kernel", [False, True])
def test_decode_chain_in_one_launch(ctx, port, in_kernel):
    """out-projection (+residual) -> gate/up of rms(resid) (shared image) ->
    down of swiglu(gate, up) (+residual) -> next projections of rms(hidden).
    The first op's image comes from the quantizer launch, or (in_kernel) is
    built by every CTA of the program itself."""
    saved = ctx.flags
    ctx.set_flags((saved & ~ob.FLAG_BUILD_IN_KERNEL) | (ob.FLAG_BUILD_IN_KERNEL if in_kernel else 0))
    try:
        _decode_chain(ctx, port)
    finally:
        ctx.set_flags(saved)


def _decode_chain(ctx, port):
    H, F = 1024, 3072
    hidden = RNG.standard_normal(H).astype(np.float32)
    xin = RNG.standard_normal(H).astype(np.float32)
    n_post = (1 + 0.1 * RNG.standard_normal(H)).astype(np.float32)
    n_next = (1 + 0.1 * RNG.standard_normal(H)).astype(np.float32)
    w_out, w_gate, w_up = weight(12, H, H, "out"), weight(12, F, H, "gate"), weight(14, F, H, "up")
    w_down, w_q, w_k = weight(14, H, F, "down"), weight(12, 2048, H, "q"), weight(12, 256, H, "k")
    d = {k: dev(v) for k, v in dict(hidden=hidden, xin=xin, n_post=n_post, n_next=n_next, w_out=w_out,
                                     w_gate=w_gate, w_up=w_up, w_down=w_down, w_q=w_q, w_k=w_k).items()}
    resid, g, u = torch.empty(H, device=DEV), torch.empty(F, device=DEV), torch.empty(F, device=DEV)
    h_out, q, k = torch.empty(H, device=DEV), torch.empty(2048, device=DEV), torch.empty(256, device=DEV)
    R = ob.XFORM_RMS
    ops = [dict(qtype=12, rows=H, cols=H, w=d["w_out"], x=d["xin"], y=resid, residual=d["hidden"]),
           dict(qtype=12, rows=F, cols=H, w=d["w_gate"], x=resid, y=g, after=True, xform=R, eps=EPS, norm=d["n_post"]),
           dict(qtype=14, rows=F, cols=H, w=d["w_up"], x=resid, y=u, after=True, xform=R, eps=EPS, norm=d["n_post"]),
           dict(qtype=14, rows=H, cols=F, w=d["w_down"], x=g, y=h_out, after=True, xform=ob.XFORM_SWIGLU, x2=u,
                residual=resid),
           dict(qtype=12, rows=2048, cols=H, w=d["w_q"], x=h_out, y=q, after=True, xform=R, eps=EPS,
                norm=d["n_next"]),
           dict(qtype=12, rows=256, cols=H, w=d["w_k"], x=h_out, y=k, after=True, xform=R, eps=EPS,
                norm=d["n_next"])]
    for _ in range(2):  # the program's counters are reused by the next launch
        ctx.matvec_program_ex(ops)
        ctx.device_status()
        c_resid = hidden + cpu_mv(port, 12, w_out, xin)
        xr = port.rms_norm_rows(c_resid[None], n_post, EPS)[0]
        c_g, c_u = cpu_mv(port, 12, w_gate, xr), cpu_mv(port, 14, w_up, xr)
        c_h = c_resid + cpu_mv(port, 14, w_down, port.swiglu(c_g, c_u))
        xn = port.rms_norm_rows(c_h[None], n_next, EPS)[0]
        for got, want in ((resid, c_resid), (g, c_g), (u, c_u), (h_out, c_h), (q, cpu_mv(port, 12, w_q, xn)),
                          (k, cpu_mv(port, 12, w_k, xn))):
            assert same(got.cpu().numpy(), want)


def test_program_ex_validation(ctx):
    w = dev(weight(12, 256, 256, "v"))
    x, y = torch.zeros(256, device=DEV), torch.zeros(256, device=DEV)
    with pytest.raises(ob.InvalidArgument, match="RMS transform needs weights"):
        ctx.matvec_program_ex([dict(qtype=12, rows=256, cols=256, w=w, x=x, y=y, xform=ob.XFORM_RMS, eps=EPS)])
    with pytest.raises(ob.InvalidArgument, match="SwiGLU transform needs up"):
        ctx.matvec_program_ex([dict(qtype=12, rows=256, cols=256, w=w, x=x, y=y, xform=ob.XFORM_SWIGLU)])
    with pytest.raises(ob.InvalidArgument, match="unknown activation transform"):
        ctx.matvec_program_ex([dict(qtype=12, rows=256, cols=256, w=w, x=x, y=y, xform=7)])


def test_gdn_core_matches_separate_kernels(ctx):
    kh, vh, D, K = 16, 32, 128, 4
    C = 2 * kh * D + vh * D
    conv_w = dev((RNG.standard_normal((C, K)) * 0.5).astype(np.float32))
    dt = dev(np.log(np.expm1(RNG.uniform(1e-3, 0.1, vh))).astype(np.float32))
    a = dev(-RNG.uniform(1, 16, vh).astype(np.float32))
    norm = dev((1 + 0.1 * RNG.standard_normal(D)).astype(np.float32))
    hist1, state1 = torch.zeros(C * K, device=DEV), torch.zeros(vh * D * D, device=DEV)
    hist2, state2 = torch.zeros(2 * C * K, device=DEV), torch.zeros(vh * D * D, device=DEV)
    pos = torch.zeros(1, dtype=torch.int32, device=DEV)
    f = lambda n: torch.empty(n, device=DEV)  # noqa: E731
    conv_out, bs, ld, rec, gated, fused = f(C), f(vh), f(vh), f(vh * D), f(vh * D), f(vh * D)
    for step in range(5):
        qkv = dev(RNG.standard_normal(C).astype(np.float32))
        z = dev(RNG.standard_normal(vh * D).astype(np.float32))
        beta, alpha = dev(RNG.standard_normal(vh).astype(np.float32)), dev(RNG.standard_normal(vh).astype(np.float32))
        ctx.gdn_gates(beta, alpha, dt, a, vh, bs, ld)
        ctx.conv_step(qkv, conv_w, hist1, C, K, True, conv_out)
        kw = kh * D
        ctx.gated_delta_step(conv_out[:kw], conv_out[kw:2 * kw], conv_out[2 * kw:], bs, ld, state1, vh, D, D, EPS,
                             rec, qk_heads=kh)
        ctx.rms_norm_rows(rec, norm, vh, D, EPS, gated)
        ctx.mul_silu(gated, z, vh * D)
        ctx.gdn_core(qkv, z, beta, alpha, dt, a, conv_w, hist2, state2, norm, kh, vh, D, K, EPS, pos, fused)
        ctx.position_advance(pos)
        ctx.device_status()
        # the fused core sums the key index as four partial sums: same terms,
        # another rounding order (the decoder's 1e-5 / 1e-6 tolerance)
        close(fused.cpu().numpy(), gated.cpu().numpy())
        close(state2.cpu().numpy(), state1.cpu().numpy())
        slot = (step + 1) & 1
        assert same(hist2[slot * C * K:(slot + 1) * C * K].cpu().numpy(), hist1.cpu().numpy()), step


def test_attention_fused_matches_separate_kernels(ctx):
    hq, hkv, D, cap, rot = 32, 4, 128, 64, 64
    table = torch.empty(cap * rot, device=DEV)
    ctx.rope_table(rot, (11, 11, 10, 0), 1.0e7, cap, table)
    qn_w = dev((1 + 0.1 * RNG.standard_normal(D)).astype(np.float32))
    kn_w = dev((1 + 0.1 * RNG.standard_normal(D)).astype(np.float32))
    f = lambda n: torch.zeros(n, device=DEV)  # noqa: E731
    keys1, vals1, keys2, vals2 = f(cap * hkv * D), f(cap * hkv * D), f(cap * hkv * D), f(cap * hkv * D)
    q, gate, qn, kn, out1, out2, qo = f(hq * D), f(hq * D), f(hq * D), f(hkv * D), f(hq * D), f(hq * D), f(hq * D)
    sc1, sc2 = f(hq * cap), f(hq * cap)
    pos = torch.zeros(1, dtype=torch.int32, device=DEV)
    for step in range(6):
        q_full = dev(RNG.standard_normal(2 * hq * D).astype(np.float32))
        k = dev(RNG.standard_normal(hkv * D).astype(np.float32))
        v = dev(RNG.standard_normal(hkv * D).astype(np.float32))
        ctx.split_query_gate(q_full, hq, D, q, gate)
        ctx.rms_norm_rows(q, qn_w, hq, D, EPS, qn)
        ctx.rms_norm_rows(k, kn_w, hkv, D, EPS, kn)
        ctx.rope_at(qn, hq, D, rot, table, cap, pos)
        ctx.rope_at(kn, hkv, D, rot, table, cap, pos)
        ctx.attention_step_at(qn, kn, v, keys1, vals1, cap, pos, hq, hkv, D, D, sc1, out1)
        ctx.gate_sigmoid_mul(out1, gate, hq * D)
        ctx.attention_prep_at(q_full, k, v, qn_w, kn_w, EPS, table, rot, hq, hkv, D, keys2, vals2, cap, pos, qo)
        ctx.attention_core_at(qo, keys2, vals2, cap, pos, hq, hkv, D, D, q_full[D:], 2 * D, sc2, out2)
        ctx.position_advance(pos)
        ctx.device_status()
        assert same(qo.cpu().numpy(), qn.cpu().numpy()), step
        assert same(keys2.cpu().numpy(), keys1.cpu().numpy()), step
        assert same(vals2.cpu().numpy(), vals1.cpu().numpy()), step
        assert same(out2.cpu().numpy(), out1.cpu().numpy()), step
