"""GPU parity: the CUDA path through the C ABI against the CPU checkers.

Bars (written into each test):
* decode, Q8_K quantization, the Q8_K integer matvec: bit-exact with the
  restatement (which is bit-exact with Oracle's compiled decoders, see
  test_oracle_pins.py);
* Oracle's f32 contract: bit-exact with the reference's own compiled
  reference_storage_matvec (and the restatement), since the kernel performs
  Oracle's operations in Oracle's order.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle_b200 as ob
from conftest import golden
from oracle_b200 import synth

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def to_dev(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a).reshape(-1)).to(DEV)


def bits_equal(a: np.ndarray, b: np.ndarray) -> bool:
    a = np.asarray(a, np.float32).reshape(-1)
    b = np.asarray(b, np.float32).reshape(-1)
    return bool(np.all((a.view(np.uint32) == b.view(np.uint32)) | (np.isnan(a) & np.isnan(b))))


# ---------------------------------------------------------------- decode (decode_storage_row)

@pytest.mark.parametrize("qtype,rows,k", [
    (ob.TYPE_Q8_0, 1, 32), (ob.TYPE_Q8_0, 7, 96), (ob.TYPE_Q8_0, 33, 4096),
    (ob.TYPE_Q4_K, 1, 256), (ob.TYPE_Q4_K, 5, 768), (ob.TYPE_Q4_K, 17, 4096),
    (ob.TYPE_Q5_K, 3, 512), (ob.TYPE_Q6_K, 1, 256), (ob.TYPE_Q6_K, 9, 1280),
    (ob.TYPE_F16, 3, 37), (ob.TYPE_BF16, 3, 37), (ob.TYPE_F32, 4, 13)])
def test_decode_rows_bit_exact(ctx, port, qtype, rows, k):
    w = synth.weight(qtype, rows, k, "gpu", f"dec_{qtype}_{rows}_{k}")
    out = torch.empty(rows * k, dtype=torch.float32, device=DEV)
    ctx.decode_rows(qtype, rows, k, to_dev(w), out)
    ctx.device_status()
    assert bits_equal(out.cpu().numpy(), port.decode_rows(qtype, rows, k, w))


def test_decode_rows_ggufpy_fixture(ctx):
    g = golden("decode_ggufpy.npz")
    for qtype, name in [(ob.TYPE_Q8_0, "Q8_0"), (ob.TYPE_Q4_K, "Q4_K"), (ob.TYPE_Q5_K, "Q5_K"),
                        (ob.TYPE_Q6_K, "Q6_K")]:
        blocks, want = g[f"{name}_blocks"], g[f"{name}_decoded"]
        out = torch.empty(want.size, dtype=torch.float32, device=DEV)
        ctx.decode_rows(qtype, blocks.shape[0], want.shape[1], to_dev(blocks), out)
        assert bits_equal(out.cpu().numpy(), want), name


def test_host_decode_rows_reference_fixture(ctx):
    g = golden("reference.npz")
    for qtype, name in [(ob.TYPE_Q8_0, "Q8_0"), (ob.TYPE_Q5_K, "Q5_K"), (ob.TYPE_Q6_K, "Q6_K"),
                        (ob.TYPE_F16, "F16"), (ob.TYPE_BF16, "BF16"), (ob.TYPE_F32, "F32")]:
        w, x = g[f"{name}_w"], g[f"{name}_x"]
        got = ctx.host_decode_rows(qtype, w.shape[0], x.size, w)
        assert bits_equal(got, g[f"{name}_decoded"]), name


# ---------------------------------------------------------------- Q8_K quantizer

def test_quantize_q8k_bit_exact(ctx, port):
    g = golden("q8k.npz")
    x = g["x"]
    rng = synth.rng_for("gpu", "q8k")
    xr = (rng.standard_normal(256 * 96) * rng.uniform(1e-3, 1e3, 256 * 96)).astype(np.float32)
    for xs, batch in [(x, 1), (xr, 3), (xr[: 256 * 5], 1)]:
        k = xs.size // batch
        q = torch.empty(xs.size // 256 * 292, dtype=torch.uint8, device=DEV)
        ctx.quantize_q8_k(to_dev(xs), k, batch, q)
        ctx.device_status()
        assert np.array_equal(q.cpu().numpy(), port.quantize_q8_k(xs.reshape(batch, k)).reshape(-1))
    assert np.array_equal(port.quantize_q8_k(x)[0], g["q8k"])


# ---------------------------------------------------------------- Q8_K integer matvec (north star)

SHAPES_Q8K = [(1, 256), (2, 512), (3, 4096), (13, 4096), (257, 4096), (149, 3072), (100, 12288),
              (37, 8192), (20, 16384), (1000, 1024)]


@pytest.mark.parametrize("qtype", [ob.TYPE_Q4_K, ob.TYPE_Q6_K])
@pytest.mark.parametrize("rows,k", SHAPES_Q8K)
def test_matvec_q8k_bit_exact(ctx, port, qtype, rows, k):
    w = synth.weight(qtype, rows, k, "gpu", f"mv_{qtype}_{rows}_{k}")
    x = synth.activations(k, 1, "gpu", f"mv_x_{k}")
    q8 = port.quantize_q8_k(x)
    want = port.matvec_q8_k(qtype, rows, k, w, q8)[0]
    wd, xd = to_dev(w), to_dev(x)
    y = torch.empty(rows, dtype=torch.float32, device=DEV)
    ctx.storage_matvec(ob.CONTRACT_Q8K, qtype, rows, k, wd, xd, y)  # quantize fused in-kernel
    ctx.device_status()
    assert bits_equal(y.cpu().numpy(), want)
    y2 = torch.empty_like(y)
    ctx.matvec_q8k_prequantized(qtype, rows, k, wd, to_dev(q8), y2)
    ctx.device_status()
    assert bits_equal(y2.cpu().numpy(), want)


@pytest.mark.parametrize("qtype", [ob.TYPE_Q4_K, ob.TYPE_Q6_K])
def test_matvec_q8k_batch(ctx, port, qtype):
    rows, k, batch = 77, 2048, 3
    w = synth.weight(qtype, rows, k, "gpu", f"mvb_{qtype}")
    x = synth.activations(k, batch, "gpu", "mvb_x")
    want = port.matvec_q8_k(qtype, rows, k, w, port.quantize_q8_k(x))
    y = torch.empty(batch * rows, dtype=torch.float32, device=DEV)
    ctx.storage_matvec(ob.CONTRACT_Q8K, qtype, rows, k, to_dev(w), to_dev(x), y)
    assert bits_equal(y.cpu().numpy(), want)


@pytest.mark.parametrize("rows,k", [(12288, 4096), (4096, 12288), (4096, 4096)])
def test_config2_full_size_q4k(ctx, port, rows, k):
    """BASELINE config 2 shapes, every element bit-exact."""
    w = synth.weight(ob.TYPE_Q4_K, rows, k, "config2", f"W_{k}_{rows}")
    x = synth.activations(k, 1, "config2", f"x_{k}")
    want = port.matvec_q8_k(ob.TYPE_Q4_K, rows, k, w, port.quantize_q8_k(x))[0]
    y = torch.empty(rows, dtype=torch.float32, device=DEV)
    ctx.storage_matvec(ob.CONTRACT_Q8K, ob.TYPE_Q4_K, rows, k, to_dev(w), to_dev(x), y)
    ctx.device_status()
    assert bits_equal(y.cpu().numpy(), want)


def test_config3_lm_head_q6k(ctx, port):
    """Q6_K 151936 x 4096 LM head, every logit bit-exact."""
    rows, k = 151936, 4096
    w = synth.weight(ob.TYPE_Q6_K, rows, k, "config3", "lm_head")
    x = synth.activations(k, 1, "config3", "x")
    want = port.matvec_q8_k(ob.TYPE_Q6_K, rows, k, w, port.quantize_q8_k(x))[0]
    y = torch.empty(rows, dtype=torch.float32, device=DEV)
    ctx.storage_matvec(ob.CONTRACT_Q8K, ob.TYPE_Q6_K, rows, k, to_dev(w), to_dev(x), y)
    ctx.device_status()
    got = y.cpu().numpy()
    assert bits_equal(got, want)
    assert int(np.argmax(got)) == int(np.argmax(want))


# ---------------------------------------------------------------- Oracle's f32 contract

@pytest.mark.parametrize("qtype,rows,k", [
    # Q8_0 with K % 256 == 0: the lane-per-row kernel (one chunk, ragged row
    # counts, several passes over the stage ring); other K: the producer kernel
    (ob.TYPE_Q8_0, 4096, 4096), (ob.TYPE_Q8_0, 33, 256), (ob.TYPE_Q8_0, 100, 2304),
    (ob.TYPE_Q8_0, 5, 32), (ob.TYPE_Q8_0, 19, 160),
    (ob.TYPE_Q4_K, 33, 4096), (ob.TYPE_Q5_K, 21, 1024), (ob.TYPE_Q6_K, 45, 4096),
    (ob.TYPE_F16, 6, 37), (ob.TYPE_BF16, 6, 300), (ob.TYPE_F32, 7, 129)])
def test_f32_contract(ctx, port, qtype, rows, k):
    w = synth.weight(qtype, rows, k, "config1" if (rows, k) == (4096, 4096) else "gpu", f"f32_{qtype}_{rows}_{k}")
    x = synth.activations(k, 1, "gpu", f"f32_x_{k}")
    want = port.storage_matvec_f32(qtype, rows, k, w, x)[0]
    y = torch.empty(rows, dtype=torch.float32, device=DEV)
    ctx.storage_matvec(ob.CONTRACT_F32, qtype, rows, k, to_dev(w), to_dev(x), y)
    ctx.device_status()
    assert bits_equal(y.cpu().numpy(), want)


def test_f32_contract_against_reference_binary(ctx, ref):
    """Oracle's own compiled reference_storage_matvec as the expected value, bit for bit."""
    for qtype, rows, k in [(ob.TYPE_Q8_0, 257, 4096), (ob.TYPE_Q6_K, 65, 2048), (ob.TYPE_Q5_K, 9, 512),
                           (ob.TYPE_Q6_K, 7, 768), (ob.TYPE_Q8_0, 3, 96), (ob.TYPE_F16, 5, 37)]:
        w = synth.weight(qtype, rows, k, "gpu", f"refbin_{qtype}_{k}")
        x = synth.activations(k, 1, "gpu", f"refbin_x_{k}")[0]
        want = ref.storage_matvec(qtype, rows, k, w, x)
        got = ctx.host_storage_matvec(ob.CONTRACT_F32, qtype, rows, k, w, x)
        assert bits_equal(got, want), (qtype, rows, k)


@pytest.mark.parametrize("qtype,rows,k,batch", [
    (ob.TYPE_Q8_0, 50, 1024, 6), (ob.TYPE_Q8_0, 70, 4096, 2), (ob.TYPE_Q6_K, 33, 512, 3),
    (ob.TYPE_Q4_K, 31, 1280, 4), (ob.TYPE_F16, 40, 301, 5), (ob.TYPE_F32, 3, 5, 4)])
def test_f32_contract_batch(ctx, port, qtype, rows, k, batch):
    w = synth.weight(qtype, rows, k, "gpu", f"f32batch_{qtype}_{k}")
    x = synth.activations(k, batch, "gpu", f"f32batch_x_{k}_{batch}")
    want = port.storage_matvec_f32(qtype, rows, k, w, x)
    y = torch.empty(batch * rows, dtype=torch.float32, device=DEV)
    ctx.storage_matvec(ob.CONTRACT_F32, qtype, rows, k, to_dev(w), to_dev(x), y)
    ctx.device_status()
    assert bits_equal(y.cpu().numpy().reshape(batch, rows), want.reshape(batch, rows))


def test_f32_contract_unaligned_rows(ctx, port):
    """Row starts that are not 4-byte aligned (Q6_K with an odd super-block count)."""
    for qtype, rows, k in [(ob.TYPE_Q6_K, 37, 768), (ob.TYPE_Q8_0, 29, 32), (ob.TYPE_BF16, 9, 7)]:
        w = synth.weight(qtype, rows, k, "gpu", f"unal_{qtype}_{k}")
        x = synth.activations(k, 2, "gpu", f"unal_x_{k}")
        y = torch.empty(2 * rows, dtype=torch.float32, device=DEV)
        ctx.storage_matvec(ob.CONTRACT_F32, qtype, rows, k, to_dev(w), to_dev(x), y)
        assert bits_equal(y.cpu().numpy(), port.storage_matvec_f32(qtype, rows, k, w, x)), (qtype, k)


# ---------------------------------------------------------------- host drop-ins: the reference's known answers

def test_host_known_answers(ctx):
    from test_oracle_pins import q5_fixture, q6_fixture, q8_0_fixture, q4_fixture
    ones = np.ones(256, np.float32)
    assert ctx.host_storage_dot(ob.CONTRACT_F32, ob.TYPE_Q5_K, 256, q5_fixture(), ones) == 4288.0
    assert ctx.host_storage_dot(ob.CONTRACT_F32, ob.TYPE_Q6_K, 256, q6_fixture(), ones) == 4480.0
    assert ctx.host_storage_dot(ob.CONTRACT_F32, ob.TYPE_Q8_0, 32, q8_0_fixture(), np.ones(32, np.float32)) == 14.0
    assert ctx.host_storage_dot(ob.CONTRACT_F32, ob.TYPE_Q4_K, 256, q4_fixture(), ones) == 192.0
    second = q5_fixture().copy()
    second[16:] = 0
    y = ctx.host_storage_matvec(ob.CONTRACT_F32, ob.TYPE_Q5_K, 2, 256, np.concatenate([q5_fixture(), second]), ones)
    assert y.tolist() == [4288.0, -192.0]
    mat8 = np.concatenate([q8_0_fixture(), q8_0_fixture(0x3800, [4] * 32)])
    assert ctx.host_storage_matvec(ob.CONTRACT_F32, ob.TYPE_Q8_0, 2, 32, mat8,
                                   np.ones(32, np.float32)).tolist() == [14.0, 64.0]
    dec = ctx.host_decode_rows(ob.TYPE_Q5_K, 1, 256, q5_fixture())
    assert np.all(dec.reshape(4, 64)[:, :32] == 16.25) and np.all(dec.reshape(4, 64)[:, 32:] == 17.25)


def test_host_q8k_matches_device(ctx, port):
    rows, k = 300, 4096
    w = synth.weight(ob.TYPE_Q4_K, rows, k, "gpu", "host_q8k")
    x = synth.activations(k, 1, "gpu", "host_q8k_x")
    got = ctx.host_storage_matvec(ob.CONTRACT_Q8K, ob.TYPE_Q4_K, rows, k, w, x)
    assert bits_equal(got, port.matvec_q8_k(ob.TYPE_Q4_K, rows, k, w, port.quantize_q8_k(x))[0])
    ctx.register_host_weight(ob.TYPE_Q4_K, rows, k, w)
    try:
        got2 = ctx.host_storage_matvec(ob.CONTRACT_Q8K, ob.TYPE_Q4_K, rows, k, w, x)  # the resident copy
    finally:
        ctx.unregister_host_weight(w)
    assert bits_equal(got, got2)


def test_host_buffer_reused_with_new_bytes(ctx, port):
    """The host-pointer calls read the caller's bytes on every call, as the
    reference does: a buffer refilled with other weights at the same address
    gives the new result.  A registered span is read from its resident copy
    (the caller promised it would not change) until it is unregistered."""
    rows, k = 96, 4096
    a = synth.weight(ob.TYPE_Q4_K, rows, k, "gpu", "reuse_a")
    b = synth.weight(ob.TYPE_Q4_K, rows, k, "gpu", "reuse_b")
    x = synth.activations(k, 1, "gpu", "reuse_x")
    q = port.quantize_q8_k(x)
    want_a = port.matvec_q8_k(ob.TYPE_Q4_K, rows, k, a, q)[0]
    want_b = port.matvec_q8_k(ob.TYPE_Q4_K, rows, k, b, q)[0]
    buf = a.copy()
    assert bits_equal(ctx.host_storage_matvec(ob.CONTRACT_Q8K, ob.TYPE_Q4_K, rows, k, buf, x), want_a)
    buf[...] = b
    assert bits_equal(ctx.host_storage_matvec(ob.CONTRACT_Q8K, ob.TYPE_Q4_K, rows, k, buf, x), want_b)
    # storage_dot on a row rebuilt at the same address (the reference's tests
    # build rows on the stack) sees the new row too
    row = a[0].copy()
    d0 = ctx.host_storage_dot(ob.CONTRACT_Q8K, ob.TYPE_Q4_K, k, row, x)
    row[...] = b[0]
    assert ctx.host_storage_dot(ob.CONTRACT_Q8K, ob.TYPE_Q4_K, k, row, x) == want_b[0] and d0 == want_a[0]
    # registered: the resident copy, until unregistered
    ctx.register_host_weight(ob.TYPE_Q4_K, rows, k, buf)
    buf[...] = a
    assert bits_equal(ctx.host_storage_matvec(ob.CONTRACT_Q8K, ob.TYPE_Q4_K, rows, k, buf, x), want_b)
    ctx.unregister_host_weight(buf)
    assert bits_equal(ctx.host_storage_matvec(ob.CONTRACT_Q8K, ob.TYPE_Q4_K, rows, k, buf, x), want_a)
    with pytest.raises(ob.OutOfRange, match="not registered"):
        ctx.unregister_host_weight(buf)


def test_host_matvec_program(ctx, port):
    """oracle_cuda_host_matvec_program: host spans in and out, one launch and
    one synchronize; an op fed by an earlier op's output (the same host array)
    reads it on the device.  Bit-identical to the restatement, registered or
    not."""
    specs = [(ob.TYPE_Q4_K, 700, 4096), (ob.TYPE_Q6_K, 300, 4096)]
    ws = [synth.weight(t, n, k, "gpu", f"hostprog{i}") for i, (t, n, k) in enumerate(specs)]
    x0 = synth.activations(4096, 1, "gpu", "hostprog_x")[0]
    ys = [np.full(n, np.nan, np.float32) for _, n, _ in specs]
    # two independent ops on x0, then a 512-row op whose whole output feeds a
    # dependent op (a dependent op reads an earlier op's whole output)
    ops = [(specs[0][0], 700, 4096, ws[0], x0, ys[0]), (specs[1][0], 300, 4096, ws[1], x0, ys[1])]
    wdep = synth.weight(ob.TYPE_Q4_K, 128, 512, "gpu", "hostprog_dep")
    wsrc = synth.weight(ob.TYPE_Q4_K, 512, 4096, "gpu", "hostprog_src")
    ysrc = np.full(512, np.nan, np.float32)
    ydep = np.full(128, np.nan, np.float32)
    ops += [(ob.TYPE_Q4_K, 512, 4096, wsrc, x0, ysrc), (ob.TYPE_Q4_K, 128, 512, wdep, ysrc, ydep)]
    q0 = port.quantize_q8_k(x0)
    want0 = port.matvec_q8_k(ob.TYPE_Q4_K, 700, 4096, ws[0], q0)[0]
    want1 = port.matvec_q8_k(ob.TYPE_Q6_K, 300, 4096, ws[1], q0)[0]
    wantsrc = port.matvec_q8_k(ob.TYPE_Q4_K, 512, 4096, wsrc, q0)[0]
    wantdep = port.matvec_q8_k(ob.TYPE_Q4_K, 128, 512, wdep, port.quantize_q8_k(wantsrc))[0]
    for registered in (False, True):
        if registered:
            for t, n, k, w, _, _ in ops:
                ctx.register_host_weight(t, n, k, w)
        for y in (ys[0], ys[1], ysrc, ydep):
            y.fill(np.nan)
        ctx.host_matvec_program(ops)
        assert bits_equal(ys[0], want0) and bits_equal(ys[1], want1)
        assert bits_equal(ysrc, wantsrc) and bits_equal(ydep, wantdep)
        # prepared once (registered weights only), run twice on changing x
        if registered:
            import torch
            for pinned in (False, True):
                xin = torch.from_numpy(x0.copy()).pin_memory().numpy() if pinned else x0.copy()
                outs = [torch.empty(n, dtype=torch.float32).pin_memory().numpy() if pinned else
                        np.empty(n, np.float32) for n in (700, 300, 512, 128)]
                prep = ctx.prepare_host_program([(t, n, k, w, xin if i < 3 else outs[2], outs[i])
                                                 for i, (t, n, k, w, _, _) in enumerate(ops)])
                for rep in range(2):
                    for o in outs:
                        o.fill(np.nan)
                    prep()
                    assert bits_equal(outs[0], want0) and bits_equal(outs[1], want1)
                    assert bits_equal(outs[2], wantsrc) and bits_equal(outs[3], wantdep)
                xin[:] = x0[::-1]
                prep()
                q1 = port.quantize_q8_k(x0[::-1].copy())
                assert bits_equal(outs[0], port.matvec_q8_k(ob.TYPE_Q4_K, 700, 4096, ws[0], q1)[0])
                prep.close()
    ctx.evict_resident()
    with pytest.raises(ob.InvalidArgument, match="needs registered weights"):
        ctx.prepare_host_program(ops)
    with pytest.raises(ob.InvalidArgument, match="op 1: reads op 0's output"):
        ctx.host_matvec_program([(ob.TYPE_Q4_K, 700, 4096, ws[0], x0, ys[0]),
                                 (ob.TYPE_Q4_K, 128, 512, wdep, ys[0], ydep)])


# ---------------------------------------------------------------- errors: same class and message as the reference

def test_validation_matches_reference(ctx, ref):
    import oracle
    w = synth.weight(ob.TYPE_Q8_0, 2, 64, "gpu", "err")
    x = np.ones(64, np.float32)
    cases = [
        (ob.TYPE_Q8_0, 0, 64, w, x, 2),          # zero rows
        (ob.TYPE_Q8_0, 2, 64, w, x[:63], 2),     # vector length
        (ob.TYPE_Q8_0, 2, 64, w, x, 3),          # output length
        (ob.TYPE_Q8_0, 2, 64, w[:, :-1], x, 2),  # matrix bytes
        (ob.TYPE_Q8_0, 2, 63, w, x[:63], 2),     # ragged row
        (999, 2, 64, w, x, 2),                   # unknown type
        (2, 2, 64, np.zeros(2 * 36, np.uint8), x, 2),  # registered, not decodable (q4_0)
    ]
    for qtype, rows, k, wb, xb, ylen in cases:
        with pytest.raises(oracle.ReferenceError_) as want:
            ref.storage_matvec(qtype, rows, k, wb, xb, y_len=ylen)
        with pytest.raises(ob.OracleCudaError) as got:
            ctx.host_storage_matvec(ob.CONTRACT_F32, qtype, rows, k, wb, xb, np.empty(ylen, np.float32))
        assert got.value.status == want.value.code, (qtype, rows, k, str(got.value), want.value.message)
        assert str(got.value) == want.value.message
    with pytest.raises(ob.Unsupported):
        ctx.host_storage_matvec(ob.CONTRACT_Q8K, ob.TYPE_Q8_0, 2, 64, w, x)


def test_device_pointer_validation(ctx):
    w = to_dev(synth.weight(ob.TYPE_Q4_K, 4, 256, "gpu", "ptr"))
    y = torch.empty(4, dtype=torch.float32, device=DEV)
    x = torch.zeros(256, dtype=torch.float32, device=DEV)
    with pytest.raises(ob.InvalidArgument, match="16-byte aligned"):
        ctx.storage_matvec(ob.CONTRACT_Q8K, ob.TYPE_Q4_K, 4, 256, w.data_ptr() + 8, x, y, w_nbytes=4 * 144)
    ctx.storage_matvec(ob.CONTRACT_Q8K, ob.TYPE_Q4_K, 4, 256, w, x, y)
    assert torch.all(y == 0)  # x = 0 quantizes to d = 0


# ---------------------------------------------------------------- failure detection without a fault

def test_bounded_wait_reports_timeout_and_context_survives(ctx, port):
    ctx.device_status()  # clean
    ctx.selftest_bounded_wait(50_000_000)  # 50 ms deadline on a barrier nobody completes
    with pytest.raises(ob.DeviceTimeout, match="site 99"):
        ctx.device_status()
    ctx.device_status()  # the status word was cleared and the context is still usable
    rows, k = 8, 512
    w = synth.weight(ob.TYPE_Q6_K, rows, k, "gpu", "after_timeout")
    x = synth.activations(k, 1, "gpu", "after_timeout_x")
    y = torch.empty(rows, dtype=torch.float32, device=DEV)
    ctx.storage_matvec(ob.CONTRACT_Q8K, ob.TYPE_Q6_K, rows, k, to_dev(w), to_dev(x), y)
    assert bits_equal(y.cpu().numpy(), port.matvec_q8_k(ob.TYPE_Q6_K, rows, k, w, port.quantize_q8_k(x))[0])


# ---------------------------------------------------------------- matvec programs (one persistent launch)

def _program_case(port, specs, cfg):
    """specs: (qtype, rows, cols, after_previous); activations chain when flagged."""
    host, dev_ops, want = [], [], []
    prev_y_host = prev_y_dev = None
    for i, (qtype, rows, cols, after) in enumerate(specs):
        w = synth.weight(qtype, rows, cols, cfg, f"prog_w{i}")
        if after:
            x_host, x_dev = prev_y_host[:cols], prev_y_dev
        else:
            x_host = synth.activations(cols, 1, cfg, f"prog_x{i}")[0]
            x_dev = to_dev(x_host)
        y_host = port.matvec_q8_k(qtype, rows, cols, w, port.quantize_q8_k(x_host))[0]
        y_dev = torch.empty(rows, dtype=torch.float32, device=DEV)
        dev_ops.append((qtype, rows, cols, to_dev(w), x_dev, y_dev, after))
        want.append(y_host)
        prev_y_host, prev_y_dev = y_host, y_dev
    return dev_ops, want


def test_program_independent_ops(ctx, port):
    specs = [(ob.TYPE_Q4_K, 1536, 4096, 0), (ob.TYPE_Q4_K, 512, 12288, 0), (ob.TYPE_Q4_K, 777, 4096, 0),
             (ob.TYPE_Q4_K, 3, 256, 0)]
    ops, want = _program_case(port, specs, "prog_ind")
    ctx.matvec_program(ops)
    ctx.device_status()
    for (_, _, _, _, _, y, _), w in zip(ops, want):
        assert bits_equal(y.cpu().numpy(), w)


def test_program_dependent_chain_and_repeat(ctx, port):
    # y0 = W0 x0 (4096 -> 12288); y1 = W1 y0 (12288 -> 4096); y2 = W2 y1 (4096 -> 4096)
    specs = [(ob.TYPE_Q4_K, 12288, 4096, 0), (ob.TYPE_Q4_K, 4096, 12288, 1), (ob.TYPE_Q4_K, 4096, 4096, 1)]
    ops, want = _program_case(port, specs, "prog_chain")
    for _ in range(3):  # completion counters reset themselves between launches
        for op in ops:
            op[5].fill_(float("nan"))
        ctx.matvec_program(ops)
        ctx.device_status()
        for (_, _, _, _, _, y, _), w in zip(ops, want):
            assert bits_equal(y.cpu().numpy(), w)


def test_program_many_images_slots(ctx, port):
    """Programs whose fed-in activation images exceed shared memory's share
    (15 distinct activations, ~150 KB of images) copy each op's image into one
    of two slots when the op starts; a dependent op's in-kernel image follows
    the slots; repeated launches reuse everything."""
    specs = [(ob.TYPE_Q4_K, 333 + 7 * i, 4096 if i % 3 else 12288, 0) for i in range(15)]
    specs.append((ob.TYPE_Q4_K, 500, 333 + 7 * 14 - (333 + 7 * 14) % 256, 1))
    ops, want = _program_case(port, specs, "prog_slots")
    for _ in range(2):
        for op in ops:
            op[5].fill_(float("nan"))
        ctx.matvec_program(ops)
        ctx.device_status()
        for (_, _, _, _, _, y, _), w in zip(ops, want):
            assert bits_equal(y.cpu().numpy(), w)


def test_program_mixed_types(ctx, port):
    specs = [(ob.TYPE_Q6_K, 1000, 4096, 0), (ob.TYPE_Q4_K, 300, 768, 0), (ob.TYPE_Q6_K, 513, 768, 0)]
    ops, want = _program_case(port, specs, "prog_mixed")
    ctx.matvec_program(ops)
    ctx.device_status()
    for (_, _, _, _, _, y, _), w in zip(ops, want):
        assert bits_equal(y.cpu().numpy(), w)


@pytest.mark.parametrize("specs", [
    [(ob.TYPE_Q6_K, 1000, 4096, 0), (ob.TYPE_Q6_K, 513, 768, 0), (ob.TYPE_Q6_K, 7, 256, 0)],  # short rows
    [(ob.TYPE_Q6_K, 300, 8192, 0), (ob.TYPE_Q6_K, 77, 512, 0)]])                              # a long row
def test_program_q6k_only(ctx, port, specs):
    """Q6_K-only programs: register-resident activation slices when every row has <= 16 super-blocks."""
    ops, want = _program_case(port, specs, f"prog_q6_{len(specs)}")
    ctx.matvec_program(ops)
    ctx.device_status()
    for (_, _, _, _, _, y, _), w in zip(ops, want):
        assert bits_equal(y.cpu().numpy(), w)


@pytest.mark.parametrize("specs", [
    # Q4_K rows of 17..136 super-blocks (ragged last passes, row counts not
    # multiples of the warps), beside short rows, and long-row ops fed by the
    # previous op
    [(ob.TYPE_Q4_K, 149, 17 * 256, 0), (ob.TYPE_Q4_K, 301, 33 * 256, 0), (ob.TYPE_Q4_K, 5, 40 * 256, 0),
     (ob.TYPE_Q4_K, 777, 48 * 256, 0), (ob.TYPE_Q4_K, 333, 4096, 0), (ob.TYPE_Q4_K, 1000, 21 * 256, 0)],
    [(ob.TYPE_Q4_K, 160, 136 * 256, 0)],
    [(ob.TYPE_Q4_K, 211, 112 * 256, 0), (ob.TYPE_Q4_K, 90, 40 * 256, 0)],
    [(ob.TYPE_Q4_K, 5000, 4096, 0), (ob.TYPE_Q4_K, 700, 19 * 256, 1), (ob.TYPE_Q4_K, 4864, 700 - 700 % 256, 1)],
    [(ob.TYPE_Q6_K, 400, 4096, 0), (ob.TYPE_Q4_K, 611, 12288, 0), (ob.TYPE_Q6_K, 99, 12288, 0)],   # mixed
    # Q6_K long rows: segment-major when every segment is a 16-byte multiple
    # (48 and 40 super-blocks), row by row otherwise (20)
    [(ob.TYPE_Q6_K, 333, 48 * 256, 0), (ob.TYPE_Q6_K, 57, 40 * 256, 0), (ob.TYPE_Q6_K, 50, 20 * 256, 0),
     (ob.TYPE_Q6_K, 29, 4096, 0)]])
def test_program_long_rows(ctx, port, specs):
    """Rows longer than 16 super-blocks (several passes over the activation
    image per row), bit-identical to the restatement."""
    ops, want = _program_case(port, specs, f"prog_long_{len(specs)}")
    for _ in range(2):
        for op in ops:
            op[5].fill_(float("nan"))
        ctx.matvec_program(ops)
        ctx.device_status()
        for (_, _, _, _, _, y, _), w in zip(ops, want):
            assert bits_equal(y.cpu().numpy(), w)


def test_program_validation(ctx):
    w = to_dev(synth.weight(ob.TYPE_Q4_K, 4, 256, "gpu", "progval"))
    x = torch.zeros(256, dtype=torch.float32, device=DEV)
    y = torch.empty(4, dtype=torch.float32, device=DEV)
    with pytest.raises(ob.InvalidArgument):
        ctx.matvec_program([])
    with pytest.raises(ob.InvalidArgument):
        ctx.matvec_program([(ob.TYPE_Q4_K, 4, 256, w, x, y, 0)] * 17)
    w8 = to_dev(synth.weight(ob.TYPE_Q8_0, 4, 256, "gpu", "progval8"))
    with pytest.raises(ob.Unsupported, match="op 1"):
        ctx.matvec_program([(ob.TYPE_Q4_K, 4, 256, w, x, y, 0), (ob.TYPE_Q8_0, 4, 256, w8, x, y, 0)])
    with pytest.raises(ob.InvalidArgument, match="op 0: reference matvec matrix byte size mismatch"):
        ctx.matvec_program([(ob.TYPE_Q4_K, 4, 256, w8, x, y, 0)])
