"""CPU: pin the restatement (oracle/quant_oracle.c) before trusting it.

1. The reference's own known answers (tests/test_phase2a.cpp in the Oracle
   repository), rebuilt here block by block, through the restatement and
   through the reference's compiled code.
2. Bit equality with the reference's compiled decoders and f32 matvec, live and
   through the committed fixture tests/golden/reference.npz.
3. Bit equality of Q8_0/Q4_K/Q5_K/Q6_K decode with gguf-py 0.19.0
   (tests/golden/decode_ggufpy.npz), the outside pin for Q4_K.
4. Q8_K quantizer properties and integer dots re-derived with numpy integer
   arithmetic, plus the committed regression fixture tests/golden/q8k.npz.
5. The integer dot's semantics (nibbles, scales, mins, the Q6_K offset) tied
   to gguf-py's dequantization in f64, and the quantizer's defining
   properties (scale from the signed largest element, nearest quants).
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import golden
from oracle_b200 import synth

T = synth


def u16le(v):
    return np.frombuffer(np.uint16(v).tobytes(), np.uint8)


# ---------------------------------------------------------------- reference fixtures (test_phase2a.cpp:50-88)

def q5_fixture():
    b = np.zeros(176, np.uint8)
    b[0:2] = u16le(0x3800)  # d = 0.5
    b[2:4] = u16le(0x3400)  # dmin = 0.25
    b[4:16] = [2, 2, 2, 2, 3, 3, 3, 3, 0x32, 0x32, 0x32, 0x32]
    b[16:48] = 0xFF
    b[48:] = 0x21
    return b


def q4_fixture():
    """Q4_K analogue of the Q5_K fixture: same header and qs, no high-bit plane."""
    b = np.zeros(144, np.uint8)
    b[0:16] = q5_fixture()[0:16]
    b[16:] = 0x21
    return b


def q6_fixture():
    b = np.zeros(210, np.uint8)
    b[0:128] = 0x21
    b[128:192] = 0xFF
    b[192:208] = 0x02
    b[208:210] = u16le(0x3800)
    return b


Q8_QUANTS = [0, 1, -1, 127, -128, 2, -2, 3, -3, 4, -4, 5, -5, 6, -6, 7,
             -7, 8, -8, 9, -9, 10, -10, 11, -11, 12, -12, 13, -13, 14, -14, 15]


def q8_0_fixture(d=0x3C00, quants=Q8_QUANTS):
    b = np.zeros(34, np.uint8)
    b[0:2] = u16le(d)
    b[2:] = np.array(quants, np.int8).view(np.uint8)
    return b


def test_half_conversions(port):
    # test_phase2a.cpp:90-106
    assert port.f16_to_f32(0x3C00) == 1.0
    assert port.f16_to_f32(0xC000) == -2.0
    assert port.f16_to_f32(0x0001) == np.ldexp(1.0, -24)
    assert np.isinf(port.f16_to_f32(0x7C00))
    assert np.isnan(port.f16_to_f32(0x7E00))
    assert np.signbit(port.f16_to_f32(0x8000))
    # every f16 bit pattern against numpy's exact conversion
    bits = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    want = bits.view(np.float16).astype(np.float32)
    got = np.array([port.lib.oq_f16_to_f32(int(b)) for b in bits[::97]], np.float32)
    want = want[::97]
    # NaNs compare by NaN-ness: Oracle keeps the payload bits (signalling NaNs
    # stay signalling, storage_decode.cpp:169-170), numpy quiets them.
    nan = np.isnan(want)
    assert np.array_equal(np.isnan(got), nan)
    assert np.array_equal(got[~nan].view(np.uint32), want[~nan].view(np.uint32))


def test_known_answers_port(port):
    ones256 = np.ones(256, np.float32)
    q5 = port.decode_rows(T.TYPE_Q5_K, 1, 256, q5_fixture())[0]
    for g in range(4):
        assert np.all(q5[64 * g:64 * g + 32] == 16.25) and np.all(q5[64 * g + 32:64 * g + 64] == 17.25)
    assert port.storage_matvec_f32(T.TYPE_Q5_K, 1, 256, q5_fixture(), ones256)[0, 0] == 4288.0
    two = np.concatenate([q5_fixture(), q5_fixture()])
    assert port.storage_matvec_f32(T.TYPE_Q5_K, 1, 512, two, np.ones(512, np.float32))[0, 0] == 8576.0
    second = q5_fixture().copy()
    second[16:] = 0
    mat = np.concatenate([q5_fixture(), second])
    assert port.storage_matvec_f32(T.TYPE_Q5_K, 2, 256, mat, ones256)[0].tolist() == [4288.0, -192.0]

    q6 = port.decode_rows(T.TYPE_Q6_K, 1, 256, q6_fixture())[0]
    for h in range(2):
        assert np.all(q6[128 * h:128 * h + 64] == 17.0) and np.all(q6[128 * h + 64:128 * h + 128] == 18.0)
    assert port.storage_matvec_f32(T.TYPE_Q6_K, 1, 256, q6_fixture(), ones256)[0, 0] == 4480.0

    q8 = port.decode_rows(T.TYPE_Q8_0, 1, 32, q8_0_fixture())[0]
    assert q8.tolist() == [float(v) for v in Q8_QUANTS]
    second8 = q8_0_fixture(0x3800, [10] * 32)
    dec = port.decode_rows(T.TYPE_Q8_0, 1, 64, np.concatenate([q8_0_fixture(), second8]))[0]
    assert dec[3] == 127.0 and dec[32] == 5.0 and dec[63] == 5.0
    mat8 = np.concatenate([q8_0_fixture(), q8_0_fixture(0x3800, [4] * 32)])
    assert port.storage_matvec_f32(T.TYPE_Q8_0, 2, 32, mat8, np.ones(32, np.float32))[0].tolist() == [14.0, 64.0]

    # Q4_K analogue: low nibble 1 -> (0.5*2)*1 - 0.25*3 = 0.25, high nibble 2 -> 1.25
    q4 = port.decode_rows(T.TYPE_Q4_K, 1, 256, q4_fixture())[0]
    for g in range(4):
        assert np.all(q4[64 * g:64 * g + 32] == 0.25) and np.all(q4[64 * g + 32:64 * g + 64] == 1.25)
    assert port.storage_matvec_f32(T.TYPE_Q4_K, 1, 256, q4_fixture(), ones256)[0, 0] == 192.0


def test_known_answers_reference(ref):
    ones256 = np.ones(256, np.float32)
    assert ref.storage_dot(T.TYPE_Q5_K, 256, q5_fixture(), ones256) == 4288.0
    assert ref.storage_dot(T.TYPE_Q6_K, 256, q6_fixture(), ones256) == 4480.0
    assert ref.storage_dot(T.TYPE_Q8_0, 32, q8_0_fixture(), np.ones(32, np.float32)) == 14.0
    second = q5_fixture().copy()
    second[16:] = 0
    assert ref.storage_matvec(T.TYPE_Q5_K, 2, 256, np.concatenate([q5_fixture(), second]),
                              ones256).tolist() == [4288.0, -192.0]
    # Oracle rejects Q4_K, the type this path adds (storage_decode.cpp:192-196)
    with pytest.raises(Exception, match="does not support GGML type 12"):
        ref.decode_row(T.TYPE_Q4_K, 256, q4_fixture())


@pytest.mark.parametrize("qtype,k", [(T.TYPE_Q8_0, 64), (T.TYPE_Q5_K, 512), (T.TYPE_Q6_K, 768),
                                     (T.TYPE_F16, 33), (T.TYPE_BF16, 33), (T.TYPE_F32, 33)])
def test_port_matches_reference_live(port, ref, qtype, k):
    rows = 9
    w = synth.weight(qtype, rows, k, "pins", f"live_{qtype}")
    x = synth.activations(k, 1, "pins", f"live_x_{qtype}")[0]
    dec = port.decode_rows(qtype, rows, k, w)
    want = np.stack([ref.decode_row(qtype, k, w[r]) for r in range(rows)])
    assert np.array_equal(dec.view(np.uint32), want.view(np.uint32))
    y = port.storage_matvec_f32(qtype, rows, k, w, x)[0]
    yr = ref.storage_matvec(qtype, rows, k, w, x)
    assert np.array_equal(y.view(np.uint32), yr.view(np.uint32))


def test_port_matches_reference_fixture(port):
    g = golden("reference.npz")
    for qtype, name in [(T.TYPE_Q8_0, "Q8_0"), (T.TYPE_Q5_K, "Q5_K"), (T.TYPE_Q6_K, "Q6_K"),
                        (T.TYPE_F16, "F16"), (T.TYPE_BF16, "BF16"), (T.TYPE_F32, "F32")]:
        w, x = g[f"{name}_w"], g[f"{name}_x"]
        rows, k = w.shape[0], x.size
        assert np.array_equal(port.decode_rows(qtype, rows, k, w).view(np.uint32),
                              g[f"{name}_decoded"].view(np.uint32)), name
        assert np.array_equal(port.storage_matvec_f32(qtype, rows, k, w, x)[0].view(np.uint32),
                              g[f"{name}_matvec"].view(np.uint32)), name


def test_port_matches_ggufpy_fixture(port):
    g = golden("decode_ggufpy.npz")
    for qtype, name in [(T.TYPE_Q8_0, "Q8_0"), (T.TYPE_Q4_K, "Q4_K"), (T.TYPE_Q5_K, "Q5_K"), (T.TYPE_Q6_K, "Q6_K")]:
        blocks, want = g[f"{name}_blocks"], g[f"{name}_decoded"]
        got = port.decode_rows(qtype, blocks.shape[0], want.shape[1], blocks)
        same = (got.view(np.uint32) == want.view(np.uint32)) | (np.isnan(got) & np.isnan(want))
        assert same.all(), name


# ---------------------------------------------------------------- Q8_K and the integer dots

def np_quantize_q8k(x: np.ndarray):
    """Independent numpy statement of the Q8_K rule, for cross-checking."""
    x = x.reshape(-1, 256).astype(np.float32)
    ax = np.abs(x)
    idx = ax.argmax(axis=1)  # first index of the maximum
    amax = ax[np.arange(len(x)), idx]
    vmax = x[np.arange(len(x)), idx]
    with np.errstate(divide="ignore", invalid="ignore"):
        iscale = np.where(amax == 0, 0, np.float32(-127.0) / vmax).astype(np.float32)
    q = np.rint((iscale[:, None] * x).astype(np.float32)).astype(np.int32)
    q = np.minimum(q, 127)
    q[amax == 0] = 0
    with np.errstate(divide="ignore"):
        d = np.where(amax == 0, 0, np.float32(1.0) / iscale).astype(np.float32)
    bs = q.reshape(len(x), 16, 16).sum(axis=2)
    return d, q.astype(np.int8), bs.astype(np.int16)


def split_q8k(raw: np.ndarray):
    raw = raw.reshape(-1, 292)
    return (raw[:, 0:4].copy().view(np.float32).reshape(-1), raw[:, 4:260].view(np.int8),
            raw[:, 260:292].copy().view(np.int16))


def test_q8k_quantizer_properties(port):
    g = golden("q8k.npz")
    x = g["x"]
    raw = port.quantize_q8_k(x)[0]
    assert np.array_equal(raw, g["q8k"])  # regression lock
    d, q, bs = split_q8k(raw)
    nd, nq, nbs = np_quantize_q8k(x)
    assert np.array_equal(d.view(np.uint32), nd.view(np.uint32))
    assert np.array_equal(q, nq) and np.array_equal(bs, nbs)
    assert np.all(q >= -127) and np.all(q <= 127)
    assert d[0] == 0 and np.all(q[0] == 0) and np.all(bs[0] == 0)  # zero block
    # ties: the first element of largest magnitude sets the sign of d (d = -max/127)
    assert d[1] < 0 and q[1, 7] == -127 and q[1, 200] == 127
    assert d[2] > 0 and q[2, 5] == -127 and q[2, 9] == 127
    rng = synth.rng_for("pins", "q8k_random")
    xr = rng.standard_normal(256 * 64).astype(np.float32) * rng.uniform(0.01, 100, 256 * 64).astype(np.float32)
    d, q, bs = split_q8k(port.quantize_q8_k(xr)[0])
    nd, nq, nbs = np_quantize_q8k(xr)
    assert np.array_equal(d.view(np.uint32), nd.view(np.uint32)) and np.array_equal(q, nq)
    assert np.array_equal(bs, q.astype(np.int32).reshape(-1, 16, 16).sum(axis=2))


def np_q4k_values(block: np.ndarray):
    sc = np.zeros(8, np.int64)
    mn = np.zeros(8, np.int64)
    s = block[4:16].astype(np.int64)
    for j in range(8):
        if j < 4:
            sc[j], mn[j] = s[j] & 63, s[j + 4] & 63
        else:
            sc[j] = (s[j + 4] & 15) | ((s[j - 4] >> 6) << 4)
            mn[j] = (s[j + 4] >> 4) | ((s[j] >> 6) << 4)
    qs = block[16:].astype(np.int64).reshape(4, 32)
    q = np.stack([qs & 15, qs >> 4], axis=1).reshape(256)
    return q, sc, mn


def np_q6k_values(block: np.ndarray):
    ql = block[0:128].astype(np.int64)
    qh = block[128:192].astype(np.int64)
    sc = block[192:208].view(np.int8).astype(np.int64)
    q = np.zeros(256, np.int64)
    for h in range(2):
        for s in range(4):
            lo = ql[64 * h + 32 * (s & 1):64 * h + 32 * (s & 1) + 32]
            lo = (lo >> 4) if s >= 2 else (lo & 15)
            hi = (qh[32 * h:32 * h + 32] >> (2 * s)) & 3
            q[128 * h + 32 * s:128 * h + 32 * s + 32] = lo | (hi << 4)
    return q, sc


def test_integer_block_sums_match_numpy(port):
    g = golden("q8k.npz")
    q8 = g["q8k"].reshape(-1, 292)
    nb = q8.shape[0]
    for r in range(3):
        for i in range(nb):
            xq = q8[i, 4:260].view(np.int8).astype(np.int64)
            xbs = q8[i, 260:292].copy().view(np.int16).astype(np.int64)
            q, sc, mn = np_q4k_values(g["w4"][r, 144 * i:144 * (i + 1)])
            isum = int(sum(sc[j] * np.dot(q[32 * j:32 * j + 32], xq[32 * j:32 * j + 32]) for j in range(8)))
            msum = int(sum(mn[j] * (xbs[2 * j] + xbs[2 * j + 1]) for j in range(8)))
            assert (isum, msum) == tuple(g["sums4"][r, i])
            q6, sc6 = np_q6k_values(g["w6"][r, 210 * i:210 * (i + 1)])
            isum6 = int(sum(sc6[s] * np.dot(q6[16 * s:16 * s + 16] - 32, xq[16 * s:16 * s + 16]) for s in range(16)))
            assert isum6 == g["sums6"][r, i][0]
            assert port.block_sums(T.TYPE_Q4_K, g["w4"][r, 144 * i:144 * (i + 1)], q8[i]) == tuple(g["sums4"][r, i])


@pytest.mark.parametrize("qtype", [T.TYPE_Q4_K, T.TYPE_Q6_K])
def test_dot_orders_agree_within_tolerance(port, qtype):
    rows, k = 64, 12288
    w = synth.weight(qtype, rows, k, "pins", f"order_{qtype}")
    x = synth.activations(k, 1, "pins", "order_x")[0]
    q8 = port.quantize_q8_k(x)[0]
    y = port.matvec_q8_k(qtype, rows, k, w, q8)[0]
    yg = np.array([port.vec_dot_q8_k_ggml_order(qtype, k, w[r], q8) for r in range(rows)], np.float32)
    # The canonical order and GGML's generic order add the same exact integer
    # sums in different f32 orders.  Rounding is relative to the summed terms,
    # not to y (a row can cancel to near zero), so the bound is 1e-6 absolute
    # + 1e-5 relative to sum_i |d_w d_x isum_i| + |dmin_w d_x msum_i|.
    bb = 144 if qtype == T.TYPE_Q4_K else 210
    q8b = q8.reshape(-1, 292)
    dx = q8b[:, 0:4].copy().view(np.float32).reshape(-1).astype(np.float64)
    scale = np.zeros(rows)
    for r in range(rows):
        for i in range(k // 256):
            blk = w[r, bb * i:bb * (i + 1)]
            isum, msum = port.block_sums(qtype, blk, q8b[i])
            if qtype == T.TYPE_Q4_K:
                d, dmin = blk[0:4].copy().view(np.float16).astype(np.float64)
            else:
                d, dmin = blk[208:210].copy().view(np.float16).astype(np.float64)[0], 0.0
            scale[r] += abs(d * dx[i] * isum) + abs(dmin * dx[i] * msum)
    assert np.all(np.abs(y - yg) <= 1e-6 + 1e-5 * scale), (np.abs(y - yg) / scale).max()


def test_matvec_q8k_fixture(port):
    g = golden("q8k.npz")
    k = g["x"].size
    assert np.array_equal(port.matvec_q8_k(T.TYPE_Q4_K, 3, k, g["w4"], g["q8k"])[0].view(np.uint32),
                          g["y4"].view(np.uint32))
    assert np.array_equal(port.matvec_q8_k(T.TYPE_Q6_K, 3, k, g["w6"], g["q8k"])[0].view(np.uint32),
                          g["y6"].view(np.uint32))


# ---------------------------------------------------------------- the integer dot against a third party

@pytest.mark.parametrize("qtype,k", [(T.TYPE_Q4_K, 4096), (T.TYPE_Q4_K, 12288), (T.TYPE_Q6_K, 4096)])
def test_integer_dot_pinned_to_ggufpy_decode(port, qtype, k):
    """The Q4_K/Q6_K x Q8_K integer dot tied to gguf-py 0.19.0 (a third
    party): for seeded rows of the config-2/3 shapes, every super-block term
    the restatement forms from its exact integer sums, d_w*d_x*isum -
    dmin_w*d_x*msum (Q4_K) or d_w*d_x*isum (Q6_K, the -32 folded through the
    bsums), equals sum_e w_e * (d_x * q8_e) computed in f64 from gguf-py's own
    dequantization of the weights and the Q8_K block's quants.  The only
    difference allowed is gguf-py's f32 rounding of each w_e (at most four
    roundings of 2^-24 each), so a wrong nibble order, scale or min index, or
    offset would miss by the size of the term itself.  The row results of the
    canonical f32 combine then sit within the north star's 1e-6 absolute +
    1e-5 relative (to the summed term magnitudes) of the f64 row sums."""
    gq = pytest.importorskip("gguf.quants")
    import gguf
    rows = 24
    w = synth.weight(qtype, rows, k, "pins", f"ggufpy_dot_{qtype}_{k}")
    x = synth.activations(k, 1, "pins", f"ggufpy_dot_x_{k}")[0]
    raw = port.quantize_q8_k(x)[0]
    d8, q8, _ = split_q8k(raw)
    xq = (q8.astype(np.float64) * d8.astype(np.float64)[:, None]).reshape(-1)
    gtype = gguf.GGMLQuantizationType(qtype)
    wf = gq.dequantize(w.reshape(rows, -1), gtype).astype(np.float64).reshape(rows, k)
    nb = k // 256
    prod = (wf * xq).reshape(rows, nb, 256)
    ref_terms = prod.sum(axis=2)
    ref_mag = np.abs(prod).sum(axis=2)
    bb = 144 if qtype == T.TYPE_Q4_K else 210
    q8b = raw.reshape(-1, 292)
    dx = d8.astype(np.float64)
    terms = np.zeros((rows, nb))
    mags = np.zeros(rows)
    for r in range(rows):
        for i in range(nb):
            blk = w[r, bb * i:bb * (i + 1)]
            isum, msum = port.block_sums(qtype, blk, q8b[i])
            if qtype == T.TYPE_Q4_K:
                d, dmin = blk[0:4].copy().view(np.float16).astype(np.float64)
            else:
                d, dmin = blk[208:210].copy().view(np.float16).astype(np.float64)[0], 0.0
            terms[r, i] = d * dx[i] * isum - dmin * dx[i] * msum
            mags[r] += abs(d * dx[i] * isum) + abs(dmin * dx[i] * msum)
    assert np.all(np.abs(terms - ref_terms) <= 4 * 2.0 ** -24 * ref_mag + 1e-30), \
        (np.abs(terms - ref_terms) / ref_mag).max()
    y = port.matvec_q8_k(qtype, rows, k, w, raw)[0].astype(np.float64)
    assert np.all(np.abs(y - ref_terms.sum(axis=1)) <= 1e-6 + 1e-5 * mags)
    # the pin has teeth: the same check against a decode with one sub-block's
    # scale index swapped fails by far more than the bound
    if qtype == T.TYPE_Q4_K:
        bad = wf.reshape(rows, nb, 8, 32).copy()
        bad[:, :, [0, 1]] = bad[:, :, [1, 0]]
        bad_terms = (bad.reshape(rows, k) * xq).reshape(rows, nb, 256).sum(axis=2)
        assert np.abs(terms - bad_terms).max() > 1e3 * (4 * 2.0 ** -24 * ref_mag).max()


def test_q8k_quantizer_rounding_properties(port):
    """What the Q8_K quantizer's definition fixes, checked on seeded config-2
    activations without a GGML vector (none exists in the reference or this
    image): d is the signed largest-magnitude element over -127 (its quant
    is -127 exactly), every quant is the nearest integer to x/d within half a
    step (clamped to [-127, 127]), and every bsum is the sum of its 16
    quants.  Bit-level choices (IEEE division for the scale, ties to even)
    stay pinned only to the restatement."""
    x = synth.activations(12288, 1, "pins", "q8k_rounding")[0]
    d, q, bs = split_q8k(port.quantize_q8_k(x)[0])
    xb = x.reshape(-1, 256).astype(np.float64)
    i = np.abs(xb).argmax(axis=1)
    assert np.all(q[np.arange(len(xb)), i] == -127)
    assert np.allclose(d.astype(np.float64), -xb[np.arange(len(xb)), i] / 127.0, rtol=2e-7)
    err = np.abs(xb - q.astype(np.float64) * d.astype(np.float64)[:, None])
    assert np.all(err <= 0.5 * np.abs(d.astype(np.float64))[:, None] * (1 + 1e-6))
    assert np.all(np.abs(q.astype(np.int32)) <= 127)
    assert np.array_equal(bs.astype(np.int32), q.astype(np.int32).reshape(-1, 16, 16).sum(axis=2))
