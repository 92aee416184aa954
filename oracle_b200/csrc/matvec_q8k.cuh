// matvec_q8k.cuh -- Q4_K x Q8_K and Q6_K x Q8_K decode matvec (the north-star op).
//
// y[b][r] = dot(W row r, Q8_K(x_b)) with GGML's integer block dot
// (ggml_vec_dot_q{4,6}_K_q8_K; Oracle has no integer dot, its f32 contract is
// quantized_reference.cpp:24-82).  Per super-block i of a row:
//   Q4_K: isum = sum_j sc_j * sum_32(q4 * q8),  msum = sum_j m_j * (bsum_2j + bsum_2j+1)
//         p_i  = (d_w * d_x) * isum - (dmin_w * d_x) * msum
//   Q6_K: isum = sum_s sc_s * (sum_16(q6 * q8) - 32 * bsum_s),  p_i = (d_w * d_x) * isum
// The integer sums are exact (dp4a).  The f32 sum over i is this build's
// canonical order: per 16-super-block segment, leaves 0 + p_i folded by a
// fixed tree (strides 8, 4, 2, 1), then a running sum of the segments in
// increasing order, starting from +0.  The CPU restatement (oq_vec_dot_q8_k)
// performs the same f32 operations, so results match bit for bit.
//
// Work mapping (one warp per row): lane = 2*j + part.  Pass k covers
// super-blocks 16k..16k+15 (segment k); lane (j, part) takes super-block
// 16k + j and the half `part` of its 256 elements (Q4_K: 64-element groups
// 2*part, 2*part+1; Q6_K: half part).  The two lanes of a pair add their
// integer sums with one shuffle; the segment's tree is the xor-16..2 lane
// butterfly, and each lane keeps the running sum of the segments.
//
// The activation is quantized once per CTA into a shared-memory image
// (q8k.cuh).  For rows of at most 16 super-blocks the lane's slice of it (32
// quant words, bsums, d_x) is held in registers for every row; longer rows
// re-read it per pass from the bank-conflict-free swizzled image.
#pragma once

#include "q8k.cuh"
#include "stream.cuh"

namespace oracle_cuda {

struct MatvecQ8KParams {
    const float* x;      // f32 activations (quantized in the prologue), or null
    const uint8_t* q8k;  // pre-quantized GGML Q8_K blocks, or null
    float* y;
    uint64_t rows;
    uint32_t nb;         // super-blocks per row (k / 256)
};

__device__ __forceinline__ int dp4a(uint32_t a, uint32_t b, int c) {
    return __dp4a(static_cast<int>(a), static_cast<int>(b), c);
}

// Unsigned bytes of a times signed bytes of b, accumulated into c.
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

__device__ __forceinline__ int ubyte(uint32_t w, int i) { return static_cast<int>((w >> (8 * i)) & 0xFFu); }

// Lane's integer sums for its half of one Q4_K super-block at `sb` (16-byte aligned).
__device__ __forceinline__ void q4k_half_sums(const uint8_t* sb, int part, const uint32_t (&xw)[32],
                                              const int (&xbs)[8], int& isum, int& msum,
                                              float& dw, float& dmw) {
    const uint4 hdr = *reinterpret_cast<const uint4*>(sb);
    dw = f16_bits_to_f32(static_cast<uint16_t>(hdr.x & 0xFFFFu));
    dmw = f16_bits_to_f32(static_cast<uint16_t>(hdr.x >> 16));
    const uint32_t sc_lo = hdr.y & 0x3F3F3F3Fu;
    const uint32_t mn_lo = hdr.z & 0x3F3F3F3Fu;
    const uint32_t sc_hi = (hdr.w & 0x0F0F0F0Fu) | ((hdr.y >> 2) & 0x30303030u);
    const uint32_t mn_hi = ((hdr.w >> 4) & 0x0F0F0F0Fu) | ((hdr.z >> 2) & 0x30303030u);
    const uint32_t scw = part ? sc_hi : sc_lo;
    const uint32_t mnw = part ? mn_hi : mn_lo;

    const uint4* qv = reinterpret_cast<const uint4*>(sb + 16 + 64 * part);
    uint32_t w[16];
#pragma unroll
    for (int v = 0; v < 4; ++v) {
        const uint4 t = qv[v];
        w[4 * v + 0] = t.x;
        w[4 * v + 1] = t.y;
        w[4 * v + 2] = t.z;
        w[4 * v + 3] = t.w;
    }
    // High nibbles are used in place (byte & 0xF0 = 16 * nibble): their dot
    // products come out 16x larger, exactly, and are shifted back.
    int d0 = 0, d1 = 0, d2 = 0, d3 = 0;
#pragma unroll
    for (int t = 0; t < 8; ++t) {
        d0 = dp4a(w[t] & 0x0F0F0F0Fu, xw[t], d0);
        d1 = dp4a_us(w[t] & 0xF0F0F0F0u, xw[8 + t], d1);
        d2 = dp4a(w[8 + t] & 0x0F0F0F0Fu, xw[16 + t], d2);
        d3 = dp4a_us(w[8 + t] & 0xF0F0F0F0u, xw[24 + t], d3);
    }
    isum = ubyte(scw, 0) * d0 + ubyte(scw, 1) * (d1 >> 4) + ubyte(scw, 2) * d2 + ubyte(scw, 3) * (d3 >> 4);
    msum = ubyte(mnw, 0) * xbs[0] + ubyte(mnw, 1) * xbs[1] + ubyte(mnw, 2) * xbs[2] +
           ubyte(mnw, 3) * xbs[3];
}

// `n` consecutive little-endian words starting at an even shared address.
template <int N>
__device__ __forceinline__ void lds_words_even(const uint8_t* p, uint32_t (&out)[N]) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    const uint32_t* base = reinterpret_cast<const uint32_t*>(a & ~uintptr_t(3));
    const uint32_t sh = static_cast<uint32_t>(a & 3u) * 8u;
    uint32_t prev = base[0];
#pragma unroll
    for (int i = 0; i < N; ++i) {
        const uint32_t next = base[i + 1];
        out[i] = __funnelshift_r(prev, next, sh);
        prev = next;
    }
}

// Lane's integer sum for half `h` of one Q6_K super-block at `sb` (even address).
// xbs holds 32 * bsum for the half's 8 sixteen-element groups.
__device__ __forceinline__ void q6k_half_sums(const uint8_t* sb, int h, const uint32_t (&xw)[32],
                                              const int (&xbs32)[8], int& isum, float& dw) {
    uint32_t lo[16], qh[8], scw[2];
    lds_words_even<16>(sb + 64 * h, lo);
    lds_words_even<8>(sb + 128 + 32 * h, qh);
    lds_words_even<2>(sb + 192 + 8 * h, scw);
    dw = f16_bits_to_f32(lds_u16(sb + 208));
    int dot[8];
#pragma unroll
    for (int t = 0; t < 8; ++t) dot[t] = 0;
#pragma unroll
    for (int w = 0; w < 8; ++w) {
        const uint32_t a = lo[w], b = lo[8 + w], c = qh[w];
        const uint32_t q0 = (a & 0x0F0F0F0Fu) | ((c << 4) & 0x30303030u);
        const uint32_t q1 = (b & 0x0F0F0F0Fu) | ((c << 2) & 0x30303030u);
        const uint32_t q2 = ((a >> 4) & 0x0F0F0F0Fu) | (c & 0x30303030u);
        const uint32_t q3 = ((b >> 4) & 0x0F0F0F0Fu) | ((c >> 2) & 0x30303030u);
        dot[0 + w / 4] = dp4a(q0, xw[w], dot[0 + w / 4]);
        dot[2 + w / 4] = dp4a(q1, xw[8 + w], dot[2 + w / 4]);
        dot[4 + w / 4] = dp4a(q2, xw[16 + w], dot[4 + w / 4]);
        dot[6 + w / 4] = dp4a(q3, xw[24 + w], dot[6 + w / 4]);
    }
    int s = 0;
#pragma unroll
    for (int t = 0; t < 8; ++t) s += sbyte(scw[t / 4], t % 4) * (dot[t] - xbs32[t]);
    isum = s;
}

// The lane's activation data for one pass: 128 quants (32 words) of half
// `part` of block i, its four 32-element sums (Q4_K) or 32 x its eight
// 16-element sums (Q6_K), and d_x.
template <uint32_t kType>
__device__ __forceinline__ void fetch_lane_x(const ActImage& img, uint32_t i, int part, uint32_t (&xw)[32],
                                             int (&xbs)[8], float& xd) {
    const uint32_t rho = 2u * i + part;
    const uint8_t* row = reinterpret_cast<const uint8_t*>(img.q) + rho * 128u;
#pragma unroll
    for (int v = 0; v < 8; ++v) {
        const uint4 t = *reinterpret_cast<const uint4*>(row + 16u * (uint32_t(v) ^ (rho & 7u)));
        xw[4 * v + 0] = t.x;
        xw[4 * v + 1] = t.y;
        xw[4 * v + 2] = t.z;
        xw[4 * v + 3] = t.w;
    }
    if (kType == 12) {
        const int4 b = *reinterpret_cast<const int4*>(img.bs32 + 8 * i + 4 * part);
        xbs[0] = b.x; xbs[1] = b.y; xbs[2] = b.z; xbs[3] = b.w;
        xbs[4] = xbs[5] = xbs[6] = xbs[7] = 0;
    } else {
        const int4 b0 = *reinterpret_cast<const int4*>(img.bs16 + 16 * i + 8 * part);
        const int4 b1 = *reinterpret_cast<const int4*>(img.bs16 + 16 * i + 8 * part + 4);
        xbs[0] = 32 * b0.x; xbs[1] = 32 * b0.y; xbs[2] = 32 * b0.z; xbs[3] = 32 * b0.w;
        xbs[4] = 32 * b1.x; xbs[5] = 32 * b1.y; xbs[6] = 32 * b1.z; xbs[7] = 32 * b1.w;
    }
    xd = img.d[i];
}

// One row's dot product in the canonical order; the result is valid on lane 0.
// kXReg: rows of at most 16 super-blocks (one pass) with the lane's activation
// slice (xw, xbs, xd) already in registers; otherwise every pass re-reads it
// from the shared-memory image (conflict-free).
// kUnroll: passes unrolled by this factor (2 lets a pass's shared loads
// overlap the previous pass's arithmetic, where registers allow).
template <uint32_t kType, bool kXReg, int kUnroll = 1>
__device__ __forceinline__ float q8k_row_dot(uint32_t nb, const ActImage& img, const uint8_t* rowp,
                                             const uint32_t (&xw)[32], const int (&xbs)[8], float xd, int lane) {
    const int j = lane >> 1, part = lane & 1;
    constexpr uint32_t kBlockBytes = kType == 12 ? 144u : 210u;
    const uint32_t passes = kXReg ? 1u : (nb + 15u) / 16u;
    float total = 0.0f;
#pragma unroll kUnroll
    for (uint32_t k = 0; k < passes; ++k) {
        const uint32_t i = 16u * k + j;
        const bool active = i < nb;
        int isum = 0, msum = 0;
        float dw = 0.0f, dmw = 0.0f, dx = 0.0f;
        if (active) {
            const uint8_t* sb = rowp + size_t(i) * kBlockBytes;
            if constexpr (kXReg) {
                dx = xd;
                if (kType == 12)
                    q4k_half_sums(sb, part, xw, xbs, isum, msum, dw, dmw);
                else
                    q6k_half_sums(sb, part, xw, xbs, isum, dw);
            } else {
                uint32_t w[32];
                int bs[8];
                fetch_lane_x<kType>(img, i, part, w, bs, dx);
                if (kType == 12)
                    q4k_half_sums(sb, part, w, bs, isum, msum, dw, dmw);
                else
                    q6k_half_sums(sb, part, w, bs, isum, dw);
            }
        }
        isum += __shfl_xor_sync(0xFFFFFFFFu, isum, 1);
        if (kType == 12) msum += __shfl_xor_sync(0xFFFFFFFFu, msum, 1);
        float leaf = 0.0f;
        if (active) {
            const float dd = __fmul_rn(dw, dx);
            float pi = __fmul_rn(dd, __int2float_rn(isum));
            if (kType == 12) {
                const float dm = __fmul_rn(dmw, dx);
                pi = __fsub_rn(pi, __fmul_rn(dm, __int2float_rn(msum)));
            }
            leaf = __fadd_rn(leaf, pi);
        }
#pragma unroll
        for (int off = 16; off >= 2; off >>= 1) leaf = __fadd_rn(leaf, __shfl_xor_sync(0xFFFFFFFFu, leaf, off));
        total = __fadd_rn(total, leaf);
    }
    return total;
}

// One segment's tree for two rows at once: leaves la (row A) and lb (row B)
// on lanes 2j + part (both lanes of a pair hold the same leaf), the two
// trees sharing their first level (lanes 0-15 keep row A's sums of leaves j
// and j + 8, lanes 16-31 row B's, by one exchange), then folding 4, 2, 1 as
// one.  Row A's segment sum on lanes 0-15, row B's on lanes 16-31.
__device__ __forceinline__ float q8k_segment_tree2(float la, float lb, int lane) {
    const bool low = lane < 16;
    float v = __fadd_rn(low ? la : lb, __shfl_xor_sync(0xFFFFFFFFu, low ? lb : la, 16));
#pragma unroll
    for (int off = 8; off >= 2; off >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xFFFFFFFFu, v, off));
    return v;
}

// Two rows at once (the same activation slice fetched once per pass for
// both): each row's terms and its per-lane accumulators exactly as
// q8k_row_dot computes them; the two butterflies share their first level
// (lanes 0-15 keep row A's sums of pairs j and j + 8, lanes 16-31 row B's,
// by one exchange), then fold 8, 4, 2 lanes as one.  The result is row A's
// dot product on lane 0 and row B's on lane 16, bit-identical to
// q8k_row_dot (every addition has the same two operands; fadd commutes).
template <uint32_t kType, bool kXReg>
__device__ __forceinline__ float q8k_row_dot2(uint32_t nb, const ActImage& img, const uint8_t* rowa,
                                              const uint8_t* rowb, const uint32_t (&xw)[32], const int (&xbs)[8],
                                              float xd, int lane) {
    const int j = lane >> 1, part = lane & 1;
    constexpr uint32_t kBlockBytes = kType == 12 ? 144u : 210u;
    const uint32_t passes = kXReg ? 1u : (nb + 15u) / 16u;
    float total = 0.0f;  // lanes 0-15: row A's running sum, lanes 16-31: row B's
#pragma unroll 1
    for (uint32_t k = 0; k < passes; ++k) {
        const uint32_t i = 16u * k + j;
        const bool active = i < nb;
        int ia = 0, ma = 0, ib = 0, mb = 0;
        float dwa = 0.0f, dmwa = 0.0f, dwb = 0.0f, dmwb = 0.0f, dx = 0.0f;
        if (active) {
            const size_t off = size_t(i) * kBlockBytes;
            if constexpr (kXReg) {
                dx = xd;
                if (kType == 12) {
                    q4k_half_sums(rowa + off, part, xw, xbs, ia, ma, dwa, dmwa);
                    q4k_half_sums(rowb + off, part, xw, xbs, ib, mb, dwb, dmwb);
                } else {
                    q6k_half_sums(rowa + off, part, xw, xbs, ia, dwa);
                    q6k_half_sums(rowb + off, part, xw, xbs, ib, dwb);
                }
            } else {
                uint32_t w[32];
                int bs[8];
                fetch_lane_x<kType>(img, i, part, w, bs, dx);
                if (kType == 12) {
                    q4k_half_sums(rowa + off, part, w, bs, ia, ma, dwa, dmwa);
                    q4k_half_sums(rowb + off, part, w, bs, ib, mb, dwb, dmwb);
                } else {
                    q6k_half_sums(rowa + off, part, w, bs, ia, dwa);
                    q6k_half_sums(rowb + off, part, w, bs, ib, dwb);
                }
            }
        }
        ia += __shfl_xor_sync(0xFFFFFFFFu, ia, 1);
        ib += __shfl_xor_sync(0xFFFFFFFFu, ib, 1);
        if (kType == 12) {
            ma += __shfl_xor_sync(0xFFFFFFFFu, ma, 1);
            mb += __shfl_xor_sync(0xFFFFFFFFu, mb, 1);
        }
        float la = 0.0f, lb = 0.0f;
        if (active) {
            float pa = __fmul_rn(__fmul_rn(dwa, dx), __int2float_rn(ia));
            float pb = __fmul_rn(__fmul_rn(dwb, dx), __int2float_rn(ib));
            if (kType == 12) {
                pa = __fsub_rn(pa, __fmul_rn(__fmul_rn(dmwa, dx), __int2float_rn(ma)));
                pb = __fsub_rn(pb, __fmul_rn(__fmul_rn(dmwb, dx), __int2float_rn(mb)));
            }
            la = __fadd_rn(la, pa);
            lb = __fadd_rn(lb, pb);
        }
        total = __fadd_rn(total, q8k_segment_tree2(la, lb, lane));
    }
    return total;
}

// Pass `seg` of q8k_row_dot2 for two rows whose super-blocks 16 * seg .. are at
// sega and segb (the segment's start): the activation slice of the segment
// is fetched once for both rows; la and lb are the rows' leaves (0 + p_i, or
// +0 past the row's end) exactly as q8k_row_dot2 forms them.
template <uint32_t kType>
__device__ __forceinline__ void q8k_segment_pass2(uint32_t nb, const ActImage& img, uint32_t seg,
                                                  const uint8_t* sega, const uint8_t* segb, int lane, float& la,
                                                  float& lb) {
    constexpr uint32_t kBlockBytes = kType == 12 ? 144u : 210u;
    const int part = lane & 1;
    const uint32_t j = static_cast<uint32_t>(lane) >> 1;
    const uint32_t i = 16u * seg + j;
    const bool active = i < nb;
    int ia = 0, ma = 0, ib = 0, mb = 0;
    float dwa = 0.0f, dmwa = 0.0f, dwb = 0.0f, dmwb = 0.0f, dx = 0.0f;
    if (active) {
        uint32_t w[32];
        int bs[8];
        fetch_lane_x<kType>(img, i, part, w, bs, dx);
        const uint32_t off = j * kBlockBytes;
        if (kType == 12) {
            q4k_half_sums(sega + off, part, w, bs, ia, ma, dwa, dmwa);
            q4k_half_sums(segb + off, part, w, bs, ib, mb, dwb, dmwb);
        } else {
            q6k_half_sums(sega + off, part, w, bs, ia, dwa);
            q6k_half_sums(segb + off, part, w, bs, ib, dwb);
        }
    }
    ia += __shfl_xor_sync(0xFFFFFFFFu, ia, 1);
    ib += __shfl_xor_sync(0xFFFFFFFFu, ib, 1);
    if (kType == 12) {
        ma += __shfl_xor_sync(0xFFFFFFFFu, ma, 1);
        mb += __shfl_xor_sync(0xFFFFFFFFu, mb, 1);
    }
    if (active) {
        float pa = __fmul_rn(__fmul_rn(dwa, dx), __int2float_rn(ia));
        float pb = __fmul_rn(__fmul_rn(dwb, dx), __int2float_rn(ib));
        if (kType == 12) {
            pa = __fsub_rn(pa, __fmul_rn(__fmul_rn(dmwa, dx), __int2float_rn(ma)));
            pb = __fsub_rn(pb, __fmul_rn(__fmul_rn(dmwb, dx), __int2float_rn(mb)));
        }
        la = __fadd_rn(0.0f, pa);
        lb = __fadd_rn(0.0f, pb);
    } else {
        la = lb = 0.0f;
    }
}

// q8k_segment_pass2 for one row (where two rows' registers would spill).
template <uint32_t kType>
__device__ __forceinline__ void q8k_segment_pass1(uint32_t nb, const ActImage& img, uint32_t seg,
                                                  const uint8_t* sega, int lane, float& la) {
    constexpr uint32_t kBlockBytes = kType == 12 ? 144u : 210u;
    const int part = lane & 1;
    const uint32_t j = static_cast<uint32_t>(lane) >> 1;
    const uint32_t i = 16u * seg + j;
    const bool active = i < nb;
    int ia = 0, ma = 0;
    float dwa = 0.0f, dmwa = 0.0f, dx = 0.0f;
    if (active) {
        uint32_t w[32];
        int bs[8];
        fetch_lane_x<kType>(img, i, part, w, bs, dx);
        if (kType == 12)
            q4k_half_sums(sega + j * kBlockBytes, part, w, bs, ia, ma, dwa, dmwa);
        else
            q6k_half_sums(sega + j * kBlockBytes, part, w, bs, ia, dwa);
    }
    ia += __shfl_xor_sync(0xFFFFFFFFu, ia, 1);
    if (kType == 12) ma += __shfl_xor_sync(0xFFFFFFFFu, ma, 1);
    if (active) {
        float pa = __fmul_rn(__fmul_rn(dwa, dx), __int2float_rn(ia));
        if (kType == 12) pa = __fsub_rn(pa, __fmul_rn(__fmul_rn(dmwa, dx), __int2float_rn(ma)));
        la = __fadd_rn(0.0f, pa);
    } else {
        la = 0.0f;
    }
}

// The lane's activation slice for register-resident rows (<= 16 super-blocks).
template <uint32_t kType>
__device__ __forceinline__ void load_lane_x(const ActImage& img, uint32_t nb, int lane, uint32_t (&xw)[32],
                                            int (&xbs)[8], float& xd) {
    const uint32_t i = lane >> 1;
    if (i < nb) {
        fetch_lane_x<kType>(img, i, lane & 1, xw, xbs, xd);
    } else {
#pragma unroll
        for (int v = 0; v < 32; ++v) xw[v] = 0u;
#pragma unroll
        for (int t = 0; t < 8; ++t) xbs[t] = 0;
        xd = 0.0f;
    }
}

template <uint32_t kType, bool kXReg, int kWarps_>
struct MatvecQ8KConsumer {
    static constexpr int kWarps = kWarps_;
    using Params = MatvecQ8KParams;

    uint32_t xw[32];
    int xbs[8];
    float xd = 0.0f;

    __device__ __forceinline__ void prologue(const Params& p, uint8_t* act, int warp, int lane) {
        const ActImage img = q8k_image(act, p.nb);
        if (p.x)
            quantize_to_image(p.x, p.nb, img, warp, kWarps, lane);
        else
            load_q8k_to_image(p.q8k, p.nb, img, warp, kWarps, lane);
    }

    __device__ __forceinline__ void load(const Params& p, uint8_t* act, int, int lane) {
        if constexpr (kXReg) load_lane_x<kType>(q8k_image(act, p.nb), p.nb, lane, xw, xbs, xd);
    }

    __device__ __forceinline__ void row(const Params& p, uint8_t* act, const uint8_t* rowp, uint64_t r,
                                        int lane) {
        const float v = q8k_row_dot<kType, kXReg>(p.nb, q8k_image(act, p.nb), rowp, xw, xbs, xd, lane);
        if (lane == 0) p.y[r] = v;
    }
};

}  // namespace oracle_cuda
