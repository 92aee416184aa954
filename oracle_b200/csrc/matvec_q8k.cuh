// matvec_q8k.cuh -- Q4_K x Q8_K and Q6_K x Q8_K decode matvec (the north-star op).
//
// y[b][r] = dot(W row r, Q8_K(x_b)) with GGML's integer block dot
// (ggml_vec_dot_q{4,6}_K_q8_K; Oracle has no integer dot, its f32 contract is
// quantized_reference.cpp:24-82).  Per super-block i of a row:
//   Q4_K: isum = sum_j sc_j * sum_32(q4 * q8),  msum = sum_j m_j * (bsum_2j + bsum_2j+1)
//         p_i  = (d_w * d_x) * isum - (dmin_w * d_x) * msum
//   Q6_K: isum = sum_s sc_s * (sum_16(q6 * q8) - 32 * bsum_s),  p_i = (d_w * d_x) * isum
// The integer sums are exact (dp4a).  The f32 sum over i is this build's
// canonical order: slot[i % 32] accumulates p_i in increasing i, then slots
// fold by strides 16, 8, 4, 2, 1.  The CPU restatement (oq_vec_dot_q8_k)
// performs the same f32 operations, so results match bit for bit.
//
// Work mapping (one warp per row): lane = 2*j + part.  Pass k covers
// super-blocks 16k..16k+15; lane (j, part) takes super-block 16k + j and the
// half `part` of its 256 elements (Q4_K: 64-element groups 2*part, 2*part+1;
// Q6_K: half part).  The two lanes of a pair add their integer sums with one
// shuffle; slot[j] and slot[j + 16] live in the pair's two accumulators, and
// the stride-8..1 folds are xor-16..2 lane shuffles.
//
// The lane's 128 activation quants (32 words), its sub-block bsums and d_x are
// loaded once into registers (kPasses compile-time) and reused for every row.
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
    int d0 = 0, d1 = 0, d2 = 0, d3 = 0;
#pragma unroll
    for (int t = 0; t < 8; ++t) {
        d0 = dp4a(w[t] & 0x0F0F0F0Fu, xw[t], d0);
        d1 = dp4a((w[t] >> 4) & 0x0F0F0F0Fu, xw[8 + t], d1);
        d2 = dp4a(w[8 + t] & 0x0F0F0F0Fu, xw[16 + t], d2);
        d3 = dp4a((w[8 + t] >> 4) & 0x0F0F0F0Fu, xw[24 + t], d3);
    }
    isum = ubyte(scw, 0) * d0 + ubyte(scw, 1) * d1 + ubyte(scw, 2) * d2 + ubyte(scw, 3) * d3;
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

// Activation image region size for nb super-blocks.
__host__ __device__ inline uint32_t q8k_image_bytes(uint32_t nb) {
    return align_up(nb * 256u, 128u) + align_up(nb * 16u * 4u, 128u) + align_up(nb * 4u, 128u);
}

__device__ __forceinline__ ActImage q8k_image(uint8_t* act, uint32_t nb) {
    ActImage img;
    img.q = reinterpret_cast<int8_t*>(act);
    img.bs = reinterpret_cast<int*>(act + align_up(nb * 256u, 128u));
    img.d = reinterpret_cast<float*>(act + align_up(nb * 256u, 128u) + align_up(nb * 64u, 128u));
    return img;
}

template <uint32_t kType, int kPasses, int kWarps_>
struct MatvecQ8KConsumer {
    static constexpr int kWarps = kWarps_;
    using Params = MatvecQ8KParams;

    uint32_t xw[kPasses][32];
    int xbs[kPasses][8];
    float xd[kPasses];

    __device__ __forceinline__ void prologue(const Params& p, uint8_t* act, int warp, int lane) {
        const ActImage img = q8k_image(act, p.nb);
        if (p.x)
            quantize_to_image(p.x, p.nb, img, warp, kWarps, lane);
        else
            load_q8k_to_image(p.q8k, p.nb, img, warp, kWarps, lane);
    }

    __device__ __forceinline__ void load(const Params& p, uint8_t* act, int, int lane) {
        const ActImage img = q8k_image(act, p.nb);
        const int j = lane >> 1, part = lane & 1;
#pragma unroll
        for (int k = 0; k < kPasses; ++k) {
            const uint32_t i = 16u * k + j;
            if (i < p.nb) {
                const uint4* src = reinterpret_cast<const uint4*>(img.q + 256 * i + 128 * part);
#pragma unroll
                for (int v = 0; v < 8; ++v) {
                    const uint4 t = src[v];
                    xw[k][4 * v + 0] = t.x;
                    xw[k][4 * v + 1] = t.y;
                    xw[k][4 * v + 2] = t.z;
                    xw[k][4 * v + 3] = t.w;
                }
                const int* bs = img.bs + 16 * i + 8 * part;
                if (kType == 12) {
                    // sub-block (32 elements) sums for sub-blocks 4*part .. 4*part+3
#pragma unroll
                    for (int t = 0; t < 4; ++t) xbs[k][t] = bs[2 * t] + bs[2 * t + 1];
#pragma unroll
                    for (int t = 4; t < 8; ++t) xbs[k][t] = 0;
                } else {
#pragma unroll
                    for (int t = 0; t < 8; ++t) xbs[k][t] = 32 * bs[t];
                }
                xd[k] = img.d[i];
            } else {
#pragma unroll
                for (int v = 0; v < 32; ++v) xw[k][v] = 0u;
#pragma unroll
                for (int t = 0; t < 8; ++t) xbs[k][t] = 0;
                xd[k] = 0.0f;
            }
        }
    }

    __device__ __forceinline__ void row(const Params& p, uint8_t*, const uint8_t* rowp, uint64_t r,
                                        int lane) {
        const int j = lane >> 1, part = lane & 1;
        constexpr uint32_t kBlockBytes = kType == 12 ? 144u : 210u;
        float acc0 = 0.0f, acc1 = 0.0f;
#pragma unroll
        for (int k = 0; k < kPasses; ++k) {
            const uint32_t i = 16u * k + j;
            const bool active = i < p.nb;
            int isum = 0, msum = 0;
            float dw = 0.0f, dmw = 0.0f;
            if (active) {
                const uint8_t* sb = rowp + size_t(i) * kBlockBytes;
                if (kType == 12)
                    q4k_half_sums(sb, part, xw[k], xbs[k], isum, msum, dw, dmw);
                else
                    q6k_half_sums(sb, part, xw[k], xbs[k], isum, dw);
            }
            isum += __shfl_xor_sync(0xFFFFFFFFu, isum, 1);
            if (kType == 12) msum += __shfl_xor_sync(0xFFFFFFFFu, msum, 1);
            if (active) {
                const float dd = __fmul_rn(dw, xd[k]);
                float pi = __fmul_rn(dd, __int2float_rn(isum));
                if (kType == 12) {
                    const float dm = __fmul_rn(dmw, xd[k]);
                    pi = __fsub_rn(pi, __fmul_rn(dm, __int2float_rn(msum)));
                }
                if (k & 1)
                    acc1 = __fadd_rn(acc1, pi);
                else
                    acc0 = __fadd_rn(acc0, pi);
            }
        }
        float v = __fadd_rn(acc0, acc1);
#pragma unroll
        for (int off = 16; off >= 2; off >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xFFFFFFFFu, v, off));
        if (lane == 0) p.y[r] = v;
    }
};

}  // namespace oracle_cuda
