// matvec_f32.cuh -- Oracle's f32 contract on the GPU: y = decode_f32(W) . x.
//
// Oracle's reference_storage_matvec (quantized_reference.cpp:128-162) decodes
// each block to f32 and adds decoded * x into one running f32 sum per row.
// Here each weight is decoded to exactly Oracle's f32 value (decode.cuh) and
// multiplied into x with a fused multiply-add; lane l owns 4-element chunks
// l, l+32, ... of the row (x is read conflict-free from shared memory), and
// the 32 lane sums fold by xor-shuffles.  Only the summation order differs
// from Oracle, and the result is at least as accurate (checked against an f64
// arbiter in the tests).
#pragma once

#include "decode.cuh"
#include "stream.cuh"

namespace oracle_cuda {

struct MatvecF32Params {
    const float* x;  // batch vectors of k floats
    float* y;        // batch * rows
    uint64_t rows;
    uint32_t k;
    uint32_t kpad;   // k rounded up to 128; the image pads with zeros
    uint32_t batch;
};

__host__ __device__ inline uint32_t f32_image_bytes(uint32_t kpad, uint32_t batch) {
    return align_up(kpad * 4u * batch, 128u);
}

template <uint32_t kType, int kWarps_>
struct MatvecF32Consumer {
    static constexpr int kWarps = kWarps_;
    using Params = MatvecF32Params;

    __device__ __forceinline__ void prologue(const Params& p, uint8_t* act, int warp, int lane) {
        float* xs = reinterpret_cast<float*>(act);
        const uint32_t n = p.kpad * p.batch;
        for (uint32_t i = warp * 32 + lane; i < n; i += kWarps * 32) {
            const uint32_t b = i / p.kpad, e = i % p.kpad;
            xs[i] = e < p.k ? p.x[uint64_t(b) * p.k + e] : 0.0f;
        }
    }

    __device__ __forceinline__ void load(const Params&, uint8_t*, int, int) {}

    __device__ __forceinline__ void row(const Params& p, uint8_t* act, const uint8_t* rowp, uint64_t r,
                                        int lane) {
        const float* xs = reinterpret_cast<const float*>(act);
        const uint32_t chunks = p.kpad / 4;
        for (uint32_t b = 0; b < p.batch; ++b) {
            const float4* xv = reinterpret_cast<const float4*>(xs + uint64_t(b) * p.kpad);
            float acc = 0.0f;
#pragma unroll 4
            for (uint32_t c = lane; c < chunks; c += 32) {
                const uint32_t e = 4 * c;
                if (e >= p.k) break;
                float w[4];
                decode4<kType, false>(rowp, e, p.k, w);
                const float4 x = xv[c];
                acc = __fmaf_rn(w[0], x.x, acc);
                acc = __fmaf_rn(w[1], x.y, acc);
                acc = __fmaf_rn(w[2], x.z, acc);
                acc = __fmaf_rn(w[3], x.w, acc);
            }
#pragma unroll
            for (int off = 16; off >= 1; off >>= 1) acc += __shfl_xor_sync(0xFFFFFFFFu, acc, off);
            if (lane == 0) p.y[uint64_t(b) * p.rows + r] = acc;
        }
    }
};

}  // namespace oracle_cuda
