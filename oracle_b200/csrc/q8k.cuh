// q8k.cuh -- Q8_K activation quantizer (f32 -> {f32 d; i8 qs[256]; i16 bsums[16]}).
//
// Restates GGML's quantize_row_q8_K_ref (ggml/src/ggml-quants.c, the commit
// Oracle's docs pin); Oracle registers only the layout (ggml_type.cpp:28,
// {15, "q8_K", 256, 292}).  Per 256-element block:
//   max    = the element of largest magnitude, the first one on ties
//   iscale = -127 / max                       (IEEE f32 division)
//   q[j]   = min(127, round_half_even(iscale * x[j]))
//   bsums  = sums of 16 consecutive q
//   d      = 1 / iscale                       (IEEE f32 division)
// An all-zero block gives d = 0, q = 0, bsums = 0.  Every f32 operation is an
// explicit round-to-nearest intrinsic, so the bytes match the CPU restatement
// exactly.  Inputs must be finite.
#pragma once

#include "common.cuh"

namespace oracle_cuda {

__host__ __device__ constexpr uint32_t align_up(uint32_t v, uint32_t a) { return (v + a - 1) / a * a; }

// One warp quantizes one 256-element block.  Lane l owns elements 8l..8l+7.
// Outputs: q_lo/q_hi = the lane's 8 quants (little-endian bytes), bsum16 = the
// sum over the 16-element group (lanes 2g, 2g+1) containing the lane, d.
struct Q8KLane {
    uint32_t q_lo, q_hi;
    int bsum16;
    float d;
};

__device__ __forceinline__ void load_lane8(const float* xb, int lane, bool aligned16, float (&v)[8]) {
    // L2 (.cg) loads: the activation may have been written by another SM
    // earlier in the same launch (matvec programs), so L1 must not serve it.
    if (aligned16) {
        const float4 a = __ldcg(reinterpret_cast<const float4*>(xb) + 2 * lane);
        const float4 b = __ldcg(reinterpret_cast<const float4*>(xb) + 2 * lane + 1);
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
        v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = __ldcg(xb + 8 * lane + j);
    }
}

// Quantize one block from the lane's 8 values (elements 8*lane .. 8*lane+7).
__device__ __forceinline__ Q8KLane quantize_q8k_lane_values(const float (&v)[8], int lane) {
    // first strictly-greater scan inside the lane, then a warp arg-max that
    // prefers the lower index on ties: the result is the sequential scan's.
    float amax = 0.0f, vmax = 0.0f;
    int idx = 0x7FFFFFFF;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const float a = fabsf(v[j]);
        if (a > amax) {
            amax = a;
            vmax = v[j];
            idx = 8 * lane + j;
        }
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) {
        const float oa = __shfl_xor_sync(0xFFFFFFFFu, amax, off);
        const float ov = __shfl_xor_sync(0xFFFFFFFFu, vmax, off);
        const int oi = __shfl_xor_sync(0xFFFFFFFFu, idx, off);
        if (oa > amax || (oa == amax && oi < idx)) {
            amax = oa;
            vmax = ov;
            idx = oi;
        }
    }
    Q8KLane out;
    if (amax == 0.0f) {
        out.q_lo = out.q_hi = 0u;
        out.bsum16 = 0;
        out.d = 0.0f;
        return out;
    }
    const float iscale = __fdiv_rn(-127.0f, vmax);
    uint32_t packed[2] = {0u, 0u};
    int sum = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        int q = __float2int_rn(__fmul_rn(iscale, v[j]));
        q = q > 127 ? 127 : q;
        sum += q;
        packed[j / 4] |= (static_cast<uint32_t>(q) & 0xFFu) << (8 * (j % 4));
    }
    out.q_lo = packed[0];
    out.q_hi = packed[1];
    out.bsum16 = sum + __shfl_xor_sync(0xFFFFFFFFu, sum, 1);
    out.d = __fdiv_rn(1.0f, iscale);
    return out;
}

__device__ __forceinline__ Q8KLane quantize_q8k_block_warp(const float* xb, int lane, bool aligned16) {
    float v[8];
    load_lane8(xb, lane, aligned16, v);
    return quantize_q8k_lane_values(v, lane);
}

// Standalone quantizer: one warp per (activation row, block); GGML byte layout
// (292 bytes per block, 4-byte aligned fields).
__global__ void __launch_bounds__(256) quantize_q8k_kernel(const float* __restrict__ x,
                                                           uint64_t k, uint64_t batch,
                                                           uint8_t* __restrict__ out) {
    const uint64_t nb = k / 256;
    const uint64_t block = (static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x) / 32;
    const int lane = threadIdx.x & 31;
    if (block >= nb * batch) return;
    const float* xb = x + block * 256;
    const bool aligned16 = (reinterpret_cast<uintptr_t>(xb) & 15u) == 0;
    const Q8KLane r = quantize_q8k_block_warp(xb, lane, aligned16);
    uint8_t* ob = out + block * 292;
    if (lane == 0) *reinterpret_cast<float*>(ob) = r.d;
    uint32_t* qs = reinterpret_cast<uint32_t*>(ob + 4);
    qs[2 * lane] = r.q_lo;
    qs[2 * lane + 1] = r.q_hi;
    if ((lane & 1) == 0) reinterpret_cast<int16_t*>(ob + 260)[lane / 2] = static_cast<int16_t>(r.bsum16);
}

// Shared-memory activation image used by the matvec kernels.  Quants are
// stored in 128-byte rows, row rho = 2*i + h holding elements 128h..128h+127 of
// block i; the 16-byte chunk v of row rho sits at chunk position
// v ^ (rho & 7), so the eight lanes of a quarter-warp reading eight consecutive
// rows hit eight different bank groups.  bs16[16*i + g] holds the sum of the
// 16-element group g, bs32[8*i + j] that of the 32-element sub-block j, d[i]
// the block scale.
struct ActImage {
    int8_t* q;
    int* bs16;
    int* bs32;
    float* d;
};

__host__ __device__ inline uint32_t q8k_image_bytes(uint32_t nb) {
    return align_up(nb * 256u, 128u) + align_up(nb * 64u, 128u) + align_up(nb * 32u, 128u) +
           align_up(nb * 4u, 128u);
}

__device__ __forceinline__ ActImage q8k_image(uint8_t* act, uint32_t nb) {
    ActImage img;
    uint32_t off = 0;
    img.q = reinterpret_cast<int8_t*>(act + off);
    off += align_up(nb * 256u, 128u);
    img.bs16 = reinterpret_cast<int*>(act + off);
    off += align_up(nb * 64u, 128u);
    img.bs32 = reinterpret_cast<int*>(act + off);
    off += align_up(nb * 32u, 128u);
    img.d = reinterpret_cast<float*>(act + off);
    return img;
}

// Byte offset of element e (0..255) of block i in the swizzled quant rows.
__device__ __forceinline__ uint32_t q8k_image_offset(uint32_t i, uint32_t e) {
    const uint32_t rho = 2u * i + (e >> 7);
    return rho * 128u + 16u * (((e >> 4) & 7u) ^ (rho & 7u)) + (e & 15u);
}

// Lane l of a warp holds elements 8l..8l+7 of block i and the sum of its
// 16-element group (lanes 2g, 2g+1 share group g); store them in the image.
__device__ __forceinline__ void store_block_to_image(ActImage img, uint32_t i, int lane, uint32_t q_lo,
                                                     uint32_t q_hi, int bsum16, float d) {
    uint2* dst = reinterpret_cast<uint2*>(img.q + q8k_image_offset(i, 8u * lane));
    *dst = make_uint2(q_lo, q_hi);
    const int bsum32 = bsum16 + __shfl_xor_sync(0xFFFFFFFFu, bsum16, 2);
    if ((lane & 1) == 0) img.bs16[16 * i + lane / 2] = bsum16;
    if ((lane & 3) == 0) img.bs32[8 * i + lane / 4] = bsum32;
    if (lane == 0) img.d[i] = d;
}

// Quantize `nb` blocks of x into the image, one block per warp, warps
// [0, nwarps) cooperating.  The caller synchronises afterwards.
// The loads of up to kBatch blocks are issued together before any of them is
// reduced, so a warp pays one memory round trip per kBatch blocks.
__device__ __forceinline__ void quantize_to_image(const float* __restrict__ x, uint32_t nb,
                                                  ActImage img, int warp, int nwarps, int lane) {
    constexpr int kBatch = 4;
    const bool aligned16 = (reinterpret_cast<uintptr_t>(x) & 15u) == 0;
    for (uint32_t base = warp; base < nb; base += uint32_t(nwarps) * kBatch) {
        float v[kBatch][8];
#pragma unroll
        for (int m = 0; m < kBatch; ++m) {
            const uint32_t i = base + uint32_t(m) * nwarps;
            if (i < nb) load_lane8(x + 256ull * i, lane, aligned16, v[m]);
        }
#pragma unroll
        for (int m = 0; m < kBatch; ++m) {
            const uint32_t i = base + uint32_t(m) * nwarps;
            if (i >= nb) break;
            const Q8KLane r = quantize_q8k_lane_values(v[m], lane);
            store_block_to_image(img, i, lane, r.q_lo, r.q_hi, r.bsum16, r.d);
        }
    }
}

// Activation transforms applied while quantizing, so that the f32 vector a
// matvec reads never has to be written out (decode programs):
//   kXformNone    v = x
//   kXformRms     v = (x * inv) * w, inv = rms_inverse(sum of x^2 over the
//                 whole vector): Oracle's rms_norm_rows for one row
//                 (qwen35_block.cpp:161-188)
//   kXformSwiglu  v = silu(x) * x2: the MLP activation (qwen35_block.cpp:315-318)
//   kXformCombineRms  (matvec programs of a sharded peer group only) v =
//                 kXformRms of x + the fold of every rank's partial sums
//                 (program.cuh, program_fold_partials)
enum : uint32_t { kXformNone = 0, kXformRms = 1, kXformSwiglu = 2, kXformCombineRms = 3 };

struct ActSource {
    const float* x;
    const float* x2;    // swiglu: up
    const float* norm;  // rms: weights
    float eps;
    uint32_t xform;
};

__device__ __forceinline__ bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// The lane's 8 transformed values of block i (inv: the rms inverse, else unused).
__device__ __forceinline__ void load_lane8_xform(const ActSource& a, uint32_t i, int lane, float inv, float (&v)[8]) {
    const float* xb = a.x + 256ull * i;
    load_lane8(xb, lane, aligned16(xb), v);
    if (a.xform == kXformRms) {
        float w[8];
        const float* wb = a.norm + 256ull * i;
        load_lane8(wb, lane, aligned16(wb), w);
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = __fmul_rn(__fmul_rn(v[j], inv), w[j]);
    } else if (a.xform == kXformSwiglu) {
        float u[8];
        const float* ub = a.x2 + 256ull * i;
        load_lane8(ub, lane, aligned16(ub), u);
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = __fmul_rn(ref_silu(v[j]), u[j]);
    }
}

// A warp's partial double sum of squares over elements [first, n) with stride
// `stride` (each product exact in double, sums rounded).
__device__ __forceinline__ double sum_squares_f64(const float* __restrict__ x, uint32_t first, uint32_t n,
                                                  uint32_t stride) {
    double s = 0.0;
    // sixteen (predicated) loads in flight per round, so a thread's share of a
    // decode-sized vector is one round; the additions keep the element order
    constexpr uint32_t kB = 16;
    for (uint32_t c = first; c < n; c += kB * stride) {
        float v[kB];
#pragma unroll
        for (uint32_t u = 0; u < kB; ++u) v[u] = c + u * stride < n ? __ldcg(x + c + u * stride) : 0.0f;
#pragma unroll
        for (uint32_t u = 0; u < kB; ++u)
            if (c + u * stride < n)
                s = __dadd_rn(s, __dmul_rn(static_cast<double>(v[u]), static_cast<double>(v[u])));
    }
    return s;
}

// Quantize `nb` transformed blocks into the image, warps [0, nwarps) of the
// calling group cooperating (inv as for load_lane8_xform).
__device__ __forceinline__ void quantize_xform_to_image(const ActSource& a, uint32_t nb, float inv, ActImage img,
                                                        int warp, int nwarps, int lane) {
    if (a.xform == kXformNone) {
        // kPlainBatch blocks per round: their loads are in flight together
        constexpr int kPlainBatch = 2;
        for (uint32_t i = warp; i < nb; i += kPlainBatch * nwarps) {
            float v[kPlainBatch][8];
#pragma unroll
            for (int m = 0; m < kPlainBatch; ++m) {
                const uint32_t im = i + m * nwarps;
                if (im < nb) load_lane8(a.x + 256ull * im, lane, aligned16(a.x + 256ull * im), v[m]);
            }
#pragma unroll
            for (int m = 0; m < kPlainBatch; ++m) {
                const uint32_t im = i + m * nwarps;
                if (im >= nb) break;
                const Q8KLane r = quantize_q8k_lane_values(v[m], lane);
                store_block_to_image(img, im, lane, r.q_lo, r.q_hi, r.bsum16, r.d);
            }
        }
        return;
    }
    // two blocks per round: both blocks' loads are in flight together
    for (uint32_t i = warp; i < nb; i += 2 * nwarps) {
        const uint32_t i2 = i + nwarps;
        float v[8], v2[8];
        load_lane8_xform(a, i, lane, inv, v);
        if (i2 < nb) load_lane8_xform(a, i2, lane, inv, v2);
        const Q8KLane r = quantize_q8k_lane_values(v, lane);
        store_block_to_image(img, i, lane, r.q_lo, r.q_hi, r.bsum16, r.d);
        if (i2 < nb) {
            const Q8KLane r2 = quantize_q8k_lane_values(v2, lane);
            store_block_to_image(img, i2, lane, r2.q_lo, r2.q_hi, r2.bsum16, r2.d);
        }
    }
}

// Quantize up to kMaxImageJobs activations, each into its own image inside
// one global buffer laid out exactly like the shared-memory images, so a
// consumer can copy the whole region into shared memory unchanged.  One warp
// per 256-element block; blocks of all jobs are numbered consecutively.
constexpr int kMaxImageJobs = 16;
struct ImageJobs {
    const float* x[kMaxImageJobs];
    const float* x2[kMaxImageJobs];
    const float* norm[kMaxImageJobs];
    float eps[kMaxImageJobs];
    uint32_t xform[kMaxImageJobs];
    uint32_t nb[kMaxImageJobs];
    uint32_t offset[kMaxImageJobs];  // byte offset of the job's image
    uint32_t first_block[kMaxImageJobs + 1];
    uint32_t n_jobs;
};

// One warp quantizes block `gw` of the jobs' concatenated blocks into its image.
__device__ __forceinline__ void quantize_image_block(const ImageJobs& jobs, uint32_t gw, uint8_t* images, int lane) {
    uint32_t j = 0;
    while (gw >= jobs.first_block[j + 1]) ++j;
    const uint32_t i = gw - jobs.first_block[j];
    const ActSource a{jobs.x[j], jobs.x2[j], jobs.norm[j], jobs.eps[j], jobs.xform[j]};
    float inv = 0.0f;
    if (a.xform == kXformRms) {
        const uint32_t n = jobs.nb[j] * 256u;
        inv = rms_inverse(warp_sum_f64(sum_squares_f64(a.x, lane, n, 32u)), n, a.eps);
    }
    float v[8];
    load_lane8_xform(a, i, lane, inv, v);
    const Q8KLane r = quantize_q8k_lane_values(v, lane);
    store_block_to_image(q8k_image(images + jobs.offset[j], jobs.nb[j]), i, lane, r.q_lo, r.q_hi, r.bsum16, r.d);
}

__global__ void __launch_bounds__(256) quantize_images_kernel(const __grid_constant__ ImageJobs jobs, uint8_t* images) {
    // The image buffer is reused by every program launch: wait until the
    // preceding kernel (possibly the previous program, still reading it) is
    // done, but let the next kernel start streaming its weights already.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const uint32_t gw = (blockIdx.x * blockDim.x + threadIdx.x) / 32;
    const int lane = threadIdx.x & 31;
    if (gw >= jobs.first_block[jobs.n_jobs]) return;
    quantize_image_block(jobs, gw, images, lane);
}

// Load pre-quantized GGML Q8_K blocks (global) into the image.
__device__ __forceinline__ void load_q8k_to_image(const uint8_t* __restrict__ q8k, uint32_t nb,
                                                  ActImage img, int warp, int nwarps, int lane) {
    for (uint32_t i = warp; i < nb; i += nwarps) {
        const uint8_t* b = q8k + 292ull * i;
        const uint32_t* qs = reinterpret_cast<const uint32_t*>(b + 4);
        const int bsum16 = reinterpret_cast<const int16_t*>(b + 260)[lane / 2];
        store_block_to_image(img, i, lane, qs[2 * lane], qs[2 * lane + 1], bsum16,
                             *reinterpret_cast<const float*>(b));
    }
}

}  // namespace oracle_cuda
