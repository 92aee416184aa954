// matvec_batch.cuh -- Q4_K / Q6_K x Q8_K matvec over up to 16 activation
// vectors at once (batched decode): every weight byte is read from HBM once
// per launch, whatever the batch.
//
// y[b][r] = dot(W row r, Q8_K(x_b)), bit-identical per vector to the batch-1
// kernels and to the CPU restatement (oq_vec_dot_q8_k): the same exact integer
// sub-block sums, the same f32 term p_i per super-block, the same canonical
// order (per 16-super-block segment the fixed tree over leaves 0 + p_i --
// strides 8, 4, 2, 1 -- then a running sum over the segments, from 0).
//
// Integer sums on the tensor cores (mma.sync, 8-bit x 8-bit -> s32): the
// ACTIVATIONS are the A operand (M = 16 vectors), 8 weight rows the B operand
// (N = 8), one sub-block the K dimension.
//   Q4_K: per 32-element sub-block j, D_j = A_j * nibbles_j (m16n8k32) and
//         isum += sc_j * D_j per (vector, row).  The min term
//         msum = sum_j m_j * bsum32_j (bsum32 = the sub-block's q8 sum) is one
//         more contraction, over j: the activation image carries each vector's
//         bsum32 split as 64 * hi + lo (hi, lo 8-bit), so msum is two
//         m16n8k16 MMAs against the row's mins.
//   Q6_K: per 16-element sub-block s, D_s = A_s * q6_s (m16n8k16, q6 in 0..63)
//         and isum += sc_s * D_s; the offset term 32 * sum_s sc_s * bsum16_s
//         is two m16n8k16 MMAs of the split bsum16 against the row's scales.
// Every sum is the exact integer the dp4a kernels form, so every p_i is
// bit-identical.
//
// Work items are (tile of 8 rows, segment).  The CTAs are shared out among the
// segments (CTA c works on segment c * G / grid) and each splits its
// segment's tiles evenly.  Per item, 8 consumer warps share a stage of
// 8 rows x the segment's super-blocks: warp r computes leaves r and r + 8
// (0 + p, or 0 past the row's end) side by side and adds them -- the tree's
// first level, N1(r) = L_r + L_{r+8} -- and, working on the same two
// super-blocks for every tile, holds their activation operands in registers
// for the whole launch.  The N1 values meet in shared memory and the rest of
// the tree runs across lanes in its own order:
// N3(0) = (N1(0) + N1(4)) + (N1(2) + N1(6)), N3(1) the same over the odd
// ones, root = N3(0) + N3(1).  With one segment per row
// y = 0 + root; with several, each root goes to a partial-sum buffer and a
// second kernel adds a row's segments in order (batch_combine_kernel).
//
// Accumulator layout (mma.sync): thread (g = lane / 4, t = lane % 4) holds
// e = 0: (vector g, row 2t), 1: (g, 2t + 1), 2: (g + 8, 2t), 3: (g + 8, 2t + 1).
#pragma once

#include "decoder_ops.cuh"
#include "q8k.cuh"

namespace oracle_cuda {

constexpr int kBatchMax = 16;             // vectors per launch (the MMA's M)
constexpr int kBatchConsumerWarps = 8;    // warp r: super-blocks r and r + 8 of a segment
constexpr int kBatchThreads = (kBatchConsumerWarps + 1) * 32;
constexpr int kBatchTileRows = 8;         // weight rows per item (the MMA's N)
constexpr int kBatchMaxStages = 12;

// Activation image of one 256-element block:
//   [0, 4096)    quants in the m16n8k32 A-fragment order: uint4 k (0..7) of
//                lane 4g + t holds words 4k + 2h + u = elements
//                32k + 16h + 4t .. +3 of vector g + 8u, stored [k][lane][4]
//                so that a warp's 16-byte reads are contiguous;
//   [4096, 4608) the 16-element sub-block sums (the Q6_K offset term), split
//                as sum = 64 * hi + lo with lo in 0..63, in the m16n8k16
//                A-fragment order: uint4 of lane 4g + t =
//                {lo(g), lo(g + 8), hi(g), hi(g + 8)}, each word the bytes for
//                sub-blocks 4t .. 4t + 3;
//   [4608, 5120) the 32-element sub-block sums (the Q4_K min term), the same
//                way (sub-blocks 8..15 zero);
//   [5120, 5184) d_x of the 16 vectors.
// Vectors past the batch are zero.  The image depends on the activations
// only, so one image serves every matrix that reads them.
constexpr uint32_t kBatchImageBlockBytes = 4096 + 512 + 512 + kBatchMax * 4;  // 5184
constexpr uint32_t kBatchImageBsum16Offset = 4096;
constexpr uint32_t kBatchImageBsum32Offset = 4608;
constexpr uint32_t kBatchImageDOffset = 5120;

// Shared-memory layout of matvec_batch_kernel: barriers, two items of the
// tree's first level (8 warps x 4 outputs x 32 lanes, each warp's block padded
// by 16 floats so that the tree's reads hit distinct banks), then the stage
// ring.
constexpr uint32_t kBatchBarrierBytes = 256;
constexpr uint32_t kBatchLeafPitch = 4 * 32 + 16;
constexpr uint32_t kBatchScratchBytes = 2 * kBatchConsumerWarps * kBatchLeafPitch * 4;
constexpr uint32_t kBatchStageOffset = align_up(kBatchBarrierBytes + kBatchScratchBytes, 128u);
// A stage row holds a segment of 16 super-blocks plus the 16-byte alignment
// window of a Q6_K row; a stride of 16 mod 128 bytes puts the 8 rows of a
// stage in different shared-memory banks.
__host__ __device__ constexpr uint32_t batch_row_stride(uint32_t type) { return type == 12 ? 2320u : 3472u; }
__host__ __device__ constexpr uint32_t batch_stage_bytes(uint32_t type) {
    return kBatchTileRows * batch_row_stride(type);
}

// One warp per (vector, block): the batch-1 quantizer's arithmetic (GGML's
// quantize_row_q8_K), scattered into the fragment order, plus the split
// sub-block sums of both widths.
// Vector v's Q8_K block i (the lane's quantized values r) into the batch image.
__device__ __forceinline__ void batch_image_store_block(uint8_t* __restrict__ image, uint32_t v, uint32_t i,
                                                        const Q8KLane& r, int lane) {
    uint8_t* blk = image + uint64_t(i) * kBatchImageBlockBytes;
    uint32_t* q = reinterpret_cast<uint32_t*>(blk);
    float* d = reinterpret_cast<float*>(blk + kBatchImageDOffset);
    const uint32_t w[2] = {r.q_lo, r.q_hi};
#pragma unroll
    for (int h2 = 0; h2 < 2; ++h2) {
        const uint32_t e = 8u * lane + 4u * h2;  // first element of the word
        const uint32_t k = e >> 5, h = (e >> 4) & 1u, t = (e >> 2) & 3u;
        const uint32_t dst_lane = 4u * (v & 7u) + t;
        q[(k * 32u + dst_lane) * 4u + 2u * h + (v >> 3)] = w[h2];
    }
    // lane s (< 16) takes the sum of 16-element sub-block s (lanes 2s, 2s + 1);
    // lane j (< 8) the sum of 32-element sub-block j
    const int b16 = __shfl_sync(0xFFFFFFFFu, r.bsum16, (2 * lane) & 31);
    const int pa = __shfl_sync(0xFFFFFFFFu, b16, (2 * lane) & 31);
    const int pb = __shfl_sync(0xFFFFFFFFu, b16, (2 * lane + 1) & 31);
#pragma unroll
    for (int width = 0; width < 2; ++width) {
        const int val = width == 0 ? (lane < 16 ? b16 : 0) : (lane < 8 ? pa + pb : 0);
        const uint32_t lo = static_cast<uint32_t>(val & 63), hi = static_cast<uint32_t>((val >> 6) & 0xFF);
        uint32_t lo_w = 0, hi_w = 0;
#pragma unroll
        for (int qq = 0; qq < 4; ++qq) {
            lo_w |= __shfl_sync(0xFFFFFFFFu, lo, (4 * (lane & 3) + qq) & 31) << (8 * qq);
            hi_w |= __shfl_sync(0xFFFFFFFFu, hi, (4 * (lane & 3) + qq) & 31) << (8 * qq);
        }
        uint32_t* bs = reinterpret_cast<uint32_t*>(blk + (width == 0 ? kBatchImageBsum16Offset
                                                                      : kBatchImageBsum32Offset));
        if (lane < 4) {
            const uint32_t dst_lane = 4u * (v & 7u) + lane;
            bs[dst_lane * 4u + (v >> 3)] = lo_w;
            bs[dst_lane * 4u + 2u + (v >> 3)] = hi_w;
        }
    }
    if (lane == 0) d[v] = r.d;
}

// One warp per (vector, block): x [batch][nb * 256] quantized into the batch image.
__global__ void __launch_bounds__(256) quantize_batch_image_kernel(const float* __restrict__ x, uint32_t batch,
                                                                   uint32_t nb, uint8_t* __restrict__ image) {
    pdl_launch_dependents();
    pdl_wait();
    const uint32_t gw = (blockIdx.x * blockDim.x + threadIdx.x) / 32;
    const int lane = threadIdx.x & 31;
    if (gw >= uint32_t(kBatchMax) * nb) return;
    const uint32_t v = gw % kBatchMax, i = gw / kBatchMax;
    Q8KLane r{0u, 0u, 0, 0.0f};
    if (v < batch) {  // warp-uniform
        const uint64_t at = (uint64_t(v) * nb + i) * 256;
        float vals[8];
        load_lane8(x + at, lane, (reinterpret_cast<uintptr_t>(x + at) & 15u) == 0, vals);
        r = quantize_q8k_lane_values(vals, lane);
    }
    batch_image_store_block(image, v, i, r, lane);
}

// One CTA (kBatchNormThreads threads) per vector: s = a (+ b), written to
// s_out when given (the residual stream), then rms_norm_rows over the row
// with weights w -- the same double sum as rms_norm_rows_kernel (thread t adds
// elements t, t + 256, ... in order, then block_sum_f64), so the same values
// -- quantized into the batch image.  The normalised row is staged in shared
// memory (width <= kBatchNormMaxWidth).  Vectors past the batch are zero.
constexpr uint32_t kBatchNormThreads = 256;
constexpr uint32_t kBatchNormMaxWidth = 8192;
__global__ void __launch_bounds__(kBatchNormThreads) batch_norm_quantize_kernel(
    const float* __restrict__ a, const float* __restrict__ b, float* __restrict__ s_out,
    const float* __restrict__ w, float eps, uint32_t batch, uint32_t width, uint8_t* __restrict__ image) {
    pdl_launch_dependents();
    pdl_wait();
    __shared__ double scratch[32];
    __shared__ __align__(16) float row[kBatchNormMaxWidth];
    const uint32_t v = blockIdx.x, nb = width / 256u;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (v >= batch) {  // CTA-uniform: zero blocks for the vectors past the batch
        for (uint32_t i = warp; i < nb; i += kBatchNormThreads / 32)
            batch_image_store_block(image, v, i, Q8KLane{0u, 0u, 0, 0.0f}, lane);
        return;
    }
    const float* av = a + uint64_t(v) * width;
    const float* bv = b ? b + uint64_t(v) * width : nullptr;
    double sum = 0.0;
    // eight elements' loads in flight per round; the squares are added in
    // element order
    constexpr uint32_t kRound = 8;
    for (uint32_t c0 = threadIdx.x; c0 < width; c0 += kRound * kBatchNormThreads) {
        float x[kRound];
#pragma unroll
        for (uint32_t u = 0; u < kRound; ++u) {
            const uint32_t c = c0 + u * kBatchNormThreads;
            x[u] = c < width ? (bv ? __fadd_rn(__ldg(av + c), __ldg(bv + c)) : __ldg(av + c)) : 0.0f;
        }
#pragma unroll
        for (uint32_t u = 0; u < kRound; ++u) {
            const uint32_t c = c0 + u * kBatchNormThreads;
            if (c < width) {
                row[c] = x[u];
                const double d = static_cast<double>(x[u]);
                sum = __dadd_rn(sum, __dmul_rn(d, d));
            }
        }
    }
    if (s_out)
        for (uint32_t c = threadIdx.x; c < width; c += kBatchNormThreads) s_out[uint64_t(v) * width + c] = row[c];
    const float inv = rms_inverse(block_sum_f64(sum, scratch), width, eps);
    for (uint32_t i = warp; i < nb; i += kBatchNormThreads / 32) {
        float vals[8], wv[8];
        const float4* rp = reinterpret_cast<const float4*>(row + 256u * i) + 2 * lane;
        const float4 lo = rp[0], hi = rp[1];
        vals[0] = lo.x; vals[1] = lo.y; vals[2] = lo.z; vals[3] = lo.w;
        vals[4] = hi.x; vals[5] = hi.y; vals[6] = hi.z; vals[7] = hi.w;
        load_lane8(w + 256ull * i, lane, (reinterpret_cast<uintptr_t>(w + 256ull * i) & 15u) == 0, wv);
#pragma unroll
        for (int j = 0; j < 8; ++j) vals[j] = __fmul_rn(__fmul_rn(vals[j], inv), wv[j]);
        batch_image_store_block(image, v, i, quantize_q8k_lane_values(vals, lane), lane);
    }
}

__device__ __forceinline__ void mma_k32_s8u8(int (&c)[4], const uint4& a, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.u8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
        : "r"(a.x), "r"(a.y), "r"(a.z), "r"(a.w), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void mma_k16_s8u8(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.s32.s8.u8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%0,%1,%2,%3};"
                 : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
                 : "r"(a0), "r"(a1), "r"(b0));
}

__device__ __forceinline__ void mma_k16_s8s8(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%0,%1,%2,%3};"
                 : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
                 : "r"(a0), "r"(a1), "r"(b0));
}

// Byte i of w, zero-extended (u8) or sign-extended (s8): one PRMT each (in
// PTX's prmt a selector nibble with bit 3 set replicates the byte's sign).
__device__ __forceinline__ int byte_u(uint32_t w, int i) { return static_cast<int>(__byte_perm(w, 0u, 0x4440u | i)); }
__device__ __forceinline__ int byte_s(uint32_t w, int i) {
    uint32_t r;
    asm("prmt.b32 %0, %1, 0, %2;" : "=r"(r) : "r"(w), "r"(static_cast<uint32_t>(i) | (0x888u | 0x111u * i) << 4));
    return static_cast<int>(r);
}

// A shared-memory row whose words sit at a fixed 2-byte misalignment: reads
// four bytes at any 4-byte multiple from `base` with two aligned loads.
struct EvenRow {
    const uint32_t* w;  // base rounded down to 4 bytes
    uint32_t shift;     // 0 or 16
    __device__ __forceinline__ explicit EvenRow(const uint8_t* base) {
        const uintptr_t a = reinterpret_cast<uintptr_t>(base);
        w = reinterpret_cast<const uint32_t*>(a & ~uintptr_t(3));
        shift = static_cast<uint32_t>(a & 2u) * 8u;
    }
    __device__ __forceinline__ uint32_t at(uint32_t off) const {  // off: multiple of 4
        return __funnelshift_r(w[off / 4], w[off / 4 + 1], shift);
    }
};

// A warp's activation operands for one super-block, held in registers for
// every tile of the launch: the lane's quant fragments, the split sums the
// weight type needs, and d_x of vectors g and g + 8.
struct BatchA {
    uint4 q[8];
    uint4 bs;
    float dxl, dxh;
};

// From the image in global memory (written by the preceding kernel: L2 reads).
__device__ __forceinline__ void batch_load_a(const uint8_t* blk, int lane, uint32_t bsum_offset, BatchA& A) {
    const uint4* src = reinterpret_cast<const uint4*>(blk) + lane;
#pragma unroll
    for (int k = 0; k < 8; ++k) A.q[k] = __ldcg(src + 32 * k);
    A.bs = __ldcg(reinterpret_cast<const uint4*>(blk + bsum_offset) + lane);
    const float* d = reinterpret_cast<const float*>(blk + kBatchImageDOffset);
    A.dxl = __ldcg(d + (lane >> 2));
    A.dxh = __ldcg(d + (lane >> 2) + 8);
}

// The term p for the thread's four (vector, row) outputs of one Q4_K
// super-block.  rg: the block in row g (the B operand); ra / rb: rows 2t and
// 2t + 1 (the outputs' scales and d); A: the activation operands.
__device__ __forceinline__ void batch_q4k_terms(const uint8_t* rg, const uint8_t* ra, const uint8_t* rb,
                                                const BatchA& A, int lane, float (&p)[4]) {
    const int t = lane & 3;
    const uint4 hg = *reinterpret_cast<const uint4*>(rg);
    const uint4 ha = *reinterpret_cast<const uint4*>(ra);
    const uint4 hb = *reinterpret_cast<const uint4*>(rb);
    // 6-bit scales of rows 2t, 2t + 1 for sub-blocks 0..3 / 4..7
    const uint32_t sa_lo = ha.y & 0x3F3F3F3Fu, sa_hi = (ha.w & 0x0F0F0F0Fu) | ((ha.y >> 2) & 0x30303030u);
    const uint32_t sb_lo = hb.y & 0x3F3F3F3Fu, sb_hi = (hb.w & 0x0F0F0F0Fu) | ((hb.y >> 2) & 0x30303030u);
    // The high-nibble sub-blocks multiply the bytes as stored (16 x nibble,
    // still u8): their scaled sums are exactly 16 x the true ones (|sum| <
    // 2^28) and are divided back once at the end, saving a shift per word.
    int isum[4] = {0, 0, 0, 0}, isum16[4] = {0, 0, 0, 0};
#pragma unroll
    for (int g64 = 0; g64 < 4; ++g64) {
        const uint32_t w0 = *reinterpret_cast<const uint32_t*>(rg + 16 + 32 * g64 + 4 * t);
        const uint32_t w1 = *reinterpret_cast<const uint32_t*>(rg + 16 + 32 * g64 + 16 + 4 * t);
#pragma unroll
        for (int hi = 0; hi < 2; ++hi) {
            const int j = 2 * g64 + hi;
            const uint32_t mask = hi ? 0xF0F0F0F0u : 0x0F0F0F0Fu;
            int c[4] = {0, 0, 0, 0};
            mma_k32_s8u8(c, A.q[j], w0 & mask, w1 & mask);
            const int sca = byte_u(j < 4 ? sa_lo : sa_hi, j & 3);
            const int scb = byte_u(j < 4 ? sb_lo : sb_hi, j & 3);
            int (&acc)[4] = hi ? isum16 : isum;
            acc[0] += sca * c[0];
            acc[1] += scb * c[1];
            acc[2] += sca * c[2];
            acc[3] += scb * c[3];
        }
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) isum[e] += isum16[e] >> 4;
    // min term: the mins of row g for sub-blocks 4t .. 4t + 3 against the split sums
    const uint32_t mn = t == 0 ? (hg.z & 0x3F3F3F3Fu)
                               : t == 1 ? (((hg.w >> 4) & 0x0F0F0F0Fu) | ((hg.z >> 2) & 0x30303030u)) : 0u;
    int mlo[4] = {0, 0, 0, 0}, mhi[4] = {0, 0, 0, 0};
    mma_k16_s8u8(mlo, A.bs.x, A.bs.y, mn);
    mma_k16_s8u8(mhi, A.bs.z, A.bs.w, mn);
    const float dxl = A.dxl, dxh = A.dxh;
    const float dwa = f16_bits_to_f32(static_cast<uint16_t>(ha.x & 0xFFFFu));
    const float dma = f16_bits_to_f32(static_cast<uint16_t>(ha.x >> 16));
    const float dwb = f16_bits_to_f32(static_cast<uint16_t>(hb.x & 0xFFFFu));
    const float dmb = f16_bits_to_f32(static_cast<uint16_t>(hb.x >> 16));
    const float dw[4] = {dwa, dwb, dwa, dwb}, dm[4] = {dma, dmb, dma, dmb}, dx[4] = {dxl, dxl, dxh, dxh};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const int msum = mlo[e] + 64 * mhi[e];
        const float q = __fmul_rn(__fmul_rn(dw[e], dx[e]), __int2float_rn(isum[e]));
        p[e] = __fsub_rn(q, __fmul_rn(__fmul_rn(dm[e], dx[e]), __int2float_rn(msum)));
    }
}

// The same for one Q6_K super-block (blocks at even shared addresses).
__device__ __forceinline__ void batch_q6k_terms(const uint8_t* rg, const uint8_t* ra, const uint8_t* rb,
                                                const BatchA& A, int lane, float (&p)[4]) {
    const int t = lane & 3;
    const EvenRow RG(rg), RA(ra), RB(rb);
    int isum[4] = {0, 0, 0, 0};
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        // row g's quant words of this half: ql[64h + 16q + 4t] (q = 0..3), qh[32h + 16 sub + 4t]
        uint32_t l[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) l[q] = RG.at(64 * h + 16 * q + 4 * t);
        const uint32_t c0 = RG.at(128 + 32 * h + 4 * t);
        const uint32_t c1 = RG.at(128 + 32 * h + 16 + 4 * t);
        // int8 scales of this half for rows 2t and 2t + 1
        const uint32_t sa0 = RA.at(192 + 8 * h), sa1 = RA.at(196 + 8 * h);
        const uint32_t sb0 = RB.at(192 + 8 * h), sb1 = RB.at(196 + 8 * h);
#pragma unroll
        for (int seg = 0; seg < 4; ++seg) {
#pragma unroll
            for (int sub = 0; sub < 2; ++sub) {
                // elements 128h + 32 seg + 16 sub + (0..15): sub-block s
                const uint32_t lo = l[2 * (seg & 1) + sub];
                const uint32_t hb = sub ? c1 : c0;
                const uint32_t nib = (seg & 2) ? ((lo >> 4) & 0x0F0F0F0Fu) : (lo & 0x0F0F0F0Fu);
                const uint32_t top =
                    (seg == 0 ? (hb << 4) : seg == 1 ? (hb << 2) : seg == 2 ? hb : (hb >> 2)) & 0x30303030u;
                const int si = 2 * seg + sub;  // sub-block within the half
                const int s = 8 * h + si;
                const int j = s >> 1, hh = s & 1;
                const uint4 aj = A.q[j];
                int c[4] = {0, 0, 0, 0};
                mma_k16_s8u8(c, hh ? aj.z : aj.x, hh ? aj.w : aj.y, nib | top);
                const int sca = byte_s(si < 4 ? sa0 : sa1, si & 3);
                const int scb = byte_s(si < 4 ? sb0 : sb1, si & 3);
                isum[0] += sca * c[0];
                isum[1] += scb * c[1];
                isum[2] += sca * c[2];
                isum[3] += scb * c[3];
            }
        }
    }
    // offset term: row g's scales for sub-blocks 4t .. 4t + 3 against the split sums
    const uint32_t scg = RG.at(192 + 4 * t);
    int olo[4] = {0, 0, 0, 0}, ohi[4] = {0, 0, 0, 0};
    mma_k16_s8s8(olo, A.bs.x, A.bs.y, scg);
    mma_k16_s8s8(ohi, A.bs.z, A.bs.w, scg);
    const float dxl = A.dxl, dxh = A.dxh;
    const float dwa = f16_bits_to_f32(static_cast<uint16_t>(RA.at(208) & 0xFFFFu));
    const float dwb = f16_bits_to_f32(static_cast<uint16_t>(RB.at(208) & 0xFFFFu));
    const float dw[4] = {dwa, dwb, dwa, dwb}, dx[4] = {dxl, dxl, dxh, dxh};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const int osum = olo[e] + 64 * ohi[e];
        p[e] = __fmul_rn(__fmul_rn(dw[e], dx[e]), __int2float_rn(isum[e] - 32 * osum));
    }
}

struct BatchParams {
    const uint8_t* w;        // 16-byte aligned
    const uint8_t* image;    // nb activation image blocks (16-byte aligned)
    float* out;              // y [batch][rows] (one segment) or partial sums [segments][batch][rows]
    uint64_t rows;
    uint64_t row_bytes;
    uint32_t nb;
    uint32_t batch;
    uint32_t stages;         // ring depth, <= kBatchMaxStages
    DeviceStatus* status;
};

template <uint32_t kType>
__global__ void __launch_bounds__(kBatchThreads, 1) matvec_batch_kernel(const __grid_constant__ BatchParams bp) {
    constexpr int NCW = kBatchConsumerWarps;
    constexpr uint32_t kBB = kType == 12 ? 144u : 210u;
    constexpr uint32_t kStride = batch_row_stride(kType);
    constexpr uint32_t kStage = batch_stage_bytes(kType);
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);
    uint64_t* empty = full + kBatchMaxStages;
    float* scratch = reinterpret_cast<float*>(smem + kBatchBarrierBytes);
    uint8_t* stage0 = smem + kBatchStageOffset;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t nb = bp.nb, S = bp.stages;
    const uint32_t G = (nb + 15u) / 16u;
    const uint32_t T = static_cast<uint32_t>((bp.rows + kBatchTileRows - 1) / kBatchTileRows);
    // this CTA's segment and its share of the segment's tiles
    const uint32_t sg = static_cast<uint32_t>(uint64_t(blockIdx.x) * G / gridDim.x);
    const uint32_t c0 = static_cast<uint32_t>((uint64_t(sg) * gridDim.x + G - 1) / G);  // first CTA of segment sg
    const uint32_t c1 = static_cast<uint32_t>((uint64_t(sg + 1) * gridDim.x + G - 1) / G);
    const uint32_t cn = c1 - c0, ci = blockIdx.x - c0;
    const uint32_t t0 = static_cast<uint32_t>(uint64_t(ci) * T / cn);
    const uint32_t t1 = static_cast<uint32_t>(uint64_t(ci + 1) * T / cn);
    const uint32_t nblk = nb - 16u * sg < 16u ? nb - 16u * sg : 16u;
    const uint64_t seg_off = uint64_t(sg) * 16u * kBB;  // the segment's first byte in a row
    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], NCW);
        }
        fence_mbar_init();
        pdl_launch_dependents();
    }
    __syncthreads();

    if (warp == NCW) {
        // ---------------- producer
        const uint64_t policy = l2_policy_evict_first();
        const uintptr_t wbase = reinterpret_cast<uintptr_t>(bp.w);
        uint32_t q = 0;  // stages issued
        for (uint32_t tile = t0; tile < t1; ++tile, ++q) {
            const uint32_t s = q % S;
            bool w_ok = true;
            if (lane == 0 && q >= S) w_ok = mbar_wait(&empty[s], ((q / S) - 1) & 1u, bp.status, 41);
            if (!__shfl_sync(0xFFFFFFFFu, w_ok ? 1 : 0, 0)) break;
            // row `lane` of the tile: the segment's super-blocks within its 16-byte window
            const uint64_t row0 = uint64_t(tile) * kBatchTileRows;
            const uint32_t n = bp.rows - row0 < kBatchTileRows ? static_cast<uint32_t>(bp.rows - row0) : 8u;
            uint32_t bytes = 0;
            uintptr_t lo = 0;
            if (static_cast<uint32_t>(lane) < n) {
                const uintptr_t o = wbase + (row0 + lane) * bp.row_bytes + seg_off;
                lo = o & ~uintptr_t(15);
                bytes = static_cast<uint32_t>(((o + nblk * kBB + 15u) & ~uintptr_t(15)) - lo);
            }
            uint32_t tx = bytes;
#pragma unroll
            for (int off = 16; off >= 1; off >>= 1) tx += __shfl_xor_sync(0xFFFFFFFFu, tx, off);
            if (lane == 0) mbar_arrive_expect_tx(&full[s], tx);
            __syncwarp();
            if (bytes)
                bulk_copy_g2s(stage0 + size_t(s) * kStage + lane * kStride, reinterpret_cast<const void*>(lo), bytes,
                              &full[s], policy);
        }
        // every copy this CTA issued lands before the CTA exits
        if (lane == 0) {
            for (uint32_t k = q > S ? q - S : 0; k < q; ++k) mbar_wait(&full[k % S], (k / S) & 1u, bp.status, 42);
        }
        return;
    }

    // ---------------- consumers.  A warp whose wait timed out skips the work
    // but takes every barrier and stage arrival, so no other warp waits on it.
    const uintptr_t wbase = reinterpret_cast<uintptr_t>(bp.w);
    pdl_wait();  // the image comes from the preceding kernel; the outputs may still be read by it
    bool failed = false;
    const int g = lane >> 2, t = lane & 3;
    // the tree's reader: output o = 16 warp + lane / 2 (e = o / 32, fragment lane o % 32), half s = lane % 2
    const uint32_t ro = 16u * warp + (lane >> 1), re = ro >> 5, rl = ro & 31u, rs = lane & 1;
    const uint32_t rvec = ((rl >> 2) + 8u * (re >> 1)), rrow = 2u * (rl & 3u) + (re & 1u);
    // this warp's two super-blocks of the segment: their activation operands, once
    const uint32_t sb0 = warp, sb1 = warp + 8;
    const uint32_t bsum = kType == 12 ? kBatchImageBsum32Offset : kBatchImageBsum16Offset;
    BatchA A0{}, A1{};
    if (t0 < t1 && sb0 < nblk) batch_load_a(bp.image + (uint64_t(sg) * 16u + sb0) * kBatchImageBlockBytes, lane, bsum, A0);
    if (t0 < t1 && sb1 < nblk) batch_load_a(bp.image + (uint64_t(sg) * 16u + sb1) * kBatchImageBlockBytes, lane, bsum, A1);
    uint32_t q = 0;
    for (uint32_t tile = t0; tile < t1; ++tile, ++q) {
        const uint32_t s = q % S;
        const uint64_t row0 = uint64_t(tile) * kBatchTileRows;
        if (!failed) {
            const bool ok = mbar_wait(&full[s], (q / S) & 1u, bp.status, 44);
            failed = !__all_sync(0xFFFFFFFFu, ok);
        }
        float p0[4] = {0.0f, 0.0f, 0.0f, 0.0f}, p1[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        if (!failed) {
            // a stage row starts at the segment's first byte rounded down to 16;
            // super-block sb sits at that remainder + sb * kBB.  Both blocks are
            // computed unconditionally (one basic block, so their instructions
            // interleave); a block past the row's end reads stale bytes inside
            // the stage row and its term is replaced by 0 below.
            const uint8_t* st = stage0 + size_t(s) * kStage;
            auto head = [&](uint32_t r) -> uint32_t {
                if (kType == 12) return r * kStride;  // rows are 16-byte multiples
                const uintptr_t o = wbase + (row0 + r) * bp.row_bytes + seg_off;
                return r * kStride + static_cast<uint32_t>(o & 15u);
            };
            const uint32_t hg = head(g), ha = head(2 * t), hb = head(2 * t + 1);
            const uint8_t* s0 = st + sb0 * kBB;
            const uint8_t* s1 = st + sb1 * kBB;
            if (kType == 12) {
                batch_q4k_terms(s0 + hg, s0 + ha, s0 + hb, A0, lane, p0);
                batch_q4k_terms(s1 + hg, s1 + ha, s1 + hb, A1, lane, p1);
            } else {
                batch_q6k_terms(s0 + hg, s0 + ha, s0 + hb, A0, lane, p0);
                batch_q6k_terms(s1 + hg, s1 + ha, s1 + hb, A1, lane, p1);
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
        // the tree's first level in registers: N1(r) = L_r + L_{r+8}, leaves
        // 0 + p (0 past the row's end)
        float* sc = scratch + (q & 1u) * (NCW * kBatchLeafPitch);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float l0 = sb0 < nblk ? __fadd_rn(0.0f, p0[e]) : 0.0f;
            const float l1 = sb1 < nblk ? __fadd_rn(0.0f, p1[e]) : 0.0f;
            sc[warp * kBatchLeafPitch + e * 32 + lane] = __fadd_rn(l0, l1);
        }
        named_barrier_sync(1, NCW * 32);
        // N3(s) = (N1(s) + N1(s+4)) + (N1(s+2) + N1(s+6)); root = N3(0) + N3(1)
        const float* lf = sc + re * 32 + rl;
        const float n3 = __fadd_rn(__fadd_rn(lf[rs * kBatchLeafPitch], lf[(rs + 4) * kBatchLeafPitch]),
                                   __fadd_rn(lf[(rs + 2) * kBatchLeafPitch], lf[(rs + 6) * kBatchLeafPitch]));
        const float root = __fadd_rn(n3, __shfl_xor_sync(0xFFFFFFFFu, n3, 1));
        if (rs == 0 && !failed && rvec < bp.batch && row0 + rrow < bp.rows) {
            const uint64_t yi = uint64_t(rvec) * bp.rows + row0 + rrow;
            if (G == 1)
                bp.out[yi] = __fadd_rn(0.0f, root);
            else
                bp.out[uint64_t(sg) * bp.batch * bp.rows + yi] = root;
        }
    }
}

// Rows of several segments: y = ((0 + P_0) + P_1) + ... in segment order.
__global__ void __launch_bounds__(256) batch_combine_kernel(const float* __restrict__ partial, float* __restrict__ y,
                                                            uint64_t n, uint32_t segments) {
    pdl_launch_dependents();
    pdl_wait();
    for (uint64_t i = blockIdx.x * uint64_t(blockDim.x) + threadIdx.x; i < n; i += uint64_t(gridDim.x) * blockDim.x) {
        float total = 0.0f;
        for (uint32_t k = 0; k < segments; ++k) total = __fadd_rn(total, __ldcg(partial + uint64_t(k) * n + i));
        y[i] = total;
    }
}

}  // namespace oracle_cuda
