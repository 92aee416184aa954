// matvec_q80_lane.cuh -- Oracle's f32 contract for Q8_0 rows, one lane per row.
//
// The same operations in the same order as matvec_seq_kernel<8, 1> (and as
// Oracle's reference_storage_dot, quantized_reference.cpp:24-82): for e = 0 ..
// K-1, w_e = d * q_e (decode4<8>'s exact decode), sum = sum + w_e * x_e, each
// product and addition rounded once.  Only the work split differs: 32 rows per
// CTA with lane = row in every warp, two product warps computing the products
// of alternate blocks and one chain warp adding them (below).  The rows arrive
// as 2-D TMA boxes (32 rows x 272 bytes = 8 Q8_0 blocks, 256 elements), with
// the matching 1 KB of x by a 1-D bulk copy on the same mbarrier, kQ80Stages
// chunks ahead.  Needs K % 256 == 0 (whole chunks; the row stride is then a
// multiple of 16 bytes) and 16-byte aligned W and x.
#pragma once

#include "decode.cuh"
#include "gemm_q4k.cuh"

namespace oracle_cuda {

constexpr uint32_t kQ80LaneRows = 32;    // rows per CTA: lane = row in every warp
constexpr uint32_t kQ80ChunkBlocks = 8;  // Q8_0 blocks per chunk (256 elements)
constexpr uint32_t kQ80ChunkBytes = kQ80ChunkBlocks * 34u;
constexpr uint32_t kQ80ChunkElems = kQ80ChunkBlocks * 32u;
constexpr uint32_t kQ80Stages = 4;
// a stage: the 32 rows' chunk bytes, then the chunk of x
constexpr uint32_t kQ80StageBytes = kQ80LaneRows * kQ80ChunkBytes + kQ80ChunkElems * 4u;

// Per 32 rows, two product warps (lane = row; warp p decodes and multiplies blocks
// p, p + 2, ... of every chunk, the block's words and x loaded one block ahead)
// write each chunk's 256 products per row into one of two product stages, and
// one chain warp (lane = row) adds them in element order, four per 128-bit
// load, so its lane issues little more than the chain of adds itself.
// Barriers (all waits bounded): raw_full / raw_empty per weight stage (every
// lane of the product warps releases it), prod_full (every product lane) /
// prod_empty (every chain lane) per product stage.
constexpr uint32_t kQ80ProdStages = 2;
constexpr uint32_t kQ80ProdWarps = 2;  // product warps per 32 rows: warp p takes blocks p, p + 2, ...
static_assert(kQ80ChunkBlocks % kQ80ProdWarps == 0 && kQ80ProdWarps % 2 == 0, "blocks per product warp");
constexpr uint32_t kQ80ProdStride = kQ80ChunkElems + 4;  // floats per row in a product stage
constexpr uint32_t kQ80ProdBytes = kQ80LaneRows * kQ80ProdStride * 4u;
__host__ __device__ constexpr uint32_t q80_split_smem_bytes() {
    return kQ80Stages * kQ80StageBytes + kQ80ProdStages * kQ80ProdBytes + (2 * kQ80Stages + 2 * kQ80ProdStages) * 8u;
}

// The 9 words of block b of a lane's 272-byte chunk row, (34 b) / 4 .. + 8, from
// three aligned 16-byte loads (rows 272 bytes apart put 4-byte loads of lanes
// l, l + 8, l + 16, l + 24 on one bank; 16-byte loads take the minimum 4
// wavefronts anyway).
template <uint32_t kB>
__device__ __forceinline__ void q80_block_words(const uint4* row4, uint32_t (&w)[9]) {
    constexpr uint32_t w0 = (34u * kB) / 4u, q0 = w0 / 4u, o = w0 % 4u;
    uint32_t u[12];
#pragma unroll
    for (uint32_t v = 0; v < 3; ++v) {
        const uint4 t = row4[q0 + v];
        u[4 * v + 0] = t.x;
        u[4 * v + 1] = t.y;
        u[4 * v + 2] = t.z;
        u[4 * v + 3] = t.w;
    }
#pragma unroll
    for (uint32_t i = 0; i < 9; ++i) w[i] = u[o + i];
}

// Product warp kP's blocks b = kP, kP + 2, ... of one chunk: d in the low (b
// even) or high (b odd) half of word 0, quant word t the funnel of words t,
// t + 1 (b even) or word t + 1 (b odd) -- the words ld_u32_even<true> reads;
// each product d * q * x rounded as decode4<8> and matvec_seq do; the next
// block's words and x loaded while this one computes.
template <uint32_t kP, uint32_t kJ = 0>
__device__ __forceinline__ void q80_products_from(const uint4* row4, const float4* x4, float4* po,
                                                  const uint32_t (&wa)[9], const float4 (&xa)[8]) {
    constexpr uint32_t b = kP + kQ80ProdWarps * kJ;
    constexpr bool kLast = kJ + 1 == kQ80ChunkBlocks / kQ80ProdWarps;
    uint32_t wn[9];
    float4 xn[8];
    if constexpr (!kLast) {
        q80_block_words<b + kQ80ProdWarps>(row4, wn);
#pragma unroll
        for (int i = 0; i < 8; ++i) xn[i] = x4[8 * (b + kQ80ProdWarps) + i];
    }
    constexpr bool odd = (b & 1u) != 0;
    const float d = f16_bits_to_f32(static_cast<uint16_t>(odd ? (wa[0] >> 16) : (wa[0] & 0xFFFFu)));
#pragma unroll
    for (int t = 0; t < 8; ++t) {
        const uint32_t qw = (odd ? wa[t + 1] : __funnelshift_r(wa[t], wa[t + 1], 16)) ^ 0x80808080u;
        float4 o;
        o.x = __fmul_rn(__fmul_rn(d, __fsub_rn(small_uint_to_f32(qw, 0), 8388736.0f)), xa[t].x);
        o.y = __fmul_rn(__fmul_rn(d, __fsub_rn(small_uint_to_f32(qw, 1), 8388736.0f)), xa[t].y);
        o.z = __fmul_rn(__fmul_rn(d, __fsub_rn(small_uint_to_f32(qw, 2), 8388736.0f)), xa[t].z);
        o.w = __fmul_rn(__fmul_rn(d, __fsub_rn(small_uint_to_f32(qw, 3), 8388736.0f)), xa[t].w);
        po[8 * b + t] = o;
    }
    if constexpr (!kLast) q80_products_from<kP, kJ + 1>(row4, x4, po, wn, xn);
}

template <uint32_t kP>
__device__ __forceinline__ void q80_products(const uint4* row4, const float4* x4, float4* po) {
    uint32_t wa[9];
    float4 xa[8];
    q80_block_words<kP>(row4, wa);
#pragma unroll
    for (int i = 0; i < 8; ++i) xa[i] = x4[8 * kP + i];
    q80_products_from<kP>(row4, x4, po, wa, xa);
}

__global__ void __launch_bounds__(32 * (1 + kQ80ProdWarps)) matvec_q80_split_kernel(const __grid_constant__ CUtensorMap wmap,
                                                              const float* __restrict__ x, float* __restrict__ y,
                                                              uint32_t rows, uint32_t k, DeviceStatus* st) {
    extern __shared__ __align__(128) uint8_t q80_smem[];
    float* prod = reinterpret_cast<float*>(q80_smem + kQ80Stages * kQ80StageBytes);
    uint64_t* raw_full = reinterpret_cast<uint64_t*>(q80_smem + kQ80Stages * kQ80StageBytes +
                                                     kQ80ProdStages * kQ80ProdBytes);
    uint64_t* raw_empty = raw_full + kQ80Stages;
    uint64_t* prod_full = raw_empty + kQ80Stages;
    uint64_t* prod_empty = prod_full + kQ80ProdStages;
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t row0 = blockIdx.x * kQ80LaneRows;
    const uint32_t chunks = k / kQ80ChunkElems;
    if (threadIdx.x == 0) {
        // every lane of the releasing warps arrives (its own reads / writes
        // ordered before its arrival)
        for (uint32_t s = 0; s < kQ80Stages; ++s) {
            mbar_init(&raw_full[s], 1);
            mbar_init(&raw_empty[s], 32 * kQ80ProdWarps);
        }
        for (uint32_t s = 0; s < kQ80ProdStages; ++s) {
            mbar_init(&prod_full[s], 32 * kQ80ProdWarps);
            mbar_init(&prod_empty[s], 32);
        }
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == 0) {
        // ------------------------------------------------ chain warp
        float sum = 0.0f;
        bool ok = true;
        for (uint32_t c = 0; c < chunks; ++c) {
            const uint32_t ps = c % kQ80ProdStages;
            ok = __all_sync(0xFFFFFFFFu, mbar_wait(&prod_full[ps], (c / kQ80ProdStages) & 1u, st, 32));
            if (!ok) break;
            const float4* pr = reinterpret_cast<const float4*>(prod + ps * (kQ80LaneRows * kQ80ProdStride) +
                                                               lane * kQ80ProdStride);
#pragma unroll 16
            for (uint32_t e = 0; e < kQ80ChunkElems / 4; ++e) {
                const float4 v = pr[e];
                sum = __fadd_rn(sum, v.x);
                sum = __fadd_rn(sum, v.y);
                sum = __fadd_rn(sum, v.z);
                sum = __fadd_rn(sum, v.w);
            }
            mbar_arrive(&prod_empty[ps]);
        }
        if (ok && row0 + lane < rows) y[row0 + lane] = sum;
        return;
    }

    // ---------------------------------------------------- product warps
    const uint32_t p = warp - 1;  // blocks p, p + kQ80ProdWarps, ... of every chunk
    const uint64_t policy = l2_policy_evict_first();
    const bool issuer = p == 0 && lane == 0;
    auto issue = [&](uint32_t c) {
        uint8_t* stage = q80_smem + (c % kQ80Stages) * kQ80StageBytes;
        uint64_t* bar = &raw_full[c % kQ80Stages];
        mbar_arrive_expect_tx(bar, kQ80StageBytes);
        tma_load_2d(smem_addr(stage), &wmap, bar, static_cast<int>(c * (kQ80ChunkBytes / 2)), static_cast<int>(row0));
        bulk_copy_g2s(stage + kQ80LaneRows * kQ80ChunkBytes, x + static_cast<uint64_t>(c) * kQ80ChunkElems,
                      kQ80ChunkElems * 4u, bar, policy);
    };
    uint32_t issued = 0;
    if (issuer)
        for (; issued < kQ80Stages && issued < chunks; ++issued) issue(issued);
    bool ok = true;
    uint32_t c = 0;
    for (; c < chunks; ++c) {
        const uint32_t s = c % kQ80Stages, ps = c % kQ80ProdStages;
        bool w_ok = mbar_wait(&raw_full[s], (c / kQ80Stages) & 1u, st, 33);
        if (w_ok && c >= kQ80ProdStages)
            w_ok = mbar_wait(&prod_empty[ps], ((c / kQ80ProdStages) - 1) & 1u, st, 34);
        ok = __all_sync(0xFFFFFFFFu, w_ok);
        if (!ok) break;
        const uint32_t* rw = reinterpret_cast<const uint32_t*>(q80_smem + s * kQ80StageBytes + lane * kQ80ChunkBytes);
        const float4* x4 = reinterpret_cast<const float4*>(q80_smem + s * kQ80StageBytes + kQ80LaneRows * kQ80ChunkBytes);
        float4* po = reinterpret_cast<float4*>(prod + ps * (kQ80LaneRows * kQ80ProdStride) + lane * kQ80ProdStride);
        if (p == 0)
            q80_products<0>(reinterpret_cast<const uint4*>(rw), x4, po);
        else
            q80_products<1>(reinterpret_cast<const uint4*>(rw), x4, po);
        mbar_arrive(&prod_full[ps]);  // this lane's products of chunk c are written
        mbar_arrive(&raw_empty[s]);   // ... and it has left weight stage s
        if (issuer && issued < chunks) {
            // both product warps have left the stage the next chunk refills
            const uint32_t n = issued;
            if (!mbar_wait(&raw_empty[n % kQ80Stages], ((n / kQ80Stages) - 1) & 1u, st, 35)) {
                ok = false;
            } else {
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                issue(issued++);
            }
        }
        if (!__shfl_sync(0xFFFFFFFFu, ok ? 1 : 0, 0)) {
            ok = false;
            break;
        }
    }
    if (!ok && issuer) {
        // let the copies already issued land (bounded) before shared memory goes away
        for (uint32_t i = c; i < issued; ++i) mbar_wait(&raw_full[i % kQ80Stages], (i / kQ80Stages) & 1u, st, 36);
    }
}

}  // namespace oracle_cuda
