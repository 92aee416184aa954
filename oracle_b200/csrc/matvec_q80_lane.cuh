// matvec_q80_lane.cuh -- Oracle's f32 contract for Q8_0 rows, one lane per row.
//
// The same operations in the same order as matvec_seq_kernel<8, 1> (and as
// Oracle's reference_storage_dot, quantized_reference.cpp:24-82): for e = 0 ..
// K-1, w_e = d * q_e (decode4<8>'s exact decode), sum = sum + w_e * x_e, each
// product and addition rounded once.  Only the work split differs: a warp owns
// 32 rows (lane = row) and every lane decodes, multiplies and adds its own row,
// so there is no producer/consumer hand-off; the chain of K dependent adds per
// lane is interleaved with the independent decode and multiply work of the
// same lane.  The rows arrive as 2-D TMA boxes (32 rows x 272 bytes = 8 Q8_0
// blocks, 256 elements), with the matching 1 KB of x by a 1-D bulk copy on the
// same mbarrier, kQ80Stages chunks ahead.  Needs K % 256 == 0 (whole chunks;
// the row stride is then a multiple of 16 bytes) and 16-byte aligned W and x.
#pragma once

#include "decode.cuh"
#include "gemm_q4k.cuh"

namespace oracle_cuda {

constexpr uint32_t kQ80LaneRows = 32;    // rows per CTA: one warp, lane = row
constexpr uint32_t kQ80ChunkBlocks = 8;  // Q8_0 blocks per chunk (256 elements)
constexpr uint32_t kQ80ChunkBytes = kQ80ChunkBlocks * 34u;
constexpr uint32_t kQ80ChunkElems = kQ80ChunkBlocks * 32u;
constexpr uint32_t kQ80Stages = 4;
// a stage: the 32 rows' chunk bytes, then the chunk of x
constexpr uint32_t kQ80StageBytes = kQ80LaneRows * kQ80ChunkBytes + kQ80ChunkElems * 4u;
__host__ __device__ constexpr uint32_t q80_lane_smem_bytes() { return kQ80Stages * kQ80StageBytes + kQ80Stages * 8u; }

__global__ void __launch_bounds__(32) matvec_q80_lane_kernel(const __grid_constant__ CUtensorMap wmap,
                                                             const float* __restrict__ x, float* __restrict__ y,
                                                             uint32_t rows, uint32_t k, DeviceStatus* st) {
    extern __shared__ __align__(128) uint8_t q80_smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(q80_smem + kQ80Stages * kQ80StageBytes);
    const uint32_t lane = threadIdx.x;
    const uint32_t row0 = blockIdx.x * kQ80LaneRows;
    const uint32_t chunks = k / kQ80ChunkElems;
    const uint64_t policy = l2_policy_evict_first();
    if (lane == 0) {
        for (uint32_t s = 0; s < kQ80Stages; ++s) mbar_init(&full[s], 1);
        fence_mbar_init();
    }
    __syncwarp();
    // lane 0: chunk c of the 32 rows (rows past the matrix read as zeros) and of x
    auto issue = [&](uint32_t c) {
        uint8_t* stage = q80_smem + (c % kQ80Stages) * kQ80StageBytes;
        uint64_t* bar = &full[c % kQ80Stages];
        mbar_arrive_expect_tx(bar, kQ80StageBytes);
        tma_load_2d(smem_addr(stage), &wmap, bar, static_cast<int>(c * (kQ80ChunkBytes / 2)), static_cast<int>(row0));
        bulk_copy_g2s(stage + kQ80LaneRows * kQ80ChunkBytes, x + static_cast<uint64_t>(c) * kQ80ChunkElems,
                      kQ80ChunkElems * 4u, bar, policy);
    };
    uint32_t issued = 0;
    if (lane == 0)
        for (; issued < kQ80Stages && issued < chunks; ++issued) issue(issued);
    float sum = 0.0f;
    bool ok = true;
    uint32_t c = 0;
    for (; c < chunks; ++c) {
        const uint32_t s = c % kQ80Stages;
        ok = __all_sync(0xFFFFFFFFu, mbar_wait(&full[s], (c / kQ80Stages) & 1u, st, 30));
        if (!ok) break;
        const uint32_t* rw = reinterpret_cast<const uint32_t*>(q80_smem + s * kQ80StageBytes + lane * kQ80ChunkBytes);
        const float4* x4 = reinterpret_cast<const float4*>(q80_smem + s * kQ80StageBytes + kQ80LaneRows * kQ80ChunkBytes);
        // Block b's 34 bytes are the 9 aligned words from (34 b) / 4: d in the
        // low (b even) or high (b odd) half of the first, quant word t the
        // funnel of words t, t + 1 (b even) or word t + 1 (b odd) -- the words
        // ld_u32_even<true> reads.  The next block's words and x are loaded
        // while this block is added (software pipeline across the unrolled blocks).
        uint32_t wa[9];
        float4 xa[8];
#pragma unroll
        for (int i = 0; i < 9; ++i) wa[i] = rw[i];
#pragma unroll
        for (int i = 0; i < 8; ++i) xa[i] = x4[i];
#pragma unroll
        for (uint32_t b = 0; b < kQ80ChunkBlocks; ++b) {
            uint32_t wn[9];
            float4 xn[8];
            if (b + 1 < kQ80ChunkBlocks) {
                const uint32_t w1 = (34u * (b + 1)) / 4u;
#pragma unroll
                for (int i = 0; i < 9; ++i) wn[i] = rw[w1 + i];
#pragma unroll
                for (int i = 0; i < 8; ++i) xn[i] = x4[8 * (b + 1) + i];
            }
            const bool odd = (b & 1u) != 0;
            const float d = f16_bits_to_f32(static_cast<uint16_t>(odd ? (wa[0] >> 16) : (wa[0] & 0xFFFFu)));
            // the block's 32 products first (independent), then the 32 adds of
            // the chain back to back
            float prod[32];
#pragma unroll
            for (int t = 0; t < 8; ++t) {
                const uint32_t qw = (odd ? wa[t + 1] : __funnelshift_r(wa[t], wa[t + 1], 16)) ^ 0x80808080u;
                const float xv[4] = {xa[t].x, xa[t].y, xa[t].z, xa[t].w};
#pragma unroll
                for (int u = 0; u < 4; ++u)
                    prod[4 * t + u] = __fmul_rn(__fmul_rn(d, __fsub_rn(small_uint_to_f32(qw, u), 8388736.0f)), xv[u]);
            }
#pragma unroll
            for (int e = 0; e < 32; ++e) sum = __fadd_rn(sum, prod[e]);
            if (b + 1 < kQ80ChunkBlocks) {
#pragma unroll
                for (int i = 0; i < 9; ++i) wa[i] = wn[i];
#pragma unroll
                for (int i = 0; i < 8; ++i) xa[i] = xn[i];
            }
        }
        __syncwarp();  // every lane has left stage s
        if (lane == 0 && issued < chunks) {
            // the generic-proxy reads of stage s before the copy engine refills it
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            issue(issued++);
        }
    }
    if (!ok) {
        // a wait gave up (recorded in the status word): let the copies already
        // issued land, each wait bounded, before the CTA's shared memory goes away
        if (lane == 0)
            for (uint32_t i = c; i < issued; ++i) mbar_wait(&full[i % kQ80Stages], (i / kQ80Stages) & 1u, st, 31);
        return;
    }
    if (row0 + lane < rows) y[row0 + lane] = sum;
}

}  // namespace oracle_cuda
