// gemm_q4k.cuh -- prefill dequant-GEMM on the 5th-generation tensor cores.
//
//   Y[m][n] = sum_k X[m][k] * W[n][k]      X: M x K activations, W: N x K Q4_K rows
//
// There is no reference counterpart: Oracle ingests prompts one matvec at a
// time (qwen35_generation.cpp:737-747).  Operands are bf16, accumulation f32:
//   * W tiles are dequantized in shared memory: each element is Oracle's f32
//     decode (d*sc)*q - dmin*m (storage_decode.cpp:44-94, Q5_K without the
//     high-bit plane), rounded once to bf16 (round to nearest even);
//   * X is converted to bf16 (round to nearest even) by a separate kernel and
//     read with tensor-memory-accelerator (TMA) tile loads.
//
// CTA tile: 128 weight rows (the MMA's M, TMEM lanes) x 256 tokens (the MMA's
// N, TMEM columns), K in stages of 64 (one 128-byte swizzle row of bf16).
// Warp roles (12 warps):
//   warp 0  lane 0: X tile loads (2-D TMA, 128-byte swizzle) into the B ring;
//                   the warp also owns the TMEM allocation (256 columns)
//   warp 1  lane 0: issues tcgen05.mma (kind::f16, bf16 x bf16 -> f32), 4 per
//                   stage, and tcgen05.commit to free stages / signal the end
//   warp 2  lane 0: raw Q4_K loads: 2-D TMA boxes of 128 rows x 144 bytes (one
//                   super-block column) into a ring of raw stages
//   warps 4-11:     dequantize raw super-blocks into the A ring (K-major,
//                   128-byte swizzle: 16-byte chunk c of row r at c ^ (r & 7));
//                   two groups of 4 warps take alternate stages, a thread
//                   per weight row,
//                   then, after the last MMA, read the accumulator out of TMEM
//                   (tcgen05.ld 32x32b) and store Y (coalesced along n)
// Every mbarrier wait is bounded (common.cuh); a timeout sets a CTA abort flag,
// the roles leave their loops, outstanding TMA loads and MMAs are waited for
// (bounded), TMEM is freed and the kernel returns with the status recorded.
#pragma once

#include <cuda.h>

#include "common.cuh"

namespace oracle_cuda {

constexpr uint32_t kGemmTileN = 128;  // weight rows per CTA (TMEM lanes)
constexpr uint32_t kGemmTileM = 256;  // tokens per CTA or CTA pair (UMMA N, TMEM columns)
constexpr uint32_t kGemmTileK = 64;   // K per stage
constexpr uint32_t kGemmRawStages = 3;
constexpr uint32_t kGemmSbBytes = 144;  // Q4_K super-block
constexpr uint32_t kGemmABytes = kGemmTileN * kGemmTileK * 2;
constexpr uint32_t kGemmRawBytes = kGemmTileN * kGemmSbBytes;
constexpr uint32_t kGemmDequantWarps = 8;
constexpr uint32_t kGemmThreads = (4 + kGemmDequantWarps) * 32;

// Shared-memory plan of one CTA.  kPair: a CTA pair (cluster of 2) shares
// each MMA: M = 256 weight rows (128 per CTA), and each CTA loads half of the
// 256 tokens, so a stage's B tile is 128 rows.
//
// kPair = false keeps the dequantized A tiles in TMEM (tcgen05.st from the
// dequant warps, tcgen05.mma reading A from tensor memory): shared memory then
// carries only B and the raw weights, which leaves its bandwidth to the MMA's
// B reads.  TMEM: columns [0, 256) accumulator, then 32 columns per stage of A
// (64 bf16 of K per row, two per column).
template <bool kPair>
struct GemmPlan {
    static constexpr bool kATmem = !kPair;
    static constexpr uint32_t kStages = 4;
    static constexpr uint32_t kTmemCols = kATmem ? 512 : 256;
    static constexpr uint32_t kATmemCol = kGemmTileM;  // first A column
    static constexpr uint32_t kBRows = kPair ? kGemmTileM / 2 : kGemmTileM;
    static constexpr uint32_t kBBytes = kBRows * kGemmTileK * 2;
    static constexpr uint32_t kOffB = kATmem ? 0 : kStages * kGemmABytes;
    static constexpr uint32_t kOffRaw = kOffB + kStages * kBBytes;
    static constexpr uint32_t kOffBars = kOffRaw + kGemmRawStages * kGemmRawBytes;
    // full_a, full_b, empty, peer_full per stage; raw_full, raw_empty per raw stage; acc_full
    static constexpr uint32_t kBars = 4 * kStages + 2 * kGemmRawStages + 1;
    static constexpr uint32_t kSmemBytes = 1024 + kOffBars + kBars * 8 + 16;
    // Instruction descriptor: D f32, A and B bf16, both K-major, M = 128 or 256 (pair), N = 256.
    static constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((kGemmTileM >> 3) << 17) |
                                       (((kPair ? 2 * kGemmTileN : kGemmTileN) >> 4) << 24);
};

struct GemmParams {
    float* y;                // m x n row-major
    uint32_t n, m, k;        // weight rows, tokens, columns
    uint32_t k_per_split;    // columns per blockIdx.z (multiple of 256)
    uint32_t accumulate;     // 1: add into y (split K), 0: store
    DeviceStatus* status;
    // tiles_m > 0: blockIdx.x numbers tiles from tile_base in m-fastest order
    // (tile t = n_tile * tiles_m + m_tile), so a launch may cover any run of
    // tiles; 0: blockIdx.x / blockIdx.y are the n / m tile
    uint32_t tile_base, tiles_m;
};

// UMMA shared-memory descriptor: K-major, 128-byte swizzle, 8-row atoms of
// 1024 bytes stacked densely (stride byte offset 1024), descriptor version 1.
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t smem) {
    return static_cast<uint64_t>((smem >> 4) & 0x3FFFu) | (1ull << 16) | (64ull << 32) | (1ull << 46) |
           (2ull << 61);
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::
            "r"(dst),
        "l"(map), "r"(smem_addr(bar)), "r"(x), "r"(y)
        : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
                 : "memory");
}

__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
          "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),
          "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]),
        "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]), "r"(v[17]),
        "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]),
        "r"(v[26]), "r"(v[27]), "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
        : "memory");
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}

// 6-bit scale and min of sub-block j from the three little-endian words
// holding the 12 packed bytes (storage_decode.cpp:44-61).
__device__ __forceinline__ void q4k_scale_min(uint32_t s0, uint32_t s1, uint32_t s2, uint32_t j, uint32_t& sc,
                                              uint32_t& mn) {
    if (j < 4) {
        sc = (s0 >> (8 * j)) & 63u;
        mn = (s1 >> (8 * j)) & 63u;
    } else {
        const uint32_t t = 8 * (j - 4);
        sc = ((s2 >> t) & 0x0Fu) | (((s0 >> t) & 0xC0u) >> 2);
        mn = ((s2 >> t) >> 4 & 0x0Fu) | (((s1 >> t) & 0xC0u) >> 2);
    }
}

__device__ __forceinline__ uint64_t f32x2(float lo, float hi) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}

// Four nibbles (one per byte of `nib4`, values 0..15) to bf16 pairs of the
// exact f32 decode (dsc * q) - dm, each operation rounded to nearest (packed
// f32x2 arithmetic: two IEEE operations per instruction), then rounded once to
// bf16.  q becomes a float exactly: the byte placed under the exponent of 2^23
// and 2^23 subtracted.
__device__ __forceinline__ uint2 dequant4(uint32_t nib4, uint64_t dsc2, uint64_t dm2) {
    const uint64_t two23 = 0x4B0000004B000000ull;
    const uint64_t m01 = f32x2(__uint_as_float(__byte_perm(nib4, 0x4B000000u, 0x7440u)),
                               __uint_as_float(__byte_perm(nib4, 0x4B000000u, 0x7441u)));
    const uint64_t m23 = f32x2(__uint_as_float(__byte_perm(nib4, 0x4B000000u, 0x7442u)),
                               __uint_as_float(__byte_perm(nib4, 0x4B000000u, 0x7443u)));
    uint64_t a, b;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(a) : "l"(m01), "l"(two23));
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(b) : "l"(m23), "l"(two23));
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(a) : "l"(a), "l"(dsc2));
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(b) : "l"(b), "l"(dsc2));
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(a) : "l"(a), "l"(dm2));
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(b) : "l"(b), "l"(dm2));
    uint2 r;
    asm("{\n\t.reg .f32 lo, hi;\n\tmov.b64 {lo, hi}, %1;\n\tcvt.rn.bf16x2.f32 %0, hi, lo;\n\t}" : "=r"(r.x) : "l"(a));
    asm("{\n\t.reg .f32 lo, hi;\n\tmov.b64 {lo, hi}, %1;\n\tcvt.rn.bf16x2.f32 %0, hi, lo;\n\t}" : "=r"(r.y) : "l"(b));
    return r;
}

__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// Address of the same shared variable in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
    return r;
}

__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// A from tensor memory (cta_group::1).
__device__ __forceinline__ void umma_bf16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                             uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
        "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

template <bool kPair>
__device__ __forceinline__ void umma_bf16_issue(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
    constexpr uint32_t idesc = GemmPlan<kPair>::kIdesc;
    if constexpr (kPair)
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "setp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
            "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
            : "memory");
    else
        umma_bf16(tmem_d, adesc, bdesc, idesc, accumulate);
}

// tcgen05.commit to a barrier given by its cluster address (own or the peer's).
template <bool kPair>
__device__ __forceinline__ void umma_commit_to(uint32_t cluster_addr) {
    if constexpr (kPair)
        asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(cluster_addr)
                     : "memory");
    else
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(cluster_addr)
                     : "memory");
}

// kPair = false: one CTA per (128 weight rows x 256 tokens) tile, tcgen05.mma
// with cta_group::1 (M = 128).  kPair = true: clusters of 2 CTAs along x, each
// CTA owning 128 weight rows and loading half of the pair's 256 tokens; the
// leader (rank 0) issues tcgen05.mma with cta_group::2 (M = 256), which reads
// A and B from both CTAs' shared memory at the same offsets and leaves each
// CTA's 128 x 256 accumulator in its own TMEM.  The peer's warp 1 relays "my
// stage is full" to the leader with a remote mbarrier arrive; the leader's
// commits arrive on both CTAs' `empty` and `acc_full` barriers.
template <bool kPair>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_q4k_bf16_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_w,
                         const GemmParams p) {
    using Plan = GemmPlan<kPair>;
    constexpr uint32_t S = Plan::kStages;
    extern __shared__ uint8_t gemm_smem[];
    const uint32_t raw_base = smem_addr(gemm_smem);
    const uint32_t base = (raw_base + 1023u) & ~1023u;
    uint8_t* smem = gemm_smem + (base - raw_base);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Plan::kOffBars);
    uint64_t* full_a = bars;                          // dequant warps -> MMA
    uint64_t* full_b = bars + S;                      // X TMA -> MMA
    uint64_t* empty = bars + 2 * S;                   // MMA commit -> producers
    uint64_t* peer_full = bars + 3 * S;               // (pair, leader) peer relay -> MMA
    uint64_t* raw_full = bars + 4 * S;                // raw TMA -> dequant
    uint64_t* raw_empty = raw_full + kGemmRawStages;  // dequant -> raw TMA
    uint64_t* acc_full = raw_empty + kGemmRawStages;  // last MMA -> epilogue
    volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(bars + Plan::kBars);
    volatile uint32_t* abort_flag = tmem_slot + 1;

    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = kPair ? cluster_rank() : 0u;
    const uint32_t tile = p.tile_base + blockIdx.x;
    const uint32_t n0 = (p.tiles_m ? tile / p.tiles_m : blockIdx.x) * kGemmTileN;
    const uint32_t m0 = (p.tiles_m ? tile % p.tiles_m : blockIdx.y) * kGemmTileM;
    const uint32_t b_row0 = m0 + rank * Plan::kBRows;  // this CTA's B rows (tokens)
    const uint32_t k_begin = blockIdx.z * p.k_per_split;
    const uint32_t k_end = p.k - k_begin < p.k_per_split ? p.k : k_begin + p.k_per_split;
    const uint32_t nk = (k_end - k_begin) / kGemmTileK;
    const uint32_t nsb = nk / 4;

    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < S; ++s) {
            mbar_init(&full_a[s], kGemmDequantWarps / 2);  // one group of 4 warps per stage
            mbar_init(&full_b[s], 1);
            mbar_init(&empty[s], 1);
            mbar_init(&peer_full[s], 1);
        }
        for (uint32_t r = 0; r < kGemmRawStages; ++r) {
            mbar_init(&raw_full[r], 1);
            mbar_init(&raw_empty[r], kGemmDequantWarps);
        }
        mbar_init(acc_full, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 0) {
        const uint32_t slot = smem_addr(const_cast<uint32_t*>(tmem_slot));
        if constexpr (kPair) {
            asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(slot),
                         "r"(Plan::kTmemCols)
                         : "memory");
            asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
        } else {
            asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(slot),
                         "r"(Plan::kTmemCols)
                         : "memory");
            asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
        }
    }
    tc_fence_before();
    __syncthreads();
    if constexpr (kPair) cluster_sync_all();  // both CTAs' barriers exist before any remote arrive
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            // ---------------------------------------------------------- X tiles
            uint32_t issued = 0;
            for (uint32_t kc = 0; kc < nk && !*abort_flag; ++kc) {
                const uint32_t s = kc % S;
                if (kc >= S && !mbar_wait(&empty[s], ((kc / S) - 1) & 1, p.status, 41)) {
                    *abort_flag = 1;
                    break;
                }
                mbar_arrive_expect_tx(&full_b[s], Plan::kBBytes);
                tma_load_2d(base + Plan::kOffB + s * Plan::kBBytes, &tmap_x, &full_b[s],
                            static_cast<int>(k_begin + kc * kGemmTileK), static_cast<int>(b_row0));
                issued = kc + 1;
            }
            // no load may still be in flight when the CTA exits
            for (uint32_t kc = issued > S ? issued - S : 0; kc < issued; ++kc)
                mbar_wait(&full_b[kc % S], (kc / S) & 1, p.status, 42);
        }
    } else if (warp == 1) {
        if (lane == 0 && rank == 0) {
            // ---------------------------------------------------------- MMA issue
            const uint32_t peer = kPair ? 1u : 0u;
            for (uint32_t kc = 0; kc < nk && !*abort_flag; ++kc) {
                const uint32_t s = kc % S, par = (kc / S) & 1;
                if (!mbar_wait(&full_b[s], par, p.status, 43) || !mbar_wait(&full_a[s], par, p.status, 44) ||
                    (kPair && !mbar_wait(&peer_full[s], par, p.status, 50))) {
                    *abort_flag = 1;
                    break;
                }
                tc_fence_after();
                const uint64_t bd = umma_desc_sw128(base + Plan::kOffB + s * Plan::kBBytes);
                if constexpr (Plan::kATmem) {
#pragma unroll
                    for (uint32_t kk = 0; kk < kGemmTileK / 16; ++kk)
                        umma_bf16_ts(tmem, tmem + Plan::kATmemCol + 32 * s + 8 * kk, bd + 2 * kk, Plan::kIdesc,
                                     (kc | kk) != 0);
                } else {
                    const uint64_t ad = umma_desc_sw128(base + s * kGemmABytes);
#pragma unroll
                    for (uint32_t kk = 0; kk < kGemmTileK / 16; ++kk)
                        umma_bf16_issue<kPair>(tmem, ad + 2 * kk, bd + 2 * kk, (kc | kk) != 0);
                }
                umma_commit_to<kPair>(smem_addr(&empty[s]));
                if (kPair) umma_commit_to<kPair>(mapa_shared(smem_addr(&empty[s]), peer));
            }
            // also after an abort: completes once the issued MMAs finish
            umma_commit_to<kPair>(smem_addr(acc_full));
            if (kPair) umma_commit_to<kPair>(mapa_shared(smem_addr(acc_full), peer));
        } else if (kPair && lane == 0) {
            // ---------------------------------------------------------- peer: relay full stages
            for (uint32_t kc = 0; kc < nk && !*abort_flag; ++kc) {
                const uint32_t s = kc % S, par = (kc / S) & 1;
                if (!mbar_wait(&full_b[s], par, p.status, 51) || !mbar_wait(&full_a[s], par, p.status, 52)) {
                    *abort_flag = 1;
                    break;
                }
                mbar_arrive_remote(mapa_shared(smem_addr(&peer_full[s]), 0));
            }
        }
    } else if (warp == 2) {
        if (lane == 0) {
            // ---------------------------------------------------------- raw Q4_K tiles
            uint32_t issued = 0;
            for (uint32_t j = 0; j < nsb && !*abort_flag; ++j) {
                const uint32_t r = j % kGemmRawStages;
                if (j >= kGemmRawStages &&
                    !mbar_wait(&raw_empty[r], ((j / kGemmRawStages) - 1) & 1, p.status, 45)) {
                    *abort_flag = 1;
                    break;
                }
                mbar_arrive_expect_tx(&raw_full[r], kGemmRawBytes);
                tma_load_2d(base + Plan::kOffRaw + r * kGemmRawBytes, &tmap_w, &raw_full[r],
                            static_cast<int>((k_begin / 256 + j) * kGemmSbBytes), static_cast<int>(n0));
                issued = j + 1;
            }
            for (uint32_t j = issued > kGemmRawStages ? issued - kGemmRawStages : 0; j < issued; ++j)
                mbar_wait(&raw_full[j % kGemmRawStages], (j / kGemmRawStages) & 1, p.status, 46);
        }
    } else if (warp >= 4) {
        // -------------------------------------------------------------- dequantize
        // Two groups of 4 warps take alternate K stages; thread = weight row,
        // the whole 64-element stage of its row (32 bytes of nibbles, two
        // sub-blocks).  A quarter-warp stores 8 consecutive rows' same logical
        // chunk, which the swizzle spreads over all banks.
        const uint32_t grp = (warp - 4) >> 2, row = (threadIdx.x - 128) & 127;
        bool ok = true;
        for (uint32_t kc = grp; kc < nk; kc += 2) {
            if (*abort_flag) {
                ok = false;
                break;
            }
            const uint32_t s = kc % S, j = kc / 4, g = kc % 4, r = j % kGemmRawStages;
            if (g == grp && !mbar_wait(&raw_full[r], (j / kGemmRawStages) & 1, p.status, 47)) ok = false;
            if (ok && kc >= S && !mbar_wait(&empty[s], ((kc / S) - 1) & 1, p.status, 48)) ok = false;
            if (!ok) {
                *abort_flag = 1;
                break;
            }
            const uint8_t* rp = smem + Plan::kOffRaw + r * kGemmRawBytes + row * kGemmSbBytes;
            const uint4 h = *reinterpret_cast<const uint4*>(rp);
            const uint4 qa = *reinterpret_cast<const uint4*>(rp + 16 + 32 * g);
            const uint4 qb = *reinterpret_cast<const uint4*>(rp + 32 + 32 * g);
            const float d = f16_bits_to_f32(static_cast<uint16_t>(h.x & 0xFFFFu));
            const float dmin = f16_bits_to_f32(static_cast<uint16_t>(h.x >> 16));
            uint32_t sc_lo, mn_lo, sc_hi, mn_hi;
            q4k_scale_min(h.y, h.z, h.w, 2 * g, sc_lo, mn_lo);
            q4k_scale_min(h.y, h.z, h.w, 2 * g + 1, sc_hi, mn_hi);
            const float dsl = __fmul_rn(d, static_cast<float>(sc_lo)), dml = __fmul_rn(dmin, static_cast<float>(mn_lo));
            const float dsh = __fmul_rn(d, static_cast<float>(sc_hi)), dmh = __fmul_rn(dmin, static_cast<float>(mn_hi));
            const uint64_t dsl2 = f32x2(dsl, dsl), dml2 = f32x2(dml, dml);
            const uint64_t dsh2 = f32x2(dsh, dsh), dmh2 = f32x2(dmh, dmh);
            const uint32_t qw[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
            // element e of the stage's 64 goes to word e / 2 (low half for even e):
            // words 0..15 = low nibbles of bytes 0..31, words 16..31 = high nibbles
            uint32_t av[32];
#pragma unroll
            for (uint32_t c = 0; c < 4; ++c) {
                const uint2 l0 = dequant4(qw[2 * c] & 0x0F0F0F0Fu, dsl2, dml2);
                const uint2 l1 = dequant4(qw[2 * c + 1] & 0x0F0F0F0Fu, dsl2, dml2);
                const uint2 h0 = dequant4((qw[2 * c] >> 4) & 0x0F0F0F0Fu, dsh2, dmh2);
                const uint2 h1 = dequant4((qw[2 * c + 1] >> 4) & 0x0F0F0F0Fu, dsh2, dmh2);
                av[4 * c + 0] = l0.x, av[4 * c + 1] = l0.y, av[4 * c + 2] = l1.x, av[4 * c + 3] = l1.y;
                av[16 + 4 * c + 0] = h0.x, av[16 + 4 * c + 1] = h0.y, av[16 + 4 * c + 2] = h1.x,
                                av[16 + 4 * c + 3] = h1.y;
            }
            if constexpr (Plan::kATmem) {
                // this warp's 32 rows are TMEM lanes 32 * (warp % 4) ...
                tmem_st_32x32b_x32(tmem + ((32u * (warp & 3u)) << 16) + Plan::kATmemCol + 32 * s, av);
                tc_fence_before();
            } else {
                // K-major, 128-byte swizzle: 16-byte chunk c of row r at c ^ (r & 7)
                uint8_t* arow = smem + s * kGemmABytes + row * 128;
#pragma unroll
                for (uint32_t c = 0; c < 8; ++c)
                    *reinterpret_cast<uint4*>(arow + ((c ^ (row & 7)) * 16)) =
                        make_uint4(av[4 * c], av[4 * c + 1], av[4 * c + 2], av[4 * c + 3]);
                fence_async_smem();
            }
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&full_a[s]);
                if (g == grp + 2) mbar_arrive(&raw_empty[r]);
            }
        }
        // ------------------------------------------------------------------ epilogue
        if (!mbar_wait(acc_full, 0, p.status, 49)) ok = false;
        tc_fence_after();
        const uint32_t q = warp & 3, half = (warp - 4) >> 2;
        const uint32_t n = n0 + 32 * q + lane;
        if (ok && !*abort_flag) {
#pragma unroll 1
            for (uint32_t cb = 0; cb < kGemmTileM / 64; ++cb) {
                const uint32_t col0 = half * (kGemmTileM / 2) + 32 * cb;
                uint32_t v[32];
                tmem_ld_32x32b_x32(tmem + ((32 * q) << 16) + col0, v);
                if (n < p.n) {
#pragma unroll
                    for (uint32_t jj = 0; jj < 32; ++jj) {
                        const uint32_t m = m0 + col0 + jj;
                        if (m < p.m) {
                            float* dst = p.y + static_cast<uint64_t>(m) * p.n + n;
                            if (p.accumulate)
                                atomicAdd(dst, __uint_as_float(v[jj]));
                            else
                                *dst = __uint_as_float(v[jj]);
                        }
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if constexpr (kPair) cluster_sync_all();  // no CTA leaves while its peer may still touch it
    if (warp == 0) {
        __syncwarp();
        tc_fence_after();
        if constexpr (kPair)
            asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(Plan::kTmemCols)
                         : "memory");
        else
            asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(Plan::kTmemCols)
                         : "memory");
    }
}

// X f32 -> bf16 (round to nearest even), 4 elements per thread-step.
// Four float4 per thread per round, their loads in flight together.
constexpr uint32_t kConvertUnroll = 4;
__global__ void __launch_bounds__(256) convert_bf16_kernel(const float* __restrict__ x, uint32_t* __restrict__ out,
                                                           uint64_t n4) {
    const uint64_t stride = uint64_t(gridDim.x) * blockDim.x;
    for (uint64_t i = blockIdx.x * uint64_t(blockDim.x) + threadIdx.x; i < n4; i += kConvertUnroll * stride) {
        float4 v[kConvertUnroll];
#pragma unroll
        for (uint32_t u = 0; u < kConvertUnroll; ++u)
            if (i + u * stride < n4) v[u] = __ldg(reinterpret_cast<const float4*>(x) + i + u * stride);
#pragma unroll
        for (uint32_t u = 0; u < kConvertUnroll; ++u)
            if (i + u * stride < n4)
                reinterpret_cast<uint2*>(out)[i + u * stride] =
                    make_uint2(pack_bf16x2(v[u].x, v[u].y), pack_bf16x2(v[u].z, v[u].w));
    }
}

}  // namespace oracle_cuda
