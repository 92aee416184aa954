// matvec_seq.cuh -- Oracle's f32 contract, bit for bit: y[r] = sequential sum.
//
// Oracle's reference_storage_dot (quantized_reference.cpp:24-82) decodes the
// row to f32 block by block and adds decoded[e] * x[e] into ONE running f32
// sum, e = 0, 1, ..., K-1, each product and each addition rounded (ISO C++ has
// no contraction).  This kernel performs exactly those operations in exactly
// that order, so its output equals the reference's bit for bit:
//   sum = __fadd_rn(sum, __fmul_rn(w_e, x_e)),  w_e = Oracle's decode (decode.cuh)
//
// The additions of one row form a serial chain of K dependent f32 adds; that
// chain, not HBM, bounds the kernel (K x add latency per row).  Everything
// else is independent work, so the CTA splits it off:
//   * chain warps (kBatch of them, warp b owns activation vector b): lane r
//     keeps the running sum of row r and does nothing but one 128-bit shared
//     load per 4 products and the adds;
//   * producer warps (the other 8 - kBatch) copy the CTA's rows a chunk of
//     C elements at a time into a ring of raw stages with cp.async (4-byte
//     words covering the chunk, so any 2-byte row alignment works), several
//     chunks ahead of use, then decode each chunk from shared memory (decode4),
//     multiply by x and store the products to a two-deep product ring.
// Product stages are handed to the chains with named barriers (FULL: producers
// arrive, chains sync; EMPTY: chains arrive, producers sync before reuse).
// Raw stages are private to the producers (cp.async groups + a producer-only
// barrier).  Product layout per stage and vector: rows of C + 4 words, so a
// chain lane's 128-bit loads hit distinct banks in every quarter-warp.
#pragma once

#include "decode.cuh"

namespace oracle_cuda {

constexpr uint32_t kSeqRows = 8;       // rows per CTA (one chain lane each; several CTAs per SM)
constexpr uint32_t kSeqThreads = 256;  // 8 warps: kBatch chain warps + producers
constexpr uint32_t kSeqStages = 2;     // product stages
constexpr uint32_t kSeqMaxBatch = 4;
constexpr uint32_t kSeqMaxRawStages = 16;
// named barrier ids: FULL 1..2, EMPTY 3..4, producers-only 5
constexpr uint32_t kSeqBarFull = 1, kSeqBarEmpty = 1 + kSeqStages, kSeqBarProducers = 1 + 2 * kSeqStages;

// Elements per chunk: whole blocks, at least 128 elements.
__host__ __device__ constexpr uint32_t seq_chunk_elems(uint32_t type) {
    return (type == 12 || type == 13 || type == 14) ? 256u : 128u;
}
__host__ __device__ constexpr uint32_t seq_chunk_bytes(uint32_t type) {
    return type == 8 ? 136u : type == 12 ? 144u : type == 13 ? 176u : type == 14 ? 210u : type == 0 ? 512u : 256u;
}
// raw slot per row: the chunk's bytes as aligned words plus one word of slack
__host__ __device__ constexpr uint32_t seq_raw_slot_bytes(uint32_t type) {
    return (((seq_chunk_bytes(type) + 3u) & ~3u) + 4u + 15u) & ~15u;
}
__host__ __device__ constexpr uint32_t seq_prod_bytes(uint32_t type, uint32_t batch) {
    return kSeqStages * batch * kSeqRows * (seq_chunk_elems(type) + 4u) * 4u;
}

struct MatvecSeqParams {
    const uint8_t* w;
    const float* x;  // batch vectors of k floats
    float* y;        // batch * rows
    uint64_t rows;
    uint64_t row_bytes;
    uint32_t k;
    uint32_t raw_stages;  // 3 .. kSeqMaxRawStages
};

__device__ __forceinline__ void cp_async_4(uint32_t dst_smem, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(dst_smem), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }
__device__ __forceinline__ void cp_async_wait_dyn(uint32_t n) {
    // wait_group takes an immediate; the prefetch distance is at most 14
    switch (n) {
        case 0: cp_async_wait<0>(); break;
        case 1: cp_async_wait<1>(); break;
        case 2: cp_async_wait<2>(); break;
        case 3: cp_async_wait<3>(); break;
        case 4: cp_async_wait<4>(); break;
        case 5: cp_async_wait<5>(); break;
        case 6: cp_async_wait<6>(); break;
        case 7: cp_async_wait<7>(); break;
        case 8: cp_async_wait<8>(); break;
        case 9: cp_async_wait<9>(); break;
        case 10: cp_async_wait<10>(); break;
        case 11: cp_async_wait<11>(); break;
        case 12: cp_async_wait<12>(); break;
        case 13: cp_async_wait<13>(); break;
        default: cp_async_wait<14>(); break;
    }
}

template <uint32_t kType, uint32_t kBatch>
__global__ void __launch_bounds__(kSeqThreads) matvec_seq_kernel(const MatvecSeqParams p) {
    constexpr uint32_t C = seq_chunk_elems(kType);
    constexpr uint32_t kStride = C + 4;
    constexpr uint32_t kVecWords = kSeqRows * kStride;
    constexpr uint32_t kSlot = seq_raw_slot_bytes(kType);
    extern __shared__ __align__(16) float prod[];  // [stage][batch][row][kStride], then the raw ring
    uint8_t* raw = reinterpret_cast<uint8_t*>(prod + kSeqStages * kBatch * kVecWords);

    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint64_t row_base = static_cast<uint64_t>(blockIdx.x) * kSeqRows;
    const uint32_t nr = p.rows - row_base < kSeqRows ? static_cast<uint32_t>(p.rows - row_base) : kSeqRows;
    const uint32_t n_chunks = (p.k + C - 1) / C;

    if (warp < kBatch) {
        // ---------------------------------------------------------- chain warp
        const uint32_t b = warp;
        float sum = 0.0f;
        for (uint32_t c = 0; c < n_chunks; ++c) {
            const uint32_t s = c % kSeqStages;
            named_barrier_sync(kSeqBarFull + s, kSeqThreads);
            const uint32_t elems = p.k - c * C < C ? p.k - c * C : C;
            const float* row = prod + (s * kBatch + b) * kVecWords + (lane < kSeqRows ? lane : 0) * kStride;
            if (elems == C) {
#pragma unroll 8
                for (uint32_t e = 0; e < C; e += 4) {
                    const float4 v = *reinterpret_cast<const float4*>(row + e);
                    sum = __fadd_rn(sum, v.x);
                    sum = __fadd_rn(sum, v.y);
                    sum = __fadd_rn(sum, v.z);
                    sum = __fadd_rn(sum, v.w);
                }
            } else {
                for (uint32_t e = 0; e < elems; ++e) sum = __fadd_rn(sum, row[e]);
            }
            if (c + kSeqStages < n_chunks) named_barrier_arrive(kSeqBarEmpty + s, kSeqThreads);
        }
        if (lane < nr) p.y[uint64_t(b) * p.rows + row_base + lane] = sum;
        return;
    }

    // ---------------------------------------------------------- producer warps
    constexpr uint32_t kProducers = kSeqThreads - 32 * kBatch;
    const uint32_t pt = threadIdx.x - 32 * kBatch;
    const uint32_t raw_base = static_cast<uint32_t>(__cvta_generic_to_shared(raw));
    const uint32_t dist = p.raw_stages - 2;  // chunks in flight ahead of the one being decoded
    constexpr uint32_t kFullBytes = seq_chunk_bytes(kType);

    // bytes of chunk c (the last one may be partial)
    auto chunk_bytes = [&](uint32_t c) -> uint32_t {
        const uint32_t elems = p.k - c * C < C ? p.k - c * C : C;
        if constexpr (kType == 8) return elems / 32u * 34u;
        else if constexpr (kType == 12 || kType == 13 || kType == 14) return kFullBytes;
        else if constexpr (kType == 0) return elems * 4u;
        else return elems * 2u;
    };
    // cp.async the aligned words covering chunk c of every row into raw stage
    // c % raw_stages: thread u of the flat (row, word) space copies one word
    constexpr uint32_t kSlotWords = kSlot / 4;
    auto issue = [&](uint32_t c) {
        if (c < n_chunks) {
            const uint32_t bytes = chunk_bytes(c);
            const uint32_t slot0 = raw_base + (c % p.raw_stages) * (kSeqRows * kSlot);
            const uintptr_t chunk0 = reinterpret_cast<uintptr_t>(p.w) + row_base * p.row_bytes +
                                     static_cast<uint64_t>(c) * kFullBytes;
            for (uint32_t u = pt; u < nr * kSlotWords; u += kProducers) {
                const uint32_t r = u / kSlotWords, j = u - r * kSlotWords;
                const uintptr_t start = chunk0 + r * p.row_bytes;
                const uintptr_t a0 = start & ~uintptr_t(3);
                if (a0 + 4u * j < start + bytes) cp_async_4(slot0 + r * kSlot + 4u * j, reinterpret_cast<const void*>(a0 + 4u * j));
            }
        }
        cp_async_commit();
    };

    for (uint32_t c = 0; c < dist; ++c) issue(c);
    for (uint32_t c = 0; c < n_chunks; ++c) {
        issue(c + dist);
        cp_async_wait_dyn(dist);                                   // this thread's copies of chunk c landed
        named_barrier_sync(kSeqBarProducers, kProducers);          // ... and every producer's
        const uint32_t s = c % kSeqStages;
        if (c >= kSeqStages) named_barrier_sync(kSeqBarEmpty + s, kSeqThreads);
        const uint32_t e0 = c * C;
        const uint32_t elems = p.k - e0 < C ? p.k - e0 : C;
        const uint32_t groups = (elems + 3) / 4;
        const uint8_t* slot0 = raw + (c % p.raw_stages) * (kSeqRows * kSlot);
        for (uint32_t u = pt; u < nr * groups; u += kProducers) {
            const uint32_t r = groups == C / 4 ? u / (C / 4) : u / groups;
            const uint32_t g = u - r * groups;
            const uintptr_t start = reinterpret_cast<uintptr_t>(p.w) + (row_base + r) * p.row_bytes +
                                    static_cast<uint64_t>(c) * kFullBytes;
            float wv[4];
            decode4<kType, true>(slot0 + r * kSlot + (start & 3u), 4 * g, elems, wv);
            const uint32_t e = e0 + 4 * g;
#pragma unroll
            for (uint32_t b = 0; b < kBatch; ++b) {
                const float* xb = p.x + uint64_t(b) * p.k + e;
                float4 xv;
                if (e + 3 < p.k && (reinterpret_cast<uintptr_t>(xb) & 15u) == 0) {
                    xv = __ldg(reinterpret_cast<const float4*>(xb));
                } else {
                    xv.x = __ldg(xb);
                    xv.y = e + 1 < p.k ? __ldg(xb + 1) : 0.0f;
                    xv.z = e + 2 < p.k ? __ldg(xb + 2) : 0.0f;
                    xv.w = e + 3 < p.k ? __ldg(xb + 3) : 0.0f;
                }
                float4 o;
                o.x = __fmul_rn(wv[0], xv.x);
                o.y = __fmul_rn(wv[1], xv.y);
                o.z = __fmul_rn(wv[2], xv.z);
                o.w = __fmul_rn(wv[3], xv.w);
                *reinterpret_cast<float4*>(prod + (s * kBatch + b) * kVecWords + r * kStride + 4 * g) = o;
            }
        }
        named_barrier_arrive(kSeqBarFull + s, kSeqThreads);
    }
    cp_async_wait<0>();
}

}  // namespace oracle_cuda
