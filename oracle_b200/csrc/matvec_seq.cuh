// matvec_seq.cuh -- Oracle's f32 contract, bit for bit: y[r] = sequential sum.
//
// Oracle's reference_storage_dot (quantized_reference.cpp:24-82) decodes the
// row to f32 block by block and adds decoded[e] * x[e] into ONE running f32
// sum, e = 0, 1, ..., K-1, each product and each addition rounded (ISO C++ has
// no contraction).  This kernel performs exactly those operations in exactly
// that order, so its output equals the reference's bit for bit:
//   sum = __fadd_rn(sum, __fmul_rn(w_e, x_e)),  w_e = Oracle's decode (decode.cuh)
//
// Mapping: one lane per row (a row's sum is a serial chain; rows run in
// parallel).  A warp owns 32 consecutive rows.  The row is walked in chunks of
// whole blocks (kChunkBlocks blocks, kChunkElems elements, kChunkBytes bytes).
// For each chunk the warp copies its 32 rows' chunk bytes into a shared slot
// per row, realigned so every slot starts at a 4-byte boundary (each slot word
// is a funnel shift of two aligned global words, read coalesced), with an odd
// slot stride in words so that lane-per-row shared reads are conflict-free.
// Each lane then decodes its own slot at compile-time offsets.  x is read with
// warp-uniform (broadcast) loads.
#pragma once

#include "decode.cuh"

namespace oracle_cuda {

template <uint32_t kType>
struct SeqChunk;
template <> struct SeqChunk<8>  { static constexpr uint32_t kBlocks = 8, kBlockElems = 32,  kBlockBytes = 34; };
template <> struct SeqChunk<12> { static constexpr uint32_t kBlocks = 1, kBlockElems = 256, kBlockBytes = 144; };
template <> struct SeqChunk<13> { static constexpr uint32_t kBlocks = 1, kBlockElems = 256, kBlockBytes = 176; };
template <> struct SeqChunk<14> { static constexpr uint32_t kBlocks = 1, kBlockElems = 256, kBlockBytes = 210; };
template <> struct SeqChunk<0>  { static constexpr uint32_t kBlocks = 64, kBlockElems = 1, kBlockBytes = 4; };
template <> struct SeqChunk<1>  { static constexpr uint32_t kBlocks = 128, kBlockElems = 1, kBlockBytes = 2; };
template <> struct SeqChunk<30> { static constexpr uint32_t kBlocks = 128, kBlockElems = 1, kBlockBytes = 2; };

constexpr int kSeqWarps = 4;
constexpr uint32_t kSeqMaxBatch = 4;

struct MatvecSeqParams {
    const uint8_t* w;
    const float* x;  // batch vectors of k floats
    float* y;        // batch * rows
    uint64_t rows;
    uint64_t row_bytes;
    uint32_t k;
    uint32_t batch;  // <= kSeqMaxBatch
};

__device__ __forceinline__ uint32_t slot_byte(const uint32_t* s, uint32_t off) {
    return (s[off >> 2] >> (8u * (off & 3u))) & 0xFFu;
}

template <uint32_t kType>
__global__ void __launch_bounds__(kSeqWarps * 32) matvec_seq_kernel(const MatvecSeqParams p) {
    using Ch = SeqChunk<kType>;
    constexpr uint32_t kChunkBytes = Ch::kBlocks * Ch::kBlockBytes;
    constexpr uint32_t kChunkElems = Ch::kBlocks * Ch::kBlockElems;
    constexpr uint32_t kWords = (kChunkBytes + 3) / 4 + 1;           // + 1: a misaligned chunk spans one more word
    constexpr uint32_t kStride = (kWords % 2) ? kWords : kWords + 1;  // odd: conflict-free lane-per-row reads
    __shared__ uint32_t slots[kSeqWarps][32 * kStride];

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint32_t* myslots = slots[warp];
    const uint64_t row_base = (static_cast<uint64_t>(blockIdx.x) * kSeqWarps + warp) * 32;
    if (row_base >= p.rows) return;
    const uint32_t nr = p.rows - row_base < 32 ? static_cast<uint32_t>(p.rows - row_base) : 32u;
    const uint64_t my_row = row_base + lane;
    const bool live = lane < static_cast<int>(nr);

    float sum[kSeqMaxBatch];
#pragma unroll
    for (uint32_t b = 0; b < kSeqMaxBatch; ++b) sum[b] = 0.0f;

    const uint32_t n_chunks = (p.k + kChunkElems - 1) / kChunkElems;
    for (uint32_t c = 0; c < n_chunks; ++c) {
        const uint32_t e0 = c * kChunkElems;
        const uint32_t elems = p.k - e0 < kChunkElems ? p.k - e0 : kChunkElems;
        const uint32_t blocks = elems / Ch::kBlockElems;  // whole blocks in this chunk
        const uint32_t cbytes = blocks * Ch::kBlockBytes;
        // ---- cooperative copy: slot word j of row i = bytes [4j, 4j+4) of the chunk
        const uint32_t words = (cbytes + 3) / 4;
        __syncwarp();
        for (uint32_t t = lane; t < nr * words; t += 32) {
            const uint32_t i = t / words, j = t % words;
            const uintptr_t start = reinterpret_cast<uintptr_t>(p.w) + (row_base + i) * p.row_bytes +
                                    static_cast<uint64_t>(c) * (kChunkElems / Ch::kBlockElems) * Ch::kBlockBytes;
            const uintptr_t aw = (start & ~uintptr_t(3)) + 4u * j;
            const uint32_t sh = static_cast<uint32_t>(start & 3u) * 8u;
            const uint32_t lo = *reinterpret_cast<const uint32_t*>(aw);
            // the next aligned word is read only if it holds wanted bytes
            const bool need_hi = sh != 0 && (aw + 4) < start + cbytes;
            const uint32_t hi = need_hi ? *reinterpret_cast<const uint32_t*>(aw + 4) : 0u;
            myslots[i * kStride + j] = sh ? __funnelshift_r(lo, hi, sh) : lo;
        }
        __syncwarp();
        if (!live) continue;
        const uint32_t* s = myslots + lane * kStride;
        // ---- decode this lane's chunk and accumulate in element order
        for (uint32_t bi = 0; bi < blocks; ++bi) {
            const uint32_t bo = bi * Ch::kBlockBytes;  // block offset in the slot
            const uint32_t eb = e0 + bi * Ch::kBlockElems;
            if constexpr (kType == 8) {
                const float d = f16_bits_to_f32(static_cast<uint16_t>(slot_byte(s, bo) | (slot_byte(s, bo + 1) << 8)));
#pragma unroll 8
                for (uint32_t l = 0; l < 32; ++l) {
                    const int q = static_cast<int>(static_cast<int8_t>(slot_byte(s, bo + 2 + l)));
                    const float wv = __fmul_rn(d, static_cast<float>(q));
#pragma unroll
                    for (uint32_t b = 0; b < kSeqMaxBatch; ++b)
                        if (b < p.batch) sum[b] = __fadd_rn(sum[b], __fmul_rn(wv, __ldg(p.x + uint64_t(b) * p.k + eb + l)));
                }
            } else if constexpr (kType == 12 || kType == 13) {
                constexpr uint32_t kQs = kType == 12 ? 16u : 48u;
                const float d = f16_bits_to_f32(static_cast<uint16_t>(slot_byte(s, bo) | (slot_byte(s, bo + 1) << 8)));
                const float dmin = f16_bits_to_f32(static_cast<uint16_t>(slot_byte(s, bo + 2) | (slot_byte(s, bo + 3) << 8)));
                for (uint32_t g = 0; g < 4; ++g) {
                    for (uint32_t up = 0; up < 2; ++up) {
                        const uint32_t jsb = 2 * g + up;
                        int sc, mn;
                        if (jsb < 4) {
                            sc = slot_byte(s, bo + 4 + jsb) & 63;
                            mn = slot_byte(s, bo + 8 + jsb) & 63;
                        } else {
                            sc = (slot_byte(s, bo + 8 + jsb) & 0x0F) | ((slot_byte(s, bo + jsb) >> 6) << 4);
                            mn = (slot_byte(s, bo + 8 + jsb) >> 4) | ((slot_byte(s, bo + 4 + jsb) >> 6) << 4);
                        }
                        const float dsc = __fmul_rn(d, static_cast<float>(sc));
                        const float dm = __fmul_rn(dmin, static_cast<float>(mn));
#pragma unroll 8
                        for (uint32_t l = 0; l < 32; ++l) {
                            const uint32_t byte = slot_byte(s, bo + kQs + 32 * g + l);
                            uint32_t q = up ? (byte >> 4) : (byte & 0x0F);
                            if constexpr (kType == 13) q |= ((slot_byte(s, bo + 16 + l) >> jsb) & 1u) << 4;
                            const float wv = __fsub_rn(__fmul_rn(dsc, static_cast<float>(q)), dm);
                            const uint32_t e = eb + 64 * g + 32 * up + l;
#pragma unroll
                            for (uint32_t b = 0; b < kSeqMaxBatch; ++b)
                                if (b < p.batch) sum[b] = __fadd_rn(sum[b], __fmul_rn(wv, __ldg(p.x + uint64_t(b) * p.k + e)));
                        }
                    }
                }
            } else if constexpr (kType == 14) {
                const float d = f16_bits_to_f32(static_cast<uint16_t>(slot_byte(s, bo + 208) | (slot_byte(s, bo + 209) << 8)));
                for (uint32_t h = 0; h < 2; ++h) {
                    for (uint32_t sg = 0; sg < 4; ++sg) {
                        for (uint32_t half16 = 0; half16 < 2; ++half16) {
                            const int scale = static_cast<int>(static_cast<int8_t>(slot_byte(s, bo + 192 + 8 * h + half16 + 2 * sg)));
                            const float dsc = __fmul_rn(d, static_cast<float>(scale));
#pragma unroll 8
                            for (uint32_t l16 = 0; l16 < 16; ++l16) {
                                const uint32_t l = 16 * half16 + l16;
                                const uint32_t lo_byte = slot_byte(s, bo + 64 * h + l + ((sg & 1u) ? 32u : 0u));
                                const uint32_t lo = sg >= 2 ? (lo_byte >> 4) : (lo_byte & 0x0F);
                                const uint32_t hi = (slot_byte(s, bo + 128 + 32 * h + l) >> (2 * sg)) & 3u;
                                const int q = static_cast<int>(lo | (hi << 4)) - 32;
                                const float wv = __fmul_rn(dsc, static_cast<float>(q));
                                const uint32_t e = eb + 128 * h + 32 * sg + l;
#pragma unroll
                                for (uint32_t b = 0; b < kSeqMaxBatch; ++b)
                                    if (b < p.batch) sum[b] = __fadd_rn(sum[b], __fmul_rn(wv, __ldg(p.x + uint64_t(b) * p.k + e)));
                            }
                        }
                    }
                }
            } else {  // f32, f16, bf16: one element per block
                float wv;
                if constexpr (kType == 0) {
                    wv = __uint_as_float(s[bo >> 2]);
                } else {
                    const uint32_t h16 = slot_byte(s, bo) | (slot_byte(s, bo + 1) << 8);
                    wv = kType == 1 ? f16_bits_to_f32(static_cast<uint16_t>(h16)) : __uint_as_float(h16 << 16);
                }
#pragma unroll
                for (uint32_t b = 0; b < kSeqMaxBatch; ++b)
                    if (b < p.batch) sum[b] = __fadd_rn(sum[b], __fmul_rn(wv, __ldg(p.x + uint64_t(b) * p.k + eb)));
            }
        }
    }
    if (live) {
#pragma unroll
        for (uint32_t b = 0; b < kSeqMaxBatch; ++b)
            if (b < p.batch) p.y[uint64_t(b) * p.rows + my_row] = sum[b];
    }
}

}  // namespace oracle_cuda
