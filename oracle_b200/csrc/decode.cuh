// decode.cuh -- GGML block decode to f32, four consecutive elements at a time.
//
// Restates Oracle's decoders (src/model/storage_decode.cpp): Q8_0 :132-139,
// Q5_K :63-94 (and Q4_K = Q5_K without the high-bit plane, qs at offset 16),
// Q6_K :96-125, f16 :150-176, bf16 :178-180.  Every product and difference is
// an explicit round-to-nearest f32 operation in Oracle's evaluation order, so
// decoded values equal Oracle's bit for bit:
//   Q8_0: d * q             Q4_K/Q5_K: (d * sc) * q - dmin * m
//   Q6_K: (d * sc) * q      f16/bf16/f32: exact conversion
// Small integers become floats through the exponent trick: the byte is placed
// under the exponent of 2^23 and 2^23 (+ offset) is subtracted, exactly.
#pragma once

#include "common.cuh"

namespace oracle_cuda {

__device__ __forceinline__ float small_uint_to_f32(uint32_t word, int byte) {
    // float bits 0x4B0000bb = 2^23 + bb
    return __int_as_float(static_cast<int>(__byte_perm(word, 0x4B000000u, 0x7440u + byte)));
}

// Little-endian word from an even address.  With kSafe, the word after is read
// only when the address is 2 mod 4 (so every aligned word read holds at least
// one requested byte); without it, one extra aligned word may be read.
template <bool kSafe>
__device__ __forceinline__ uint32_t ld_u32_even(const uint8_t* p) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    const uint32_t* base = reinterpret_cast<const uint32_t*>(a & ~uintptr_t(3));
    if (kSafe) {
        if ((a & 3u) == 0) return base[0];
        return __funnelshift_r(base[0], base[1], 16);
    }
    return __funnelshift_r(base[0], base[1], static_cast<uint32_t>(a & 3u) * 8u);
}

__device__ __forceinline__ void k4_scale_min(const uint8_t* scales4, int j, float& sc, float& mn) {
    // scales4 is 4-byte aligned (super-block base + 4)
    const uint32_t* s = reinterpret_cast<const uint32_t*>(scales4);
    const uint32_t s0 = s[0], s1 = s[1], s2 = s[2];
    int a, b;
    if (j < 4) {
        a = (s0 >> (8 * j)) & 63;
        b = (s1 >> (8 * j)) & 63;
    } else {
        const int t = 8 * (j - 4);
        a = ((s2 >> t) & 0x0F) | (((s0 >> t) & 0xC0) >> 2);
        b = ((s2 >> t) & 0xF0) >> 4 | (((s1 >> t) & 0xC0) >> 2);
    }
    sc = static_cast<float>(a);
    mn = static_cast<float>(b);
}

// Decode elements e..e+3 (e a multiple of 4, e < k) of a row starting at `row`.
// K-quant and Q8_0 rows start at an even address; Q4_K/Q5_K rows 4-aligned.
template <uint32_t kType, bool kSafe>
__device__ __forceinline__ void decode4(const uint8_t* row, uint32_t e, uint32_t k, float (&w)[4]) {
    if constexpr (kType == 8) {  // Q8_0
        const uint8_t* blk = row + 34u * (e / 32u);
        const float d = f16_bits_to_f32(*reinterpret_cast<const uint16_t*>(blk));
        const uint32_t qw = ld_u32_even<kSafe>(blk + 2 + (e % 32u)) ^ 0x80808080u;
#pragma unroll
        for (int t = 0; t < 4; ++t) w[t] = __fmul_rn(d, __fsub_rn(small_uint_to_f32(qw, t), 8388736.0f));
    } else if constexpr (kType == 12 || kType == 13) {  // Q4_K, Q5_K
        constexpr uint32_t kBB = kType == 12 ? 144u : 176u;
        constexpr uint32_t kQs = kType == 12 ? 16u : 48u;
        const uint8_t* sb = row + kBB * (e / 256u);
        const uint32_t ep = e % 256u, g = ep / 64u, up = (ep / 32u) & 1u, l = ep % 32u;
        const uint32_t dd = *reinterpret_cast<const uint32_t*>(sb);
        const float d = f16_bits_to_f32(static_cast<uint16_t>(dd & 0xFFFFu));
        const float dmin = f16_bits_to_f32(static_cast<uint16_t>(dd >> 16));
        float sc, mn;
        k4_scale_min(sb + 4, static_cast<int>(2 * g + up), sc, mn);
        const uint32_t qw = *reinterpret_cast<const uint32_t*>(sb + kQs + 32u * g + l);
        uint32_t q = up ? ((qw >> 4) & 0x0F0F0F0Fu) : (qw & 0x0F0F0F0Fu);
        if constexpr (kType == 13) {
            const uint32_t hw = *reinterpret_cast<const uint32_t*>(sb + 16 + l);
            q |= ((hw >> (2 * g + up)) & 0x01010101u) << 4;
        }
        const float dsc = __fmul_rn(d, sc);
        const float dm = __fmul_rn(dmin, mn);
#pragma unroll
        for (int t = 0; t < 4; ++t)
            w[t] = __fsub_rn(__fmul_rn(dsc, __fsub_rn(small_uint_to_f32(q, t), 8388608.0f)), dm);
    } else if constexpr (kType == 14) {  // Q6_K
        const uint8_t* sb = row + 210u * (e / 256u);
        const uint32_t ep = e % 256u, h = ep / 128u, s = (ep % 128u) / 32u, l = ep % 32u;
        const uint32_t lw = ld_u32_even<kSafe>(sb + 64u * h + l + ((s & 1u) ? 32u : 0u));
        const uint32_t hw = ld_u32_even<kSafe>(sb + 128u + 32u * h + l);
        const uint32_t lo = (s >= 2u) ? ((lw >> 4) & 0x0F0F0F0Fu) : (lw & 0x0F0F0F0Fu);
        const uint32_t q = lo | (((hw >> (2u * s)) & 0x03030303u) << 4);
        const int scale = static_cast<int8_t>(sb[192u + 8u * h + l / 16u + 2u * s]);
        const float d = f16_bits_to_f32(static_cast<uint16_t>(sb[208] | (sb[209] << 8)));
        const float dsc = __fmul_rn(d, static_cast<float>(scale));
#pragma unroll
        for (int t = 0; t < 4; ++t) w[t] = __fmul_rn(dsc, __fsub_rn(small_uint_to_f32(q, t), 8388640.0f));
    } else if constexpr (kType == 0) {  // f32
#pragma unroll
        for (int t = 0; t < 4; ++t) w[t] = e + t < k ? reinterpret_cast<const float*>(row)[e + t] : 0.0f;
    } else if constexpr (kType == 1) {  // f16
#pragma unroll
        for (int t = 0; t < 4; ++t)
            w[t] = e + t < k ? f16_bits_to_f32(reinterpret_cast<const uint16_t*>(row)[e + t]) : 0.0f;
    } else if constexpr (kType == 30) {  // bf16
#pragma unroll
        for (int t = 0; t < 4; ++t)
            w[t] = e + t < k ? __uint_as_float(uint32_t(reinterpret_cast<const uint16_t*>(row)[e + t]) << 16)
                             : 0.0f;
    }
}

// decode_storage_row over `rows` rows: thread per 4-element chunk, reading the
// packed bytes straight from global memory (safe word reads), f32 out.
template <uint32_t kType>
__global__ void __launch_bounds__(256) decode_rows_kernel(const uint8_t* __restrict__ w, uint64_t rows,
                                                          uint32_t k, uint64_t row_bytes,
                                                          float* __restrict__ out) {
    const uint32_t chunks = (k + 3) / 4;
    const uint64_t total = rows * chunks;
    for (uint64_t c = blockIdx.x * uint64_t(blockDim.x) + threadIdx.x; c < total;
         c += uint64_t(gridDim.x) * blockDim.x) {
        const uint64_t r = c / chunks;
        const uint32_t e = static_cast<uint32_t>(c % chunks) * 4u;
        float v[4];
        decode4<kType, true>(w + r * row_bytes, e, k, v);
        float* o = out + r * k + e;
#pragma unroll
        for (int t = 0; t < 4; ++t)
            if (e + t < k) o[t] = v[t];
    }
}

}  // namespace oracle_cuda
