// gather.cuh -- the steps either side of the matvecs: embedding-row gather and
// greedy argmax over logits.
//
// gather_rows_kernel restates Oracle's embedding lookup (embedding_row,
// src/runtime/qwen35_forward.cpp:51-70: bounds check of the token id, then
// decode_storage_row of that row) for a batch of token ids held in device
// memory; every element is Oracle's exact f32 decode (decode4).  A token id
// outside the table is not read: the kernel records it in the status word
// (kDevBadIndex) and leaves that output row untouched.
//
// argmax_kernel restates the greedy branch of Oracle's sampler
// (src/runtime/sampler.cpp:22-46): the first index holding the largest value,
// NaN anywhere is an error, a non-finite maximum is an error.  Each value maps
// to a 64-bit key, (order-preserving bits of the value) << 32 | ~index, so
// the largest key is the largest value at the lowest index; -0.0 counts as
// +0.0 (the reference compares with `>`), and a NaN maps to the all-ones key,
// which no number reaches.  Blocks reduce their keys and combine them with one
// 64-bit atomicMax into a key the caller zeroed.
#pragma once

#include "decode.cuh"

namespace oracle_cuda {

enum : unsigned int { kDevBadIndex = 2 };

template <uint32_t kType>
__global__ void __launch_bounds__(256) gather_rows_kernel(const uint8_t* __restrict__ w, uint64_t rows, uint32_t k,
                                                          uint64_t row_bytes, const uint32_t* __restrict__ ids,
                                                          uint64_t n_ids, float* __restrict__ out,
                                                          DeviceStatus* st) {
    pdl_enter();
    const uint32_t chunks = (k + 3) / 4;
    const uint64_t total = n_ids * chunks;
    for (uint64_t c = blockIdx.x * uint64_t(blockDim.x) + threadIdx.x; c < total;
         c += uint64_t(gridDim.x) * blockDim.x) {
        const uint64_t t = c / chunks;
        const uint32_t e = static_cast<uint32_t>(c % chunks) * 4u;
        const uint32_t id = __ldg(ids + t);
        if (id >= rows) {
            if (e == 0 && st && atomicCAS(&st->code, kDevOk, kDevBadIndex) == kDevOk) {
                st->where = id;
                st->block = static_cast<unsigned int>(t);
            }
            continue;
        }
        float v[4];
        decode4<kType, true>(w + id * row_bytes, e, k, v);
        float* o = out + t * k + e;
#pragma unroll
        for (int q = 0; q < 4; ++q)
            if (e + q < k) o[q] = v[q];
    }
}

__device__ __forceinline__ unsigned long long argmax_key(float v, uint32_t index) {
    if (v != v) return ~0ull;  // NaN
    uint32_t b = __float_as_uint(v == 0.0f ? 0.0f : v);
    b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);  // order-preserving
    return (static_cast<unsigned long long>(b) << 32) | static_cast<unsigned long long>(~index);
}

__global__ void __launch_bounds__(256) argmax_kernel(const float* __restrict__ x, uint64_t n, uint32_t index_base,
                                                     unsigned long long* __restrict__ key_out) {
    pdl_enter();
    x += blockIdx.y * n;  // row blockIdx.y of a batch of logits vectors, one key each
    key_out += blockIdx.y;
    __shared__ unsigned long long warp_best[8];
    unsigned long long best = 0;
    for (uint64_t i = blockIdx.x * uint64_t(blockDim.x) + threadIdx.x; i < n; i += uint64_t(gridDim.x) * blockDim.x) {
        const unsigned long long k = argmax_key(__ldg(x + i), index_base + static_cast<uint32_t>(i));
        best = k > best ? k : best;
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) {
        const unsigned long long o = __shfl_xor_sync(0xFFFFFFFFu, best, off);
        best = o > best ? o : best;
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) warp_best[warp] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < static_cast<int>(blockDim.x >> 5); ++w) best = warp_best[w] > best ? warp_best[w] : best;
        atomicMax(key_out, best);
    }
}

// Host-side decode of an argmax key: token index and whether the maximum is
// a finite number; `nan` when some value was NaN.
struct ArgmaxResult {
    uint32_t index;
    bool nan;
    bool finite;
    float value;
};

__host__ __device__ inline ArgmaxResult decode_argmax_key(unsigned long long key) {
    ArgmaxResult r{};
    if (key == ~0ull) {
        r.nan = true;
        return r;
    }
    uint32_t b = static_cast<uint32_t>(key >> 32);
    b = (b & 0x80000000u) ? (b & 0x7FFFFFFFu) : ~b;
    float v;
#ifdef __CUDA_ARCH__
    v = __uint_as_float(b);
#else
    static_assert(sizeof v == sizeof b, "float width");
    memcpy(&v, &b, sizeof v);
#endif
    r.value = v;
    r.index = ~static_cast<uint32_t>(key & 0xFFFFFFFFull);
    r.finite = v == v && v - v == 0.0f;
    return r;
}

enum : unsigned int { kDevLogitsNaN = 5, kDevLogitsNonFinite = 6 };

// One decode step's bookkeeping on the device, so that a step captured in a
// CUDA graph can be replayed token after token without the host: the argmax
// key of the step's logits becomes the sampled token (Sampler::sample at
// temperature 0), and the next step's input id is the next prompt token while
// the prompt lasts (the reference ingests prompts one token at a time,
// qwen35_generation.cpp:737-747), else the sampled token, which is also
// appended to tokens_out.  Then the position advances.  A NaN or non-finite
// maximum is reported (the sampler's invalid_argument) and ends sampling:
// the position does not advance.
__global__ void token_commit_kernel(const unsigned long long* __restrict__ key, const uint32_t* __restrict__ prompt,
                                    uint32_t n_prompt, uint32_t* pos, uint32_t* next_id, uint32_t* tokens_out,
                                    uint32_t out_capacity, DeviceStatus* st) {
    pdl_enter();
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    const ArgmaxResult r = decode_argmax_key(*key);
    const uint32_t p = *pos;
    if (r.nan || !r.finite) {
        if (st && atomicCAS(&st->code, kDevOk, r.nan ? kDevLogitsNaN : kDevLogitsNonFinite) == kDevOk) {
            st->where = p;
            st->block = 0;
        }
        return;
    }
    if (p + 1 < n_prompt) {
        *next_id = prompt[p + 1];
    } else {
        *next_id = r.index;
        const uint32_t i = p + 1 - n_prompt;
        if (i < out_capacity) tokens_out[i] = r.index;
    }
    *pos = p + 1;
}

// token_commit_kernel for a batch of sequences decoded in lockstep (one
// position): sequence b's key is keys[b], its prompt prompt[b * n_prompt ..],
// its next input next_id[b] and its tokens tokens_out[b * out_capacity ..].
// Each key is cleared after it is read (the next step's argmax accumulates
// into it).  A NaN or non-finite maximum in any sequence is reported and
// stops the batch: the position does not advance.
__global__ void __launch_bounds__(256) token_commit_rows_kernel(unsigned long long* __restrict__ keys, uint32_t rows,
                                                                const uint32_t* __restrict__ prompt,
                                                                uint32_t n_prompt, uint32_t* pos,
                                                                uint32_t* __restrict__ next_id,
                                                                uint32_t* __restrict__ tokens_out,
                                                                uint32_t out_capacity, DeviceStatus* st) {
    pdl_enter();
    __shared__ int bad;
    if (threadIdx.x == 0) bad = 0;
    __syncthreads();
    const uint32_t p = *pos;
    for (uint32_t b = threadIdx.x; b < rows; b += blockDim.x) {
        const ArgmaxResult r = decode_argmax_key(keys[b]);
        if (r.nan || !r.finite) {
            bad = 1;
            if (st && atomicCAS(&st->code, kDevOk, r.nan ? kDevLogitsNaN : kDevLogitsNonFinite) == kDevOk) {
                st->where = p;
                st->block = b;
            }
        }
    }
    __syncthreads();
    if (bad) return;
    for (uint32_t b = threadIdx.x; b < rows; b += blockDim.x) {
        const ArgmaxResult r = decode_argmax_key(keys[b]);
        keys[b] = 0ull;
        if (p + 1 < n_prompt) {
            next_id[b] = prompt[uint64_t(b) * n_prompt + p + 1];
        } else {
            next_id[b] = r.index;
            const uint32_t i = p + 1 - n_prompt;
            if (i < out_capacity) tokens_out[uint64_t(b) * out_capacity + i] = r.index;
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) *pos = p + 1;
}

}  // namespace oracle_cuda
