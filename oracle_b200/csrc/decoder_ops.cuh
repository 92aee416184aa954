// decoder_ops.cuh -- the decoder's glue between the matvecs, one decode step.
//
// Each kernel restates one of Oracle's CPU functions and keeps its arithmetic:
// the same f32 / f64 types, the same rounding of every product and sum
// (explicit _rn intrinsics: ISO C++ does not contract), and the same order
// wherever the order is a sequential sum.  Where the reference sums
// sequentially in double, these kernels sum in double in a tree; the double
// result is then rounded to float, so the float outputs agree except when the
// double sums straddle a float rounding boundary.  exp() and log1p() are the
// host C library's float functions bit for bit (ref_expf / ref_log1pf,
// common.cuh).
//   rms_norm_rows_kernel   <- rms_norm_rows           (qwen35_block.cpp:161-188)
//   rope_kernel            <- apply_qwen35_rope       (reference_kernels.cpp:74-123),
//                             cos/sin from a table the host computes with the
//                             reference's own expressions
//   attention_*_kernel     <- causal_attention_step   (reference_kernels.cpp:125-190)
//   conv_step_kernel       <- causal_depthwise_convolution_step (:192-219)
//   gated_delta_kernel     <- gated_delta_step        (:221-335)
//   swiglu_kernel          <- silu(gate) * up         (qwen35_block.cpp:138-159, 315-318)
//   add_kernel             <- add_vectors             (qwen35_block.cpp:190-200)
#pragma once

#include "common.cuh"

namespace oracle_cuda {

// Block-wide double sum (blockDim.x a multiple of 32, <= 1024); every thread gets it.
__device__ __forceinline__ double block_sum_f64(double v, double* scratch) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    v = warp_sum_f64(v);
    __syncthreads();
    if (lane == 0) scratch[warp] = v;
    __syncthreads();
    double t = lane < nw ? scratch[lane] : 0.0;
    return warp_sum_f64(t);
}

// Two block_sum_f64 reductions at once (scratch of 64 doubles), each with
// the same additions in the same order as a block_sum_f64 of its own.
__device__ __forceinline__ void block_sum2_f64(double a, double b, double* scratch, double& sa, double& sb) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    a = warp_sum_f64(a);
    b = warp_sum_f64(b);
    __syncthreads();
    if (lane == 0) {
        scratch[warp] = a;
        scratch[32 + warp] = b;
    }
    __syncthreads();
    sa = warp_sum_f64(lane < nw ? scratch[lane] : 0.0);
    sb = warp_sum_f64(lane < nw ? scratch[32 + lane] : 0.0);
}

// One CTA per row.
__global__ void __launch_bounds__(256) rms_norm_rows_kernel(const float* __restrict__ in, const float* __restrict__ w,
                                                            uint32_t width, float eps, float* __restrict__ out) {
    __shared__ double scratch[32];
    const float* x = in + static_cast<uint64_t>(blockIdx.x) * width;
    float* y = out + static_cast<uint64_t>(blockIdx.x) * width;
    double s = 0.0;
    for (uint32_t c = threadIdx.x; c < width; c += blockDim.x) {
        const double v = static_cast<double>(x[c]);
        s = __dadd_rn(s, __dmul_rn(v, v));  // product and sum each rounded, as in the reference
    }
    const float inv = rms_inverse(block_sum_f64(s, scratch), width, eps);
    for (uint32_t c = threadIdx.x; c < width; c += blockDim.x) y[c] = __fmul_rn(__fmul_rn(x[c], inv), w[c]);
}

constexpr uint32_t kRopeMaxHalf = 128;
struct RopeTable {
    float cosv[kRopeMaxHalf];
    float sinv[kRopeMaxHalf];
    uint32_t half;
};

__global__ void __launch_bounds__(256) rope_kernel(float* __restrict__ heads, uint32_t n_heads, uint32_t head_dim,
                                                   const __grid_constant__ RopeTable t) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n_heads * t.half) return;
    const uint32_t h = i / t.half, f = i % t.half;
    float* base = heads + static_cast<uint64_t>(h) * head_dim;
    const float a = base[f], b = base[t.half + f], c = t.cosv[f], s = t.sinv[f];
    base[f] = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
    base[t.half + f] = __fadd_rn(__fmul_rn(b, c), __fmul_rn(a, s));
}

// KV cache layout as Oracle's KvCache (hybrid_cache.cpp): keys[token][kv_head][key_dim],
// values[token][kv_head][value_dim].  Appends the new token at `length`.
__global__ void __launch_bounds__(256) attention_append_kernel(const float* __restrict__ k_new,
                                                               const float* __restrict__ v_new, float* keys,
                                                               float* values, uint64_t length, uint32_t nk,
                                                               uint32_t nv) {
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < nk + nv; i += gridDim.x * blockDim.x) {
        if (i < nk)
            keys[length * nk + i] = k_new[i];
        else
            values[length * nv + (i - nk)] = v_new[i - nk];
    }
}

// scores[h][t] = float(double dot(q_h, key_t)) * scale; a warp per (head, token).
__global__ void __launch_bounds__(256) attention_scores_kernel(const float* __restrict__ q,
                                                               const float* __restrict__ keys, uint32_t tokens,
                                                               uint32_t q_heads, uint32_t kv_heads, uint32_t key_dim,
                                                               float scale, float* __restrict__ scores) {
    const uint32_t gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (gw >= q_heads * tokens) return;
    const uint32_t h = gw / tokens, t = gw % tokens, kvh = h / (q_heads / kv_heads);
    const float* qh = q + static_cast<uint64_t>(h) * key_dim;
    const float* kt = keys + (static_cast<uint64_t>(t) * kv_heads + kvh) * key_dim;
    double s = 0.0;
    for (uint32_t d = lane; d < key_dim; d += 32)
        s = __dadd_rn(s, __dmul_rn(static_cast<double>(qh[d]), static_cast<double>(kt[d])));
    s = warp_sum_f64(s);
    if (lane == 0) scores[static_cast<uint64_t>(h) * tokens + t] = __fmul_rn(__double2float_rn(s), scale);
}

// Per head (one CTA): softmax of the scores into probabilities (float of the
// double quotient), then out[h][d] = sum over tokens, in token order, of
// probability * value (each product and sum rounded in float).
__global__ void __launch_bounds__(256) attention_output_kernel(float* __restrict__ scores,
                                                               const float* __restrict__ values, uint32_t tokens,
                                                               uint32_t q_heads, uint32_t kv_heads,
                                                               uint32_t value_dim, float* __restrict__ out,
                                                               DeviceStatus* st) {
    __shared__ double scratch[32];
    __shared__ float fmax_s[32];
    const uint32_t h = blockIdx.x, kvh = h / (q_heads / kv_heads);
    float* sc = scores + static_cast<uint64_t>(h) * tokens;
    float m = -INFINITY;
    for (uint32_t t = threadIdx.x; t < tokens; t += blockDim.x) m = fmaxf(m, sc[t]);
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, off));
    if ((threadIdx.x & 31) == 0) fmax_s[threadIdx.x >> 5] = m;
    __syncthreads();
    m = -INFINITY;
    for (uint32_t w = 0; w < (blockDim.x >> 5); ++w) m = fmaxf(m, fmax_s[w]);
    double den = 0.0;
    for (uint32_t t = threadIdx.x; t < tokens; t += blockDim.x) {
        const float e = ref_expf(__fsub_rn(sc[t], m));
        sc[t] = e;
        den = __dadd_rn(den, static_cast<double>(e));
    }
    den = block_sum_f64(den, scratch);
    if (!(den > 0.0) || !isfinite(den)) {
        if (threadIdx.x == 0 && st) atomicCAS(&st->code, kDevOk, 3u);  // softmax normalisation failed
        return;
    }
    for (uint32_t t = threadIdx.x; t < tokens; t += blockDim.x)
        sc[t] = __double2float_rn(__ddiv_rn(static_cast<double>(sc[t]), den));
    __syncthreads();
    for (uint32_t d = threadIdx.x; d < value_dim; d += blockDim.x) {
        const float* vp = values + static_cast<uint64_t>(kvh) * value_dim + d;
        const uint64_t stride = static_cast<uint64_t>(kv_heads) * value_dim;
        float acc = 0.0f;
        for (uint32_t t = 0; t < tokens; ++t) acc = __fadd_rn(acc, __fmul_rn(sc[t], __ldg(vp + t * stride)));
        out[static_cast<uint64_t>(h) * value_dim + d] = acc;
    }
}

// One thread per channel: shift the history, insert the input, double sum of
// the taps in order, optional SiLU.
__global__ void __launch_bounds__(256) conv_step_kernel(const float* __restrict__ in, const float* __restrict__ w,
                                                        float* history, uint32_t channels, uint32_t kernel,
                                                        int apply_silu, float* __restrict__ out) {
    const uint32_t c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= channels) return;
    float* hc = history + static_cast<uint64_t>(c) * kernel;
    const float* wc = w + static_cast<uint64_t>(c) * kernel;
    for (uint32_t i = 1; i < kernel; ++i) hc[i - 1] = hc[i];
    hc[kernel - 1] = in[c];
    double s = 0.0;
    for (uint32_t i = 0; i < kernel; ++i)
        s = __dadd_rn(s, __dmul_rn(static_cast<double>(hc[i]), static_cast<double>(wc[i])));
    const float v = __double2float_rn(s);
    out[c] = apply_silu ? ref_silu(v) : v;
}

// One CTA per head, thread per value index v (blockDim.x = value_dim <= 1024);
// recurrent state[head][key][value].  q and k hold qk_heads rows; head h reads
// row h % qk_heads, which is Oracle's repeat_heads_tiled (qwen35_block.cpp:225-243)
// applied before the step (qwen35_block.cpp:531-538).
__global__ void gated_delta_kernel(const float* __restrict__ q, const float* __restrict__ k,
                                   const float* __restrict__ v, const float* __restrict__ beta,
                                   const float* __restrict__ log_decay, float* state, uint32_t qk_heads,
                                   uint32_t key_dim, uint32_t value_dim, float eps, float* __restrict__ out) {
    extern __shared__ float gd_smem[];  // normalized q, normalized k
    __shared__ double scratch[32];
    float* nq = gd_smem;
    float* nk = gd_smem + key_dim;
    const uint32_t h = blockIdx.x, vi = threadIdx.x;
    const float* qh = q + static_cast<uint64_t>(h % qk_heads) * key_dim;
    const float* kh = k + static_cast<uint64_t>(h % qk_heads) * key_dim;
    double qs = 0.0, ks = 0.0;
    for (uint32_t d = threadIdx.x; d < key_dim; d += blockDim.x) {
        const double a = qh[d], b = kh[d];
        qs = __dadd_rn(qs, __dmul_rn(a, a));
        ks = __dadd_rn(ks, __dmul_rn(b, b));
    }
    const double q_norm = block_sum_f64(qs, scratch);
    const double k_norm = block_sum_f64(ks, scratch);
    const double e = static_cast<double>(eps);
    const float inv_q = __double2float_rn(__ddiv_rn(1.0, fmax(__dsqrt_rn(q_norm), e)));
    const float inv_k = __double2float_rn(__ddiv_rn(1.0, fmax(__dsqrt_rn(k_norm), e)));
    const float q_scale = __fdiv_rn(1.0f, __fsqrt_rn(static_cast<float>(key_dim)));
    for (uint32_t d = threadIdx.x; d < key_dim; d += blockDim.x) {
        nq[d] = __fmul_rn(__fmul_rn(qh[d], inv_q), q_scale);
        nk[d] = __fmul_rn(kh[d], inv_k);
    }
    __syncthreads();
    if (vi >= value_dim) return;
    const float decay = ref_expf(log_decay[h]);
    const float b = beta[h];
    float* sh = state + static_cast<uint64_t>(h) * key_dim * value_dim + vi;
    float mem = 0.0f;
    for (uint32_t d = 0; d < key_dim; ++d) {
        const float s = __fmul_rn(sh[static_cast<uint64_t>(d) * value_dim], decay);
        sh[static_cast<uint64_t>(d) * value_dim] = s;
        mem = __fadd_rn(mem, __fmul_rn(s, nk[d]));
    }
    const float delta = __fmul_rn(__fsub_rn(v[static_cast<uint64_t>(h) * value_dim + vi], mem), b);
    double o = 0.0;
    for (uint32_t d = 0; d < key_dim; ++d) {
        const float s = __fadd_rn(sh[static_cast<uint64_t>(d) * value_dim], __fmul_rn(nk[d], delta));
        sh[static_cast<uint64_t>(d) * value_dim] = s;
        o = __dadd_rn(o, __dmul_rn(static_cast<double>(s), static_cast<double>(nq[d])));
    }
    out[static_cast<uint64_t>(h) * value_dim + vi] = __double2float_rn(o);
}

__global__ void __launch_bounds__(256) swiglu_kernel(const float* __restrict__ gate, const float* __restrict__ up,
                                                     uint64_t n, float* __restrict__ out) {
    for (uint64_t i = blockIdx.x * uint64_t(blockDim.x) + threadIdx.x; i < n; i += uint64_t(gridDim.x) * blockDim.x)
        out[i] = __fmul_rn(ref_silu(gate[i]), up[i]);
}

__global__ void __launch_bounds__(256) add_kernel(const float* __restrict__ a, const float* __restrict__ b, uint64_t n,
                                                  float* __restrict__ out) {
    for (uint64_t i = blockIdx.x * uint64_t(blockDim.x) + threadIdx.x; i < n; i += uint64_t(gridDim.x) * blockDim.x)
        out[i] = __fadd_rn(a[i], b[i]);
}

}  // namespace oracle_cuda
