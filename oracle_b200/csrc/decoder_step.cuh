// decoder_step.cuh -- graph-replayable forms of the decode step's glue.
//
// A decode step captured once in a CUDA graph is replayed for every token, so
// nothing that changes per token may live in kernel parameters: the token
// position is a device counter (`pos`, advanced by step_advance_kernel at the
// end of a step), RoPE reads its cos/sin from a table of every position the
// host computed once by the reference's expressions, and the attention kernels
// read the cache length from `pos`.  Arithmetic is that of decoder_ops.cuh.
// A position at or past the cache capacity (or the RoPE table) is not
// processed: the kernels skip it and report kDevKvOverflow, which
// oracle_cuda_device_status returns as OVERFLOW, the class KvCache::append
// throws (hybrid_cache.cpp).
// The small elementwise kernels restate Oracle's block code
// (src/runtime/qwen35_block.cpp):
//   split_query_gate_kernel  joint query/gate projection -> query, gate (:676-688)
//   gate_sigmoid_mul_kernel  attention *= sigmoid(gate)                (:738-742)
//   gdn_gates_kernel         beta = sigmoid(beta), log_decay =
//                            softplus(alpha + time_step_bias) * decay  (:472-489)
//   mul_silu_kernel          gated *= silu(z)                          (:589-592)
#pragma once

#include "decoder_ops.cuh"

namespace oracle_cuda {

enum : unsigned int { kDevKvOverflow = 4 };

__device__ __forceinline__ void report_overflow(DeviceStatus* st, uint32_t pos) {
    if (st && atomicCAS(&st->code, kDevOk, kDevKvOverflow) == kDevOk) {
        st->where = pos;
        st->block = blockIdx.x;
    }
}

__device__ __forceinline__ float ref_softplus(float v) {
    // qwen35_block.cpp:147-155
    if (v > 20.0f) return v;
    if (v < -20.0f) return ref_expf(v);
    return ref_log1pf(ref_expf(v));
}

// One recurrent head's gates (qwen35_block.cpp:472-489), computed by a whole
// warp so that the library functions' table reads overlap: beta =
// sigmoid(beta_in), decay = exp(softplus(alpha + dt_bias) * a).  The first
// round evaluates, side by side, expf(-|beta_in|) (lane 0), expf(v) (lane 1)
// and log1pf at the three floats expf(v) can be -- its correctly rounded
// value and the two neighbours, since the library is within one float of it
// (lanes 2-4); the lane that guessed expf(v) supplies softplus.  The second
// round is the decay's expf.  Same values as ref_sigmoid / ref_softplus.
__device__ __forceinline__ void gdn_gates_warp(float beta_in, float alpha, float dt_bias, float a, uint32_t lane,
                                               float* gate_s) {
    const float v = __fadd_rn(alpha, dt_bias);
    const float ycr = __double2float_rn(exp(static_cast<double>(v)));
    const uint32_t nb = lane == 2 ? 0u : lane == 3 ? 1u : 0xFFFFFFFFu;
    const bool log = lane >= 2 && lane <= 4;
    const float arg = lane == 0 ? -fabsf(beta_in) : lane == 1 ? v : log ? __uint_as_float(__float_as_uint(ycr) + nb) : 0.0f;
    const float r = libm_eval(log, arg);
    const float e_beta = __shfl_sync(0xFFFFFFFFu, r, 0);
    const float y = __shfl_sync(0xFFFFFFFFu, r, 1);
    const uint32_t dy = __float_as_uint(y) - __float_as_uint(ycr);
    const float l1p = __shfl_sync(0xFFFFFFFFu, r, dy == 0u ? 2 : dy == 1u ? 3 : 4);
    const float s = v > 20.0f ? v : v < -20.0f ? y : l1p;
    const float decay = ref_expf(__fmul_rn(s, a));
    if (lane == 0) {
        gate_s[0] = beta_in >= 0.0f ? __fdiv_rn(1.0f, __fadd_rn(1.0f, e_beta)) : __fdiv_rn(e_beta, __fadd_rn(1.0f, e_beta));
        gate_s[1] = decay;
    }
}

__global__ void __launch_bounds__(256) rope_pos_kernel(float* __restrict__ heads, uint32_t n_heads, uint32_t head_dim,
                                                       uint32_t half, const float* __restrict__ table,
                                                       const uint32_t* __restrict__ pos, uint32_t positions,
                                                       DeviceStatus* st) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n_heads * half) return;
    if (*pos >= positions) {
        if (i == 0) report_overflow(st, *pos);
        return;
    }
    const uint32_t h = i / half, f = i % half;
    const float* row = table + (static_cast<uint64_t>(*pos) * half + f) * 2;
    float* base = heads + static_cast<uint64_t>(h) * head_dim;
    const float a = base[f], b = base[half + f], c = row[0], s = row[1];
    base[f] = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
    base[half + f] = __fadd_rn(__fmul_rn(b, c), __fmul_rn(a, s));
}

__global__ void __launch_bounds__(256) attention_append_pos_kernel(const float* __restrict__ k_new,
                                                                   const float* __restrict__ v_new, float* keys,
                                                                   float* values, const uint32_t* __restrict__ pos,
                                                                   uint32_t capacity, uint32_t nk, uint32_t nv,
                                                                   DeviceStatus* st) {
    const uint64_t length = *pos;
    if (length >= capacity) {
        if (blockIdx.x == 0 && threadIdx.x == 0) report_overflow(st, static_cast<uint32_t>(length));
        return;
    }
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < nk + nv; i += gridDim.x * blockDim.x) {
        if (i < nk)
            keys[length * nk + i] = k_new[i];
        else
            values[length * nv + (i - nk)] = v_new[i - nk];
    }
}

// grid (q_heads, chunks); warps of all chunks of a head stride over tokens.
__global__ void __launch_bounds__(256) attention_scores_pos_kernel(const float* __restrict__ q,
                                                                   const float* __restrict__ keys,
                                                                   const uint32_t* __restrict__ pos, uint32_t capacity,
                                                                   uint32_t q_heads, uint32_t kv_heads,
                                                                   uint32_t key_dim, float scale,
                                                                   float* __restrict__ scores) {
    pdl_enter();
    if (*pos >= capacity) return;
    const uint32_t tokens = *pos + 1;
    const uint32_t h = blockIdx.x, lane = threadIdx.x & 31;
    const uint32_t w = blockIdx.y * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const uint32_t nw = gridDim.y * (blockDim.x >> 5);
    const uint32_t kvh = h / (q_heads / kv_heads);
    const float* qh = q + static_cast<uint64_t>(h) * key_dim;
    // four of the warp's tokens at a time (their loads in flight together);
    // each token's sum is the lane sums in dimension order, then warp_sum_f64
    constexpr uint32_t kU = 4;
    for (uint32_t t0 = w; t0 < tokens; t0 += kU * nw) {
        double s[kU];
#pragma unroll
        for (uint32_t u = 0; u < kU; ++u) {
            const uint32_t t = t0 + u * nw;
            s[u] = 0.0;
            if (t < tokens) {
                const float* kt = keys + (static_cast<uint64_t>(t) * kv_heads + kvh) * key_dim;
                for (uint32_t d = lane; d < key_dim; d += 32)
                    s[u] = __dadd_rn(s[u], __dmul_rn(static_cast<double>(qh[d]), static_cast<double>(kt[d])));
            }
        }
#pragma unroll
        for (uint32_t u = 0; u < kU; ++u) s[u] = warp_sum_f64(s[u]);
        if (lane == 0) {
#pragma unroll
            for (uint32_t u = 0; u < kU; ++u) {
                const uint32_t t = t0 + u * nw;
                if (t < tokens)
                    scores[static_cast<uint64_t>(h) * capacity + t] = __fmul_rn(__double2float_rn(s[u]), scale);
            }
        }
    }
}

__global__ void __launch_bounds__(256) attention_output_pos_kernel(float* __restrict__ scores,
                                                                   const float* __restrict__ values,
                                                                   const uint32_t* __restrict__ pos, uint32_t capacity,
                                                                   uint32_t q_heads, uint32_t kv_heads,
                                                                   uint32_t value_dim, const float* __restrict__ gate,
                                                                   uint32_t gate_stride, float* __restrict__ out,
                                                                   DeviceStatus* st) {
    pdl_enter();
    __shared__ double scratch[32];
    __shared__ float fmax_s[32];
    if (*pos >= capacity) return;
    const uint32_t tokens = *pos + 1;
    const uint32_t h = blockIdx.x, kvh = h / (q_heads / kv_heads);
    float* sc = scores + static_cast<uint64_t>(h) * capacity;
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
        if (threadIdx.x == 0 && st) atomicCAS(&st->code, kDevOk, 3u);
        return;
    }
    for (uint32_t t = threadIdx.x; t < tokens; t += blockDim.x)
        sc[t] = __double2float_rn(__ddiv_rn(static_cast<double>(sc[t]), den));
    if (!values) return;  // the weighted sum is attention_values_pos_kernel's
    __syncthreads();
    for (uint32_t d = threadIdx.x; d < value_dim; d += blockDim.x) {
        const float* vp = values + static_cast<uint64_t>(kvh) * value_dim + d;
        const uint64_t stride = static_cast<uint64_t>(kv_heads) * value_dim;
        float acc = 0.0f;
        for (uint32_t t = 0; t < tokens; ++t) acc = __fadd_rn(acc, __fmul_rn(sc[t], __ldg(vp + t * stride)));
        // the output gate, attention *= sigmoid(gate) (qwen35_block.cpp:738-742)
        if (gate) acc = __fmul_rn(acc, ref_sigmoid(gate[static_cast<uint64_t>(h) * gate_stride + d]));
        out[static_cast<uint64_t>(h) * value_dim + d] = acc;
    }
}

// The weighted sum of the values for every query head of one KV head and a
// kAttnDims-wide slice of the value dimensions: grid (kv_heads, value_dim /
// kAttnDims), block (q_heads / kv_heads) * kAttnDims threads, thread (head hl,
// dim dl).  Each thread adds p[t] * v[t] in token order in f32 (the order of
// attention_output_pos_kernel's loop, bit for bit).  Chunks of kAttnChunk
// positions of the value slice and of the group's probabilities are staged
// in shared memory by asynchronous copies, two chunks in flight, so the
// dependent chain reads shared memory while the next chunk loads.
constexpr uint32_t kAttnDims = 16;
constexpr uint32_t kAttnChunk = 256;
__host__ __device__ constexpr uint32_t attn_values_smem_floats(uint32_t group) {
    return 2u * kAttnChunk * (kAttnDims + group);
}
__global__ void __launch_bounds__(1024) attention_values_pos_kernel(const float* __restrict__ probs,
                                                                    const float* __restrict__ values,
                                                                    const uint32_t* __restrict__ pos,
                                                                    uint32_t capacity, uint32_t q_heads,
                                                                    uint32_t kv_heads, uint32_t value_dim,
                                                                    const float* __restrict__ gate,
                                                                    uint32_t gate_stride, float* __restrict__ out) {
    pdl_enter();
    extern __shared__ __align__(16) float attn_smem[];
    if (*pos >= capacity) return;
    const uint32_t tokens = *pos + 1;
    const uint32_t group = q_heads / kv_heads;
    const uint32_t kvh = blockIdx.x, d0 = blockIdx.y * kAttnDims;
    const uint32_t hl = threadIdx.x / kAttnDims, dl = threadIdx.x % kAttnDims;
    const uint32_t h = kvh * group + hl;
    const uint32_t buf_floats = kAttnChunk * (kAttnDims + group);  // [kAttnChunk][kAttnDims], then [group][kAttnChunk]
    const uint64_t vstride = static_cast<uint64_t>(kv_heads) * value_dim;
    // probability rows may be copied 16 bytes at a time when every chunk start is
    // 16-byte aligned; the rounded-up tail stays inside the row (capacity % 4 == 0)
    const bool p16 = capacity % 4 == 0 && reinterpret_cast<uintptr_t>(probs) % 16 == 0;
    auto stage = [&](uint32_t c0, uint32_t b) {
        float* vs = attn_smem + b * buf_floats;
        float* ps = vs + kAttnChunk * kAttnDims;
        const uint32_t n = tokens - c0 < kAttnChunk ? tokens - c0 : kAttnChunk;
        for (uint32_t i = threadIdx.x; i < n * (kAttnDims / 4); i += blockDim.x) {
            const uint32_t t = i / (kAttnDims / 4), q4 = i % (kAttnDims / 4);
            async_copy16(vs + 4 * i, values + (c0 + t) * vstride + static_cast<uint64_t>(kvh) * value_dim + d0 + 4 * q4);
        }
        if (p16) {
            const uint32_t n4 = (n + 3) / 4;
            for (uint32_t i = threadIdx.x; i < group * n4; i += blockDim.x) {
                const uint32_t g = i / n4, t4 = i % n4;
                async_copy16(ps + g * kAttnChunk + 4 * t4,
                             probs + static_cast<uint64_t>(kvh * group + g) * capacity + c0 + 4 * t4);
            }
        } else {
            for (uint32_t i = threadIdx.x; i < group * n; i += blockDim.x) {
                const uint32_t g = i / n, t = i % n;
                async_copy4(ps + g * kAttnChunk + t, probs + static_cast<uint64_t>(kvh * group + g) * capacity + c0 + t);
            }
        }
        async_commit();
    };
    const uint32_t chunks = (tokens + kAttnChunk - 1) / kAttnChunk;
    stage(0, 0);
    // the output gate's sigmoid (qwen35_block.cpp:738-742) needs only the
    // projection: evaluated while the first chunk loads
    const uint32_t d = d0 + dl;
    const float sg = gate ? ref_sigmoid(gate[static_cast<uint64_t>(h) * gate_stride + d]) : 1.0f;
    float acc = 0.0f;
    for (uint32_t c = 0; c < chunks; ++c) {
        if (c + 1 < chunks) {
            stage((c + 1) * kAttnChunk, (c + 1) & 1u);
            async_wait<1>();
        } else {
            async_wait<0>();
        }
        __syncthreads();
        const float* vs = attn_smem + (c & 1u) * buf_floats;
        const float* pr = vs + kAttnChunk * kAttnDims + hl * kAttnChunk;
        const uint32_t c0 = c * kAttnChunk;
        const uint32_t n = tokens - c0 < kAttnChunk ? tokens - c0 : kAttnChunk;
#pragma unroll 8
        for (uint32_t t = 0; t < n; ++t) acc = __fadd_rn(acc, __fmul_rn(pr[t], vs[t * kAttnDims + dl]));
        __syncthreads();  // the buffer is refilled by the stage after next
    }
    // the output gate, attention *= sigmoid(gate)
    if (gate) acc = __fmul_rn(acc, sg);
    out[static_cast<uint64_t>(h) * value_dim + d] = acc;
}

__global__ void step_advance_kernel(uint32_t* pos) {
    if (threadIdx.x == 0 && blockIdx.x == 0) *pos += 1u;
}

// query_full [heads][2 * width] (query then gate per head) -> query, gate [heads][width]
__global__ void __launch_bounds__(256) split_query_gate_kernel(const float* __restrict__ full, uint32_t heads,
                                                               uint32_t width, float* __restrict__ query,
                                                               float* __restrict__ gate) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= heads * width) return;
    const uint32_t h = i / width, c = i % width;
    query[i] = full[static_cast<uint64_t>(h) * 2 * width + c];
    gate[i] = full[static_cast<uint64_t>(h) * 2 * width + width + c];
}

__global__ void __launch_bounds__(256) gate_sigmoid_mul_kernel(float* __restrict__ x, const float* __restrict__ gate,
                                                               uint32_t n) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) x[i] = __fmul_rn(x[i], ref_sigmoid(gate[i]));
}

__global__ void __launch_bounds__(256) gdn_gates_kernel(const float* __restrict__ beta_in,
                                                        const float* __restrict__ alpha,
                                                        const float* __restrict__ time_step_bias,
                                                        const float* __restrict__ decay, uint32_t heads,
                                                        float* __restrict__ beta_out,
                                                        float* __restrict__ log_decay) {
    const uint32_t h = blockIdx.x * blockDim.x + threadIdx.x;
    if (h >= heads) return;
    beta_out[h] = ref_sigmoid(beta_in[h]);
    log_decay[h] = __fmul_rn(ref_softplus(__fadd_rn(alpha[h], time_step_bias[h])), decay[h]);
}

__global__ void __launch_bounds__(256) mul_silu_kernel(float* __restrict__ x, const float* __restrict__ z, uint32_t n) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) x[i] = __fmul_rn(x[i], ref_silu(z[i]));
}

// ---------------------------------------------------------------- fused block cores
//
// A Gated DeltaNet block between its input projections and its output
// projection, as ONE kernel: Oracle's recurrent block (qwen35_block.cpp:
// 472-592) from the projected qkv / z / beta / alpha to the gated vector the
// output projection reads.  One CTA per value head, key_dim == value_dim ==
// kD, 4 * kD threads:
//   conv       the depthwise causal conv + SiLU of the head's q, k (key head
//              h % key_heads, repeat_heads_tiled) and v channels, one channel
//              per thread; the history is double-buffered by position parity
//              (read slot pos & 1, write the other), so the CTAs that share a
//              key head read a history nobody writes during the step; the CTA
//              h < key_heads writes the shared q / k channels
//   gates      beta = sigmoid(beta), log_decay = softplus(alpha + dt_bias) * a
//   delta      gated_delta_step (reference_kernels.cpp:221-335) on the head's
//              [key][value] state: thread (t, part) keeps rows part * kD/4 ..
//              of state column t in registers; the two sums over the key
//              index (the f32 memory read-out and the f64 output) are one
//              chain from key row 0 to kD - 1 each, the reference's order
//              (the column's four threads add their quarters in turn), so the
//              block matches gated_delta_kernel bit for bit
//   out        rms_norm_rows over the head's row, then * silu(z)
// A batched decode runs its sequences as grid rows (blockIdx.y), each on its
// own stacked buffers (the history [2][channels][conv_kernel] per sequence).
template <int kD>
__global__ void __launch_bounds__(4 * kD) gdn_core_kernel(const float* __restrict__ qkv, const float* __restrict__ z,
                                                          const float* __restrict__ beta_in,
                                                          const float* __restrict__ alpha,
                                                          const float* __restrict__ dt_bias,
                                                          const float* __restrict__ decay_a,
                                                          const float* __restrict__ conv_w, float* hist, float* state,
                                                          const float* __restrict__ norm_w, uint32_t key_heads,
                                                          uint32_t value_heads, uint32_t conv_kernel, float eps,
                                                          const uint32_t* __restrict__ pos, float* __restrict__ out) {
    constexpr int kQ = kD / 4;  // key rows per thread
    pdl_launch_dependents();
    {
        // blockIdx.y: the sequence of a batched decode, with its own inputs,
        // history, state and output stacked after the previous sequence's
        const uint64_t seq = blockIdx.y;
        const uint64_t ch = 2ull * key_heads * kD + uint64_t(value_heads) * kD;
        qkv += seq * ch;
        z += seq * value_heads * kD;
        beta_in += seq * value_heads;
        alpha += seq * value_heads;
        hist += seq * 2 * ch * conv_kernel;
        state += seq * value_heads * kD * kD;
        out += seq * value_heads * kD;
    }
    __shared__ float q_s[kD], k_s[kD], v_s[kD], nq[kD], nk[kD], o_s[kD];
    __shared__ double scratch[64];
    __shared__ float gate_s[2];
    __shared__ float zs_s[kD];  // silu(z) of the head
    const uint32_t h = blockIdx.x, tid = threadIdx.x;
    const uint32_t t = tid >> 2, part = tid & 3u;  // state column, quarter of the key rows
    // the state rows of this thread, loaded up front: only this block's own
    // earlier steps write the state, so the loads may overlap the tail of the
    // preceding kernel (programmatic launch)
    float* sh = state + static_cast<uint64_t>(h) * kD * kD + static_cast<uint64_t>(part) * kQ * kD + t;
    float col[kQ];
#pragma unroll
    for (int j = 0; j < kQ; ++j) col[j] = sh[j * kD];
    const uint32_t kh = h % key_heads;
    const uint32_t key_width = key_heads * kD;
    const uint32_t channels = 2 * key_width + value_heads * kD;
    const uint32_t K = conv_kernel;
    // the position, the conv weights and the history this step reads are
    // written by no kernel of this step (the history slot by this layer's core
    // one step earlier), so they load with the state, before the wait
    const uint32_t slot = *pos & 1u;
    const float* hin = hist + static_cast<uint64_t>(slot) * channels * K;
    float* hout = hist + static_cast<uint64_t>(slot ^ 1u) * channels * K;
    const uint32_t which = tid / kD, ci = tid % kD;  // 0: q, 1: k, 2: v
    const uint32_t c = which == 0 ? kh * kD + ci : which == 1 ? key_width + kh * kD + ci : 2 * key_width + h * kD + ci;
    constexpr uint32_t kMaxK = 8;
    float hv[kMaxK], wv[kMaxK];
    const bool conv = tid < 3 * kD && K <= kMaxK;
    if (conv) {
#pragma unroll
        for (uint32_t j = 0; j < kMaxK; ++j) {
            if (j < K) {
                hv[j] = j + 1 < K ? hin[static_cast<uint64_t>(c) * K + j + 1] : 0.0f;
                wv[j] = conv_w[static_cast<uint64_t>(c) * K + j];
            }
        }
    }
    pdl_wait();
    if (tid < 3 * kD) {
        const bool write = which == 2 || h < key_heads;
        const float* hc = hin + static_cast<uint64_t>(c) * K;
        const float* wc = conv_w + static_cast<uint64_t>(c) * K;
        float* oc = hout + static_cast<uint64_t>(c) * K;
        double sum = 0.0;
        if (conv) {
#pragma unroll
            for (uint32_t j = 0; j < kMaxK; ++j) {
                if (j < K) {
                    const float v = j + 1 < K ? hv[j] : qkv[c];
                    if (write) oc[j] = v;
                    sum = __dadd_rn(sum, __dmul_rn(static_cast<double>(v), static_cast<double>(wv[j])));
                }
            }
        } else {
            for (uint32_t j = 0; j < K; ++j) {
                const float v = j + 1 < K ? hc[j + 1] : qkv[c];
                if (write) oc[j] = v;
                sum = __dadd_rn(sum, __dmul_rn(static_cast<double>(v), static_cast<double>(wc[j])));
            }
        }
        const float r = ref_silu(__double2float_rn(sum));
        (which == 0 ? q_s : which == 1 ? k_s : v_s)[ci] = r;
    } else {
        // the threads the conv leaves idle: one warp computes the gates, the
        // others silu(z) of the head, which only the last phase needs
        const uint32_t u = tid - 3 * kD;
        if (u < 32) {
            gdn_gates_warp(beta_in[h], alpha[h], dt_bias[h], decay_a[h], u, gate_s);
        } else {
            for (uint32_t i = u - 32; i < kD; i += kD - 32) zs_s[i] = ref_silu(z[static_cast<uint64_t>(h) * kD + i]);
        }
    }
    __syncthreads();
    // gated_delta_step: l2-normalised q (scaled by 1/sqrt(key_dim)) and k
    const double qv = tid < kD ? static_cast<double>(q_s[tid]) : 0.0;
    const double kv = tid < kD ? static_cast<double>(k_s[tid]) : 0.0;
    // both sums in one block reduction (each in block_sum_f64's order)
    double q_norm, k_norm;
    block_sum2_f64(__dmul_rn(qv, qv), __dmul_rn(kv, kv), scratch, q_norm, k_norm);
    if (tid < kD) {
        const double e = static_cast<double>(eps);
        const float inv_q = __double2float_rn(__ddiv_rn(1.0, fmax(__dsqrt_rn(q_norm), e)));
        const float inv_k = __double2float_rn(__ddiv_rn(1.0, fmax(__dsqrt_rn(k_norm), e)));
        const float q_scale = __fdiv_rn(1.0f, __fsqrt_rn(static_cast<float>(kD)));
        nq[tid] = __fmul_rn(__fmul_rn(q_s[tid], inv_q), q_scale);
        nk[tid] = __fmul_rn(k_s[tid], inv_k);
    }
    __syncthreads();
    const float b = gate_s[0], decay = gate_s[1];
    const float* nkp = nk + part * kQ;
    const float* nqp = nq + part * kQ;
    // Both sums over the key rows run in gated_delta_step's order, one chain
    // from row 0 to row kD - 1: the four threads of column t (adjacent lanes)
    // add their quarters in turn, handing the running sum on by shuffle.
    const uint32_t lane = tid & 31u, group = lane & ~3u;
#pragma unroll
    for (int j = 0; j < kQ; ++j) col[j] = __fmul_rn(col[j], decay);
    float mem = 0.0f;
#pragma unroll
    for (uint32_t p = 0; p < 4; ++p) {
        if (part == p) {
#pragma unroll
            for (int j = 0; j < kQ; ++j) mem = __fadd_rn(mem, __fmul_rn(col[j], nkp[j]));
        }
        mem = __shfl_sync(0xFFFFFFFFu, mem, group | p);
    }
    const float delta = __fmul_rn(__fsub_rn(v_s[t], mem), b);
#pragma unroll
    for (int j = 0; j < kQ; ++j) col[j] = __fadd_rn(col[j], __fmul_rn(nkp[j], delta));
    double o = 0.0;
#pragma unroll
    for (uint32_t p = 0; p < 4; ++p) {
        if (part == p) {
#pragma unroll
            for (int j = 0; j < kQ; ++j)
                o = __dadd_rn(o, __dmul_rn(static_cast<double>(col[j]), static_cast<double>(nqp[j])));
        }
        o = __shfl_sync(0xFFFFFFFFu, o, group | p);
    }
#pragma unroll
    for (int j = 0; j < kQ; ++j) sh[j * kD] = col[j];
    if (part == 0) o_s[t] = __double2float_rn(o);
    __syncthreads();
    // rms_norm_rows over the head's row, then gated *= silu(z)
    const float of = tid < kD ? o_s[tid] : 0.0f;
    const float inv = rms_inverse(block_sum_f64(__dmul_rn(static_cast<double>(of), static_cast<double>(of)), scratch),
                                  kD, eps);
    if (tid < kD) {
        const float g = __fmul_rn(__fmul_rn(of, inv), norm_w[tid]);
        out[static_cast<uint64_t>(h) * kD + tid] = __fmul_rn(g, zs_s[tid]);
    }
}

// The gated attention block up to its softmax, as one kernel per query head
// (thread t = dimension, blockDim.x = head_dim): the query half of the joint
// query/gate projection (qwen35_block.cpp:676-688), its per-head RMSNorm
// (:693-700) and RoPE at *pos; the CTA h = group * kv_head also normalises
// and rotates that KV head's key and appends key and value to the cache at
// *pos (KvCache::append).  Position-table overflow: kDevKvOverflow.
__global__ void attention_prep_kernel(const float* __restrict__ q_full, const float* __restrict__ k_proj,
                                      const float* __restrict__ v_proj, const float* __restrict__ q_norm,
                                      const float* __restrict__ k_norm, float eps, const float* __restrict__ table,
                                      uint32_t half, uint32_t q_heads, uint32_t kv_heads, float* keys, float* values,
                                      uint32_t capacity, const uint32_t* __restrict__ pos, float* __restrict__ q_out,
                                      DeviceStatus* st) {
    pdl_enter();
    __shared__ double scratch[32];
    __shared__ float row[1024];
    const uint32_t D = blockDim.x, h = blockIdx.x, t = threadIdx.x;
    const uint32_t p = *pos;
    if (p >= capacity) {
        if (h == 0 && t == 0) report_overflow(st, p);
        return;
    }
    const float* rope = table + static_cast<uint64_t>(p) * half * 2;
    auto norm_rope = [&](float x, const float* w) -> float {
        const float inv = rms_inverse(block_sum_f64(__dmul_rn(static_cast<double>(x), static_cast<double>(x)), scratch),
                                      D, eps);
        row[t] = __fmul_rn(__fmul_rn(x, inv), w[t]);
        __syncthreads();
        float r = row[t];
        if (t < half) {
            const float a = row[t], b = row[t + half], c = rope[2 * t], s = rope[2 * t + 1];
            r = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
        } else if (t < 2 * half) {
            const uint32_t f = t - half;
            const float a = row[f], b = row[t], c = rope[2 * f], s = rope[2 * f + 1];
            r = __fadd_rn(__fmul_rn(b, c), __fmul_rn(a, s));
        }
        __syncthreads();
        return r;
    };
    q_out[static_cast<uint64_t>(h) * D + t] = norm_rope(q_full[static_cast<uint64_t>(h) * 2 * D + t], q_norm);
    const uint32_t group = q_heads / kv_heads;
    if (h % group == 0) {
        const uint32_t kvh = h / group;
        const float kr = norm_rope(k_proj[static_cast<uint64_t>(kvh) * D + t], k_norm);
        const uint64_t at = (static_cast<uint64_t>(p) * kv_heads + kvh) * D + t;
        keys[at] = kr;
        values[at] = v_proj[static_cast<uint64_t>(kvh) * D + t];
    }
}

}  // namespace oracle_cuda
