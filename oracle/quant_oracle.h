/*
 * quant_oracle.h -- CPU restatement of Oracle's quantized-weight path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity checker for the CUDA
 * path in oracle_b200/.  Only tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline / --impl reference legs may load it.  The product library
 * (liboracle_cuda.so) never links, loads or calls it.
 *
 * Provenance of each function (paths relative to the Oracle repository):
 *   - f16/bf16 conversion, Q8_0 / Q5_K / Q6_K block decode, row validation:
 *     src/model/storage_decode.cpp:44-176, :182-198, :244-294 (restated, not
 *     copied; pinned bit-for-bit against the reference's own compiled code by
 *     tests/test_oracle_pin.py).
 *   - Q4_K block decode: Oracle has no Q4_K decoder (storage_decode.cpp:192-196
 *     rejects type 12).  It is Oracle's Q5_K decode (storage_decode.cpp:63-94)
 *     with the 32-byte high-bit plane removed and qs moved from offset 48 to
 *     offset 16, i.e. the GGML block_q4_K layout {f16 d, f16 dmin, u8
 *     scales[12], u8 qs[128]}.  Pinned against gguf-py 0.19.0
 *     Q4_K.dequantize_blocks via tests/golden/.
 *   - Row geometry: src/model/ggml_type.cpp:12-56 (table), :77-94 (row bytes).
 *   - f32-activation dot / matvec (Oracle's contract): a sequential f32 sum,
 *     src/backend/cpu/quantized_reference.cpp:24-82 and :128-162.
 *   - Q8_K quantizer and the Q4_K x Q8_K / Q6_K x Q8_K integer dots: not in
 *     Oracle (only the q8_K layout is registered, ggml_type.cpp:28).  They
 *     restate GGML's published algorithm (ggml/src/ggml-quants.c,
 *     quantize_row_q8_K_ref and ggml_vec_dot_q{4,6}_K_q8_K_generic, at the
 *     commit Oracle's docs pin, a620cbd481d16d3ccb5c8c96fa2fbd70191bea38).
 *     GGML itself is not vendored, so byte parity of these two against GGML
 *     is UNPINNED; the integer super-block sums are exact integers and the
 *     f32 combination order across super-blocks is this build's documented
 *     contract (oq_vec_dot_q8_k below).
 */
#ifndef ORACLE_QUANT_ORACLE_H
#define ORACLE_QUANT_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
    OQ_TYPE_F32 = 0,
    OQ_TYPE_F16 = 1,
    OQ_TYPE_Q8_0 = 8,
    OQ_TYPE_Q4_K = 12,
    OQ_TYPE_Q5_K = 13,
    OQ_TYPE_Q6_K = 14,
    OQ_TYPE_Q8_K = 15,
    OQ_TYPE_BF16 = 30
};

enum { OQ_QK_K = 256, OQ_Q8_K_BLOCK_BYTES = 292 };

/* Status codes: 0 ok, 1 invalid argument, 2 unsupported type. */
enum { OQ_OK = 0, OQ_EINVAL = 1, OQ_EUNSUPPORTED = 2 };

float oq_f16_to_f32(uint16_t bits);
float oq_bf16_to_f32(uint16_t bits);
uint16_t oq_f32_to_bf16_rne(float value);

/* Bytes of one row of `k` elements, or 0 when the type is unknown or k is not
 * a whole number of blocks (ggml_type.cpp:77-94). */
uint64_t oq_row_bytes(uint32_t type, uint64_t k);

/* Decode one row to f32 (decode_storage_row, storage_decode.cpp:244-294).
 * Types: f32, f16, bf16, q8_0, q4_K, q5_K, q6_K. */
int oq_decode_row(uint32_t type, uint64_t k, const uint8_t* row, float* out);

/* Q8_K: per 256 elements {f32 d; i8 qs[256]; i16 bsums[16]} = 292 bytes. */
int oq_quantize_row_q8_k(const float* x, uint64_t k, uint8_t* q8k);

/* Exact integer super-block sums against one Q8_K block.
 * Q4_K: *isum = sum_j sc_j * sum_{32} q4*q8, *msum = sum_j m_j * (bsum_2j + bsum_2j+1).
 * Q6_K: *isum = sum_s sc_s * (sum_{16} q6*q8 - 32*bsum_s), *msum = 0. */
void oq_block_sums_q4_k(const uint8_t* wblock, const uint8_t* q8block, int32_t* isum,
                        int32_t* msum);
void oq_block_sums_q6_k(const uint8_t* wblock, const uint8_t* q8block, int32_t* isum,
                        int32_t* msum);

/* Row dot against Q8_K activations in this build's canonical f32 order:
 *   p_i   = (d_w * d_x) * (float)isum_i - (dmin_w * d_x) * (float)msum_i
 *   per 16-super-block segment g: leaf[j] = 0.0f + p_{16g+j} (+0.0f past the
 *   row's end); for stride in 8, 4, 2, 1: leaf[s] += leaf[s + stride] for
 *   s < stride; seg_g = leaf[0]
 *   total = ((0.0f + seg_0) + seg_1) + ...   (increasing g)
 * A fixed tree inside a segment (lanes of a warp, or the super-blocks of a
 * stage), a running sum across segments (stages streamed in order).
 * Types: q4_K, q6_K. */
float oq_vec_dot_q8_k(uint32_t type, uint64_t k, const uint8_t* wrow, const uint8_t* q8row);

/* The same dot in GGML's generic summation order (8 partial f32 sums per
 * super-block lane group), for the tolerance cross-check only. */
float oq_vec_dot_q8_k_ggml_order(uint32_t type, uint64_t k, const uint8_t* wrow,
                                 const uint8_t* q8row);

/* y[b*rows + r] = dot(row r, q8k of activation b).  q8k holds batch rows of
 * (k/256) Q8_K blocks each. */
int oq_matvec_q8_k(uint32_t type, uint64_t rows, uint64_t k, const uint8_t* w,
                   const uint8_t* q8k, uint64_t batch, float* y);

/* Oracle's f32 contract: decode each block to f32, then `sum += w * x`
 * sequentially over the whole row (quantized_reference.cpp:24-82).  Compiled
 * with -ffp-contract=off so no multiply-add is fused. */
float oq_storage_dot_f32(uint32_t type, uint64_t k, const uint8_t* row, const float* x);
int oq_storage_matvec_f32(uint32_t type, uint64_t rows, uint64_t k, const uint8_t* w,
                          const float* x, uint64_t batch, float* y);

/* Arbiter: decoded f32 weights times f32 x, products and sum in double. */
int oq_storage_matvec_f64(uint32_t type, uint64_t rows, uint64_t k, const uint8_t* w,
                          const float* x, uint64_t batch, double* y);

/* Prefill GEMM references, Y[m][n] = sum_k X[m][k] * W[n][k], evaluated only
 * at the `count` sampled (m, n) pairs.  f64 accumulation throughout.
 *   mode 0: f32 operands (X as given, W = Oracle's f32 decode);
 *   mode 1: both operands rounded to bf16 (round-to-nearest-even) first;
 *   mode 2: sum of |products| of the mode-1 operands (error scale);
 *   mode 3: sum of |products| of the mode-0 operands. */
int oq_gemm_sampled(uint32_t type, uint64_t n, uint64_t k, const uint8_t* w, uint64_t m,
                    const float* x, uint64_t count, const uint64_t* m_index,
                    const uint64_t* n_index, int mode, double* y);

/* Decoder glue restated from Oracle's block code (anonymous-namespace
 * helpers of src/runtime/qwen35_block.cpp, not linkable):
 *   rms_norm_rows (:161-188): per row, sum of squares in double, inverse RMS
 *   as float(1 / sqrt(mean + eps)), out = (x * inv) * w in float;
 *   swiglu (:138-159, :315-318): silu(gate) * up with the two-branch sigmoid. */
int oq_rms_norm_rows(const float* in, const float* weight, uint64_t rows, uint64_t width, float eps, float* out);
void oq_swiglu(const float* gate, const float* up, uint64_t n, float* out);

#ifdef __cplusplus
}
#endif

#endif
