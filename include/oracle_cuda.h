/*
 * oracle_cuda.h -- C ABI of the B200 (sm_100a) quantized-weight path.
 *
 * This library replaces Oracle's stubbed CUDA hook
 * (src/backend/cuda/cuda_backend.cu:1-4, built under ORACLE_ENABLE_CUDA,
 * CMakeLists.txt:53-58) for the path Oracle runs through the free functions in
 * include/oracle/backend/cpu/quantized_reference.hpp:12-27 and
 * include/oracle/model/storage_decode.hpp:38-41.  Paths below are relative to
 * the Oracle repository.
 *
 * Conventions
 *   - Plain pointers and sizes only.  "Device" pointers address GPU memory of
 *     the context's device; "host" pointers address CPU memory.
 *   - Matrices are GGML row-major: `rows` rows of `cols` elements, each row
 *     ggml_row_byte_size(cols, type) bytes (GGUF dims[0] = cols, dims[1] =
 *     rows, quantized_reference.cpp:118-119).
 *   - Activations x are `batch` contiguous f32 vectors of `cols` elements;
 *     outputs y are `batch` contiguous f32 vectors of `rows` elements.
 *   - Device-pointer calls are asynchronous on `stream` (a cudaStream_t; NULL
 *     is the legacy default stream).  Host-pointer calls are synchronous, like
 *     the reference.
 *   - Every call validates its arguments on the host first, in the order the
 *     reference does, and returns the status class of the C++ exception the
 *     reference would throw; oracle_cuda_last_error() gives the message, which
 *     repeats the reference's text.  Nothing is launched when validation fails.
 *   - One context per device; calls on one context come from one host thread.
 *
 * Two arithmetic contracts
 *   ORACLE_CUDA_CONTRACT_F32  Oracle's own: weights decoded to f32 exactly as
 *                             Oracle decodes them, products added into one
 *                             running f32 sum in element order
 *                             (quantized_reference.cpp:24-82): results are
 *                             bit-identical to the reference.  Types f32,
 *                             f16, bf16, q8_0, q4_K, q5_K, q6_K.
 *   ORACLE_CUDA_CONTRACT_Q8K  GGML's integer contract: x quantized to Q8_K
 *                             (f32 d, int8 qs[256], int16 bsums[16]), exact
 *                             integer super-block dots, f32 combination in a
 *                             fixed documented order.  Types q4_K, q6_K.
 */
#ifndef ORACLE_CUDA_H
#define ORACLE_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ORACLE_CUDA_ABI_VERSION 1

/* Status codes.  1..5 name the C++ exception class the reference throws for the
 * same input, so a C++ adapter can rethrow the same type. */
typedef enum oracle_cuda_status {
    ORACLE_CUDA_OK = 0,
    ORACLE_CUDA_INVALID_ARGUMENT = 1, /* std::invalid_argument */
    ORACLE_CUDA_OUT_OF_RANGE = 2,     /* std::out_of_range */
    ORACLE_CUDA_OVERFLOW = 3,         /* std::overflow_error */
    ORACLE_CUDA_RUNTIME_ERROR = 4,    /* std::runtime_error */
    ORACLE_CUDA_LOGIC_ERROR = 5,      /* std::logic_error */
    ORACLE_CUDA_CUDA_ERROR = 6,       /* a CUDA runtime call failed */
    ORACLE_CUDA_OUT_OF_MEMORY = 7,    /* device or pinned allocation failed */
    ORACLE_CUDA_DEVICE_TIMEOUT = 8,   /* a kernel wait hit its deadline and returned early */
    ORACLE_CUDA_UNSUPPORTED = 9       /* valid input this path does not implement */
} oracle_cuda_status;

typedef enum oracle_cuda_contract {
    ORACLE_CUDA_CONTRACT_F32 = 0,
    ORACLE_CUDA_CONTRACT_Q8K = 1
} oracle_cuda_contract;

typedef struct oracle_cuda_context oracle_cuda_context;
typedef struct oracle_cuda_weight oracle_cuda_weight;

/* ------------------------------------------------------------------ library */

int oracle_cuda_abi_version(void);
const char* oracle_cuda_status_name(oracle_cuda_status status);

/* Message of the last failed call on `ctx` (or of the calling thread when ctx
 * is NULL, e.g. after a failed create).  Valid until the next call. */
const char* oracle_cuda_last_error(const oracle_cuda_context* ctx);

/* ------------------------------------------------------------------ layout
 * Host-only; no GPU needed.  Replaces ggml_type_layout / ggml_row_byte_size
 * (include/oracle/model/ggml_type.hpp:17-19, src/model/ggml_type.cpp:69-94). */

/* OK and the layout of a registered type; INVALID_ARGUMENT for an unknown or
 * removed id (the reference returns nullptr). `name` may be NULL. */
oracle_cuda_status oracle_ggml_type_layout(uint32_t type, uint64_t* block_elements,
                                           uint64_t* bytes_per_block, int* quantized,
                                           const char** name);

/* ggml_row_byte_size: RUNTIME_ERROR for an unknown type or a ragged row,
 * INVALID_ARGUMENT for zero elements, OVERFLOW on overflow. */
oracle_cuda_status oracle_ggml_row_byte_size(uint64_t row_elements, uint32_t type,
                                             uint64_t* out);

/* ------------------------------------------------------------------ context */

/* Create a context on CUDA device `device`: sets the device current, reads its
 * SM count, allocates the device status word and pinned staging.  Replaces the
 * reference's backend selection by name (src/runtime/engine.cpp:64-70). */
oracle_cuda_status oracle_cuda_create(int device, oracle_cuda_context** out);
oracle_cuda_status oracle_cuda_destroy(oracle_cuda_context* ctx);

/* Context options (bit flags).  ORACLE_CUDA_FLAG_PDL launches the matvec
 * kernels with programmatic dependent launch: a kernel may start streaming its
 * weights before the preceding kernel in the stream finishes, and waits for it
 * only before reading activations.  Only safe when the preceding kernel does
 * not write the weight bytes. */
#define ORACLE_CUDA_FLAG_PDL 1u
/* ORACLE_CUDA_FLAG_BUILD_IN_KERNEL: matvec programs quantize the activations
 * of their first ops inside the program kernel (every CTA its own copy)
 * instead of a separate quantizer launch before it: one launch fewer per
 * program, for chains of short programs (a decode step).  Programs whose
 * fed-in images would not fit in shared memory keep the quantizer launch. */
#define ORACLE_CUDA_FLAG_BUILD_IN_KERNEL 2u
oracle_cuda_status oracle_cuda_set_flags(oracle_cuda_context* ctx, uint32_t flags);

/* Device status word written by kernels whose bounded waits expired.  Reads it
 * (synchronising the device), clears it, and returns OK or DEVICE_TIMEOUT. */
oracle_cuda_status oracle_cuda_device_status(oracle_cuda_context* ctx);

/* Failure-detection self-test: launches one kernel whose only thread waits
 * on a barrier that never completes, with a deadline of `limit_ns`.  The wait
 * gives up, records a timeout in the device status word and the kernel ends;
 * the context stays usable.  The next oracle_cuda_device_status() returns
 * DEVICE_TIMEOUT. */
oracle_cuda_status oracle_cuda_selftest_bounded_wait(oracle_cuda_context* ctx, uint64_t limit_ns);

/* Number of kernels this context has launched (for launch accounting). */
uint64_t oracle_cuda_launch_count(const oracle_cuda_context* ctx);

/* ------------------------------------------------------------------ device-pointer path */

/* decode_storage_row / reference_decode_mapped_tensor
 * (storage_decode.cpp:244-294, quantized_reference.cpp:85-105): decode `rows`
 * rows to f32, out_len == rows * cols. */
oracle_cuda_status oracle_cuda_decode_rows(oracle_cuda_context* ctx, uint32_t type, uint64_t rows,
                                           uint64_t cols, const void* w_dev, uint64_t w_nbytes,
                                           float* out_dev, uint64_t out_len, void* stream);

/* Q8_K activation quantizer: `batch` vectors of `cols` floats (cols % 256 == 0)
 * into batch * (cols / 256) GGML block_q8_K records of 292 bytes.  No Oracle
 * counterpart (only the layout is registered, ggml_type.cpp:28). */
oracle_cuda_status oracle_cuda_quantize_q8_k(oracle_cuda_context* ctx, const float* x_dev,
                                             uint64_t cols, uint64_t batch, void* q8k_dev,
                                             uint64_t q8k_nbytes, void* stream);

/* reference_storage_matvec (quantized_reference.cpp:128-162) on device
 * buffers, for `batch` activation vectors: x_len == batch * cols, y_len ==
 * batch * rows.  With CONTRACT_Q8K the activations are quantized to Q8_K
 * inside the kernel (no intermediate buffer). */
oracle_cuda_status oracle_cuda_storage_matvec(oracle_cuda_context* ctx, int contract, uint32_t type,
                                              uint64_t rows, uint64_t cols, const void* w_dev,
                                              uint64_t w_nbytes, const float* x_dev, uint64_t x_len,
                                              float* y_dev, uint64_t y_len, void* stream);

/* Q8_K contract with activations already quantized by oracle_cuda_quantize_q8_k
 * (q8k_nbytes == batch * cols / 256 * 292). */
oracle_cuda_status oracle_cuda_matvec_q8k_prequantized(oracle_cuda_context* ctx, uint32_t type,
                                                       uint64_t rows, uint64_t cols,
                                                       const void* w_dev, uint64_t w_nbytes,
                                                       const void* q8k_dev, uint64_t q8k_nbytes,
                                                       float* y_dev, uint64_t y_len, void* stream);

/* Batched decode: the Q8_K matvec of up to 16 activation vectors in one pass
 * over the weights (each weight byte read once, not once per vector).  Two
 * steps, so that one quantization serves every matrix that reads the same
 * activations (a block's q / k / v, gate / up):
 *   oracle_cuda_batch_quantize  x[batch][cols] (batch 1..16, cols a multiple
 *       of 256) -> a batch image of oracle_cuda_batch_image_bytes(cols) bytes
 *       (16-byte aligned device buffer): GGML's quantize_row_q8_K per vector,
 *       laid out for the tensor-core kernel;
 *   oracle_cuda_batch_matvec    y[b][r] = the Q8_K-contract dot of weight row r
 *       (q4_K / q6_K, 16-byte aligned) with vector b of the image, for
 *       b < batch; y_len == batch * rows.  Bit-identical, vector by vector, to
 *       oracle_cuda_storage_matvec with CONTRACT_Q8K.
 * These replace a loop of reference_storage_matvec calls over the batch
 * (quantized_reference.cpp:128-162), which reads the weights once per vector.
 * oracle_cuda_storage_matvec with CONTRACT_Q8K and 2..16 vectors takes the
 * same path internally. */
uint64_t oracle_cuda_batch_image_bytes(uint64_t cols);
oracle_cuda_status oracle_cuda_batch_quantize(oracle_cuda_context* ctx, const float* x_dev, uint64_t cols,
                                              uint32_t batch, void* image_dev, uint64_t image_nbytes, void* stream);
oracle_cuda_status oracle_cuda_batch_matvec(oracle_cuda_context* ctx, uint32_t type, uint64_t rows, uint64_t cols,
                                            const void* w_dev, uint64_t w_nbytes, const void* image_dev,
                                            uint64_t image_nbytes, uint32_t batch, float* y_dev, uint64_t y_len,
                                            void* stream);
/* The residual add and RMSNorm before a projection, fused into its
 * quantization (arguments and checks as oracle_cuda_batch_quantize): s = a + b
 * (b may be NULL: s = a), written to sum_dev when it is not NULL (the
 * residual stream; not one of the inputs), then rms_norm_rows of s with
 * weight_dev / eps (src/runtime/qwen35_block.cpp:161-188, 190-200; the same
 * double sum as oracle_cuda_rms_norm_rows) quantized into the batch image;
 * cols at most 8192.  The same image as oracle_cuda_add,
 * oracle_cuda_rms_norm_rows and oracle_cuda_batch_quantize in one launch
 * instead of three. */
oracle_cuda_status oracle_cuda_batch_norm_quantize(oracle_cuda_context* ctx, const float* a_dev, const float* b_dev,
                                                   float* sum_dev, const float* weight_dev, float eps, uint64_t cols,
                                                   uint32_t batch, void* image_dev, uint64_t image_nbytes,
                                                   void* stream);

/* Matvec program: up to ORACLE_CUDA_PROGRAM_MAX_OPS Q8_K-contract matvecs
 * (q4_K / q6_K weights) in ONE persistent launch.  The weights of all ops
 * stream through one shared-memory ring without pausing at op boundaries;
 * each op quantizes its f32 activation in-kernel, exactly like
 * oracle_cuda_storage_matvec (bit-identical results).  An op with
 * after_previous = 1 reads an activation written by an earlier op of the same
 * call: it waits, on the device, for every CTA to finish all earlier ops
 * (bounded; a timeout is reported by oracle_cuda_device_status).  Ops without
 * it must not read what an earlier op of the call writes.  Programs launched
 * from one context must not run concurrently with each other (they share the
 * completion counters).  No Oracle counterpart: Oracle runs each projection
 * as its own call (src/runtime/qwen35_block.cpp:108-119). */
#define ORACLE_CUDA_PROGRAM_MAX_OPS 16
typedef struct oracle_cuda_matvec_op {
    uint32_t type;           /* 12 (q4_K) or 14 (q6_K) */
    uint32_t after_previous; /* 1: x is produced by an earlier op of this call */
    uint64_t rows;
    uint64_t cols;
    const void* w_dev;
    uint64_t w_nbytes;
    const float* x_dev;      /* cols floats */
    float* y_dev;            /* rows floats */
} oracle_cuda_matvec_op;

oracle_cuda_status oracle_cuda_matvec_program(oracle_cuda_context* ctx, const oracle_cuda_matvec_op* ops,
                                              uint32_t n_ops, void* stream);

/* Matvec program with activation transforms and residual outputs: the decode
 * step of a transformer block as few launches.  Per op, on top of
 * oracle_cuda_matvec_op:
 *   xform         ORACLE_CUDA_XFORM_NONE: the activation is x_dev;
 *                 ORACLE_CUDA_XFORM_RMS: (x * inv) * norm_dev[i] with inv =
 *                 1 / sqrt(sum(x^2) / cols + eps) (double sum, float inverse):
 *                 Oracle's rms_norm_rows over one row (src/runtime/
 *                 qwen35_block.cpp:161-188), never written out;
 *                 ORACLE_CUDA_XFORM_SWIGLU: silu(x) * x2_dev[i] (the MLP
 *                 activation, qwen35_block.cpp:315-318);
 *   residual_dev  optional (rows floats): y = residual + W.x, Oracle's
 *                 add_vectors of the block input and the branch
 *                 (qwen35_block.cpp:190-200, 333, 349);
 * each then quantized to Q8_K exactly as oracle_cuda_quantize_q8_k would
 * quantize the transformed vector.  Ops whose sources (x, xform, x2 / norm,
 * eps) are identical share one image: an op repeating an earlier op's source
 * needs no wait (after_previous is then ignored).  A SWIGLU op whose gate and
 * up are outputs of two earlier ops of the call over the same rows gets the
 * SwiGLU vector formed once, in the epilogue of the later of the two, at
 * act_dev (or in context scratch when act_dev is NULL).  No Oracle
 * counterpart: Oracle runs each projection, norm and add as its own call. */
#define ORACLE_CUDA_XFORM_NONE 0u
#define ORACLE_CUDA_XFORM_RMS 1u
#define ORACLE_CUDA_XFORM_SWIGLU 2u
typedef struct oracle_cuda_matvec_op_ex {
    oracle_cuda_matvec_op base;
    uint32_t xform;
    float eps;
    const float* x2_dev;
    const float* norm_dev;
    const float* residual_dev;
    float* act_dev;      /* optional (SWIGLU ops): where the SwiGLU vector (cols floats) is formed */
} oracle_cuda_matvec_op_ex;

oracle_cuda_status oracle_cuda_matvec_program_ex(oracle_cuda_context* ctx, const oracle_cuda_matvec_op_ex* ops,
                                                 uint32_t n_ops, void* stream);

/* The same matvec program for callers that cannot allocate device memory:
 * e.g. an engine that has already reserved nearly all of HBM for its own
 * pools, or a latency-critical path on which cudaMalloc, which can synchronise
 * the device, is not allowed.  It takes no context and allocates nothing: its
 * scratch (activation images of at most ORACLE_CUDA_NOALLOC_IMAGE_BYTES, the
 * completion counters and a status word) is one static device array that every
 * GPU loading this library holds until the process exits.  Works on the
 * current CUDA device.  The first call on a device looks the array up
 * (cudaGetSymbolAddress) and sets kernel attributes; make that first call
 * before any stream capture.  Each call clears the counters on `stream` and
 * then overwrites the images, so calls that overlap on the GPU (other streams,
 * other threads) race with each other.  Programs whose activation images need
 * more than ORACLE_CUDA_NOALLOC_IMAGE_BYTES are rejected with
 * INVALID_ARGUMENT.  Errors are reported through oracle_cuda_last_error(NULL);
 * a device-side wait that expired is reported by oracle_cuda_noalloc_status
 * (below), which reads the status word of the last call.  Results equal those
 * of oracle_cuda_matvec_program.  No counterpart in the reference (Oracle's
 * path never touches device memory). */
#define ORACLE_CUDA_NOALLOC_IMAGE_BYTES 65536
oracle_cuda_status oracle_cuda_matvec_program_noalloc(const oracle_cuda_matvec_op* ops, uint32_t n_ops,
                                                      void* stream);

/* The status of the last oracle_cuda_matvec_program_noalloc (or no-allocation
 * self-test) call on `device`: waits for that device's work to finish, then
 * returns ORACLE_CUDA_DEVICE_TIMEOUT (with the site in
 * oracle_cuda_last_error(NULL)) if one of the call's bounded device-side waits
 * expired -- its outputs are then incomplete -- else OK.  Reads the static
 * array's status word with a device-to-host copy; allocates nothing.  No
 * counterpart in the reference. */
oracle_cuda_status oracle_cuda_noalloc_status(int device);

/* A test of that status path: one kernel waits, on the no-allocation status
 * word of the current device, for a barrier nothing completes, and gives up
 * after limit_ns (0 < limit_ns <= 2 s); oracle_cuda_noalloc_status then reports
 * the timeout.  No counterpart in the reference. */
oracle_cuda_status oracle_cuda_noalloc_selftest_bounded_wait(uint64_t limit_ns, void* stream);

/* ------------------------------------------------------------------ either side of the matvecs
 * Embedding gather: out[t][0..cols) = the exact f32 decode of row ids[t] of a
 * GGML table (rows x cols, device memory), for n_ids token ids in device
 * memory; Oracle's embedding_row (src/runtime/qwen35_forward.cpp:51-70) for a
 * batch.  An id >= rows is not read: its output row is left as it was and the
 * next oracle_cuda_device_status reports OUT_OF_RANGE ("token id N exceeds the
 * embedding row count").  Asynchronous on `stream`. */
oracle_cuda_status oracle_cuda_gather_rows(oracle_cuda_context* ctx, uint32_t type, uint64_t rows, uint64_t cols,
                                           const void* w_dev, uint64_t w_nbytes, const uint32_t* ids_dev,
                                           uint64_t n_ids, float* out_dev, void* stream);

/* Greedy token of Oracle's sampler (src/runtime/sampler.cpp:22-46): the first
 * index of the largest logit.  oracle_cuda_argmax writes a 64-bit key to
 * key_dev (zeroed on `stream` first; asynchronous, graph-capturable) for the
 * n logits whose token ids start at index_base (a rank's shard of the vocabulary);
 * oracle_cuda_argmax_decode turns a key into the token, failing like the
 * reference (INVALID_ARGUMENT "logits contain NaN" / "logits contain no finite
 * candidates").  Keys of several shards combine by taking their maximum, so the
 * argmax of row-sharded logits needs only one key per rank.
 * oracle_cuda_greedy_token is the synchronous form (empty input: "cannot
 * sample an empty logits vector"). */
oracle_cuda_status oracle_cuda_argmax(oracle_cuda_context* ctx, const float* x_dev, uint64_t n,
                                      uint32_t index_base, unsigned long long* key_dev, void* stream);
oracle_cuda_status oracle_cuda_argmax_decode(unsigned long long key, uint32_t* token, float* value);
oracle_cuda_status oracle_cuda_greedy_token(oracle_cuda_context* ctx, const float* logits_dev, uint64_t n,
                                            uint32_t* token);

/* ------------------------------------------------------------------ decoder glue, one decode step
 * Device-memory, stream-ordered restatements of Oracle's decoder helpers, same
 * arithmetic (f32 / f64 as the reference; every product and sum rounded; the
 * reference's order wherever it sums sequentially; double sums in a tree).
 *   rms_norm_rows   rms_norm_rows, src/runtime/qwen35_block.cpp:161-188
 *   rope            apply_qwen35_rope, src/runtime/reference_kernels.cpp:74-123
 *                   (in place on heads [n_heads][head_dim]; cos/sin on the host
 *                   by the reference's expressions)
 *   attention_step  causal_attention_step, reference_kernels.cpp:125-190: appends
 *                   k_new/v_new at `length` of a KV cache laid out as Oracle's
 *                   (keys[token][kv_head][key_dim]); scores_dev holds
 *                   q_heads * (length + 1) floats of scratch
 *   conv_step       causal_depthwise_convolution_step, reference_kernels.cpp:192-219
 *                   (history [channels][kernel], updated in place)
 *   gated_delta_step gated_delta_step, reference_kernels.cpp:221-335 (state
 *                   [heads][key_dim][value_dim], updated in place); q and k
 *                   hold qk_heads rows of key_dim, head h reading row
 *                   h % qk_heads: the block's repeat_heads_tiled
 *                   (qwen35_block.cpp:225-243, 531-538) folded into the step
 *   swiglu          silu(gate) * up, qwen35_block.cpp:138-159 and 315-318
 *   add             add_vectors, qwen35_block.cpp:190-200 */
oracle_cuda_status oracle_cuda_rms_norm_rows(oracle_cuda_context* ctx, const float* in_dev, const float* weight_dev,
                                             uint64_t rows, uint64_t width, float eps, float* out_dev, void* stream);
oracle_cuda_status oracle_cuda_rope(oracle_cuda_context* ctx, float* heads_dev, uint64_t n_heads, uint64_t head_dim,
                                    uint64_t rotary_dim, const int32_t* sections, float base, uint64_t pos_temporal,
                                    uint64_t pos_height, uint64_t pos_width, void* stream);
oracle_cuda_status oracle_cuda_attention_step(oracle_cuda_context* ctx, const float* q_dev, const float* k_new_dev,
                                              const float* v_new_dev, float* keys_dev, float* values_dev,
                                              uint64_t capacity, uint64_t length, uint32_t q_heads,
                                              uint32_t kv_heads, uint32_t key_dim, uint32_t value_dim,
                                              float* scores_dev, float* out_dev, void* stream);
oracle_cuda_status oracle_cuda_conv_step(oracle_cuda_context* ctx, const float* in_dev, const float* weights_dev,
                                         float* history_dev, uint64_t channels, uint32_t kernel, int apply_silu,
                                         float* out_dev, void* stream);
oracle_cuda_status oracle_cuda_gated_delta_step(oracle_cuda_context* ctx, const float* q_dev, const float* k_dev,
                                                const float* v_dev, const float* beta_dev, const float* log_decay_dev,
                                                float* state_dev, uint32_t heads, uint32_t qk_heads,
                                                uint32_t key_dim, uint32_t value_dim, float eps, float* out_dev,
                                                void* stream);
oracle_cuda_status oracle_cuda_swiglu(oracle_cuda_context* ctx, const float* gate_dev, const float* up_dev, uint64_t n,
                                      float* out_dev, void* stream);
oracle_cuda_status oracle_cuda_add(oracle_cuda_context* ctx, const float* a_dev, const float* b_dev, uint64_t n,
                                   float* out_dev, void* stream);

/* ------------------------------------------------------------------ graph-replayable decode step
 * A decode step captured once in a CUDA graph and replayed for every token
 * keeps the token position in device memory (pos_dev, one uint32): the forms
 * below read it there, and oracle_cuda_position_advance adds one at the end
 * of a step.  Same arithmetic as oracle_cuda_rope / oracle_cuda_attention_step.
 * A position >= the cache capacity (or the table's positions) is skipped and
 * reported by the next oracle_cuda_device_status as OVERFLOW ("KV cache
 * capacity exceeded ..."), the class KvCache::append throws.
 *   rope_table        cos/sin of every text position p < positions
 *                     (RopePosition::text, reference_kernels.hpp:18-20) by
 *                     apply_qwen35_rope's expressions, reference_kernels.cpp:104-113;
 *                     table_dev holds positions * rotary_dim floats; synchronous
 *   rope_at           apply_qwen35_rope at position *pos_dev
 *   attention_step_at causal_attention_step at length *pos_dev; scores_dev
 *                     holds q_heads * capacity floats
 *   split_query_gate  the joint query/gate projection [heads][2 * width] split
 *                     into query and gate [heads][width], qwen35_block.cpp:676-688
 *   gate_sigmoid_mul  x[i] *= sigmoid(gate[i]), qwen35_block.cpp:738-742
 *   mul_silu          x[i] *= silu(z[i]), qwen35_block.cpp:589-592
 *   gdn_gates         beta_out = sigmoid(beta), log_decay = softplus(alpha +
 *                     time_step_bias) * decay, qwen35_block.cpp:472-489 */
oracle_cuda_status oracle_cuda_rope_table(oracle_cuda_context* ctx, uint64_t rotary_dim, const int32_t* sections,
                                          float base, uint64_t positions, float* table_dev);
oracle_cuda_status oracle_cuda_rope_at(oracle_cuda_context* ctx, float* heads_dev, uint64_t n_heads, uint64_t head_dim,
                                       uint64_t rotary_dim, const float* table_dev, uint64_t positions,
                                       const uint32_t* pos_dev, void* stream);
oracle_cuda_status oracle_cuda_attention_step_at(oracle_cuda_context* ctx, const float* q_dev, const float* k_new_dev,
                                                 const float* v_new_dev, float* keys_dev, float* values_dev,
                                                 uint64_t capacity, const uint32_t* pos_dev, uint32_t q_heads,
                                                 uint32_t kv_heads, uint32_t key_dim, uint32_t value_dim,
                                                 float* scores_dev, float* out_dev, void* stream);
oracle_cuda_status oracle_cuda_position_advance(oracle_cuda_context* ctx, uint32_t* pos_dev, void* stream);
oracle_cuda_status oracle_cuda_split_query_gate(oracle_cuda_context* ctx, const float* full_dev, uint32_t heads,
                                                uint32_t width, float* query_dev, float* gate_dev, void* stream);
oracle_cuda_status oracle_cuda_gate_sigmoid_mul(oracle_cuda_context* ctx, float* x_dev, const float* gate_dev,
                                                uint64_t n, void* stream);
oracle_cuda_status oracle_cuda_mul_silu(oracle_cuda_context* ctx, float* x_dev, const float* z_dev, uint64_t n,
                                        void* stream);
/* token_commit: after oracle_cuda_argmax into key_dev, the sampled token
 * (Sampler::sample at temperature 0, src/runtime/sampler.cpp:22-46) and the
 * next step's input: *next_id_dev = prompt[*pos + 1] while *pos + 1 < n_prompt
 * (prompt ingestion one token at a time, qwen35_generation.cpp:737-747), else
 * the sampled token, also stored at tokens_dev[*pos + 1 - n_prompt] when that
 * index is < tokens_capacity; then *pos_dev += 1.  NaN / no finite logit:
 * INVALID_ARGUMENT from the next oracle_cuda_device_status with the sampler's
 * message, and the position does not advance. */
oracle_cuda_status oracle_cuda_token_commit(oracle_cuda_context* ctx, const unsigned long long* key_dev,
                                            const uint32_t* prompt_dev, uint32_t n_prompt, uint32_t* pos_dev,
                                            uint32_t* next_id_dev, uint32_t* tokens_dev, uint32_t tokens_capacity,
                                            void* stream);
/* Batched greedy sampling for sequences decoded in lockstep (one shared
 * position): oracle_cuda_argmax_rows writes the argmax key of each logits row
 * x[b][n] (b < rows) to keys_dev[b]; oracle_cuda_token_commit_rows applies
 * token_commit to each sequence b (prompt_dev[b * n_prompt ..], next_id_dev[b],
 * tokens_dev[b * tokens_capacity ..]), clears the keys and advances *pos_dev
 * once.  A NaN / non-finite maximum in any row is reported like
 * oracle_cuda_token_commit and stops the batch (no advance). */
oracle_cuda_status oracle_cuda_argmax_rows(oracle_cuda_context* ctx, const float* x_dev, uint32_t rows, uint64_t n,
                                           unsigned long long* keys_dev, void* stream);
oracle_cuda_status oracle_cuda_token_commit_rows(oracle_cuda_context* ctx, unsigned long long* keys_dev,
                                                 uint32_t rows, const uint32_t* prompt_dev, uint32_t n_prompt,
                                                 uint32_t* pos_dev, uint32_t* next_id_dev, uint32_t* tokens_dev,
                                                 uint32_t tokens_capacity, void* stream);
/* Fused block cores (graph-replayable, position in device memory):
 *   gdn_core        a Gated DeltaNet block from its projections to the vector
 *                   its output projection reads (qwen35_block.cpp:472-592):
 *                   gates, depthwise conv + SiLU (history [2][channels][kernel],
 *                   double-buffered by position parity: zero both halves to
 *                   reset), gated_delta_step on state [value_heads][head_dim]
 *                   [head_dim] with q / k of key head h % key_heads, RMSNorm
 *                   of each head's output, * silu(z); key and value head widths
 *                   equal (Oracle's layout: both ssm.state_size)
 *   attention_prep_at  per query head: the query half of q_full [heads][2 *
 *                   head_dim], its RMSNorm and RoPE (q_out); per KV head the
 *                   same for the key, appended with the value at *pos
 *   attention_core_at  scores, softmax and values over the cache (no append),
 *                   times sigmoid(gate) when gate_dev is given (gate of head h
 *                   at gate_dev + h * gate_stride) */
oracle_cuda_status oracle_cuda_gdn_core(oracle_cuda_context* ctx, const float* qkv_dev, const float* z_dev,
                                        const float* beta_dev, const float* alpha_dev,
                                        const float* time_step_bias_dev, const float* decay_dev,
                                        const float* conv_weights_dev, float* history_dev, float* state_dev,
                                        const float* norm_dev, uint32_t key_heads, uint32_t value_heads,
                                        uint32_t head_dim, uint32_t conv_kernel, float eps, const uint32_t* pos_dev,
                                        float* out_dev, void* stream);
/* gdn_core for `seqs` sequences decoded in lockstep: sequence s reads and
 * writes its own stacked buffers (qkv_dev + s * channels, z / out + s *
 * value_heads * head_dim, beta / alpha + s * value_heads, history + s * 2 *
 * channels * conv_kernel, state + s * value_heads * head_dim^2); the weights
 * and the position are shared.  seqs == 1 is oracle_cuda_gdn_core. */
oracle_cuda_status oracle_cuda_gdn_core_seqs(oracle_cuda_context* ctx, const float* qkv_dev, const float* z_dev,
                                             const float* beta_dev, const float* alpha_dev,
                                             const float* time_step_bias_dev, const float* decay_dev,
                                             const float* conv_weights_dev, float* history_dev, float* state_dev,
                                             const float* norm_dev, uint32_t key_heads, uint32_t value_heads,
                                             uint32_t head_dim, uint32_t conv_kernel, float eps,
                                             const uint32_t* pos_dev, uint32_t seqs, float* out_dev, void* stream);
oracle_cuda_status oracle_cuda_attention_prep_at(oracle_cuda_context* ctx, const float* q_full_dev, const float* k_dev,
                                                 const float* v_dev, const float* q_norm_dev, const float* k_norm_dev,
                                                 float eps, const float* table_dev, uint64_t rotary_dim,
                                                 uint32_t q_heads, uint32_t kv_heads, uint32_t head_dim,
                                                 float* keys_dev, float* values_dev, uint64_t capacity,
                                                 const uint32_t* pos_dev, float* q_out_dev, void* stream);
oracle_cuda_status oracle_cuda_attention_core_at(oracle_cuda_context* ctx, const float* q_dev, const float* keys_dev,
                                                 const float* values_dev, uint64_t capacity, const uint32_t* pos_dev,
                                                 uint32_t q_heads, uint32_t kv_heads, uint32_t key_dim,
                                                 uint32_t value_dim, const float* gate_dev, uint32_t gate_stride,
                                                 float* scores_dev, float* out_dev, void* stream);
oracle_cuda_status oracle_cuda_gdn_gates(oracle_cuda_context* ctx, const float* beta_dev, const float* alpha_dev,
                                         const float* time_step_bias_dev, const float* decay_dev, uint32_t heads,
                                         float* beta_out_dev, float* log_decay_dev, void* stream);

/* ------------------------------------------------------------------ row-sharded programs over GPUs
 * Tensor-parallel decode on the GPUs of one node, one process per GPU: every
 * rank holds an equal contiguous row range of each weight matrix and runs the
 * same matvec program on it; every output row is stored both locally and,
 * over NVLink, into every peer's gather buffer at the same offset, so that
 * when the launch completes each rank holds all ranks' rows (the all-gather
 * of the outputs happens inside the matvec kernel; no NCCL call).
 *   1. oracle_cuda_peer_group_create on every rank: allocates the rank's
 *      gather buffer (data_bytes, device memory) and returns its CUDA IPC
 *      handle (ORACLE_CUDA_IPC_HANDLE_BYTES) to publish to the other ranks;
 *   2. oracle_cuda_peer_group_connect with all ranks' handles, in rank order;
 *   3. oracle_cuda_matvec_program_allgather: like oracle_cuda_matvec_program,
 *      with every op's y_dev inside this rank's gather data region
 *      (oracle_cuda_peer_group_data) at the offset of this rank's rows; all
 *      ranks must run the same program shapes, launch for launch.
 * The gather buffer is overwritten by peers on their next launch: a caller
 * that needs the previous gathered output while peers run ahead alternates
 * two groups.  A peer that does not launch makes the waiting kernel give up
 * after one second and record a device timeout (oracle_cuda_device_status).
 * No counterpart in the reference (Oracle runs on one CPU thread); the north
 * star's per-layer NCCL all-gather is what this replaces. */
#define ORACLE_CUDA_IPC_HANDLE_BYTES 64
#define ORACLE_CUDA_MAX_PEERS 8
typedef struct oracle_cuda_peer_group oracle_cuda_peer_group;
oracle_cuda_status oracle_cuda_peer_group_create(oracle_cuda_context* ctx, uint32_t rank, uint32_t world,
                                                 uint64_t data_bytes, oracle_cuda_peer_group** out,
                                                 void* ipc_handle_out);
oracle_cuda_status oracle_cuda_peer_group_connect(oracle_cuda_peer_group* group, const void* handles);
oracle_cuda_status oracle_cuda_peer_group_data(oracle_cuda_peer_group* group, float** data_dev);
oracle_cuda_status oracle_cuda_peer_group_destroy(oracle_cuda_peer_group* group);
/* The extended program over a peer group: every op's rows are this rank's
 * shard, outputs (y, residual outputs, SwiGLU vectors at act_dev) lie in the
 * gather buffer and reach every rank; an op with after_previous (or a
 * transform of an earlier op's output) waits until EVERY rank has finished the
 * op before it, so transforms see whole vectors.  Results on every rank equal
 * the single-GPU program's bit for bit. */
oracle_cuda_status oracle_cuda_matvec_program_ex_allgather(oracle_cuda_context* ctx, oracle_cuda_peer_group* group,
                                                           const oracle_cuda_matvec_op_ex* ops, uint32_t n_ops,
                                                           void* stream);
oracle_cuda_status oracle_cuda_matvec_program_allgather(oracle_cuda_context* ctx, oracle_cuda_peer_group* group,
                                                        const oracle_cuda_matvec_op* ops, uint32_t n_ops,
                                                        void* stream);

/* ------------------------------------------------------------------ head-sharded programs
 * The decode step with heads sharded over the ranks (one process per GPU): a
 * rank computes its own heads' input projections (rows of its heads only)
 * and, for a projection whose input is sharded (the block output projection
 * over the rank's heads, the MLP down projection over the rank's FFN
 * columns), PARTIAL sums of every row over its own super-blocks.  Rank q of
 * `world` (1, 2, 4 or 8) owns super-blocks j with j % world == q of every
 * 16-super-block segment; its partial of a row is the canonical fold of
 * those leaves (a row of that rank's columns only, one matvec per segment),
 * and the next op's transform ORACLE_CUDA_XFORM_COMBINE_RMS folds every
 * rank's partials by the remaining strides, adds the segments in order and
 * the residual, so every rank obtains the unsharded program's vector bit for
 * bit.  Per op, on top of oracle_cuda_matvec_op_ex:
 *   push      1: y_dev lies in the gather buffer and every row is also stored
 *             into every peer's buffer at the same offset (NVLink stores);
 *   wait      0: x is produced before the call; 1: x is produced by the op
 *             before (this rank's CTAs are waited for); 2: as 1, and the op
 *             before must `announce`: its outputs from EVERY rank are waited
 *             for; 3: x is produced by an earlier op that a previous op of
 *             this call already waited for (no wait; the image is built when
 *             the op starts);
 *   announce  1: once this rank finished the op (and all before it), every
 *             peer is told (one cross-rank dependency; numbered within the
 *             step from `first_dep`);
 *   segments  XFORM_COMBINE_RMS: x_dev = the residual vector (cols floats),
 *             x2_dev = the partial sums [world][segments][cols] inside the
 *             gather buffer, norm_dev / eps as for XFORM_RMS; with wait 2, or
 *             wait 3 when an earlier op of the call has the same source;
 *   swiglu_gate  optional: after the op, act_dev[r] = silu(swiglu_gate[r]) *
 *             y[r] for the op's rows (the MLP activation from the gate
 *             rows of an earlier op and this op's up rows);
 *   combined_dev  XFORM_COMBINE_RMS: receives the combined vector (cols
 *             floats, before the norm; device memory other than x_dev).
 * `step`: first_dep = the index within the decode step of this call's first
 * announcement, deps_per_step = announcements per step (the same on every
 * rank), end_of_step = 1 on the step's last call, tail_wait = 1: the call's
 * grid ends only once every peer announced this call's last announcement
 * (outputs the next kernel reads from every rank).  Every rank issues the
 * same calls in the same order; peers waited for longer than one second make
 * the kernel record a device timeout (oracle_cuda_device_status).  No
 * counterpart in the reference (Oracle runs on one CPU thread); the north
 * star's head-sharded decoder with per-layer collectives is what this
 * replaces, with two cross-rank dependencies per block. */
#define ORACLE_CUDA_XFORM_COMBINE_RMS 3u
typedef struct oracle_cuda_sharded_op {
    oracle_cuda_matvec_op_ex ex;
    uint32_t push;
    uint32_t wait;
    uint32_t announce;
    uint32_t segments;
    const float* swiglu_gate;
    float* combined_dev;
} oracle_cuda_sharded_op;
typedef struct oracle_cuda_sharded_step {
    uint32_t first_dep;
    uint32_t deps_per_step;
    uint32_t end_of_step;
    uint32_t tail_wait;
} oracle_cuda_sharded_step;
oracle_cuda_status oracle_cuda_matvec_program_sharded(oracle_cuda_context* ctx, oracle_cuda_peer_group* group,
                                                      const oracle_cuda_sharded_op* ops, uint32_t n_ops,
                                                      const oracle_cuda_sharded_step* step, void* stream);

/* Launch trace of the matvec programs (all entry points that launch one):
 * with `records` > 0, the programs launched from now on write global-timer
 * stamps (ns) into trace_dev (device memory, 8-byte aligned, 1 + records *
 * ORACLE_CUDA_TRACE_WORDS words, word 0 zero to start): word 0 counts
 * launches; launch r (while r < records) fills words 1 + r * TRACE_WORDS
 * onward, as seen by CTA 0: [0] consumers start (after the wait for the
 * preceding kernel), per op k [1 + 3k] its wait for earlier ops done,
 * [2 + 3k] its activation image built, [3 + 3k] its rows written and
 * published, [TRACE_WORDS - 1] CTA 0 done.  records = 0 switches it off.
 * Launches captured in a CUDA graph keep the setting of their capture. */
#define ORACLE_CUDA_TRACE_WORDS 50
oracle_cuda_status oracle_cuda_set_program_trace(oracle_cuda_context* ctx, unsigned long long* trace_dev,
                                                 uint32_t records);

/* ------------------------------------------------------------------ prefill dequant-GEMM
 * Y[m][n] = sum_k X[m][k] * W[n][k] for m < m_tokens: the batched form of the
 * matvec for prompt ingestion (M >= 64 tokens).  W: `rows` GGML rows of `cols`
 * columns (Q4_K only), device memory, 16-byte aligned.  X: m_tokens x cols f32,
 * row-major, 16-byte aligned.  Y: m_tokens x rows f32, row-major.  Both operands
 * are rounded to bf16 (round to nearest even; W from its exact f32 decode) and
 * multiplied on the tensor cores with f32 accumulation; when K is split across
 * CTAs (small grids) the partial sums are added atomically, so the last bits
 * may vary between runs.  Asynchronous on `stream`.  No counterpart in the
 * reference: Oracle ingests prompts one matvec at a time
 * (src/runtime/qwen35_generation.cpp:737-747). */
oracle_cuda_status oracle_cuda_prefill_gemm(oracle_cuda_context* ctx, uint32_t type, uint64_t rows, uint64_t cols,
                                            const void* w_dev, uint64_t w_nbytes, const float* x_dev,
                                            uint64_t m_tokens, float* y_dev, void* stream);

/* ------------------------------------------------------------------ resident weights
 * Oracle's weights are immutable GGUF bytes in a read-only mapping
 * (MappedGgufModel, include/oracle/model/mapped_gguf.hpp:56-59).  They are
 * copied to HBM once; a shard keeps rows [row_begin, row_end). */

oracle_cuda_status oracle_cuda_weight_upload(oracle_cuda_context* ctx, uint32_t type, uint64_t rows,
                                             uint64_t cols, const void* host_bytes, uint64_t nbytes,
                                             uint64_t row_begin, uint64_t row_end,
                                             oracle_cuda_weight** out);
oracle_cuda_status oracle_cuda_weight_free(oracle_cuda_weight* weight);
/* Device address, byte size and shard geometry of an uploaded weight. */
oracle_cuda_status oracle_cuda_weight_info(const oracle_cuda_weight* weight, uint32_t* type,
                                           uint64_t* rows, uint64_t* cols, uint64_t* row_begin,
                                           const void** dev, uint64_t* nbytes);

/* ------------------------------------------------------------------ host-pointer drop-ins
 * Synchronous, host spans in and out, exactly the reference's signatures (the
 * reference's functions are pure: they read the caller's bytes on every call).
 * A weight span the caller has REGISTERED (below) is read from its resident
 * copy in HBM; any other span is copied to the device on every call, so a
 * buffer whose bytes change between calls always gives the new result. */

/* Register host weight bytes (rows x cols of `type`, exactly `nbytes`): they
 * are copied to HBM now and the host-pointer calls given the same (address,
 * nbytes, type, rows, cols) read that copy from then on.  The caller promises
 * the bytes do not change while registered -- true of Oracle's GGUF tensors,
 * read-only MAP_PRIVATE pages owned by MappedGgufModel
 * (include/oracle/model/mapped_gguf.hpp:56-59).  Registering the same span
 * again is a no-op.  No counterpart in the reference (it has no device). */
oracle_cuda_status oracle_cuda_register_host_weight(oracle_cuda_context* ctx, uint32_t type, uint64_t rows,
                                                    uint64_t cols, const void* host, uint64_t nbytes);
/* Drop the resident copy of a registered span (OUT_OF_RANGE if it is not
 * registered).  No counterpart in the reference. */
oracle_cuda_status oracle_cuda_unregister_host_weight(oracle_cuda_context* ctx, const void* host, uint64_t nbytes);

/* reference_storage_matvec (quantized_reference.cpp:128-162). */
oracle_cuda_status oracle_cuda_host_storage_matvec(oracle_cuda_context* ctx, int contract,
                                                   uint32_t type, uint64_t rows, uint64_t cols,
                                                   const void* w_host, uint64_t w_nbytes,
                                                   const float* x_host, uint64_t x_len,
                                                   float* y_host, uint64_t y_len);

/* reference_storage_dot (quantized_reference.cpp:24-82): one row. */
oracle_cuda_status oracle_cuda_host_storage_dot(oracle_cuda_context* ctx, int contract,
                                                uint32_t type, uint64_t cols, const void* row_host,
                                                uint64_t row_nbytes, const float* x_host,
                                                uint64_t x_len, float* out);

/* decode_storage_row (storage_decode.cpp:244-294) and
 * reference_decode_mapped_tensor (quantized_reference.cpp:85-105). */
oracle_cuda_status oracle_cuda_host_decode_rows(oracle_cuda_context* ctx, uint32_t type,
                                                uint64_t rows, uint64_t cols, const void* w_host,
                                                uint64_t w_nbytes, float* out_host,
                                                uint64_t out_len);

/* Unregister every registered weight span (drops their resident copies). */
oracle_cuda_status oracle_cuda_evict_resident(oracle_cuda_context* ctx);

/* A matvec program over host spans: several Q8_K-contract matvecs (q4_K /
 * q6_K weights) in ONE device launch with one synchronize, e.g. a layer's
 * projections.  Every x is copied in and every y out in one transfer each.
 * An op whose x_host is the y_host of an earlier op of the same call reads
 * that op's result on the device (cols must equal that op's rows): a
 * dependent op, as in oracle_cuda_matvec_program.  Weights as for the
 * host-pointer calls above (registered: resident; otherwise copied per call).
 * Results equal oracle_cuda_matvec_program's.  No counterpart in the
 * reference (its products run one at a time, qwen35_block.cpp:108-119). */
typedef struct oracle_cuda_host_matvec_op {
    uint32_t type;
    uint64_t rows;
    uint64_t cols;
    const void* w_host;
    uint64_t w_nbytes;
    const float* x_host;  /* cols floats, or an earlier op's y_host */
    float* y_host;        /* rows floats */
} oracle_cuda_host_matvec_op;
oracle_cuda_status oracle_cuda_host_matvec_program(oracle_cuda_context* ctx, const oracle_cuda_host_matvec_op* ops,
                                                   uint32_t n_ops);

/* The same call prepared once for a caller that repeats it (a decode step
 * over the same buffers): the op list is validated and planned, and the
 * copy-in, the program launch and the copy-out are captured into one CUDA
 * graph on a stream of the prepared call's own.  Every weight must be
 * registered (INVALID_ARGUMENT otherwise); x and y stay the caller's arrays,
 * read and written at each run.  When every x and y is page-locked host
 * memory mapped for the device (cudaHostAlloc, cudaHostRegister) two small
 * kernels of the graph read x and write y there in place; otherwise the run
 * copies them through page-locked buffers the prepared call owns.  run() is
 * synchronous and gives exactly what
 * oracle_cuda_host_matvec_program gives for the arrays' current contents.
 * The context must outlive the prepared call.  No counterpart in the
 * reference. */
typedef struct oracle_cuda_host_program oracle_cuda_host_program;
oracle_cuda_status oracle_cuda_host_program_create(oracle_cuda_context* ctx, const oracle_cuda_host_matvec_op* ops,
                                                   uint32_t n_ops, oracle_cuda_host_program** out);
oracle_cuda_status oracle_cuda_host_program_run(oracle_cuda_host_program* program);
oracle_cuda_status oracle_cuda_host_program_destroy(oracle_cuda_host_program* program);

#ifdef __cplusplus
}
#endif

#endif /* ORACLE_CUDA_H */
