// oracle_cuda.cu -- C ABI over the sm_100a kernels of the quantized-weight path.
//
// Host-side validation restates the reference's checks in its order and with
// its messages (quantized_reference.cpp:128-153, storage_decode.cpp:182-198,
// ggml_type.cpp:77-94), so the status code names the exception class the
// reference would throw.  Nothing is launched unless validation passes.
#include "../../include/oracle_cuda.h"

#include <cuda_runtime.h>

#include <cmath>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <set>
#include <string>
#include <tuple>
#include <vector>

#include "decoder_ops.cuh"
#include "decoder_step.cuh"
#include "gather.cuh"
#include "gemm_q4k.cuh"
#include "layout.hpp"
#include "matvec_batch.cuh"
#include "matvec_q80_lane.cuh"
#include "matvec_seq.cuh"
#include "matvec_q8k.cuh"
#include "program.cuh"
#include "q8k.cuh"

using namespace oracle_cuda;

struct oracle_cuda_weight {
    oracle_cuda_context* ctx;
    uint32_t type;
    uint64_t rows;       // rows held (the shard)
    uint64_t cols;
    uint64_t row_begin;  // first global row of the shard
    uint64_t nbytes;
    void* dev;
    bool owned_by_cache;
};

struct oracle_cuda_context {
    int device = 0;
    int sm_count = 0;
    int max_smem_optin = 0;
    uint64_t smem_budget = 0;  // per-CTA shared memory for stream kernels (0 = all)
    uint64_t stage_target = 36864;  // bytes per stage the stage plan aims for
    // matvec programs: bytes per stage (two rows per consumer warp, e.g. 28
    // rows of 16 super-blocks) while at least kProgramMinStages stages fit
    uint64_t program_stage_target = 65536;
    uint32_t copy_chunk = 32768;    // largest single bulk copy
    uint32_t max_inflight = 16;     // stages a program producer keeps in flight
    uint32_t jit_image_threshold = 48 * 1024;  // prebuilt image bytes above which programs copy per op
    uint32_t flags = 0;
    uint64_t launches = 0;
    DeviceStatus* status = nullptr;
    unsigned int* program_counters = nullptr;  // kProgramCounters, zero between launches
    unsigned long long* trace = nullptr;       // matvec program launch trace (caller's memory), or null
    uint32_t trace_records = 0;
    uint8_t* image_scratch = nullptr;          // prebuilt activation images of programs
    uint64_t image_scratch_bytes = 0;
    uint8_t* act_scratch = nullptr;            // SwiGLU activations formed in program epilogues
    uint64_t act_scratch_bytes = 0;
    std::string last_error;
    std::set<const void*> smem_configured;
    // registered host weight spans and their resident copies (host-pointer calls)
    std::map<std::tuple<const void*, uint64_t, uint32_t, uint64_t, uint64_t>, oracle_cuda_weight*> resident;
    // device copies of unregistered weight spans, made on every host-pointer call
    uint8_t* stage_w = nullptr;
    uint64_t stage_w_len = 0;
    // staging for the host-pointer drop-ins (grown on demand)
    float* pin_x = nullptr;
    float* pin_y = nullptr;
    uint64_t pin_x_len = 0, pin_y_len = 0;
    float* dev_x = nullptr;
    float* dev_y = nullptr;
    uint64_t dev_x_len = 0, dev_y_len = 0;
    // prefill GEMM: bf16 copy of the activations
    uint16_t* gemm_x = nullptr;
    uint64_t gemm_x_len = 0;
    bool gemm_pair = false;
    unsigned long long* argmax_key = nullptr;  // one key for oracle_cuda_greedy_token  // prefill GEMM on CTA pairs (cta_group::2); ORACLE_CUDA_GEMM_PAIR=1
    // batched Q8_K matvec: activation images and per-segment partial sums
    uint8_t* batch_image = nullptr;
    uint64_t batch_image_len = 0;
    float* batch_partial = nullptr;
    uint64_t batch_partial_len = 0;
};

namespace {

thread_local std::string g_thread_error;

oracle_cuda_status fail(oracle_cuda_context* ctx, oracle_cuda_status s, const std::string& msg) {
    if (ctx)
        ctx->last_error = msg;
    else
        g_thread_error = msg;
    return s;
}

oracle_cuda_status fail(oracle_cuda_context* ctx, const Error& e) {
    return fail(ctx, static_cast<oracle_cuda_status>(static_cast<int>(e.kind)), e.message);
}

oracle_cuda_status cuda_fail(oracle_cuda_context* ctx, cudaError_t err, const char* what) {
    return fail(ctx, err == cudaErrorMemoryAllocation ? ORACLE_CUDA_OUT_OF_MEMORY : ORACLE_CUDA_CUDA_ERROR,
                std::string(what) + ": " + cudaGetErrorString(err));
}

#define ORACLE_CUDA_TRY(ctx, call, what)                  \
    do {                                                  \
        cudaError_t _e = (call);                          \
        if (_e != cudaSuccess) return cuda_fail(ctx, _e, what); \
    } while (0)

oracle_cuda_status ok(oracle_cuda_context* ctx) {
    if (ctx) ctx->last_error.clear();
    return ORACLE_CUDA_OK;
}

// The reference's row-view type gate (storage_decode.cpp:192-196), widened by q4_K.
Error check_decodable(uint32_t type) {
    if (!decodable(type))
        return make_error(ErrorKind::InvalidArgument,
                          "storage decoder does not support GGML type " + std::to_string(type));
    return {};
}

// Pointer alignment the kernels rely on: 16 bytes for q4_K/q5_K (vector loads
// of 16-byte aligned super-blocks), 4 for f32, 2 otherwise.
Error check_weight_pointer(uint32_t type, const void* p) {
    if (!p) return make_error(ErrorKind::InvalidArgument, "weight pointer is null");
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    const uintptr_t need = (type == kTypeQ4_K || type == kTypeQ5_K) ? 16 : type == kTypeF32 ? 4 : 2;
    if (a % need)
        return make_error(ErrorKind::InvalidArgument,
                          "weight pointer must be " + std::to_string(need) + "-byte aligned for GGML type " +
                              std::to_string(type));
    return {};
}

// reference_storage_matvec's validation (quantized_reference.cpp:134-153),
// generalised to `batch` activation vectors, plus the per-row type gate.
Error check_matvec(uint32_t type, uint64_t rows, uint64_t cols, uint64_t w_nbytes, uint64_t x_len,
                   uint64_t y_len, uint64_t* row_bytes, uint64_t* batch) {
    if (rows == 0 || cols == 0)
        return make_error(ErrorKind::InvalidArgument, "reference matvec dimensions must be non-zero");
    if (x_len == 0 || x_len % cols != 0)
        return make_error(ErrorKind::InvalidArgument, "reference matvec vector length mismatch");
    *batch = x_len / cols;
    uint64_t expect_y;
    if (!checked_mul(rows, *batch, &expect_y) || y_len != expect_y)
        return make_error(ErrorKind::InvalidArgument, "reference matvec output length mismatch");
    if (Error e = row_byte_size(cols, type, row_bytes)) return e;
    uint64_t total;
    if (!checked_mul(rows, *row_bytes, &total))
        return make_error(ErrorKind::Overflow, "reference matvec matrix size overflow");
    if (w_nbytes != total)
        return make_error(ErrorKind::InvalidArgument, "reference matvec matrix byte size mismatch");
    return check_decodable(type);
}

// ---------------------------------------------------------------- launches

template <typename Kernel, typename... Args>
oracle_cuda_status launch(oracle_cuda_context* ctx, Kernel kernel, dim3 grid, dim3 block, size_t smem,
                          cudaStream_t stream, bool pdl, Args... args) {
    const void* key = reinterpret_cast<const void*>(kernel);
    if (smem > 48 * 1024 && !ctx->smem_configured.count(key)) {
        ORACLE_CUDA_TRY(ctx,
                        cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             ctx->max_smem_optin),
                        "cudaFuncSetAttribute");
        ctx->smem_configured.insert(key);
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    if (pdl) {
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
    }
    ORACLE_CUDA_TRY(ctx, cudaLaunchKernelEx(&cfg, kernel, args...), "kernel launch");
    ctx->launches += 1;
    return ORACLE_CUDA_OK;
}

// Stage plan for the row-streaming kernels: up to one row per consumer warp
// and about stage_target bytes per stage, as many stages as the
// CTA's shared-memory budget allows (<= 16).
bool plan_stream(oracle_cuda_context* ctx, uint64_t rows, uint64_t row_bytes, uint32_t act_bytes, int ncw,
                 StreamParams& sp, uint32_t& grid) {
    grid = static_cast<uint32_t>(rows < uint64_t(ctx->sm_count) ? rows : ctx->sm_count);
    const uint64_t cta_budget = ctx->smem_budget ? ctx->smem_budget : uint64_t(ctx->max_smem_optin);
    if (act_bytes + stream_barrier_bytes(16) + 2 * 128 > cta_budget) return false;
    const uint64_t budget = cta_budget - stream_barrier_bytes(16) - act_bytes;
    // one row per consumer warp per stage when rows are short, fewer when long
    uint64_t R = ctx->stage_target / row_bytes;
    if (R > uint64_t(ncw)) R = ncw;
    if (R < 1) R = 1;
    uint64_t stage = align_up(static_cast<uint32_t>(R * row_bytes + 32), 128u);
    while (R > 1 && stage * 2 > budget) {
        R -= 1;
        stage = align_up(static_cast<uint32_t>(R * row_bytes + 32), 128u);
    }
    if (row_bytes + 32 > (1u << 30) || stage * 2 > budget) return false;
    const uint64_t rows_per_cta = (rows + grid - 1) / grid;
    const uint64_t tmax = (rows_per_cta + R - 1) / R;
    uint64_t S = budget / stage;
    if (S > 16) S = 16;
    if (S > tmax) S = tmax < 1 ? 1 : tmax;
    sp.rows = rows;
    sp.row_bytes = row_bytes;
    sp.rows_per_stage = static_cast<uint32_t>(R);
    sp.stages = static_cast<uint32_t>(S);
    sp.stage_bytes = static_cast<uint32_t>(stage);
    sp.act_bytes = act_bytes;
    sp.copy_chunk = ctx->copy_chunk;
    sp.status = ctx->status;
    return true;
}

constexpr int kQ8KConsumerWarps = 16;
// The program kernel carries several ops' code paths and may use 128 registers
// unspilled; 14 consumer warps + 1 producer take 61,440 of the SM's 65,536
// registers, which leaves room for one warp of the next step's quantizer
// (quantize_images_kernel, one warp per CTA) to run beside a program CTA.
constexpr int kProgramWarps = 14;
constexpr uint64_t kProgramMinStages = 3;

template <class Consumer>
oracle_cuda_status launch_stream(oracle_cuda_context* ctx, const uint8_t* w, uint64_t rows, uint64_t row_bytes,
                                 uint32_t act_bytes, const typename Consumer::Params& cp, cudaStream_t stream) {
    StreamParams sp{};
    uint32_t grid = 0;
    if (!plan_stream(ctx, rows, row_bytes, act_bytes, Consumer::kWarps, sp, grid))
        return fail(ctx, ORACLE_CUDA_UNSUPPORTED, "weight rows too long for the shared-memory stage ring");
    sp.w = w;
    const size_t smem = stream_smem_bytes(sp);
    return launch(ctx, stream_rows_kernel<Consumer>, dim3(grid), dim3((Consumer::kWarps + 1) * 32), smem,
                  stream, (ctx->flags & ORACLE_CUDA_FLAG_PDL) != 0, sp, cp);
}

template <uint32_t kType>
oracle_cuda_status launch_q8k_typed(oracle_cuda_context* ctx, const uint8_t* w, uint64_t rows, uint64_t row_bytes,
                                    const MatvecQ8KParams& cp, cudaStream_t stream) {
    const uint32_t act = q8k_image_bytes(cp.nb);
    if (cp.nb <= 16)
        return launch_stream<MatvecQ8KConsumer<kType, true, kQ8KConsumerWarps>>(ctx, w, rows, row_bytes, act, cp,
                                                                                stream);
    return launch_stream<MatvecQ8KConsumer<kType, false, kQ8KConsumerWarps>>(ctx, w, rows, row_bytes, act, cp,
                                                                             stream);
}

// Q8_K contract, one activation vector per launch (x f32 or pre-quantized).
oracle_cuda_status launch_q8k(oracle_cuda_context* ctx, uint32_t type, const void* w, uint64_t rows, uint64_t cols,
                              uint64_t row_bytes, const float* x, const uint8_t* q8k, float* y, cudaStream_t stream) {
    MatvecQ8KParams cp{};
    cp.x = x;
    cp.q8k = q8k;
    cp.y = y;
    cp.rows = rows;
    cp.nb = static_cast<uint32_t>(cols / 256);
    const uint8_t* wb = static_cast<const uint8_t*>(w);
    if (type == kTypeQ4_K) return launch_q8k_typed<12>(ctx, wb, rows, row_bytes, cp, stream);
    return launch_q8k_typed<14>(ctx, wb, rows, row_bytes, cp, stream);
}

oracle_cuda_status launch_q80_split(oracle_cuda_context* ctx, const MatvecSeqParams& sp, cudaStream_t stream);
bool q80_split_fits(const MatvecSeqParams& sp);

template <uint32_t kType, uint32_t kBatch>
oracle_cuda_status launch_seq_batch(oracle_cuda_context* ctx, MatvecSeqParams sp, cudaStream_t stream) {
    // Q8_0 vectors one at a time: lane-per-row kernel (same operations, same order)
    if constexpr (kType == 8 && kBatch == 1)
        if (q80_split_fits(sp)) return launch_q80_split(ctx, sp, stream);
    const uint64_t grid = (sp.rows + kSeqRows - 1) / kSeqRows;
    if (grid > 0x7FFFFFFFull) return fail(ctx, ORACLE_CUDA_UNSUPPORTED, "too many rows for one launch");
    const uint64_t budget = ctx->smem_budget ? ctx->smem_budget : uint64_t(ctx->max_smem_optin);
    const uint64_t prod = seq_prod_bytes(kType, kBatch);
    const uint64_t stage = uint64_t(kSeqRows) * seq_raw_slot_bytes(kType);
    uint64_t raw_stages = budget > prod ? (budget - prod) / stage : 0;
    if (raw_stages > kSeqMaxRawStages) raw_stages = kSeqMaxRawStages;
    if (raw_stages < 3) return fail(ctx, ORACLE_CUDA_UNSUPPORTED, "shared-memory budget too small for the f32-contract kernel");
    sp.raw_stages = static_cast<uint32_t>(raw_stages);
    return launch(ctx, matvec_seq_kernel<kType, kBatch>, dim3(static_cast<uint32_t>(grid)), dim3(kSeqThreads),
                  static_cast<size_t>(prod + raw_stages * stage), stream, false, sp);
}

template <uint32_t kType>
oracle_cuda_status launch_seq_typed(oracle_cuda_context* ctx, const MatvecSeqParams& sp, uint32_t batch,
                                    cudaStream_t stream) {
    switch (batch) {
        case 1: return launch_seq_batch<kType, 1>(ctx, sp, stream);
        case 2: return launch_seq_batch<kType, 2>(ctx, sp, stream);
        case 3: return launch_seq_batch<kType, 3>(ctx, sp, stream);
        default: return launch_seq_batch<kType, 4>(ctx, sp, stream);
    }
}

// Oracle's f32 contract, bit-exact: sequential f32 sum per row (matvec_seq.cuh).
// Up to 4 activation vectors per launch (2 for the K-quants, whose chunks are longer).
oracle_cuda_status launch_f32(oracle_cuda_context* ctx, uint32_t type, const void* w, uint64_t rows, uint64_t cols,
                              uint64_t row_bytes, const float* x, uint64_t batch, float* y, cudaStream_t stream) {
    if (cols > 0xFFFFFFFFull) return fail(ctx, ORACLE_CUDA_UNSUPPORTED, "rows longer than 2^32 elements");
    const uint64_t per_launch = seq_chunk_elems(type) > 128 ? 2 : kSeqMaxBatch;
    for (uint64_t b0 = 0; b0 < batch; b0 += per_launch) {
        MatvecSeqParams sp{};
        sp.w = static_cast<const uint8_t*>(w);
        sp.x = x + b0 * cols;
        sp.y = y + b0 * rows;
        sp.rows = rows;
        sp.row_bytes = row_bytes;
        sp.k = static_cast<uint32_t>(cols);
        const uint32_t nb = static_cast<uint32_t>(batch - b0 < per_launch ? batch - b0 : per_launch);
        oracle_cuda_status s;
        switch (type) {
            case kTypeF32: s = launch_seq_typed<0>(ctx, sp, nb, stream); break;
            case kTypeF16: s = launch_seq_typed<1>(ctx, sp, nb, stream); break;
            case kTypeBF16: s = launch_seq_typed<30>(ctx, sp, nb, stream); break;
            case kTypeQ8_0: s = launch_seq_typed<8>(ctx, sp, nb, stream); break;
            case kTypeQ4_K: s = launch_seq_typed<12>(ctx, sp, nb, stream); break;
            case kTypeQ5_K: s = launch_seq_typed<13>(ctx, sp, nb, stream); break;
            case kTypeQ6_K: s = launch_seq_typed<14>(ctx, sp, nb, stream); break;
            default: return fail(ctx, check_decodable(type));
        }
        if (s != ORACLE_CUDA_OK) return s;
    }
    return ORACLE_CUDA_OK;
}

template <uint32_t kType>
oracle_cuda_status launch_decode_typed(oracle_cuda_context* ctx, const uint8_t* w, uint64_t rows, uint64_t cols,
                                       uint64_t row_bytes, float* out, cudaStream_t stream) {
    const uint64_t total = rows * ((cols + 3) / 4);
    uint64_t blocks = (total + 255) / 256;
    const uint64_t cap = uint64_t(ctx->sm_count) * 8;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    return launch(ctx, decode_rows_kernel<kType>, dim3(static_cast<uint32_t>(blocks)), dim3(256), 0, stream, false, w,
                  rows, static_cast<uint32_t>(cols), row_bytes, out);
}

oracle_cuda_status launch_decode(oracle_cuda_context* ctx, uint32_t type, const void* w, uint64_t rows, uint64_t cols,
                                 uint64_t row_bytes, float* out, cudaStream_t stream) {
    const uint8_t* wb = static_cast<const uint8_t*>(w);
    switch (type) {
        case kTypeF32: return launch_decode_typed<0>(ctx, wb, rows, cols, row_bytes, out, stream);
        case kTypeF16: return launch_decode_typed<1>(ctx, wb, rows, cols, row_bytes, out, stream);
        case kTypeBF16: return launch_decode_typed<30>(ctx, wb, rows, cols, row_bytes, out, stream);
        case kTypeQ8_0: return launch_decode_typed<8>(ctx, wb, rows, cols, row_bytes, out, stream);
        case kTypeQ4_K: return launch_decode_typed<12>(ctx, wb, rows, cols, row_bytes, out, stream);
        case kTypeQ5_K: return launch_decode_typed<13>(ctx, wb, rows, cols, row_bytes, out, stream);
        case kTypeQ6_K: return launch_decode_typed<14>(ctx, wb, rows, cols, row_bytes, out, stream);
        default: return fail(ctx, check_decodable(type));
    }
}

bool batch_q8k_fits(oracle_cuda_context* ctx, const void* w, uint64_t rows, uint64_t cols);
oracle_cuda_status launch_q8k_batch(oracle_cuda_context* ctx, uint32_t type, const void* w, uint64_t rows,
                                    uint64_t cols, uint64_t row_bytes, const float* x, uint32_t batch, float* y,
                                    cudaStream_t stream);

// Validation shared by the device and host matvec entry points.
oracle_cuda_status validate_matvec(oracle_cuda_context* ctx, int contract, uint32_t type, uint64_t rows, uint64_t cols,
                                   uint64_t w_nbytes, uint64_t x_len, uint64_t y_len, uint64_t* row_bytes,
                                   uint64_t* batch) {
    if (contract != ORACLE_CUDA_CONTRACT_F32 && contract != ORACLE_CUDA_CONTRACT_Q8K)
        return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "unknown arithmetic contract " + std::to_string(contract));
    if (Error e = check_matvec(type, rows, cols, w_nbytes, x_len, y_len, row_bytes, batch)) return fail(ctx, e);
    if (contract == ORACLE_CUDA_CONTRACT_Q8K && !q8k_dot_type(type))
        return fail(ctx, ORACLE_CUDA_UNSUPPORTED,
                    "Q8_K integer dot supports q4_K and q6_K weights, not GGML type " + std::to_string(type));
    return ORACLE_CUDA_OK;
}

oracle_cuda_status run_matvec(oracle_cuda_context* ctx, int contract, uint32_t type, uint64_t rows, uint64_t cols,
                              uint64_t row_bytes, const void* w, const float* x, uint64_t batch, float* y,
                              cudaStream_t stream) {
    if (contract == ORACLE_CUDA_CONTRACT_F32) return launch_f32(ctx, type, w, rows, cols, row_bytes, x, batch, y, stream);
    if (batch > 1 && batch_q8k_fits(ctx, w, rows, cols)) {
        // up to 16 vectors per launch, each weight byte read once per launch
        for (uint64_t b0 = 0; b0 < batch; b0 += kBatchMax) {
            const uint64_t nbv = batch - b0 < uint64_t(kBatchMax) ? batch - b0 : uint64_t(kBatchMax);
            oracle_cuda_status s = nbv == 1 ? launch_q8k(ctx, type, w, rows, cols, row_bytes, x + b0 * cols, nullptr,
                                                         y + b0 * rows, stream)
                                            : launch_q8k_batch(ctx, type, w, rows, cols, row_bytes, x + b0 * cols,
                                                               static_cast<uint32_t>(nbv), y + b0 * rows, stream);
            if (s != ORACLE_CUDA_OK) return s;
        }
        return ORACLE_CUDA_OK;
    }
    for (uint64_t b = 0; b < batch; ++b) {
        oracle_cuda_status s = launch_q8k(ctx, type, w, rows, cols, row_bytes, x + b * cols, nullptr, y + b * rows, stream);
        if (s != ORACLE_CUDA_OK) return s;
    }
    return ORACLE_CUDA_OK;
}

template <typename T>
oracle_cuda_status grow_pinned(oracle_cuda_context* ctx, T*& p, uint64_t& have, uint64_t need) {
    if (have >= need) return ORACLE_CUDA_OK;
    if (p) cudaFreeHost(p);
    p = nullptr;
    have = 0;
    ORACLE_CUDA_TRY(ctx, cudaHostAlloc(reinterpret_cast<void**>(&p), need * sizeof(T), cudaHostAllocDefault),
                    "cudaHostAlloc");
    have = need;
    return ORACLE_CUDA_OK;
}

template <typename T>
oracle_cuda_status grow_device(oracle_cuda_context* ctx, T*& p, uint64_t& have, uint64_t need) {
    if (have >= need) return ORACLE_CUDA_OK;
    if (p) cudaFree(p);
    p = nullptr;
    have = 0;
    ORACLE_CUDA_TRY(ctx, cudaMalloc(reinterpret_cast<void**>(&p), need * sizeof(T)), "cudaMalloc");
    have = need;
    return ORACLE_CUDA_OK;
}

// The batched Q8_K kernel's limits: 16-byte aligned weights, at least one CTA
// per segment, and tile counts in 32 bits.
bool batch_q8k_fits(oracle_cuda_context* ctx, const void* w, uint64_t rows, uint64_t cols) {
    if (reinterpret_cast<uintptr_t>(w) & 15u) return false;
    const uint64_t nb = cols / 256, G = (nb + 15) / 16, T = (rows + kBatchTileRows - 1) / kBatchTileRows;
    return nb > 0 && G <= uint64_t(ctx->sm_count) && T < 0x7FFFFFFFull &&
           kBatchStageOffset + 2 * batch_stage_bytes(kTypeQ6_K) <=
               uint64_t(ctx->max_smem_optin);
}

// Batch image of x[batch][cols] (batch <= 16) into `image` (nb blocks).
oracle_cuda_status launch_batch_quantize(oracle_cuda_context* ctx, const float* x, uint32_t batch, uint32_t nb,
                                         uint8_t* image, cudaStream_t stream) {
    return launch(ctx, quantize_batch_image_kernel, dim3(2 * nb), dim3(256), 0, stream,
                  (ctx->flags & ORACLE_CUDA_FLAG_PDL) != 0, x, batch, nb, image);
}

// Batched Q8_K matvec (matvec_batch.cuh) of a batch image -> y[b][rows].
oracle_cuda_status launch_batch_matvec(oracle_cuda_context* ctx, uint32_t type, const void* w, uint64_t rows,
                                       uint64_t cols, uint64_t row_bytes, const uint8_t* image, uint32_t batch,
                                       float* y, cudaStream_t stream) {
    const uint32_t nb = static_cast<uint32_t>(cols / 256), G = (nb + 15) / 16;
    const uint64_t T = (rows + kBatchTileRows - 1) / kBatchTileRows;
    if (G > 1)
        if (oracle_cuda_status s =
                grow_device(ctx, ctx->batch_partial, ctx->batch_partial_len, G * uint64_t(batch) * rows))
            return s;
    const bool pdl = (ctx->flags & ORACLE_CUDA_FLAG_PDL) != 0;
    BatchParams bp{};
    bp.w = static_cast<const uint8_t*>(w);
    bp.image = image;
    bp.out = G > 1 ? ctx->batch_partial : y;
    bp.rows = rows;
    bp.row_bytes = row_bytes;
    bp.nb = nb;
    bp.batch = batch;
    bp.status = ctx->status;
    const uint64_t items = T * G;
    const uint32_t grid = static_cast<uint32_t>(items < uint64_t(ctx->sm_count) ? items : ctx->sm_count);
    const uint64_t budget = ctx->smem_budget ? ctx->smem_budget : uint64_t(ctx->max_smem_optin);
    const uint32_t off = kBatchStageOffset;
    const uint32_t stage = type == kTypeQ4_K ? batch_stage_bytes(12) : batch_stage_bytes(14);
    uint64_t stages = budget > off ? (budget - off) / stage : 0;
    if (stages > uint64_t(kBatchMaxStages)) stages = kBatchMaxStages;
    if (stages < 2) return fail(ctx, ORACLE_CUDA_UNSUPPORTED, "shared-memory budget too small for the batched matvec");
    bp.stages = static_cast<uint32_t>(stages);
    const size_t smem = off + stages * stage;
    oracle_cuda_status s =
        type == kTypeQ4_K
            ? launch(ctx, matvec_batch_kernel<12>, dim3(grid), dim3(kBatchThreads), smem, stream, pdl, bp)
            : launch(ctx, matvec_batch_kernel<14>, dim3(grid), dim3(kBatchThreads), smem, stream, pdl, bp);
    if (s != ORACLE_CUDA_OK || G == 1) return s;
    const uint64_t n = uint64_t(batch) * rows;
    const uint64_t blocks = (n + 255) / 256;
    return launch(ctx, batch_combine_kernel, dim3(static_cast<uint32_t>(blocks < 4096 ? blocks : 4096)), dim3(256), 0,
                  stream, pdl, static_cast<const float*>(ctx->batch_partial), y, n, G);
}

// 2..16 vectors x[b][cols] -> y[b][rows] through the context's image buffer.
oracle_cuda_status launch_q8k_batch(oracle_cuda_context* ctx, uint32_t type, const void* w, uint64_t rows,
                                    uint64_t cols, uint64_t row_bytes, const float* x, uint32_t batch, float* y,
                                    cudaStream_t stream) {
    const uint32_t nb = static_cast<uint32_t>(cols / 256);
    if (oracle_cuda_status s = grow_device(ctx, ctx->batch_image, ctx->batch_image_len,
                                           uint64_t(nb) * kBatchImageBlockBytes))
        return s;
    if (oracle_cuda_status s = launch_batch_quantize(ctx, x, batch, nb, ctx->batch_image, stream)) return s;
    return launch_batch_matvec(ctx, type, w, rows, cols, row_bytes, ctx->batch_image, batch, y, stream);
}

// The device bytes a host-pointer call reads for a weight span: the resident
// copy of a registered span, else a fresh copy into the staging buffer at
// byte `stage_off` (16-byte aligned; the caller advances it by the span).
// The reference reads the caller's bytes on every call; so does this, unless
// the caller has promised (by registering) that they never change.
oracle_cuda_status weight_bytes_for_call(oracle_cuda_context* ctx, uint32_t type, uint64_t rows, uint64_t cols,
                                         const void* host, uint64_t nbytes, uint64_t stage_off, cudaStream_t stream,
                                         const void** dev) {
    auto it = ctx->resident.find(std::make_tuple(host, nbytes, type, rows, cols));
    if (it != ctx->resident.end()) {
        *dev = it->second->dev;
        return ORACLE_CUDA_OK;
    }
    ORACLE_CUDA_TRY(ctx, cudaMemcpyAsync(ctx->stage_w + stage_off, host, nbytes, cudaMemcpyHostToDevice, stream),
                    "cudaMemcpyAsync(weight)");
    *dev = ctx->stage_w + stage_off;
    return ORACLE_CUDA_OK;
}

// Bytes of staging needed for an unregistered span (0 for a registered one).
uint64_t weight_stage_need(const oracle_cuda_context* ctx, uint32_t type, uint64_t rows, uint64_t cols,
                           const void* host, uint64_t nbytes) {
    if (ctx->resident.count(std::make_tuple(host, nbytes, type, rows, cols))) return 0;
    return (nbytes + 16 + 15) / 16 * 16;  // +16: aligned word reads stay inside
}

// Page-locked host memory the device reaches at the same address (unified
// addressing maps cudaHostAlloc'd and registered memory so).
bool is_device_mapped_host(const void* p) {
    cudaPointerAttributes attr{};
    if (cudaPointerGetAttributes(&attr, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return attr.type == cudaMemoryTypeHost && attr.devicePointer == p;
}

bool is_pinned(const void* p) {
    cudaPointerAttributes attr{};
    if (cudaPointerGetAttributes(&attr, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return attr.type == cudaMemoryTypeHost;
}

}  // namespace

// ====================================================================== C ABI

extern "C" {

int oracle_cuda_abi_version(void) { return ORACLE_CUDA_ABI_VERSION; }

const char* oracle_cuda_status_name(oracle_cuda_status s) {
    switch (s) {
        case ORACLE_CUDA_OK: return "OK";
        case ORACLE_CUDA_INVALID_ARGUMENT: return "INVALID_ARGUMENT";
        case ORACLE_CUDA_OUT_OF_RANGE: return "OUT_OF_RANGE";
        case ORACLE_CUDA_OVERFLOW: return "OVERFLOW";
        case ORACLE_CUDA_RUNTIME_ERROR: return "RUNTIME_ERROR";
        case ORACLE_CUDA_LOGIC_ERROR: return "LOGIC_ERROR";
        case ORACLE_CUDA_CUDA_ERROR: return "CUDA_ERROR";
        case ORACLE_CUDA_OUT_OF_MEMORY: return "OUT_OF_MEMORY";
        case ORACLE_CUDA_DEVICE_TIMEOUT: return "DEVICE_TIMEOUT";
        case ORACLE_CUDA_UNSUPPORTED: return "UNSUPPORTED";
    }
    return "UNKNOWN";
}

const char* oracle_cuda_last_error(const oracle_cuda_context* ctx) {
    return ctx ? ctx->last_error.c_str() : g_thread_error.c_str();
}

oracle_cuda_status oracle_ggml_type_layout(uint32_t type, uint64_t* block_elements, uint64_t* bytes_per_block,
                                           int* quantized, const char** name) {
    const TypeLayout* l = type_layout(type);
    if (!l) return fail(nullptr, ORACLE_CUDA_INVALID_ARGUMENT, "unsupported GGML tensor type: " + std::to_string(type));
    if (block_elements) *block_elements = l->block_elements;
    if (bytes_per_block) *bytes_per_block = l->bytes_per_block;
    if (quantized) *quantized = l->quantized ? 1 : 0;
    if (name) *name = l->name;
    return ORACLE_CUDA_OK;
}

oracle_cuda_status oracle_ggml_row_byte_size(uint64_t row_elements, uint32_t type, uint64_t* out) {
    if (!out) return fail(nullptr, ORACLE_CUDA_INVALID_ARGUMENT, "output pointer is null");
    if (Error e = row_byte_size(row_elements, type, out)) return fail(nullptr, e);
    return ORACLE_CUDA_OK;
}

// The host C library's expf / log1pf corrections (common.cuh, g_libm), generated
// at build time by csrc/libm_tables.c and linked into this library as a blob.
extern "C" const unsigned char oracle_libm_blob[];
extern "C" const unsigned char oracle_libm_blob_end[];

namespace {

std::mutex g_libm_mutex;
bool g_libm_loaded[64] = {};

// Once per device, with that device current: copy the tables into g_libm.
oracle_cuda_status libm_tables_load(int device) {
    if (device < 0 || device >= 64) return fail(nullptr, ORACLE_CUDA_UNSUPPORTED, "device index too large");
    std::lock_guard<std::mutex> lock(g_libm_mutex);
    if (g_libm_loaded[device]) return ORACLE_CUDA_OK;
    const uint64_t bytes = static_cast<uint64_t>(oracle_libm_blob_end - oracle_libm_blob);
    uint32_t hdr[kLibmHeaderWords] = {};
    if (bytes >= sizeof hdr) std::memcpy(hdr, oracle_libm_blob, sizeof hdr);
    const auto pow2 = [](uint32_t v) { return v != 0 && (v & (v - 1)) == 0; };
    const uint64_t words = kLibmHeaderWords + 33ull * hdr[1] + 32ull * hdr[2] + 2ull * (uint64_t(hdr[3]) + hdr[4]);
    if (bytes < sizeof hdr || hdr[0] != 0x324D424Cu || !pow2(hdr[1]) || !pow2(hdr[2]) || bytes != words * 4 ||
        words > kLibmMaxWords)
        return fail(nullptr, ORACLE_CUDA_CUDA_ERROR, "the library's expf/log1pf tables are missing or malformed");
    const cudaError_t e = cudaMemcpyToSymbol(g_libm, oracle_libm_blob, bytes);
    if (e != cudaSuccess) return cuda_fail(nullptr, e, "cudaMemcpyToSymbol(expf/log1pf tables)");
    g_libm_loaded[device] = true;
    return ORACLE_CUDA_OK;
}

}  // namespace

oracle_cuda_status oracle_cuda_create(int device, oracle_cuda_context** out) {
    if (!out) return fail(nullptr, ORACLE_CUDA_INVALID_ARGUMENT, "output pointer is null");
    *out = nullptr;
    int count = 0;
    cudaError_t e = cudaGetDeviceCount(&count);
    if (e != cudaSuccess) return cuda_fail(nullptr, e, "cudaGetDeviceCount");
    if (device < 0 || device >= count)
        return fail(nullptr, ORACLE_CUDA_OUT_OF_RANGE, "CUDA device index " + std::to_string(device) + " out of range");
    if ((e = cudaSetDevice(device)) != cudaSuccess) return cuda_fail(nullptr, e, "cudaSetDevice");
    cudaDeviceProp prop{};
    if ((e = cudaGetDeviceProperties(&prop, device)) != cudaSuccess)
        return cuda_fail(nullptr, e, "cudaGetDeviceProperties");
    if (prop.major != 10)
        return fail(nullptr, ORACLE_CUDA_UNSUPPORTED,
                    std::string("this library is built for sm_100a (B200); device is ") + prop.name);
    if (oracle_cuda_status ls = libm_tables_load(device)) return ls;
    auto* ctx = new oracle_cuda_context();
    ctx->device = device;
    ctx->sm_count = prop.multiProcessorCount;
    ctx->max_smem_optin = static_cast<int>(prop.sharedMemPerBlockOptin);
    // All of it: with 16 consumer warps the register file already holds one
    // stream CTA per SM, so a deep stage ring (prefetching while a programmatic
    // dependent launch waits for its predecessor) is worth more than room for a
    // second CTA.  ORACLE_CUDA_SMEM_BUDGET (bytes) overrides it for tuning.
    ctx->smem_budget = prop.sharedMemPerBlockOptin;
    if (const char* env = std::getenv("ORACLE_CUDA_STAGE_BYTES")) {
        const unsigned long long v = std::strtoull(env, nullptr, 10);
        if (v >= 4096 && v <= 200000) ctx->stage_target = v;
    }
    if (const char* env = std::getenv("ORACLE_CUDA_PROGRAM_STAGE_BYTES")) {
        const unsigned long long v = std::strtoull(env, nullptr, 10);
        if (v >= 4096 && v <= 200000) ctx->program_stage_target = v;
    }
    if (const char* env = std::getenv("ORACLE_CUDA_MAX_INFLIGHT")) {
        const unsigned long long v = std::strtoull(env, nullptr, 10);
        if (v >= 1 && v <= 16) ctx->max_inflight = static_cast<uint32_t>(v);
    }
    if (const char* env = std::getenv("ORACLE_CUDA_COPY_CHUNK")) {
        const unsigned long long v = std::strtoull(env, nullptr, 10);
        if (v >= 4096 && v <= 196608 && v % 16 == 0) ctx->copy_chunk = static_cast<uint32_t>(v);
    }
    if (const char* env = std::getenv("ORACLE_CUDA_SMEM_BUDGET")) {
        const unsigned long long v = std::strtoull(env, nullptr, 10);
        if (v >= 16384 && v <= static_cast<unsigned long long>(ctx->max_smem_optin)) ctx->smem_budget = v;
    }
    if (const char* env = std::getenv("ORACLE_CUDA_GEMM_PAIR")) ctx->gemm_pair = std::strtoull(env, nullptr, 10) != 0;
    if ((e = cudaMalloc(reinterpret_cast<void**>(&ctx->status), sizeof(DeviceStatus))) != cudaSuccess) {
        delete ctx;
        return cuda_fail(nullptr, e, "cudaMalloc(status)");
    }
    cudaMemset(ctx->status, 0, sizeof(DeviceStatus));
    if ((e = cudaMalloc(reinterpret_cast<void**>(&ctx->program_counters),
                        kProgramCounters * sizeof(unsigned int))) != cudaSuccess) {
        cudaFree(ctx->status);
        delete ctx;
        return cuda_fail(nullptr, e, "cudaMalloc(program counters)");
    }
    cudaMemset(ctx->program_counters, 0, kProgramCounters * sizeof(unsigned int));
    *out = ctx;
    return ORACLE_CUDA_OK;
}

oracle_cuda_status oracle_cuda_destroy(oracle_cuda_context* ctx) {
    if (!ctx) return ORACLE_CUDA_OK;
    cudaSetDevice(ctx->device);
    cudaDeviceSynchronize();
    for (auto& kv : ctx->resident) {
        cudaFree(kv.second->dev);
        delete kv.second;
    }
    if (ctx->stage_w) cudaFree(ctx->stage_w);
    if (ctx->pin_x) cudaFreeHost(ctx->pin_x);
    if (ctx->pin_y) cudaFreeHost(ctx->pin_y);
    if (ctx->dev_x) cudaFree(ctx->dev_x);
    if (ctx->dev_y) cudaFree(ctx->dev_y);
    if (ctx->status) cudaFree(ctx->status);
    if (ctx->program_counters) cudaFree(ctx->program_counters);
    if (ctx->image_scratch) cudaFree(ctx->image_scratch);
    if (ctx->act_scratch) cudaFree(ctx->act_scratch);
    if (ctx->gemm_x) cudaFree(ctx->gemm_x);
    if (ctx->argmax_key) cudaFree(ctx->argmax_key);
    if (ctx->batch_image) cudaFree(ctx->batch_image);
    if (ctx->batch_partial) cudaFree(ctx->batch_partial);
    delete ctx;
    return ORACLE_CUDA_OK;
}

oracle_cuda_status oracle_cuda_set_flags(oracle_cuda_context* ctx, uint32_t flags) {
    if (!ctx) return fail(nullptr, ORACLE_CUDA_INVALID_ARGUMENT, "context is null");
    ctx->flags = flags;
    return ok(ctx);
}

uint64_t oracle_cuda_launch_count(const oracle_cuda_context* ctx) { return ctx ? ctx->launches : 0; }

oracle_cuda_status oracle_cuda_device_status(oracle_cuda_context* ctx) {
    if (!ctx) return fail(nullptr, ORACLE_CUDA_INVALID_ARGUMENT, "context is null");
    ORACLE_CUDA_TRY(ctx, cudaSetDevice(ctx->device), "cudaSetDevice");
    DeviceStatus st{};
    ORACLE_CUDA_TRY(ctx, cudaDeviceSynchronize(), "cudaDeviceSynchronize");
    ORACLE_CUDA_TRY(ctx, cudaMemcpy(&st, ctx->status, sizeof st, cudaMemcpyDeviceToHost), "cudaMemcpy(status)");
    ORACLE_CUDA_TRY(ctx, cudaMemset(ctx->status, 0, sizeof st), "cudaMemset(status)");
    if (st.code != kDevOk)  // an aborted program may have left its counters set
        ORACLE_CUDA_TRY(ctx, cudaMemset(ctx->program_counters, 0, kProgramCounters * sizeof(unsigned int)),
                        "cudaMemset(program counters)");
    if (st.code == 3u)  // causal_attention_step (reference_kernels.cpp:170-172)
        return fail(ctx, ORACLE_CUDA_RUNTIME_ERROR, "causal attention softmax normalization failed");
    if (st.code == kDevKvOverflow)  // KvCache::append (hybrid_cache.cpp)
        return fail(ctx, ORACLE_CUDA_OVERFLOW,
                    "KV cache capacity exceeded at position " + std::to_string(st.where));
    if (st.code == kDevLogitsNaN)  // Sampler::sample (sampler.cpp:34-36)
        return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "logits contain NaN");
    if (st.code == kDevLogitsNonFinite)  // Sampler::sample (sampler.cpp:42-44)
        return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "logits contain no finite candidates");
    if (st.code == kDevBadIndex)  // embedding_row (qwen35_forward.cpp:59-61)
        return fail(ctx, ORACLE_CUDA_OUT_OF_RANGE,
                    "token id " + std::to_string(st.where) + " exceeds the embedding row count");
    if (st.code != kDevOk)
        return fail(ctx, ORACLE_CUDA_DEVICE_TIMEOUT,
                    "kernel wait timed out at site " + std::to_string(st.where) + " in block " +
                        std::to_string(st.block));
    return ok(ctx);
}

oracle_cuda_status oracle_cuda_selftest_bounded_wait(oracle_cuda_context* ctx, uint64_t limit_ns) {
    if (!ctx) return fail(nullptr, ORACLE_CUDA_INVALID_ARGUMENT, "context is null");
    if (limit_ns == 0 || limit_ns > 2000000000ull)
        return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "self-test deadline must be in (0, 2 s]");
    ORACLE_CUDA_TRY(ctx, cudaSetDevice(ctx->device), "cudaSetDevice");
    oracle_cuda_status s = launch(ctx, bounded_wait_selftest_kernel, dim3(1), dim3(32), 0, nullptr, false,
                                  ctx->status, static_cast<unsigned long long>(limit_ns));
    return s == ORACLE_CUDA_OK ? ok(ctx) : s;
}

oracle_cuda_status oracle_cuda_decode_rows(oracle_cuda_context* ctx, uint32_t type, uint64_t rows, uint64_t cols,
                                           const void* w_dev, uint64_t w_nbytes, float* out_dev, uint64_t out_len,
                                           void* stream) {
    if (!ctx) return fail(nullptr, ORACLE_CUDA_INVALID_ARGUMENT, "context is null");
    uint64_t rb = 0, total = 0, elems = 0;
    if (rows == 0) return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "GGUF tensor must have at least one dimension");
    if (Error e = row_byte_size(cols, type, &rb)) return fail(ctx, e);
    if (!checked_mul(rows, rb, &total))
        return fail(ctx, ORACLE_CUDA_OVERFLOW, "GGUF tensor byte size exceeds addressable size");
    if (w_nbytes != total)
        return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "GGUF tensor byte size does not match row geometry");
    if (Error e = check_decodable(type)) return fail(ctx, e);
    if (!checked_mul(rows, cols, &elems))
        return fail(ctx, ORACLE_CUDA_OVERFLOW, "mapped tensor element count overflow");
    if (out_len != elems)
        return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "mapped tensor decode output length mismatch");
    if (cols > 0xFFFFFFFFull) return fail(ctx, ORACLE_CUDA_UNSUPPORTED, "rows longer than 2^32 elements");
    if (Error e = check_weight_pointer(type, w_dev)) return fail(ctx, e);
    if (!out_dev) return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "output pointer is null");
    ORACLE_CUDA_TRY(ctx, cudaSetDevice(ctx->device), "cudaSetDevice");
    oracle_cuda_status s = launch_decode(ctx, type, w_dev, rows, cols, rb, out_dev, static_cast<cudaStream_t>(stream));
    return s == ORACLE_CUDA_OK ? ok(ctx) : s;
}

oracle_cuda_status oracle_cuda_quantize_q8_k(oracle_cuda_context* ctx, const float* x_dev, uint64_t cols,
                                             uint64_t batch, void* q8k_dev, uint64_t q8k_nbytes, void* stream) {
    if (!ctx) return fail(nullptr, ORACLE_CUDA_INVALID_ARGUMENT, "context is null");
    if (cols == 0 || batch == 0) return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "Q8_K quantize dimensions must be non-zero");
    uint64_t rb = 0;
    if (Error e = row_byte_size(cols, kTypeQ8_K, &rb)) return fail(ctx, e);
    uint64_t need = 0;
    if (!checked_mul(rb, batch, &need)) return fail(ctx, ORACLE_CUDA_OVERFLOW, "Q8_K output size overflow");
    if (q8k_nbytes != need) return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "Q8_K output byte size mismatch");
    if (!x_dev || !q8k_dev) return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "null pointer");
    if (reinterpret_cast<uintptr_t>(x_dev) % 4 || reinterpret_cast<uintptr_t>(q8k_dev) % 4)
        return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "Q8_K buffers must be 4-byte aligned");
    ORACLE_CUDA_TRY(ctx, cudaSetDevice(ctx->device), "cudaSetDevice");
    const uint64_t blocks = (cols / 256) * batch;
    const uint64_t grid = (blocks * 32 + 255) / 256;
    if (grid > 0x7FFFFFFFull) return fail(ctx, ORACLE_CUDA_UNSUPPORTED, "too many Q8_K blocks for one launch");
    oracle_cuda_status s = launch(ctx, quantize_q8k_kernel, dim3(static_cast<uint32_t>(grid)), dim3(256), 0,
                                  static_cast<cudaStream_t>(stream), false, x_dev, cols, batch,
                                  static_cast<uint8_t*>(q8k_dev));
    return s == ORACLE_CUDA_OK ? ok(ctx) : s;
}

oracle_cuda_status oracle_cuda_storage_matvec(oracle_cuda_context* ctx, int contract, uint32_t type, uint64_t rows,
                                              uint64_t cols, const void* w_dev, uint64_t w_nbytes, const float* x_dev,
                                              uint64_t x_len, float* y_dev, uint64_t y_len, void* stream) {
    if (!ctx) return fail(nullptr, ORACLE_CUDA_INVALID_ARGUMENT, "context is null");
    uint64_t rb = 0, batch = 0;
    oracle_cuda_status s = validate_matvec(ctx, contract, type, rows, cols, w_nbytes, x_len, y_len, &rb, &batch);
    if (s != ORACLE_CUDA_OK) return s;
    if (Error e = check_weight_pointer(type, w_dev)) return fail(ctx, e);
    if (!x_dev || !y_dev) return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "activation or output pointer is null");
    ORACLE_CUDA_TRY(ctx, cudaSetDevice(ctx->device), "cudaSetDevice");
    s = run_matvec(ctx, contract, type, rows, cols, rb, w_dev, x_dev, batch, y_dev, static_cast<cudaStream_t>(stream));
    return s == ORACLE_CUDA_OK ? ok(ctx) : s;
}

uint64_t oracle_cuda_batch_image_bytes(uint64_t cols) {
    return cols == 0 || cols % 256 != 0 ? 0 : cols / 256 * kBatchImageBlockBytes;
}

oracle_cuda_status oracle_cuda_batch_quantize(oracle_cuda_context* ctx, const float* x_dev, uint64_t cols,
                                              uint32_t batch, void* image_dev, uint64_t image_nbytes, void* stream) {
    if (!ctx) return fail(nullptr, ORACLE_CUDA_INVALID_ARGUMENT, "context is null");
    if (cols == 0 || cols % 256 != 0)
        return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "Q8_K activations need a multiple of 256 columns");
    if (batch == 0 || batch > uint32_t(kBatchMax))
        return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "a batch image holds 1 to 16 vectors");
    if (cols / 256 > 0xFFFFFFFull) return fail(ctx, ORACLE_CUDA_UNSUPPORTED, "rows longer than 2^36 elements");
    if (image_nbytes < oracle_cuda_batch_image_bytes(cols))
        return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "batch image buffer too small");
    if (!x_dev || !image_dev || (reinterpret_cast<uintptr_t>(image_dev) & 15u))
        return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "activation pointer null or image pointer not 16-byte aligned");
    ORACLE_CUDA_TRY(ctx, cudaSetDevice(ctx->device), "cudaSetDevice");
    const oracle_cuda_status s = launch_batch_quantize(ctx, x_dev, batch, static_cast<uint32_t>(cols / 256),
                                                       static_cast<uint8_t*>(image_dev),
                                                       static_cast<cudaStream_t>(stream));
    return s == ORACLE_CUDA_OK ? ok(ctx) : s;
}

namespace {
// The checks of oracle_cuda_batch_quantize, shared by the fused form.
oracle_cuda_status check_batch_image_args(oracle_cuda_context* ctx, const float* x_dev, uint64_t cols, uint32_t batch,
                                          const void* image_dev, uint64_t image_nbytes) {
    if (cols == 0 || cols % 256 != 0)
        return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "Q8_K activations need a multiple of 256 columns");
    if (batch == 0 || batch > uint32_t(kBatchMax))
        return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "a batch image holds 1 to 16 vectors");
    if (cols / 256 > 0xFFFFFFFull) return fail(ctx, ORACLE_CUDA_UNSUPPORTED, "rows longer than 2^36 elements");
    if (image_nbytes < oracle_cuda_batch_image_bytes(cols))
        return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "batch image buffer too small");
    if (!x_dev || !image_dev || (reinterpret_cast<uintptr_t>(image_dev) & 15u))
        return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "activation pointer null or image pointer not 16-byte aligned");
    return ORACLE_CUDA_OK;
}
}  // namespace

oracle_cuda_status oracle_cuda_batch_norm_quantize(oracle_cuda_context* ctx, const float* a_dev, const float* b_dev,
                                                   float* sum_dev, const float* weight_dev, float eps, uint64_t cols,
                                                   uint32_t batch, void* image_dev, uint64_t image_nbytes,
                                                   void* stream) {
    if (!ctx) return fail(nullptr, ORACLE_CUDA_INVALID_ARGUMENT, "context is null");
    if (oracle_cuda_status s = check_batch_image_args(ctx, a_dev, cols, batch, image_dev, image_nbytes)) return s;
    if (cols > kBatchNormMaxWidth)
        return fail(ctx, ORACLE_CUDA_UNSUPPORTED, "batched norm rows of more than 8192 columns");
    if (!weight_dev || !(eps > 0.0f) || !std::isfinite(eps))
        return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "norm weights null or epsilon not positive and finite");
    if (sum_dev && (sum_dev == a_dev || sum_dev == b_dev))
        return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "the sum must not overwrite an input");
    ORACLE_CUDA_TRY(ctx, cudaSetDevice(ctx->device), "cudaSetDevice");
    const oracle_cuda_status s =
        launch(ctx, batch_norm_quantize_kernel, dim3(kBatchMax), dim3(kBatchNormThreads), 0,
               static_cast<cudaStream_t>(stream), (ctx->flags & ORACLE_CUDA_FLAG_PDL) != 0, a_dev, b_dev, sum_dev,
               weight_dev, eps, batch, static_cast<uint32_t>(cols), static_cast<uint8_t*>(image_dev));
    return s == ORACLE_CUDA_OK ? ok(ctx) : s;
}

oracle_cuda_status oracle_cuda_batch_matvec(oracle_cuda_context* ctx, uint32_t type, uint64_t rows, uint64_t cols,
                                            const void* w_dev, uint64_t w_nbytes, const void* image_dev,
                                            uint64_t image_nbytes, uint32_t batch, float* y_dev, uint64_t y_len,
                                            void* stream) {
    if (!ctx) return fail(nullptr, ORACLE_CUDA_INVALID_ARGUMENT, "context is null");
    if (batch == 0 || batch > uint32_t(kBatchMax))
        return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "a batch image holds 1 to 16 vectors");
    uint64_t rb = 0, nvec = 0;
    oracle_cuda_status s = validate_matvec(ctx, ORACLE_CUDA_CONTRACT_Q8K, type, rows, cols, w_nbytes,
                                           uint64_t(batch) * cols, y_len, &rb, &nvec);
    if (s != ORACLE_CUDA_OK) return s;
    if (image_nbytes < oracle_cuda_batch_image_bytes(cols))
        return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "batch image buffer too small");
    if (!image_dev || !y_dev || (reinterpret_cast<uintptr_t>(image_dev) & 15u))
        return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "output pointer null or image pointer not 16-byte aligned");
    if (!batch_q8k_fits(ctx, w_dev, rows, cols))
        return fail(ctx, ORACLE_CUDA_UNSUPPORTED,
                    "batched matvec needs 16-byte aligned weights and at most one 4096-column segment per SM");
    ORACLE_CUDA_TRY(ctx, cudaSetDevice(ctx->device), "cudaSetDevice");
    s = launch_batch_matvec(ctx, type, w_dev, rows, cols, rb, static_cast<const uint8_t*>(image_dev), batch, y_dev,
                            static_cast<cudaStream_t>(stream));
    return s == ORACLE_CUDA_OK ? ok(ctx) : s;
}

oracle_cuda_status oracle_cuda_matvec_q8k_prequantized(oracle_cuda_context* ctx, uint32_t type, uint64_t rows,
                                                       uint64_t cols, const void* w_dev, uint64_t w_nbytes,
                                                       const void* q8k_dev, uint64_t q8k_nbytes, float* y_dev,
                                                       uint64_t y_len, void* stream) {
    if (!ctx) return fail(nullptr, ORACLE_CUDA_INVALID_ARGUMENT, "context is null");
    uint64_t qrb = 0;
    if (cols == 0 || rows == 0)
        return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "reference matvec dimensions must be non-zero");
    if (Error e = row_byte_size(cols, kTypeQ8_K, &qrb)) return fail(ctx, e);
    if (q8k_nbytes == 0 || q8k_nbytes % qrb)
        return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "reference matvec vector length mismatch");
    const uint64_t batch = q8k_nbytes / qrb;
    uint64_t rb = 0, b2 = 0;
    oracle_cuda_status s = validate_matvec(ctx, ORACLE_CUDA_CONTRACT_Q8K, type, rows, cols, w_nbytes, batch * cols,
                                           y_len, &rb, &b2);
    if (s != ORACLE_CUDA_OK) return s;
    if (Error e = check_weight_pointer(type, w_dev)) return fail(ctx, e);
    if (!q8k_dev || !y_dev) return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "activation or output pointer is null");
    if (reinterpret_cast<uintptr_t>(q8k_dev) % 4)
        return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "Q8_K buffers must be 4-byte aligned");
    ORACLE_CUDA_TRY(ctx, cudaSetDevice(ctx->device), "cudaSetDevice");
    for (uint64_t b = 0; b < batch; ++b) {
        s = launch_q8k(ctx, type, w_dev, rows, cols, rb, nullptr, static_cast<const uint8_t*>(q8k_dev) + b * qrb,
                       y_dev + b * rows, static_cast<cudaStream_t>(stream));
        if (s != ORACLE_CUDA_OK) return s;
    }
    return ok(ctx);
}

struct oracle_cuda_peer_group {
    oracle_cuda_context* ctx = nullptr;
    uint32_t rank = 0, world = 1;
    uint64_t data_bytes = 0;
    uint8_t* local = nullptr;                 // 256-byte header (counter, epoch) + data
    uint8_t* mapped[kMaxPeers] = {};          // every rank's allocation, mapped here (own = local)
    bool connected = false;
};

namespace {

constexpr uint64_t kGatherHeader = 256;  // arrival counter, epoch, ..., op counters
constexpr uint32_t kGatherOpCounters = 16;  // uint index of the [2][kProgramMaxOps] op counters
constexpr uint32_t kGatherXdep = 2;         // uint index of the sharded programs' announcement counter
constexpr uint32_t kGatherStep = 3;         // uint index of the sharded programs' step counter

// sh / step: head-sharded programs (oracle_cuda_matvec_program_sharded), else null.
oracle_cuda_status program_run(oracle_cuda_context* ctx, const oracle_cuda_matvec_op_ex* ops, uint32_t n_ops,
                               void* stream, const oracle_cuda_peer_group* group,
                               const oracle_cuda_sharded_op* sh = nullptr,
                               const oracle_cuda_sharded_step* step = nullptr);

oracle_cuda_status program_run_base(oracle_cuda_context* ctx, const oracle_cuda_matvec_op* ops, uint32_t n_ops,
                                    void* stream, const oracle_cuda_peer_group* group) {
    if (!ctx) return fail(nullptr, ORACLE_CUDA_INVALID_ARGUMENT, "context is null");
    if (!ops || n_ops == 0 || n_ops > kProgramMaxOps)
        return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT,
                    "a matvec program holds 1 to " + std::to_string(kProgramMaxOps) + " ops");
    oracle_cuda_matvec_op_ex ex[kProgramMaxOps] = {};
    for (uint32_t k = 0; k < n_ops; ++k) ex[k].base = ops[k];
    return program_run(ctx, ex, n_ops, stream, group);
}

}  // namespace

oracle_cuda_status oracle_cuda_matvec_program(oracle_cuda_context* ctx, const oracle_cuda_matvec_op* ops,
                                              uint32_t n_ops, void* stream) {
    return program_run_base(ctx, ops, n_ops, stream, nullptr);
}

oracle_cuda_status oracle_cuda_matvec_program_ex(oracle_cuda_context* ctx, const oracle_cuda_matvec_op_ex* ops,
                                                 uint32_t n_ops, void* stream) {
    return program_run(ctx, ops, n_ops, stream, nullptr);
}

namespace {

// Rows per stage, segment-major streaming and the shared-memory stage ring of
// a program whose ops and activation image bytes (pp.act_bytes) are set.  One
// planner for every entry point that launches matvec_program_kernel, so they
// all stream the same stages for the same ops.
oracle_cuda_status plan_program_ring(ProgramParams& pp, uint64_t smem_budget, uint64_t stage_target,
                                     std::string& why) {
    why = "matvec program rows too long for the shared-memory stage ring";
    if (pp.act_bytes > 96 * 1024) return ORACLE_CUDA_UNSUPPORTED;
    const uint64_t budget = smem_budget - stream_barrier_bytes(16) - pp.act_bytes;
    uint64_t stage = 0;
    // rows per stage: up to two per consumer warp (Q4_K rows of <= 16
    // super-blocks are computed in pairs), within the stage target, and
    // small enough that kProgramMinStages stages fit beside the images
    uint64_t target = budget / kProgramMinStages;
    if (target > stage_target) target = stage_target;
    // Q4_K rows of more than 16 super-blocks stream segment-major: a stage
    // holds one 16-super-block segment of up to two rows per consumer warp
    for (uint32_t k = 0; k < pp.n_ops; ++k) {
        ProgramOp& p = pp.ops[k];
        // Q6_K: every segment a 16-byte multiple (nb % 8 == 0) from a
        // 16-byte aligned weight pointer (bulk copies), one row per warp
        const bool q6 = p.type == kTypeQ6_K;
        p.segmented = (p.nb > kSegmentBlocks &&
                       (p.type == kTypeQ4_K || (q6 && p.nb % 8 == 0 && reinterpret_cast<uintptr_t>(p.w) % 16 == 0)))
                          ? 1u
                          : 0u;
        const uint64_t rb = p.segmented ? uint64_t(kSegmentBlocks) * (q6 ? 210u : 144u) : p.row_bytes;
        uint64_t R = target > 32 ? (target - 32) / rb : 0;
        const uint64_t cap = (p.segmented && q6) ? kProgramWarps : 2 * kProgramWarps;
        if (R > cap) R = cap;
        if (R < 1) R = 1;
        p.rows_per_stage = static_cast<uint32_t>(R);
        const uint64_t sb = align_up(static_cast<uint32_t>(R * rb + 32), 128u);
        if (sb > stage) stage = sb;
    }
    if (stage * 2 > budget) return ORACLE_CUDA_UNSUPPORTED;
    uint64_t S = budget / stage;
    if (S > 16) S = 16;
    pp.stages = static_cast<uint32_t>(S);
    pp.stage_bytes = static_cast<uint32_t>(stage);
    return ORACLE_CUDA_OK;
}

using ProgramKernel = void (*)(const ProgramParams);

// The program kernel specialised for the ops' weight types (and, in a peer
// group, with the peer stores compiled in).
ProgramKernel select_program_kernel(const ProgramParams& pp, bool peers) {
    int types = 0;
    bool short_rows = true;
    for (uint32_t k = 0; k < pp.n_ops; ++k) {
        types |= pp.ops[k].type == kTypeQ4_K ? 1 : 2;
        short_rows = short_rows && pp.ops[k].nb <= 16;
    }
    if (types == 2 && short_rows) types = 4;
    if (peers)
        return types == 1   ? matvec_program_kernel<kProgramWarps, 1, true>
               : types == 2 ? matvec_program_kernel<kProgramWarps, 2, true>
               : types == 4 ? matvec_program_kernel<kProgramWarps, 4, true>
                            : matvec_program_kernel<kProgramWarps, 3, true>;
    return types == 1   ? matvec_program_kernel<kProgramWarps, 1>
           : types == 2 ? matvec_program_kernel<kProgramWarps, 2>
           : types == 4 ? matvec_program_kernel<kProgramWarps, 4>
                        : matvec_program_kernel<kProgramWarps, 3>;
}

// Two ops read the same activation image when their sources are identical.
bool same_source(const oracle_cuda_matvec_op_ex& a, const oracle_cuda_matvec_op_ex& b) {
    return a.base.x_dev == b.base.x_dev && a.base.cols == b.base.cols && a.xform == b.xform &&
           (a.xform != ORACLE_CUDA_XFORM_SWIGLU || a.x2_dev == b.x2_dev) &&
           (a.xform != ORACLE_CUDA_XFORM_RMS || (a.norm_dev == b.norm_dev && a.eps == b.eps));
}

oracle_cuda_status program_run(oracle_cuda_context* ctx, const oracle_cuda_matvec_op_ex* ops, uint32_t n_ops,
                               void* stream, const oracle_cuda_peer_group* group, const oracle_cuda_sharded_op* sh,
                               const oracle_cuda_sharded_step* step) {
    if (!ctx) return fail(nullptr, ORACLE_CUDA_INVALID_ARGUMENT, "context is null");
    if (!ops || n_ops == 0 || n_ops > kProgramMaxOps)
        return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT,
                    "a matvec program holds 1 to " + std::to_string(kProgramMaxOps) + " ops");
    ProgramParams pp{};
    pp.n_ops = n_ops;
    uint64_t max_rows = 0;
    for (uint32_t k = 0; k < n_ops; ++k) {
        const oracle_cuda_matvec_op_ex& e = ops[k];
        const std::string at = "op " + std::to_string(k) + ": ";
        if (e.xform > ORACLE_CUDA_XFORM_SWIGLU && !(sh && e.xform == ORACLE_CUDA_XFORM_COMBINE_RMS))
            return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, at + "unknown activation transform");
        if (sh) {
            if (sh[k].wait > 3) return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, at + "wait must be 0, 1, 2 or 3");
            if (sh[k].wait != 0 && k == 0)
                return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, at + "the first op cannot wait for an earlier op");
            if (sh[k].wait == 2 && !sh[k - 1].announce)
                return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, at + "waiting for every rank needs the op before to announce");
            if (e.xform == ORACLE_CUDA_XFORM_COMBINE_RMS) {
                if (sh[k].wait < 2 || !e.x2_dev || sh[k].segments == 0 || !e.norm_dev || !(e.eps > 0.0f) ||
                    !std::isfinite(e.eps))
                    return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT,
                                at + "the combine transform needs wait 2 or 3, partial sums, segments, norm weights "
                                     "and a positive finite epsilon");
                if (!sh[k].combined_dev || sh[k].combined_dev == e.base.x_dev)
                    return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT,
                                at + "the combine transform needs combined_dev, distinct from x_dev");
                if (reinterpret_cast<uintptr_t>(e.x2_dev) % 4 || reinterpret_cast<uintptr_t>(e.base.x_dev) % 4 ||
                    reinterpret_cast<uintptr_t>(sh[k].combined_dev) % 4)
                    return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, at + "combine vectors must be 4-byte aligned");
            }
            if (sh[k].swiglu_gate && !e.act_dev)
                return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, at + "a SwiGLU epilogue needs act_dev");
        }
        if (e.xform == ORACLE_CUDA_XFORM_RMS && (!e.norm_dev || !(e.eps > 0.0f) || !std::isfinite(e.eps)))
            return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT,
                        "op " + std::to_string(k) + ": RMS transform needs weights and a positive finite epsilon");
        if (e.xform == ORACLE_CUDA_XFORM_SWIGLU && !e.x2_dev)
            return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "op " + std::to_string(k) + ": SwiGLU transform needs up");
        const oracle_cuda_matvec_op& o = e.base;
        uint64_t rb = 0, batch = 0;
        oracle_cuda_status st = validate_matvec(ctx, ORACLE_CUDA_CONTRACT_Q8K, o.type, o.rows, o.cols, o.w_nbytes,
                                                o.cols, o.rows, &rb, &batch);
        if (st != ORACLE_CUDA_OK) {
            ctx->last_error = "op " + std::to_string(k) + ": " + ctx->last_error;
            return st;
        }
        if (Error e = check_weight_pointer(o.type, o.w_dev)) return fail(ctx, e);
        if (!o.x_dev || !o.y_dev)
            return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "op " + std::to_string(k) + ": null activation or output");
        ProgramOp& p = pp.ops[k];
        p.w = static_cast<const uint8_t*>(o.w_dev);
        p.x = o.x_dev;
        p.y = o.y_dev;
        p.rows = o.rows;
        p.row_bytes = rb;
        p.type = o.type;
        p.nb = static_cast<uint32_t>(o.cols / 256);
        p.after_previous = sh ? ((sh[k].wait == 1 || sh[k].wait == 2) ? 1u : 0u)
                              : ((o.after_previous && k > 0) ? 1u : 0u);
        p.push = sh ? (sh[k].push ? 1u : 0u) : (group ? 1u : 0u);
        pp.ext[k].xform = e.xform;
        pp.ext[k].eps = e.eps;
        pp.ext[k].x2 = e.x2_dev;
        pp.ext[k].norm = e.norm_dev;
        p.residual = e.residual_dev;
        if (sh && e.xform == ORACLE_CUDA_XFORM_COMBINE_RMS) {
            pp.ext[k].partials = e.x2_dev;
            pp.ext[k].x2 = nullptr;
            pp.ext[k].segments = sh[k].segments;
            pp.ext[k].combined = sh[k].combined_dev;
        }
        if (sh && sh[k].swiglu_gate) {
            pp.ext[k].act = e.act_dev;
            pp.ext[k].other = sh[k].swiglu_gate;
            pp.ext[k].other_is_gate = 1u;
        }
        if (o.rows > max_rows) max_rows = o.rows;
    }
    // A SwiGLU op whose gate and up are outputs of two earlier ops of this
    // launch over the same rows: the later of the two forms silu(gate) * up
    // row by row in its epilogue (once per element, by the CTA that owns the
    // row in both ops), and the SwiGLU op reads that vector plainly.
    // (Sharded programs name their SwiGLU epilogues explicitly: swiglu_gate.)
    if (!sh) {
        uint64_t need = 0;
        for (uint32_t j = 0; j < n_ops; ++j)
            if (ops[j].xform == ORACLE_CUDA_XFORM_SWIGLU && !ops[j].act_dev) need += ops[j].base.cols * sizeof(float);
        if (need > 0 && !group) {
            oracle_cuda_status gs = grow_device(ctx, ctx->act_scratch, ctx->act_scratch_bytes, need);
            if (gs != ORACLE_CUDA_OK) return gs;
        }
        uint64_t used = 0;
        for (uint32_t j = 0; j < n_ops; ++j) {
            if (ops[j].xform != ORACLE_CUDA_XFORM_SWIGLU) continue;
            if (group && !ops[j].act_dev) continue;  // peers need the vector in the gather buffer
            // gate = the earlier op whose rows lie in x, up = the one whose rows lie
            // in x2, over the same rows at the same offsets (a row shard of the
            // vector when the ranks of a peer group split it)
            auto inside = [&](const oracle_cuda_matvec_op_ex& o, const float* v) {
                return o.base.y_dev >= v && o.base.y_dev + o.base.rows <= v + ops[j].base.cols;
            };
            int a = -1, b = -1;
            for (uint32_t i = 0; i < j; ++i) {
                if (inside(ops[i], ops[j].base.x_dev)) a = static_cast<int>(i);
                if (inside(ops[i], ops[j].x2_dev)) b = static_cast<int>(i);
            }
            if (a < 0 || b < 0 || a == b || ops[a].base.rows != ops[b].base.rows ||
                ops[a].base.y_dev - ops[j].base.x_dev != ops[b].base.y_dev - ops[j].x2_dev || pp.ext[a].act ||
                pp.ext[b].act)
                continue;
            // single GPU: the two producers must cover the whole vector
            if (!group && ops[a].base.rows != ops[j].base.cols) continue;
            const int later = a > b ? a : b;
            float* act = ops[j].act_dev;
            if (!act) {
                act = reinterpret_cast<float*>(ctx->act_scratch + used);
                used += ops[j].base.cols * sizeof(float);
            }
            // the later op writes its rows at the same offsets as in its own output
            pp.ext[later].act = act + (ops[later].base.y_dev - (later == b ? ops[j].x2_dev : ops[j].base.x_dev));
            // later == b: this op computes up, `other` is the gate output; else the reverse
            pp.ext[later].other = later == b ? ops[a].base.y_dev : ops[b].base.y_dev;
            pp.ext[later].other_is_gate = later == b ? 1u : 0u;
            pp.ops[j].x = act;
            pp.ext[j].xform = kXformNone;
            pp.ext[j].x2 = nullptr;
        }
    }
    // Images of ops whose activation comes from outside the launch are built
    // once by quantize_images_kernel into the scratch region, laid out with
    // the dependent ops' images last, so one contiguous copy serves them.  An
    // op whose source equals an earlier op's shares that op's image: it needs
    // neither a build nor a wait of its own.
    ImageJobs jobs{};
    uint32_t prebuilt = 0, blocks = 0, act_total = 0;
    {
        // produced[k]: x comes from earlier ops of this launch (waited for by
        // this op, or, sharded wait 3, by an earlier one): built in the kernel
        bool produced[kProgramMaxOps];
        for (uint32_t k = 0; k < n_ops; ++k)
            produced[k] = pp.ops[k].after_previous != 0 || (sh && sh[k].wait == 3);
        auto same = [&](uint32_t j, uint32_t k) {
            if (!same_source(ops[j], ops[k])) return false;
            if (!sh) return true;
            if (produced[j] != produced[k]) return false;
            return ops[j].xform != ORACLE_CUDA_XFORM_COMBINE_RMS ||
                   (ops[j].x2_dev == ops[k].x2_dev && sh[j].segments == sh[k].segments &&
                    sh[j].combined_dev == sh[k].combined_dev && ops[j].norm_dev == ops[k].norm_dev &&
                    ops[j].eps == ops[k].eps);
        };
        int owner[kProgramMaxOps];
        for (uint32_t k = 0; k < n_ops; ++k) {
            owner[k] = -1;
            for (uint32_t j = 0; j < k && owner[k] < 0; ++j)
                if (owner[j] < 0 && same(j, k)) owner[k] = static_cast<int>(j);
            if (owner[k] >= 0) pp.ops[k].after_previous = 0u;
            // a combine reads every rank's partials: the op that builds it waits for them
            if (sh && owner[k] < 0 && ops[k].xform == ORACLE_CUDA_XFORM_COMBINE_RMS && sh[k].wait != 2)
                return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT,
                            "op " + std::to_string(k) + ": a combine transform not shared with an earlier op needs wait 2");
        }
        // in-kernel builds of fed-in images only while they all fit in shared
        // memory beside the ring; otherwise prebuilt images (slots when large)
        uint64_t fed = 0;
        for (uint32_t k = 0; k < n_ops; ++k)
            if (owner[k] < 0 && !produced[k]) fed += q8k_image_bytes(pp.ops[k].nb);
        const bool in_kernel = (ctx->flags & ORACLE_CUDA_FLAG_BUILD_IN_KERNEL) != 0 && fed <= ctx->jit_image_threshold;
        uint32_t off = 0;
        for (uint32_t k = 0; k < n_ops; ++k)
            if (owner[k] < 0 && !produced[k] && !in_kernel) {
                pp.ops[k].act_offset = off;
                pp.ops[k].prebuilt = 1u;
                const uint32_t jn = jobs.n_jobs;
                jobs.x[jn] = pp.ops[k].x;
                jobs.x2[jn] = pp.ext[k].x2;
                jobs.norm[jn] = pp.ext[k].norm;
                jobs.eps[jn] = pp.ext[k].eps;
                jobs.xform[jn] = pp.ext[k].xform;
                jobs.nb[jn] = pp.ops[k].nb;
                jobs.offset[jn] = off;
                jobs.first_block[jn] = blocks;
                blocks += pp.ops[k].nb;
                jobs.n_jobs++;
                off += q8k_image_bytes(pp.ops[k].nb);
            }
        prebuilt = off;
        jobs.first_block[jobs.n_jobs] = blocks;
        for (uint32_t k = 0; k < n_ops; ++k)
            if (owner[k] < 0 && (produced[k] || in_kernel)) {
                pp.ops[k].act_offset = off;
                pp.ext[k].build = 1u;
                off += q8k_image_bytes(pp.ops[k].nb);
            }
        for (uint32_t k = 0; k < n_ops; ++k)
            if (owner[k] >= 0) pp.ops[k].act_offset = pp.ops[owner[k]].act_offset;
        for (uint32_t k = 1; k < n_ops; ++k)
            if (pp.ops[k].after_previous) pp.ops[k - 1].publish = 1u;
        act_total = off + 256;  // + reduction scratch
        // Images that would crowd the stage ring out of shared memory stay in
        // global memory; each op copies its own into one of two slots.
        if (prebuilt > ctx->jit_image_threshold) {
            uint32_t slot = 0, old_offset[kProgramMaxOps];
            bool pre[kProgramMaxOps];
            for (uint32_t k = 0; k < n_ops; ++k) {
                old_offset[k] = pp.ops[k].act_offset;
                pre[k] = pp.ops[k].prebuilt || (owner[k] >= 0 && pp.ops[owner[k]].prebuilt);
                if (pre[k] && q8k_image_bytes(pp.ops[k].nb) > slot) slot = q8k_image_bytes(pp.ops[k].nb);
            }
            uint32_t jit_index = 0;
            for (uint32_t k = 0; k < n_ops; ++k) {
                if (pre[k]) {  // a fed-in image (its own or one it shares): copied into a slot
                    pp.ext[k].jit_src = old_offset[k];
                    pp.ops[k].prebuilt = 1u;
                    pp.ops[k].act_offset = (jit_index++ & 1u) * slot;
                } else {       // built in the kernel: after the two slots
                    pp.ops[k].act_offset = old_offset[k] - prebuilt + 2 * slot;
                }
            }
            pp.jit_slot_bytes = slot;
            act_total = act_total - prebuilt + 2 * slot;
        }
    }
    pp.act_bytes = act_total;
    {
        std::string why;
        const oracle_cuda_status rs = plan_program_ring(pp, ctx->smem_budget, ctx->program_stage_target, why);
        if (rs != ORACLE_CUDA_OK) return fail(ctx, rs, why);
    }
    pp.copy_chunk = ctx->copy_chunk;
    pp.max_inflight = ctx->max_inflight < pp.stages ? ctx->max_inflight : pp.stages;
    pp.prebuilt_bytes = prebuilt;
    pp.counters = ctx->program_counters;
    pp.status = ctx->status;
    pp.trace = ctx->trace;
    pp.trace_records = ctx->trace_records;
    pp.px.world = 1;
    if (group) {
        if (!group->connected) return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "peer group is not connected");
        if (group->ctx != ctx) return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "peer group belongs to another context");
        const float* lo = reinterpret_cast<const float*>(group->local + kGatherHeader);
        const float* hi = lo + group->data_bytes / sizeof(float);
        for (uint32_t k = 0; k < n_ops; ++k) {
            const float* y0 = ops[k].base.y_dev;
            if (pp.ops[k].push && (y0 < lo || y0 + ops[k].base.rows > hi))
                return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT,
                            "op " + std::to_string(k) + ": output must lie inside the peer group's gather buffer");
        }
        if (sh) {
            const uint32_t w = group->world;
            if (w & (w - 1)) return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "sharded programs need 1, 2, 4 or 8 ranks");
            if (!step) return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "sharded program without step information");
            uint32_t j = step->first_dep, last = 0;
            for (uint32_t k = 0; k < n_ops; ++k) {
                if (pp.ext[k].partials) {
                    const float* p0 = pp.ext[k].partials;
                    if (p0 < lo || p0 + uint64_t(w) * pp.ext[k].segments * ops[k].base.cols > hi)
                        return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT,
                                    "op " + std::to_string(k) + ": partial sums must lie inside the gather buffer");
                }
                if (sh[k].announce) {
                    pp.ext[k].announce = 1u + j++;
                    pp.ops[k].publish = 1u;
                    last = pp.ext[k].announce;
                }
                if (sh[k].wait == 2) pp.ext[k].xwait = pp.ext[k - 1].announce;
            }
            if (j > step->deps_per_step)
                return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "more announcements than deps_per_step");
            if (step->tail_wait && last == 0)
                return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "tail_wait needs an announcing op");
            pp.px.sharded = 1u;
            pp.px.deps_per_step = step->deps_per_step;
            pp.px.end_of_step = step->end_of_step ? 1u : 0u;
            pp.px.tail_wait = step->tail_wait ? last : 0u;
            pp.px.my_xdep = reinterpret_cast<unsigned int*>(group->local) + kGatherXdep;
            pp.px.my_step = reinterpret_cast<unsigned int*>(group->local) + kGatherStep;
            for (uint32_t r = 0; r < w; ++r)
                pp.px.peer_xdep[r] = reinterpret_cast<unsigned int*>(group->mapped[r]) + kGatherXdep;
        }
        pp.px.world = group->world;
        pp.px.rank = group->rank;
        pp.px.local_base = lo;
        for (uint32_t r = 0; r < group->world; ++r) {
            pp.px.peer_base[r] = reinterpret_cast<float*>(group->mapped[r] + kGatherHeader);
            pp.px.peer_counter[r] = reinterpret_cast<unsigned int*>(group->mapped[r]);
        }
        pp.px.my_counter = reinterpret_cast<unsigned int*>(group->local);
        pp.px.my_epoch = reinterpret_cast<unsigned int*>(group->local) + 1;
        pp.px.my_op = reinterpret_cast<unsigned int*>(group->local) + kGatherOpCounters;
        for (uint32_t r = 0; r < group->world; ++r)
            pp.px.peer_op[r] = reinterpret_cast<unsigned int*>(group->mapped[r]) + kGatherOpCounters;
        // SwiGLU vectors and residual outputs reach the peers from the end-of-op
        // passes: they must sit in the gather buffer too
        for (uint32_t k = 0; k < n_ops; ++k)
            if (pp.ext[k].act && pp.ops[k].push && (pp.ext[k].act < lo || pp.ext[k].act + pp.ops[k].rows > hi))
                return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT,
                            "op " + std::to_string(k) + ": the SwiGLU vector must lie inside the peer group's gather buffer");
    }
    const uint32_t grid = static_cast<uint32_t>(max_rows < uint64_t(ctx->sm_count) ? max_rows : ctx->sm_count);
    const size_t smem = stream_barrier_bytes(pp.stages) + pp.act_bytes + size_t(pp.stages) * pp.stage_bytes;
    ORACLE_CUDA_TRY(ctx, cudaSetDevice(ctx->device), "cudaSetDevice");
    if (prebuilt > 0) {
        oracle_cuda_status gs = grow_device(ctx, ctx->image_scratch, ctx->image_scratch_bytes, prebuilt);
        if (gs != ORACLE_CUDA_OK) return gs;
        pp.images = ctx->image_scratch;
        // one warp per CTA: a warp fits beside a program CTA on every SM, so the
        // quantizer starts the moment its predecessor completes
        gs = launch(ctx, quantize_images_kernel, dim3(blocks), dim3(32), 0, static_cast<cudaStream_t>(stream),
                    (ctx->flags & ORACLE_CUDA_FLAG_PDL) != 0, jobs, ctx->image_scratch);
        if (gs != ORACLE_CUDA_OK) return gs;
    }
    const auto kernel = select_program_kernel(pp, group != nullptr);
    oracle_cuda_status st = launch(ctx, kernel, dim3(grid), dim3((kProgramWarps + 1) * 32), smem,
                                   static_cast<cudaStream_t>(stream), (ctx->flags & ORACLE_CUDA_FLAG_PDL) != 0, pp);
    return st == ORACLE_CUDA_OK ? ok(ctx) : st;
}

}  // namespace

// ---------------------------------------------------------------- row-sharded programs over peers

extern "C" oracle_cuda_status oracle_cuda_peer_group_create(oracle_cuda_context* ctx, uint32_t rank, uint32_t world,
                                                            uint64_t data_bytes, oracle_cuda_peer_group** out,
                                                            void* ipc_handle_out) {
    if (!ctx || !out || !ipc_handle_out) return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "null argument");
    *out = nullptr;
    if (world < 1 || world > kMaxPeers || rank >= world)
        return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT,
                    "peer group needs 1 <= world <= " + std::to_string(kMaxPeers) + " and rank < world");
    if (data_bytes == 0 || data_bytes % 16) return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "gather data size must be a positive multiple of 16");
    ORACLE_CUDA_TRY(ctx, cudaSetDevice(ctx->device), "cudaSetDevice");
    auto* g = new oracle_cuda_peer_group();
    g->ctx = ctx;
    g->rank = rank;
    g->world = world;
    g->data_bytes = data_bytes;
    cudaError_t e = cudaMalloc(reinterpret_cast<void**>(&g->local), kGatherHeader + data_bytes);
    if (e == cudaSuccess) e = cudaMemset(g->local, 0, kGatherHeader + data_bytes);
    cudaIpcMemHandle_t h{};
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, g->local);
    if (e != cudaSuccess) {
        if (g->local) cudaFree(g->local);
        delete g;
        return cuda_fail(ctx, e, "peer group gather buffer");
    }
    static_assert(sizeof(cudaIpcMemHandle_t) == ORACLE_CUDA_IPC_HANDLE_BYTES, "IPC handle size");
    std::memcpy(ipc_handle_out, &h, sizeof h);
    g->mapped[rank] = g->local;
    if (world == 1) g->connected = true;
    *out = g;
    return ok(ctx);
}

extern "C" oracle_cuda_status oracle_cuda_peer_group_connect(oracle_cuda_peer_group* g, const void* handles) {
    if (!g || !handles) return fail(g ? g->ctx : nullptr, ORACLE_CUDA_INVALID_ARGUMENT, "null argument");
    oracle_cuda_context* ctx = g->ctx;
    if (g->connected) return ok(ctx);
    ORACLE_CUDA_TRY(ctx, cudaSetDevice(ctx->device), "cudaSetDevice");
    const uint8_t* hb = static_cast<const uint8_t*>(handles);
    for (uint32_t r = 0; r < g->world; ++r) {
        if (r == g->rank) continue;
        cudaIpcMemHandle_t h;
        std::memcpy(&h, hb + size_t(r) * ORACLE_CUDA_IPC_HANDLE_BYTES, sizeof h);
        void* p = nullptr;
        const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) {
            for (uint32_t q = 0; q < r; ++q)
                if (q != g->rank && g->mapped[q]) {
                    cudaIpcCloseMemHandle(g->mapped[q]);
                    g->mapped[q] = nullptr;
                }
            return cuda_fail(ctx, e, ("cudaIpcOpenMemHandle (rank " + std::to_string(r) + ")").c_str());
        }
        g->mapped[r] = static_cast<uint8_t*>(p);
    }
    g->connected = true;
    return ok(ctx);
}

extern "C" oracle_cuda_status oracle_cuda_peer_group_data(oracle_cuda_peer_group* g, float** data_dev) {
    if (!g || !data_dev) return fail(g ? g->ctx : nullptr, ORACLE_CUDA_INVALID_ARGUMENT, "null argument");
    *data_dev = reinterpret_cast<float*>(g->local + kGatherHeader);
    return ok(g->ctx);
}

extern "C" oracle_cuda_status oracle_cuda_peer_group_destroy(oracle_cuda_peer_group* g) {
    if (!g) return ORACLE_CUDA_OK;
    cudaSetDevice(g->ctx->device);
    cudaDeviceSynchronize();
    for (uint32_t r = 0; r < g->world; ++r)
        if (r != g->rank && g->mapped[r]) cudaIpcCloseMemHandle(g->mapped[r]);
    if (g->local) cudaFree(g->local);
    delete g;
    return ORACLE_CUDA_OK;
}

extern "C" oracle_cuda_status oracle_cuda_matvec_program_allgather(oracle_cuda_context* ctx,
                                                                   oracle_cuda_peer_group* group,
                                                                   const oracle_cuda_matvec_op* ops, uint32_t n_ops,
                                                                   void* stream) {
    if (!group) return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "peer group is null");
    return program_run_base(ctx, ops, n_ops, stream, group);
}

oracle_cuda_status oracle_cuda_weight_upload(oracle_cuda_context* ctx, uint32_t type, uint64_t rows, uint64_t cols,
                                             const void* host_bytes, uint64_t nbytes, uint64_t row_begin,
                                             uint64_t row_end, oracle_cuda_weight** out) {
    if (!ctx) return fail(nullptr, ORACLE_CUDA_INVALID_ARGUMENT, "context is null");
    if (!out || !host_bytes) return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "null pointer");
    *out = nullptr;
    uint64_t rb = 0, total = 0;
    if (rows == 0) return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "GGUF tensor must have at least one dimension");
    if (Error e = row_byte_size(cols, type, &rb)) return fail(ctx, e);
    if (!checked_mul(rows, rb, &total))
        return fail(ctx, ORACLE_CUDA_OVERFLOW, "GGUF tensor byte size exceeds addressable size");
    if (nbytes != total)
        return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "GGUF tensor byte size does not match row geometry");
    if (row_begin >= row_end || row_end > rows)
        return fail(ctx, ORACLE_CUDA_OUT_OF_RANGE, "GGUF tensor row index exceeds row count");
    ORACLE_CUDA_TRY(ctx, cudaSetDevice(ctx->device), "cudaSetDevice");
    auto* w = new oracle_cuda_weight{ctx, type, row_end - row_begin, cols, row_begin, (row_end - row_begin) * rb,
                                     nullptr, false};
    // +16 bytes of tail padding keeps every aligned word read inside the allocation.
    cudaError_t e = cudaMalloc(&w->dev, w->nbytes + 16);
    if (e != cudaSuccess) {
        delete w;
        return cuda_fail(ctx, e, "cudaMalloc(weight)");
    }
    e = cudaMemcpy(w->dev, static_cast<const uint8_t*>(host_bytes) + row_begin * rb, w->nbytes,
                   cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        cudaFree(w->dev);
        delete w;
        return cuda_fail(ctx, e, "cudaMemcpy(weight)");
    }
    *out = w;
    return ok(ctx);
}

oracle_cuda_status oracle_cuda_weight_free(oracle_cuda_weight* w) {
    if (!w) return ORACLE_CUDA_OK;
    if (w->owned_by_cache) return fail(w->ctx, ORACLE_CUDA_INVALID_ARGUMENT, "registered host weights are freed by oracle_cuda_unregister_host_weight or oracle_cuda_evict_resident");
    cudaSetDevice(w->ctx->device);
    cudaFree(w->dev);
    delete w;
    return ORACLE_CUDA_OK;
}

oracle_cuda_status oracle_cuda_weight_info(const oracle_cuda_weight* w, uint32_t* type, uint64_t* rows, uint64_t* cols,
                                           uint64_t* row_begin, const void** dev, uint64_t* nbytes) {
    if (!w) return fail(nullptr, ORACLE_CUDA_INVALID_ARGUMENT, "weight is null");
    if (type) *type = w->type;
    if (rows) *rows = w->rows;
    if (cols) *cols = w->cols;
    if (row_begin) *row_begin = w->row_begin;
    if (dev) *dev = w->dev;
    if (nbytes) *nbytes = w->nbytes;
    return ORACLE_CUDA_OK;
}

oracle_cuda_status oracle_cuda_register_host_weight(oracle_cuda_context* ctx, uint32_t type, uint64_t rows,
                                                    uint64_t cols, const void* host, uint64_t nbytes) {
    if (!ctx) return fail(nullptr, ORACLE_CUDA_INVALID_ARGUMENT, "context is null");
    const auto key = std::make_tuple(host, nbytes, type, rows, cols);
    if (ctx->resident.count(key)) return ok(ctx);
    oracle_cuda_weight* w = nullptr;
    oracle_cuda_status s = oracle_cuda_weight_upload(ctx, type, rows, cols, host, nbytes, 0, rows, &w);
    if (s != ORACLE_CUDA_OK) return s;
    w->owned_by_cache = true;
    ctx->resident[key] = w;
    return ok(ctx);
}

oracle_cuda_status oracle_cuda_unregister_host_weight(oracle_cuda_context* ctx, const void* host, uint64_t nbytes) {
    if (!ctx) return fail(nullptr, ORACLE_CUDA_INVALID_ARGUMENT, "context is null");
    bool found = false;
    for (auto it = ctx->resident.begin(); it != ctx->resident.end();) {
        if (std::get<0>(it->first) == host && std::get<1>(it->first) == nbytes) {
            if (!found) {
                cudaSetDevice(ctx->device);
                cudaDeviceSynchronize();  // no launch may still read the copy
            }
            found = true;
            cudaFree(it->second->dev);
            delete it->second;
            it = ctx->resident.erase(it);
        } else {
            ++it;
        }
    }
    if (!found) return fail(ctx, ORACLE_CUDA_OUT_OF_RANGE, "host weight span is not registered");
    return ok(ctx);
}

oracle_cuda_status oracle_cuda_host_matvec_program(oracle_cuda_context* ctx, const oracle_cuda_host_matvec_op* ops,
                                                   uint32_t n_ops) {
    if (!ctx) return fail(nullptr, ORACLE_CUDA_INVALID_ARGUMENT, "context is null");
    if (!ops || n_ops == 0 || n_ops > kProgramMaxOps)
        return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT,
                    "a matvec program holds 1 to " + std::to_string(kProgramMaxOps) + " ops");
    // layout of the call's device buffers: fed-in x vectors, every y, staged weights
    int src[kProgramMaxOps];
    uint64_t x_off[kProgramMaxOps], y_off[kProgramMaxOps], w_off[kProgramMaxOps];
    uint64_t x_total = 0, y_total = 0, w_total = 0;
    for (uint32_t k = 0; k < n_ops; ++k) {
        const oracle_cuda_host_matvec_op& o = ops[k];
        uint64_t rb = 0, batch = 0;
        oracle_cuda_status s = validate_matvec(ctx, ORACLE_CUDA_CONTRACT_Q8K, o.type, o.rows, o.cols, o.w_nbytes,
                                               o.cols, o.rows, &rb, &batch);
        if (s != ORACLE_CUDA_OK) {
            ctx->last_error = "op " + std::to_string(k) + ": " + ctx->last_error;
            return s;
        }
        if (!o.w_host || !o.x_host || !o.y_host)
            return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "op " + std::to_string(k) + ": null pointer");
        src[k] = -1;
        for (uint32_t j = 0; j < k; ++j)
            if (ops[j].y_host == o.x_host) src[k] = static_cast<int>(j);
        if (src[k] >= 0 && ops[src[k]].rows != o.cols)
            return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT,
                        "op " + std::to_string(k) + ": reads op " + std::to_string(src[k]) +
                            "'s output, whose length is not its column count");
        x_off[k] = x_total;
        if (src[k] < 0) x_total += o.cols;
        y_off[k] = y_total;
        y_total += o.rows;
        w_off[k] = w_total;
        w_total += weight_stage_need(ctx, o.type, o.rows, o.cols, o.w_host, o.w_nbytes);
    }
    ORACLE_CUDA_TRY(ctx, cudaSetDevice(ctx->device), "cudaSetDevice");
    oracle_cuda_status s = ORACLE_CUDA_OK;
    if ((x_total && (s = grow_device(ctx, ctx->dev_x, ctx->dev_x_len, x_total)) != ORACLE_CUDA_OK) ||
        (s = grow_device(ctx, ctx->dev_y, ctx->dev_y_len, y_total)) != ORACLE_CUDA_OK ||
        (x_total && (s = grow_pinned(ctx, ctx->pin_x, ctx->pin_x_len, x_total)) != ORACLE_CUDA_OK) ||
        (s = grow_pinned(ctx, ctx->pin_y, ctx->pin_y_len, y_total)) != ORACLE_CUDA_OK ||
        (w_total && (s = grow_device(ctx, ctx->stage_w, ctx->stage_w_len, w_total)) != ORACLE_CUDA_OK))
        return s;
    cudaStream_t st = nullptr;
    oracle_cuda_matvec_op dops[kProgramMaxOps] = {};
    for (uint32_t k = 0; k < n_ops; ++k) {
        const oracle_cuda_host_matvec_op& o = ops[k];
        const void* wdev = nullptr;
        if ((s = weight_bytes_for_call(ctx, o.type, o.rows, o.cols, o.w_host, o.w_nbytes, w_off[k], st, &wdev)) !=
            ORACLE_CUDA_OK)
            return s;
        if (src[k] < 0) std::memcpy(ctx->pin_x + x_off[k], o.x_host, o.cols * sizeof(float));
        dops[k] = oracle_cuda_matvec_op{o.type, src[k] >= 0 ? 1u : 0u, o.rows, o.cols, wdev, o.w_nbytes,
                                        src[k] >= 0 ? ctx->dev_y + y_off[src[k]] : ctx->dev_x + x_off[k],
                                        ctx->dev_y + y_off[k]};
    }
    if (x_total)
        ORACLE_CUDA_TRY(ctx, cudaMemcpyAsync(ctx->dev_x, ctx->pin_x, x_total * sizeof(float), cudaMemcpyHostToDevice, st),
                        "cudaMemcpyAsync(x)");
    // a synchronous call pays every launch's latency: the program quantizes
    // its activations itself (no quantizer launch before it)
    const uint32_t saved_flags = ctx->flags;
    ctx->flags |= ORACLE_CUDA_FLAG_BUILD_IN_KERNEL;
    s = program_run_base(ctx, dops, n_ops, st, nullptr);
    ctx->flags = saved_flags;
    if (s != ORACLE_CUDA_OK) return s;
    ORACLE_CUDA_TRY(ctx, cudaMemcpyAsync(ctx->pin_y, ctx->dev_y, y_total * sizeof(float), cudaMemcpyDeviceToHost, st),
                    "cudaMemcpyAsync(y)");
    ORACLE_CUDA_TRY(ctx, cudaStreamSynchronize(st), "cudaStreamSynchronize");
    for (uint32_t k = 0; k < n_ops; ++k) std::memcpy(ops[k].y_host, ctx->pin_y + y_off[k], ops[k].rows * sizeof(float));
    return ok(ctx);
}

}  // extern "C"

// Copies between page-locked host arrays (device-mapped) and device buffers
// for prepared host programs: one launch moves every op's vector, so the
// captured graph holds no copy-engine transfers (each costs microseconds of
// latency for a few kilobytes).
struct HostCopies {
    const float* src[kProgramMaxOps];
    float* dst[kProgramMaxOps];
    uint32_t n[kProgramMaxOps];
    uint32_t count;
    uint32_t wait_previous;  // 1: griddepcontrol.wait first (y after the program)
};

__global__ void __launch_bounds__(256) host_copies_kernel(const __grid_constant__ HostCopies c) {
    pdl_launch_dependents();
    if (c.wait_previous) pdl_wait();
    for (uint32_t k = 0; k < c.count; ++k) {
        const float* src = c.src[k];
        float* dst = c.dst[k];
        for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < c.n[k]; i += gridDim.x * blockDim.x)
            dst[i] = src[i];
    }
}

struct oracle_cuda_host_program {
    oracle_cuda_context* ctx = nullptr;
    uint32_t n_ops = 0;
    oracle_cuda_host_matvec_op ops[kProgramMaxOps] = {};
    int src[kProgramMaxOps] = {};
    uint64_t x_off[kProgramMaxOps] = {}, y_off[kProgramMaxOps] = {};
    uint64_t x_total = 0, y_total = 0;
    bool direct = false;  // every x and y is device-mapped page-locked memory: read and written in place
    float* pin_x = nullptr;
    float* pin_y = nullptr;
    float* dev_x = nullptr;
    float* dev_y = nullptr;
    cudaStream_t stream = nullptr;
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
};

namespace {

void host_program_free(oracle_cuda_host_program* p) {
    if (!p) return;
    if (p->ctx) cudaSetDevice(p->ctx->device);
    if (p->stream) cudaStreamSynchronize(p->stream);
    if (p->exec) cudaGraphExecDestroy(p->exec);
    if (p->graph) cudaGraphDestroy(p->graph);
    if (p->stream) cudaStreamDestroy(p->stream);
    if (p->pin_x) cudaFreeHost(p->pin_x);
    if (p->pin_y) cudaFreeHost(p->pin_y);
    if (p->dev_x) cudaFree(p->dev_x);
    if (p->dev_y) cudaFree(p->dev_y);
    delete p;
}

}  // namespace

extern "C" {

oracle_cuda_status oracle_cuda_host_program_create(oracle_cuda_context* ctx, const oracle_cuda_host_matvec_op* ops,
                                                   uint32_t n_ops, oracle_cuda_host_program** out) {
    if (!ctx) return fail(nullptr, ORACLE_CUDA_INVALID_ARGUMENT, "context is null");
    if (!out) return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "output pointer is null");
    *out = nullptr;
    if (!ops || n_ops == 0 || n_ops > kProgramMaxOps)
        return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT,
                    "a matvec program holds 1 to " + std::to_string(kProgramMaxOps) + " ops");
    auto* p = new oracle_cuda_host_program();
    p->ctx = ctx;
    p->n_ops = n_ops;
    const void* wdev[kProgramMaxOps];
    bool pinned = true;
    for (uint32_t k = 0; k < n_ops; ++k) {
        const oracle_cuda_host_matvec_op& o = ops[k];
        p->ops[k] = o;
        uint64_t rb = 0, batch = 0;
        oracle_cuda_status s = validate_matvec(ctx, ORACLE_CUDA_CONTRACT_Q8K, o.type, o.rows, o.cols, o.w_nbytes,
                                               o.cols, o.rows, &rb, &batch);
        if (s != ORACLE_CUDA_OK) {
            ctx->last_error = "op " + std::to_string(k) + ": " + ctx->last_error;
            host_program_free(p);
            return s;
        }
        if (!o.w_host || !o.x_host || !o.y_host) {
            host_program_free(p);
            return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "op " + std::to_string(k) + ": null pointer");
        }
        auto it = ctx->resident.find(std::make_tuple(o.w_host, o.w_nbytes, o.type, o.rows, o.cols));
        if (it == ctx->resident.end()) {
            host_program_free(p);
            return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT,
                        "op " + std::to_string(k) + ": a prepared host program needs registered weights");
        }
        wdev[k] = it->second->dev;
        p->src[k] = -1;
        for (uint32_t j = 0; j < k; ++j)
            if (ops[j].y_host == o.x_host) p->src[k] = static_cast<int>(j);
        if (p->src[k] >= 0 && ops[p->src[k]].rows != o.cols) {
            host_program_free(p);
            return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT,
                        "op " + std::to_string(k) + ": reads op " + std::to_string(p->src[k]) +
                            "'s output, whose length is not its column count");
        }
        p->x_off[k] = p->x_total;
        if (p->src[k] < 0) {
            p->x_total += o.cols;
            pinned = pinned && is_device_mapped_host(o.x_host);
        }
        p->y_off[k] = p->y_total;
        p->y_total += o.rows;
        pinned = pinned && is_device_mapped_host(o.y_host);
    }
    p->direct = pinned;
    cudaError_t e = cudaSetDevice(ctx->device);
    if (e == cudaSuccess && p->x_total) e = cudaMalloc(reinterpret_cast<void**>(&p->dev_x), p->x_total * sizeof(float));
    if (e == cudaSuccess) e = cudaMalloc(reinterpret_cast<void**>(&p->dev_y), p->y_total * sizeof(float));
    if (e == cudaSuccess && !p->direct && p->x_total)
        e = cudaHostAlloc(reinterpret_cast<void**>(&p->pin_x), p->x_total * sizeof(float), cudaHostAllocDefault);
    if (e == cudaSuccess && !p->direct)
        e = cudaHostAlloc(reinterpret_cast<void**>(&p->pin_y), p->y_total * sizeof(float), cudaHostAllocDefault);
    if (e == cudaSuccess) e = cudaStreamCreate(&p->stream);
    if (e != cudaSuccess) {
        host_program_free(p);
        return cuda_fail(ctx, e, "prepared host program buffers");
    }
    oracle_cuda_matvec_op dops[kProgramMaxOps] = {};
    for (uint32_t k = 0; k < n_ops; ++k) {
        const oracle_cuda_host_matvec_op& o = ops[k];
        dops[k] = oracle_cuda_matvec_op{o.type, p->src[k] >= 0 ? 1u : 0u, o.rows, o.cols, wdev[k], o.w_nbytes,
                                        p->src[k] >= 0 ? p->dev_y + p->y_off[p->src[k]] : p->dev_x + p->x_off[k],
                                        p->dev_y + p->y_off[k]};
    }
    // capture: x in, the program (quantizing its activations in the kernel), y out
    oracle_cuda_status s = ORACLE_CUDA_OK;
    HostCopies xin{}, yout{};
    for (uint32_t k = 0; k < n_ops; ++k) {
        if (p->src[k] < 0) {
            xin.src[xin.count] = p->direct ? ops[k].x_host : p->pin_x + p->x_off[k];
            xin.dst[xin.count] = p->dev_x + p->x_off[k];
            xin.n[xin.count++] = static_cast<uint32_t>(ops[k].cols);
        }
        yout.src[yout.count] = p->dev_y + p->y_off[k];
        yout.dst[yout.count] = p->direct ? ops[k].y_host : p->pin_y + p->y_off[k];
        yout.n[yout.count++] = static_cast<uint32_t>(ops[k].rows);
    }
    yout.wait_previous = 1;
    e = cudaStreamBeginCapture(p->stream, cudaStreamCaptureModeThreadLocal);
    if (e == cudaSuccess) {
        // x in, the program (quantizing its activations in the kernel; its
        // weight stream starts beside the copy), y out after it
        if (xin.count) s = launch(ctx, host_copies_kernel, dim3(16), dim3(256), 0, p->stream, false, xin);
        if (s == ORACLE_CUDA_OK) {
            const uint32_t saved_flags = ctx->flags;
            ctx->flags |= ORACLE_CUDA_FLAG_BUILD_IN_KERNEL | ORACLE_CUDA_FLAG_PDL;
            s = program_run_base(ctx, dops, n_ops, p->stream, nullptr);
            ctx->flags = saved_flags;
        }
        if (s == ORACLE_CUDA_OK) s = launch(ctx, host_copies_kernel, dim3(16), dim3(256), 0, p->stream, true, yout);
        const cudaError_t e2 = cudaStreamEndCapture(p->stream, &p->graph);
        if (e == cudaSuccess) e = e2;
    }
    if (e == cudaSuccess && s == ORACLE_CUDA_OK) e = cudaGraphInstantiate(&p->exec, p->graph, 0);
    if (s != ORACLE_CUDA_OK || e != cudaSuccess) {
        const std::string msg = ctx->last_error;
        host_program_free(p);
        cudaGetLastError();
        if (s != ORACLE_CUDA_OK) return fail(ctx, s, msg);
        return cuda_fail(ctx, e, "prepared host program capture");
    }
    *out = p;
    return ok(ctx);
}

oracle_cuda_status oracle_cuda_host_program_run(oracle_cuda_host_program* p) {
    if (!p) return fail(nullptr, ORACLE_CUDA_INVALID_ARGUMENT, "prepared host program is null");
    oracle_cuda_context* ctx = p->ctx;
    ORACLE_CUDA_TRY(ctx, cudaSetDevice(ctx->device), "cudaSetDevice");
    if (!p->direct)
        for (uint32_t k = 0; k < p->n_ops; ++k)
            if (p->src[k] < 0)
                std::memcpy(p->pin_x + p->x_off[k], p->ops[k].x_host, p->ops[k].cols * sizeof(float));
    ORACLE_CUDA_TRY(ctx, cudaGraphLaunch(p->exec, p->stream), "cudaGraphLaunch");
    ORACLE_CUDA_TRY(ctx, cudaStreamSynchronize(p->stream), "cudaStreamSynchronize");
    ctx->launches += 1;
    if (!p->direct)
        for (uint32_t k = 0; k < p->n_ops; ++k)
            std::memcpy(p->ops[k].y_host, p->pin_y + p->y_off[k], p->ops[k].rows * sizeof(float));
    return ok(ctx);
}

oracle_cuda_status oracle_cuda_host_program_destroy(oracle_cuda_host_program* p) {
    host_program_free(p);
    return ORACLE_CUDA_OK;
}

oracle_cuda_status oracle_cuda_evict_resident(oracle_cuda_context* ctx) {
    if (!ctx) return fail(nullptr, ORACLE_CUDA_INVALID_ARGUMENT, "context is null");
    cudaSetDevice(ctx->device);
    cudaDeviceSynchronize();
    for (auto& kv : ctx->resident) {
        cudaFree(kv.second->dev);
        delete kv.second;
    }
    ctx->resident.clear();
    return ok(ctx);
}

oracle_cuda_status oracle_cuda_host_storage_matvec(oracle_cuda_context* ctx, int contract, uint32_t type,
                                                   uint64_t rows, uint64_t cols, const void* w_host, uint64_t w_nbytes,
                                                   const float* x_host, uint64_t x_len, float* y_host,
                                                   uint64_t y_len) {
    if (!ctx) return fail(nullptr, ORACLE_CUDA_INVALID_ARGUMENT, "context is null");
    uint64_t rb = 0, batch = 0;
    oracle_cuda_status s = validate_matvec(ctx, contract, type, rows, cols, w_nbytes, x_len, y_len, &rb, &batch);
    if (s != ORACLE_CUDA_OK) return s;
    if (!w_host || !x_host || !y_host) return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "null pointer");
    ORACLE_CUDA_TRY(ctx, cudaSetDevice(ctx->device), "cudaSetDevice");
    cudaStream_t st = nullptr;
    const uint64_t need = weight_stage_need(ctx, type, rows, cols, w_host, w_nbytes);
    if (need && (s = grow_device(ctx, ctx->stage_w, ctx->stage_w_len, need)) != ORACLE_CUDA_OK) return s;
    const void* wdev = nullptr;
    if ((s = weight_bytes_for_call(ctx, type, rows, cols, w_host, w_nbytes, 0, st, &wdev)) != ORACLE_CUDA_OK) return s;
    if ((s = grow_device(ctx, ctx->dev_x, ctx->dev_x_len, x_len)) != ORACLE_CUDA_OK) return s;
    if ((s = grow_device(ctx, ctx->dev_y, ctx->dev_y_len, y_len)) != ORACLE_CUDA_OK) return s;
    const bool x_pinned = is_pinned(x_host), y_pinned = is_pinned(y_host);
    const float* xsrc = x_host;
    if (!x_pinned) {
        if ((s = grow_pinned(ctx, ctx->pin_x, ctx->pin_x_len, x_len)) != ORACLE_CUDA_OK) return s;
        std::memcpy(ctx->pin_x, x_host, x_len * sizeof(float));
        xsrc = ctx->pin_x;
    }
    float* ydst = y_host;
    if (!y_pinned) {
        if ((s = grow_pinned(ctx, ctx->pin_y, ctx->pin_y_len, y_len)) != ORACLE_CUDA_OK) return s;
        ydst = ctx->pin_y;
    }
    ORACLE_CUDA_TRY(ctx, cudaMemcpyAsync(ctx->dev_x, xsrc, x_len * sizeof(float), cudaMemcpyHostToDevice, st),
                    "cudaMemcpyAsync(x)");
    s = run_matvec(ctx, contract, type, rows, cols, rb, wdev, ctx->dev_x, batch, ctx->dev_y, st);
    if (s != ORACLE_CUDA_OK) return s;
    ORACLE_CUDA_TRY(ctx, cudaMemcpyAsync(ydst, ctx->dev_y, y_len * sizeof(float), cudaMemcpyDeviceToHost, st),
                    "cudaMemcpyAsync(y)");
    ORACLE_CUDA_TRY(ctx, cudaStreamSynchronize(st), "cudaStreamSynchronize");
    if (!y_pinned) std::memcpy(y_host, ctx->pin_y, y_len * sizeof(float));
    return ok(ctx);
}

oracle_cuda_status oracle_cuda_host_storage_dot(oracle_cuda_context* ctx, int contract, uint32_t type, uint64_t cols,
                                                const void* row_host, uint64_t row_nbytes, const float* x_host,
                                                uint64_t x_len, float* out) {
    if (!ctx) return fail(nullptr, ORACLE_CUDA_INVALID_ARGUMENT, "context is null");
    uint64_t rb = 0;
    // make_storage_row_view (storage_decode.cpp:182-198), then the dot's length check (:27-29).
    if (Error e = row_byte_size(cols, type, &rb)) return fail(ctx, e);
    if (row_nbytes != rb)
        return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT,
                    "storage row byte size mismatch: expected " + std::to_string(rb) + ", received " +
                        std::to_string(row_nbytes));
    if (Error e = check_decodable(type)) return fail(ctx, e);
    if (x_len != cols) return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "reference dot vector length mismatch");
    if (!out) return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "output pointer is null");
    return oracle_cuda_host_storage_matvec(ctx, contract, type, 1, cols, row_host, row_nbytes, x_host, x_len, out, 1);
}

oracle_cuda_status oracle_cuda_host_decode_rows(oracle_cuda_context* ctx, uint32_t type, uint64_t rows, uint64_t cols,
                                                const void* w_host, uint64_t w_nbytes, float* out_host,
                                                uint64_t out_len) {
    if (!ctx) return fail(nullptr, ORACLE_CUDA_INVALID_ARGUMENT, "context is null");
    uint64_t rb = 0, total = 0, elems = 0;
    if (rows == 0) return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "GGUF tensor must have at least one dimension");
    if (Error e = row_byte_size(cols, type, &rb)) return fail(ctx, e);
    if (!checked_mul(rows, rb, &total) || w_nbytes != total)
        return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "GGUF tensor byte size does not match row geometry");
    if (Error e = check_decodable(type)) return fail(ctx, e);
    if (!checked_mul(rows, cols, &elems) || out_len != elems)
        return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "mapped tensor decode output length mismatch");
    if (!w_host || !out_host) return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "null pointer");
    ORACLE_CUDA_TRY(ctx, cudaSetDevice(ctx->device), "cudaSetDevice");
    oracle_cuda_status s = ORACLE_CUDA_OK;
    const uint64_t need = weight_stage_need(ctx, type, rows, cols, w_host, w_nbytes);
    if (need && (s = grow_device(ctx, ctx->stage_w, ctx->stage_w_len, need)) != ORACLE_CUDA_OK) return s;
    const void* wdev = nullptr;
    if ((s = weight_bytes_for_call(ctx, type, rows, cols, w_host, w_nbytes, 0, nullptr, &wdev)) != ORACLE_CUDA_OK)
        return s;
    if ((s = grow_device(ctx, ctx->dev_y, ctx->dev_y_len, out_len)) != ORACLE_CUDA_OK) return s;
    s = launch_decode(ctx, type, wdev, rows, cols, rb, ctx->dev_y, nullptr);
    if (s != ORACLE_CUDA_OK) return s;
    ORACLE_CUDA_TRY(ctx, cudaMemcpy(out_host, ctx->dev_y, out_len * sizeof(float), cudaMemcpyDeviceToHost),
                    "cudaMemcpy(out)");
    return ok(ctx);
}

}  // extern "C"

// ====================================================================== no-allocation program
//
// oracle_cuda_matvec_program_noalloc: the matvec program for callers that may
// not allocate device memory themselves -- for instance an engine that has
// already reserved nearly all of HBM for its own pools, or a latency-critical
// path where cudaMalloc (which can synchronise the device) is not allowed.  It
// needs no context: its scratch (the prebuilt activation images, the
// completion counters and the device status word) is one file-scope device
// array, present on every GPU that loads this library until the process exits.

namespace {

constexpr uint64_t kNoAllocImageBytes = ORACLE_CUDA_NOALLOC_IMAGE_BYTES;
constexpr uint64_t kNoAllocCountersOffset = kNoAllocImageBytes;
static_assert(kProgramCounters * sizeof(unsigned int) <= 256, "no-allocation counters fit before the status word");
constexpr uint64_t kNoAllocStatusOffset = kNoAllocImageBytes + 256;
constexpr uint64_t kNoAllocScratchBytes = kNoAllocImageBytes + 512;
constexpr int kNoAllocMaxDevices = 64;

}  // namespace

// Host code must not use this name as an address: on the host it is only a
// stand-in for the symbol.  The device address comes from cudaGetSymbolAddress.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

namespace {

struct NoAllocDevice {
    bool ready = false;
    unsigned char* scratch = nullptr;  // device address of g_noalloc_scratch
    int sm_count = 0;
    int smem_optin = 0;
};

NoAllocDevice g_noalloc_devices[kNoAllocMaxDevices];
std::mutex g_noalloc_mutex;

// Once per device, with that device current: resolve the array's device
// address, read the SM count and shared-memory limit, and allow the program
// kernels their dynamic shared memory.
oracle_cuda_status noalloc_setup(int device, NoAllocDevice** out) {
    if (device < 0 || device >= kNoAllocMaxDevices)
        return fail(nullptr, ORACLE_CUDA_UNSUPPORTED, "device index too large for the no-allocation entry point");
    std::lock_guard<std::mutex> lock(g_noalloc_mutex);
    NoAllocDevice& d = g_noalloc_devices[device];
    if (!d.ready) {
        cudaError_t e = cudaGetSymbolAddress(reinterpret_cast<void**>(&d.scratch), g_noalloc_scratch);
        if (e != cudaSuccess) return cuda_fail(nullptr, e, "cudaGetSymbolAddress(g_noalloc_scratch)");
        int major = 0;
        if ((e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device)) != cudaSuccess)
            return cuda_fail(nullptr, e, "cudaDeviceGetAttribute");
        if (major != 10) return fail(nullptr, ORACLE_CUDA_UNSUPPORTED, "this library is built for sm_100a (B200)");
        if ((e = cudaDeviceGetAttribute(&d.sm_count, cudaDevAttrMultiProcessorCount, device)) != cudaSuccess ||
            (e = cudaDeviceGetAttribute(&d.smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device)) !=
                cudaSuccess)
            return cuda_fail(nullptr, e, "cudaDeviceGetAttribute");
        const void* kernels[3] = {reinterpret_cast<const void*>(matvec_program_kernel<kProgramWarps, 1>),
                                  reinterpret_cast<const void*>(matvec_program_kernel<kProgramWarps, 2>),
                                  reinterpret_cast<const void*>(matvec_program_kernel<kProgramWarps, 3>)};
        for (const void* k : kernels)
            if ((e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, d.smem_optin)) !=
                cudaSuccess)
                return cuda_fail(nullptr, e, "cudaFuncSetAttribute");
        d.ready = true;
    }
    *out = &d;
    return ORACLE_CUDA_OK;
}

}  // namespace

extern "C" oracle_cuda_status oracle_cuda_matvec_program_noalloc(const oracle_cuda_matvec_op* ops, uint32_t n_ops,
                                                                 void* stream) {
    if (!ops || n_ops == 0 || n_ops > kProgramMaxOps)
        return fail(nullptr, ORACLE_CUDA_INVALID_ARGUMENT,
                    "a matvec program holds 1 to " + std::to_string(kProgramMaxOps) + " ops");
    int device = 0;
    cudaError_t e = cudaGetDevice(&device);
    if (e != cudaSuccess) return cuda_fail(nullptr, e, "cudaGetDevice");
    NoAllocDevice* dev = nullptr;
    oracle_cuda_status st = noalloc_setup(device, &dev);
    if (st != ORACLE_CUDA_OK) return st;

    ProgramParams pp{};
    pp.n_ops = n_ops;
    uint64_t max_rows = 0, prebuilt = 0;
    for (uint32_t k = 0; k < n_ops; ++k) {
        const oracle_cuda_matvec_op& o = ops[k];
        uint64_t rb = 0, batch = 0;
        st = validate_matvec(nullptr, ORACLE_CUDA_CONTRACT_Q8K, o.type, o.rows, o.cols, o.w_nbytes, o.cols, o.rows, &rb,
                             &batch);
        if (st != ORACLE_CUDA_OK)
            return fail(nullptr, st, "op " + std::to_string(k) + ": " + oracle_cuda_last_error(nullptr));
        if (Error err = check_weight_pointer(o.type, o.w_dev)) return fail(nullptr, err);
        if (!o.x_dev || !o.y_dev)
            return fail(nullptr, ORACLE_CUDA_INVALID_ARGUMENT, "op " + std::to_string(k) + ": null activation or output");
        ProgramOp& p = pp.ops[k];
        p.w = static_cast<const uint8_t*>(o.w_dev);
        p.x = o.x_dev;
        p.y = o.y_dev;
        p.rows = o.rows;
        p.row_bytes = rb;
        p.type = o.type;
        p.nb = static_cast<uint32_t>(o.cols / 256);
        p.after_previous = (o.after_previous && k > 0) ? 1u : 0u;
        if (p.after_previous) pp.ops[k - 1].publish = 1u;
        if (o.rows > max_rows) max_rows = o.rows;
        if (!p.after_previous) prebuilt += q8k_image_bytes(p.nb);
    }
    // The activation images of ops fed from outside the call live in the
    // static array; they must fit its stated size.
    if (prebuilt > kNoAllocImageBytes)
        return fail(nullptr, ORACLE_CUDA_INVALID_ARGUMENT,
                    "the activation images of this program need " + std::to_string(prebuilt) +
                        " bytes; the no-allocation entry point holds at most " + std::to_string(kNoAllocImageBytes));
    ImageJobs jobs{};
    uint32_t off = 0, blocks = 0;
    for (uint32_t k = 0; k < n_ops; ++k)
        if (!pp.ops[k].after_previous) {
            pp.ops[k].act_offset = off;
            pp.ops[k].prebuilt = 1u;
            jobs.x[jobs.n_jobs] = pp.ops[k].x;
            jobs.nb[jobs.n_jobs] = pp.ops[k].nb;
            jobs.offset[jobs.n_jobs] = off;
            jobs.first_block[jobs.n_jobs] = blocks;
            blocks += pp.ops[k].nb;
            jobs.n_jobs++;
            off += q8k_image_bytes(pp.ops[k].nb);
        }
    jobs.first_block[jobs.n_jobs] = blocks;
    const uint32_t prebuilt_bytes = off;
    for (uint32_t k = 0; k < n_ops; ++k)
        if (pp.ops[k].after_previous) {
            pp.ops[k].act_offset = off;
            pp.ext[k].build = 1u;
            off += q8k_image_bytes(pp.ops[k].nb);
        }
    pp.act_bytes = off + 256;  // + reduction scratch
    {
        // the same stage planning as the context entry points, with their defaults
        const oracle_cuda_context defaults{};
        std::string why;
        st = plan_program_ring(pp, uint64_t(dev->smem_optin), defaults.program_stage_target, why);
        if (st != ORACLE_CUDA_OK) return fail(nullptr, st, why);
        pp.copy_chunk = defaults.copy_chunk;
        pp.max_inflight = defaults.max_inflight < pp.stages ? defaults.max_inflight : pp.stages;
    }
    pp.images = dev->scratch;
    pp.prebuilt_bytes = prebuilt_bytes;
    pp.counters = reinterpret_cast<unsigned int*>(dev->scratch + kNoAllocCountersOffset);
    pp.status = reinterpret_cast<DeviceStatus*>(dev->scratch + kNoAllocStatusOffset);
    pp.px.world = 1;  // one GPU: the single-GPU release path for dependent ops

    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // Counters and status must start at zero; the array keeps whatever the
    // previous call left there.
    if ((e = cudaMemsetAsync(dev->scratch + kNoAllocCountersOffset, 0, 512, s)) != cudaSuccess)
        return cuda_fail(nullptr, e, "cudaMemsetAsync(no-allocation counters)");
    if (prebuilt_bytes > 0) {
        // one warp per 256-block, as the context entry points launch it
        quantize_images_kernel<<<blocks, 32, 0, s>>>(jobs, dev->scratch);
        if ((e = cudaGetLastError()) != cudaSuccess) return cuda_fail(nullptr, e, "quantize_images_kernel launch");
    }
    const uint32_t grid = static_cast<uint32_t>(max_rows < uint64_t(dev->sm_count) ? max_rows : dev->sm_count);
    const size_t smem = stream_barrier_bytes(pp.stages) + pp.act_bytes + size_t(pp.stages) * pp.stage_bytes;
    select_program_kernel(pp, false)<<<grid, dim3((kProgramWarps + 1) * 32), smem, s>>>(pp);
    if ((e = cudaGetLastError()) != cudaSuccess) return cuda_fail(nullptr, e, "matvec_program_kernel launch");
    return ORACLE_CUDA_OK;
}

extern "C" oracle_cuda_status oracle_cuda_noalloc_status(int device) {
    int current = 0;
    cudaError_t e = cudaGetDevice(&current);
    if (e != cudaSuccess) return cuda_fail(nullptr, e, "cudaGetDevice");
    if (current != device && (e = cudaSetDevice(device)) != cudaSuccess) return cuda_fail(nullptr, e, "cudaSetDevice");
    NoAllocDevice* dev = nullptr;
    oracle_cuda_status st = noalloc_setup(device, &dev);  // with `device` current
    if (st != ORACLE_CUDA_OK) {
        if (current != device) cudaSetDevice(current);
        return st;
    }
    // a plain device-to-host copy of the status word (it waits for the device's
    // work to finish and allocates nothing); the next call clears the word
    DeviceStatus h{};
    e = cudaMemcpy(&h, dev->scratch + kNoAllocStatusOffset, sizeof(h), cudaMemcpyDeviceToHost);
    if (current != device) cudaSetDevice(current);
    if (e != cudaSuccess) return cuda_fail(nullptr, e, "cudaMemcpy(no-allocation status)");
    if (h.code != kDevOk)
        return fail(nullptr, ORACLE_CUDA_DEVICE_TIMEOUT,
                    "kernel wait timed out at site " + std::to_string(h.where) + " in block " +
                        std::to_string(h.block) + " (last no-allocation call)");
    return ORACLE_CUDA_OK;
}

extern "C" oracle_cuda_status oracle_cuda_noalloc_selftest_bounded_wait(uint64_t limit_ns, void* stream) {
    if (limit_ns == 0 || limit_ns > 2000000000ull)
        return fail(nullptr, ORACLE_CUDA_INVALID_ARGUMENT, "self-test deadline must be in (0, 2 s]");
    int device = 0;
    cudaError_t e = cudaGetDevice(&device);
    if (e != cudaSuccess) return cuda_fail(nullptr, e, "cudaGetDevice");
    NoAllocDevice* dev = nullptr;
    oracle_cuda_status st = noalloc_setup(device, &dev);
    if (st != ORACLE_CUDA_OK) return st;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if ((e = cudaMemsetAsync(dev->scratch + kNoAllocCountersOffset, 0, 512, s)) != cudaSuccess)
        return cuda_fail(nullptr, e, "cudaMemsetAsync(no-allocation counters)");
    bounded_wait_selftest_kernel<<<1, 32, 0, s>>>(reinterpret_cast<DeviceStatus*>(dev->scratch + kNoAllocStatusOffset),
                                                 limit_ns);
    if ((e = cudaGetLastError()) != cudaSuccess) return cuda_fail(nullptr, e, "bounded_wait_selftest_kernel launch");
    return ORACLE_CUDA_OK;
}

// ---------------------------------------------------------------- prefill dequant-GEMM

namespace {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_tiled() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

bool q80_split_fits(const MatvecSeqParams& sp) {
    return sp.k % kQ80ChunkElems == 0 && sp.rows > 0 && sp.rows <= 0x7FFFFFFFull &&
           reinterpret_cast<uintptr_t>(sp.w) % 16 == 0 && reinterpret_cast<uintptr_t>(sp.x) % 16 == 0 &&
           sp.row_bytes == uint64_t(sp.k) / 32u * 34u;
}

oracle_cuda_status launch_q80_split(oracle_cuda_context* ctx, const MatvecSeqParams& sp, cudaStream_t stream) {
    const EncodeTiledFn encode = encode_tiled();
    if (!encode) return fail(ctx, ORACLE_CUDA_CUDA_ERROR, "cuTensorMapEncodeTiled is unavailable");
    CUtensorMap tw{};
    // the rows as 2-byte elements (Q8_0 blocks are 34 bytes): a box of 136 x 32
    // is 8 blocks of 32 rows, 272 bytes per row (a multiple of 16)
    const cuuint64_t dims[2] = {sp.row_bytes / 2, sp.rows};
    const cuuint64_t strides[1] = {sp.row_bytes};
    const cuuint32_t box[2] = {kQ80ChunkBytes / 2, kQ80LaneRows};
    const cuuint32_t estr[2] = {1, 1};
    if (encode(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<uint8_t*>(sp.w), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return fail(ctx, ORACLE_CUDA_CUDA_ERROR, "tensor map for the Q8_0 rows rejected");
    const uint32_t grid = static_cast<uint32_t>((sp.rows + kQ80LaneRows - 1) / kQ80LaneRows);
    return launch(ctx, matvec_q80_split_kernel, dim3(grid), dim3(32 * (1 + kQ80ProdWarps)), q80_split_smem_bytes(),
                  stream, false, tw, sp.x,
                  sp.y, static_cast<uint32_t>(sp.rows), sp.k, ctx->status);
}

// Columns per split of K: halve while the grid is at most half the SMs and
// each split keeps at least 1024 columns of whole super-blocks.
uint32_t gemm_k_per_split(uint64_t tiles, uint64_t cols, int sm_count) {
    uint64_t splits = 1;
    while (tiles * splits * 2 <= uint64_t(sm_count) && (cols / 256) % (splits * 2) == 0 &&
           cols / (splits * 2) >= 1024)
        splits *= 2;
    return static_cast<uint32_t>(cols / splits);
}

}  // namespace

extern "C" oracle_cuda_status oracle_cuda_prefill_gemm(oracle_cuda_context* ctx, uint32_t type, uint64_t rows,
                                                       uint64_t cols, const void* w_dev, uint64_t w_nbytes,
                                                       const float* x_dev, uint64_t m, float* y_dev,
                                                       void* stream_handle) {
    const cudaStream_t stream = static_cast<cudaStream_t>(stream_handle);
    if (!ctx) return fail(nullptr, ORACLE_CUDA_INVALID_ARGUMENT, "context is null");
    if (rows == 0 || cols == 0 || m == 0)
        return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "prefill GEMM dimensions must be positive");
    uint64_t row_bytes = 0;
    if (Error e = row_byte_size(cols, type, &row_bytes)) return fail(ctx, e);
    if (type != kTypeQ4_K) return fail(ctx, ORACLE_CUDA_UNSUPPORTED, "prefill GEMM supports Q4_K weights only");
    uint64_t total = 0;
    if (!checked_mul(rows, row_bytes, &total)) return fail(ctx, ORACLE_CUDA_OVERFLOW, "prefill GEMM weight size overflow");
    if (w_nbytes != total) return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "prefill GEMM weight byte size mismatch");
    if (Error e = check_weight_pointer(type, w_dev)) return fail(ctx, e);
    if (!x_dev || (reinterpret_cast<uintptr_t>(x_dev) & 15u))
        return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "activation pointer must be non-null and 16-byte aligned");
    if (!y_dev) return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "output pointer is null");
    if (rows > 0x7FFFFFFFull || m > 0x7FFFFFFFull || cols > 0x7FFFFFFFull)
        return fail(ctx, ORACLE_CUDA_UNSUPPORTED, "prefill GEMM dimensions above 2^31");
    const EncodeTiledFn encode = encode_tiled();
    if (!encode) return fail(ctx, ORACLE_CUDA_CUDA_ERROR, "cuTensorMapEncodeTiled is unavailable");
    ORACLE_CUDA_TRY(ctx, cudaSetDevice(ctx->device), "cudaSetDevice");
    oracle_cuda_status s = grow_device(ctx, ctx->gemm_x, ctx->gemm_x_len, m * cols);
    if (s != ORACLE_CUDA_OK) return s;

    // activations to bf16
    const uint64_t n4 = m * cols / 4;
    uint64_t blocks = (n4 + 256 * kConvertUnroll - 1) / (256 * kConvertUnroll);
    if (blocks > uint64_t(ctx->sm_count) * 8) blocks = uint64_t(ctx->sm_count) * 8;
    s = launch(ctx, convert_bf16_kernel, dim3(static_cast<uint32_t>(blocks)), dim3(256), 0, stream, false, x_dev,
               reinterpret_cast<uint32_t*>(ctx->gemm_x), n4);
    if (s != ORACLE_CUDA_OK) return s;

    const uint64_t tiles_m = (m + kGemmTileM - 1) / kGemmTileM, tiles_n = (rows + kGemmTileN - 1) / kGemmTileN;
    // CTA pairs (cta_group::2) when enabled (ORACLE_CUDA_GEMM_PAIR=1)
    const bool pair = ctx->gemm_pair && tiles_n >= 2;
    const uint64_t grid_n = pair ? (tiles_n + 1) / 2 * 2 : tiles_n;
    if (grid_n > 0x7FFFFFFFull || tiles_m > 65535)
        return fail(ctx, ORACLE_CUDA_UNSUPPORTED, "prefill GEMM grid too large for one launch");
    CUtensorMap tx{}, tw{};
    {
        const cuuint64_t dims[2] = {cols, m};
        const cuuint64_t strides[1] = {cols * 2};
        const cuuint32_t box[2] = {kGemmTileK, pair ? GemmPlan<true>::kBRows : GemmPlan<false>::kBRows};
        const cuuint32_t estr[2] = {1, 1};
        if (encode(&tx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, ctx->gemm_x, dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return fail(ctx, ORACLE_CUDA_CUDA_ERROR, "tensor map for the activations rejected");
    }
    {
        const cuuint64_t dims[2] = {row_bytes, rows};
        const cuuint64_t strides[1] = {row_bytes};
        const cuuint32_t box[2] = {kGemmSbBytes, kGemmTileN};
        const cuuint32_t estr[2] = {1, 1};
        if (encode(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(w_dev), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return fail(ctx, ORACLE_CUDA_CUDA_ERROR, "tensor map for the weights rejected");
    }
    GemmParams gp{};
    gp.y = y_dev;
    gp.n = static_cast<uint32_t>(rows);
    gp.m = static_cast<uint32_t>(m);
    gp.k = static_cast<uint32_t>(cols);
    gp.status = ctx->status;
    const uint64_t tiles = tiles_m * grid_n;
    const uint64_t sms = static_cast<uint64_t>(ctx->sm_count);
    // Whole waves of whole tiles, then the remaining tiles (rounded up to
    // whole weight-row tiles, so their outputs are whole column ranges of y)
    // split along K so that they fill the last wave: one launch each, when
    // splitting the remainder shortens it (else one launch of every tile).
    uint64_t tail = tiles % sms, best_splits = 1;
    tail = (tail + tiles_m - 1) / tiles_m * tiles_m;
    if (!pair && tiles > sms && tail < tiles) {
        double best_cost = static_cast<double>((tail + sms - 1) / sms);
        for (uint64_t sp = 2; sp <= 8; sp *= 2) {
            if ((cols / 256) % sp != 0 || cols / sp < 1024) break;
            const double cost = static_cast<double>((tail * sp + sms - 1) / sms) / static_cast<double>(sp);
            if (cost < best_cost - 1e-9) {
                best_cost = cost;
                best_splits = sp;
            }
        }
    }
    if (best_splits > 1) {
        const uint64_t head = tiles - tail;
        gp.tiles_m = static_cast<uint32_t>(tiles_m);
        if (head > 0) {
            gp.tile_base = 0;
            gp.k_per_split = static_cast<uint32_t>(cols);
            gp.accumulate = 0;
            oracle_cuda_status ls = launch(ctx, gemm_q4k_bf16_kernel<false>, dim3(static_cast<uint32_t>(head), 1, 1),
                                           dim3(kGemmThreads), GemmPlan<false>::kSmemBytes, stream, false, tx, tw, gp);
            if (ls != ORACLE_CUDA_OK) return ls;
        }
        gp.tile_base = static_cast<uint32_t>(head);
        gp.k_per_split = static_cast<uint32_t>(cols / best_splits);
        gp.accumulate = 1u;
        const uint64_t n_first = head / tiles_m * kGemmTileN;  // first weight row of the tail tiles
        ORACLE_CUDA_TRY(ctx,
                        cudaMemset2DAsync(y_dev + n_first, rows * sizeof(float), 0, (rows - n_first) * sizeof(float),
                                          m, stream),
                        "cudaMemset2DAsync");
        return launch(ctx, gemm_q4k_bf16_kernel<false>,
                      dim3(static_cast<uint32_t>(tail), 1, static_cast<uint32_t>(best_splits)), dim3(kGemmThreads),
                      GemmPlan<false>::kSmemBytes, stream, false, tx, tw, gp);
    }
    gp.k_per_split = gemm_k_per_split(tiles, cols, ctx->sm_count);
    gp.accumulate = gp.k_per_split < cols ? 1u : 0u;
    if (gp.accumulate) ORACLE_CUDA_TRY(ctx, cudaMemsetAsync(y_dev, 0, m * rows * sizeof(float), stream), "cudaMemsetAsync");
    const dim3 grid(static_cast<uint32_t>(grid_n), static_cast<uint32_t>(tiles_m),
                    static_cast<uint32_t>(cols / gp.k_per_split));
    if (!pair)
        return launch(ctx, gemm_q4k_bf16_kernel<false>, grid, dim3(kGemmThreads), GemmPlan<false>::kSmemBytes, stream,
                      false, tx, tw, gp);
    // clusters of two CTAs along x
    const void* key = reinterpret_cast<const void*>(gemm_q4k_bf16_kernel<true>);
    if (!ctx->smem_configured.count(key)) {
        ORACLE_CUDA_TRY(ctx,
                        cudaFuncSetAttribute(gemm_q4k_bf16_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             ctx->max_smem_optin),
                        "cudaFuncSetAttribute");
        ctx->smem_configured.insert(key);
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(kGemmThreads);
    cfg.dynamicSmemBytes = GemmPlan<true>::kSmemBytes;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    ORACLE_CUDA_TRY(ctx, cudaLaunchKernelEx(&cfg, gemm_q4k_bf16_kernel<true>, tx, tw, gp), "kernel launch");
    ctx->launches += 1;
    return ORACLE_CUDA_OK;
}

// ---------------------------------------------------------------- embedding gather, greedy argmax

namespace {

template <uint32_t kType>
oracle_cuda_status launch_gather_typed(oracle_cuda_context* ctx, const uint8_t* w, uint64_t rows, uint64_t cols,
                                       uint64_t row_bytes, const uint32_t* ids, uint64_t n_ids, float* out,
                                       cudaStream_t stream) {
    const uint64_t total = n_ids * ((cols + 3) / 4);
    uint64_t blocks = (total + 255) / 256;
    const uint64_t cap = uint64_t(ctx->sm_count) * 8;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    return launch(ctx, gather_rows_kernel<kType>, dim3(static_cast<uint32_t>(blocks)), dim3(256), 0, stream,
                  (ctx->flags & ORACLE_CUDA_FLAG_PDL) != 0, w,
                  rows, static_cast<uint32_t>(cols), row_bytes, ids, n_ids, out, ctx->status);
}

}  // namespace

extern "C" oracle_cuda_status oracle_cuda_gather_rows(oracle_cuda_context* ctx, uint32_t type, uint64_t rows,
                                                      uint64_t cols, const void* w_dev, uint64_t w_nbytes,
                                                      const uint32_t* ids_dev, uint64_t n_ids, float* out_dev,
                                                      void* stream) {
    if (!ctx) return fail(nullptr, ORACLE_CUDA_INVALID_ARGUMENT, "context is null");
    uint64_t rb = 0, total = 0;
    if (rows == 0) return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "GGUF tensor must have at least one dimension");
    if (Error e = row_byte_size(cols, type, &rb)) return fail(ctx, e);
    if (!checked_mul(rows, rb, &total))
        return fail(ctx, ORACLE_CUDA_OVERFLOW, "GGUF tensor byte size exceeds addressable size");
    if (w_nbytes != total)
        return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "GGUF tensor byte size does not match row geometry");
    if (Error e = check_decodable(type)) return fail(ctx, e);
    if (cols > 0xFFFFFFFFull || rows > 0xFFFFFFFFull)
        return fail(ctx, ORACLE_CUDA_UNSUPPORTED, "tables above 2^32 rows or columns");
    if (Error e = check_weight_pointer(type, w_dev)) return fail(ctx, e);
    if (n_ids == 0) return ok(ctx);
    if (!ids_dev || !out_dev) return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "null token ids or output");
    ORACLE_CUDA_TRY(ctx, cudaSetDevice(ctx->device), "cudaSetDevice");
    const uint8_t* wb = static_cast<const uint8_t*>(w_dev);
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    oracle_cuda_status s;
    switch (type) {
        case kTypeF32: s = launch_gather_typed<0>(ctx, wb, rows, cols, rb, ids_dev, n_ids, out_dev, st); break;
        case kTypeF16: s = launch_gather_typed<1>(ctx, wb, rows, cols, rb, ids_dev, n_ids, out_dev, st); break;
        case kTypeBF16: s = launch_gather_typed<30>(ctx, wb, rows, cols, rb, ids_dev, n_ids, out_dev, st); break;
        case kTypeQ8_0: s = launch_gather_typed<8>(ctx, wb, rows, cols, rb, ids_dev, n_ids, out_dev, st); break;
        case kTypeQ4_K: s = launch_gather_typed<12>(ctx, wb, rows, cols, rb, ids_dev, n_ids, out_dev, st); break;
        case kTypeQ5_K: s = launch_gather_typed<13>(ctx, wb, rows, cols, rb, ids_dev, n_ids, out_dev, st); break;
        case kTypeQ6_K: s = launch_gather_typed<14>(ctx, wb, rows, cols, rb, ids_dev, n_ids, out_dev, st); break;
        default: return fail(ctx, check_decodable(type));
    }
    return s == ORACLE_CUDA_OK ? ok(ctx) : s;
}

extern "C" oracle_cuda_status oracle_cuda_argmax(oracle_cuda_context* ctx, const float* x_dev, uint64_t n,
                                                 uint32_t index_base, unsigned long long* key_dev, void* stream) {
    if (!ctx) return fail(nullptr, ORACLE_CUDA_INVALID_ARGUMENT, "context is null");
    if (n == 0) return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "cannot sample an empty logits vector");
    if (n + index_base > 0xFFFFFFFFull)
        return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "logits vector exceeds token-id range");
    if (!x_dev || !key_dev) return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "null logits or key");
    ORACLE_CUDA_TRY(ctx, cudaSetDevice(ctx->device), "cudaSetDevice");
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    ORACLE_CUDA_TRY(ctx, cudaMemsetAsync(key_dev, 0, sizeof(unsigned long long), st), "cudaMemsetAsync");
    uint64_t blocks = (n + 255) / 256;
    if (blocks > uint64_t(ctx->sm_count) * 4) blocks = uint64_t(ctx->sm_count) * 4;
    const oracle_cuda_status s =
        launch(ctx, argmax_kernel, dim3(static_cast<uint32_t>(blocks)), dim3(256), 0, st,
               (ctx->flags & ORACLE_CUDA_FLAG_PDL) != 0, x_dev, n, index_base,
               key_dev);
    return s == ORACLE_CUDA_OK ? ok(ctx) : s;
}

extern "C" oracle_cuda_status oracle_cuda_argmax_decode(unsigned long long key, uint32_t* token, float* value) {
    const ArgmaxResult r = decode_argmax_key(key);
    if (r.nan) return fail(nullptr, ORACLE_CUDA_INVALID_ARGUMENT, "logits contain NaN");
    if (!r.finite) return fail(nullptr, ORACLE_CUDA_INVALID_ARGUMENT, "logits contain no finite candidates");
    if (token) *token = r.index;
    if (value) *value = r.value;
    return ORACLE_CUDA_OK;
}

extern "C" oracle_cuda_status oracle_cuda_greedy_token(oracle_cuda_context* ctx, const float* logits_dev, uint64_t n,
                                                       uint32_t* token) {
    if (!ctx) return fail(nullptr, ORACLE_CUDA_INVALID_ARGUMENT, "context is null");
    if (!token) return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "token pointer is null");
    ORACLE_CUDA_TRY(ctx, cudaSetDevice(ctx->device), "cudaSetDevice");
    if (!ctx->argmax_key)
        ORACLE_CUDA_TRY(ctx, cudaMalloc(reinterpret_cast<void**>(&ctx->argmax_key), sizeof(unsigned long long)),
                        "cudaMalloc");
    oracle_cuda_status s = oracle_cuda_argmax(ctx, logits_dev, n, 0, ctx->argmax_key, nullptr);
    if (s != ORACLE_CUDA_OK) return s;
    unsigned long long key = 0;
    ORACLE_CUDA_TRY(ctx, cudaMemcpy(&key, ctx->argmax_key, sizeof key, cudaMemcpyDeviceToHost), "cudaMemcpy");
    s = oracle_cuda_argmax_decode(key, token, nullptr);
    if (s != ORACLE_CUDA_OK) return fail(ctx, s, oracle_cuda_last_error(nullptr));
    return ok(ctx);
}

// ---------------------------------------------------------------- decoder glue (decoder_ops.cuh)

namespace {

uint32_t grid_for(uint64_t n, int sm_count) {
    uint64_t b = (n + 255) / 256;
    const uint64_t cap = uint64_t(sm_count) * 16;
    if (b > cap) b = cap;
    return static_cast<uint32_t>(b < 1 ? 1 : b);
}

// position_for_frequency (reference_kernels.cpp:28-40)
uint64_t rope_coordinate(size_t f, uint64_t pt, uint64_t ph, uint64_t pw, const int32_t* sections) {
    const size_t height_count = static_cast<size_t>(sections[1]);
    const size_t width_count = static_cast<size_t>(sections[2]);
    if (f % 3u == 1u && f / 3u < height_count) return ph;
    if (f % 3u == 2u && f / 3u < width_count) return pw;
    return pt;
}

}  // namespace

extern "C" oracle_cuda_status oracle_cuda_rms_norm_rows(oracle_cuda_context* ctx, const float* in_dev,
                                                        const float* weight_dev, uint64_t rows, uint64_t width,
                                                        float eps, float* out_dev, void* stream) {
    if (!ctx) return fail(nullptr, ORACLE_CUDA_INVALID_ARGUMENT, "context is null");
    if (width == 0 || rows == 0) return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "Qwen3.5 RMSNorm dimensions are incompatible");
    if (!(eps > 0.0f) || !std::isfinite(eps))
        return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "Qwen3.5 RMSNorm epsilon must be positive and finite");
    if (rows > 0x7FFFFFFFull || width > 0xFFFFFFFFull) return fail(ctx, ORACLE_CUDA_UNSUPPORTED, "RMSNorm shape too large");
    ORACLE_CUDA_TRY(ctx, cudaSetDevice(ctx->device), "cudaSetDevice");
    const oracle_cuda_status s = launch(ctx, rms_norm_rows_kernel, dim3(static_cast<uint32_t>(rows)), dim3(256), 0,
                                        static_cast<cudaStream_t>(stream), false, in_dev, weight_dev,
                                        static_cast<uint32_t>(width), eps, out_dev);
    return s == ORACLE_CUDA_OK ? ok(ctx) : s;
}

extern "C" oracle_cuda_status oracle_cuda_rope(oracle_cuda_context* ctx, float* heads_dev, uint64_t n_heads,
                                               uint64_t head_dim, uint64_t rotary_dim, const int32_t* sections,
                                               float base, uint64_t pos_temporal, uint64_t pos_height,
                                               uint64_t pos_width, void* stream) {
    if (!ctx) return fail(nullptr, ORACLE_CUDA_INVALID_ARGUMENT, "context is null");
    // apply_qwen35_rope's checks (reference_kernels.cpp:79-99), same messages
    if (rotary_dim == 0 || rotary_dim % 2 != 0 || rotary_dim > head_dim)
        return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "RoPE dimension must be non-zero, even, and within head width");
    if (!(base > 0.0f) || !std::isfinite(base))
        return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "RoPE frequency base must be positive and finite");
    if (!sections) return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "RoPE sections pointer is null");
    int64_t section_sum = 0;
    for (int i = 0; i < 4; ++i) {
        if (sections[i] < 0) return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "RoPE dimension sections must be non-negative");
        section_sum += sections[i];
    }
    if (section_sum != static_cast<int64_t>(rotary_dim / 2))
        return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "RoPE dimension sections must sum to half the rotary dimension");
    if (rotary_dim / 2 > kRopeMaxHalf || n_heads * (rotary_dim / 2) > 0xFFFFFFFFull)
        return fail(ctx, ORACLE_CUDA_UNSUPPORTED, "rotary dimension above 256");
    // the cos/sin table, by the reference's own expressions (reference_kernels.cpp:104-113)
    RopeTable t{};
    t.half = static_cast<uint32_t>(rotary_dim / 2);
    for (size_t f = 0; f < t.half; ++f) {
        const double exponent = (2.0 * static_cast<double>(f)) / static_cast<double>(rotary_dim);
        const double inverse_frequency = 1.0 / std::pow(base, exponent);
        const uint64_t coordinate = rope_coordinate(f, pos_temporal, pos_height, pos_width, sections);
        const double angle = static_cast<double>(coordinate) * inverse_frequency;
        t.cosv[f] = static_cast<float>(std::cos(angle));
        t.sinv[f] = static_cast<float>(std::sin(angle));
    }
    ORACLE_CUDA_TRY(ctx, cudaSetDevice(ctx->device), "cudaSetDevice");
    const uint64_t n = n_heads * t.half;
    const oracle_cuda_status s = launch(ctx, rope_kernel, dim3(static_cast<uint32_t>((n + 255) / 256)), dim3(256), 0,
                                        static_cast<cudaStream_t>(stream), false, heads_dev,
                                        static_cast<uint32_t>(n_heads), static_cast<uint32_t>(head_dim), t);
    return s == ORACLE_CUDA_OK ? ok(ctx) : s;
}

extern "C" oracle_cuda_status oracle_cuda_attention_step(oracle_cuda_context* ctx, const float* q_dev,
                                                         const float* k_new_dev, const float* v_new_dev,
                                                         float* keys_dev, float* values_dev, uint64_t capacity,
                                                         uint64_t length, uint32_t q_heads, uint32_t kv_heads,
                                                         uint32_t key_dim, uint32_t value_dim, float* scores_dev,
                                                         float* out_dev, void* stream) {
    if (!ctx) return fail(nullptr, ORACLE_CUDA_INVALID_ARGUMENT, "context is null");
    if (kv_heads == 0 || q_heads % kv_heads != 0 || key_dim == 0 || value_dim == 0)
        return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "causal_attention_step dimensions are incompatible");
    if (length >= capacity) return fail(ctx, ORACLE_CUDA_OVERFLOW, "KV cache capacity exceeded");
    if (length + 1 > 0xFFFFFFFFull) return fail(ctx, ORACLE_CUDA_UNSUPPORTED, "attention over more than 2^32 tokens");
    ORACLE_CUDA_TRY(ctx, cudaSetDevice(ctx->device), "cudaSetDevice");
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    const uint32_t tokens = static_cast<uint32_t>(length + 1);
    const uint32_t nk = kv_heads * key_dim, nv = kv_heads * value_dim;
    oracle_cuda_status s = launch(ctx, attention_append_kernel, dim3(grid_for(nk + nv, ctx->sm_count)), dim3(256), 0,
                                  st, false, k_new_dev, v_new_dev, keys_dev, values_dev, length, nk, nv);
    if (s != ORACLE_CUDA_OK) return s;
    const float scale = 1.0f / std::sqrt(static_cast<float>(key_dim));
    const uint64_t warps = uint64_t(q_heads) * tokens;
    s = launch(ctx, attention_scores_kernel, dim3(static_cast<uint32_t>((warps * 32 + 255) / 256)), dim3(256), 0, st,
               false, q_dev, static_cast<const float*>(keys_dev), tokens, q_heads, kv_heads, key_dim, scale,
               scores_dev);
    if (s != ORACLE_CUDA_OK) return s;
    s = launch(ctx, attention_output_kernel, dim3(q_heads), dim3(256), 0, st, false, scores_dev,
               static_cast<const float*>(values_dev), tokens, q_heads, kv_heads, value_dim, out_dev, ctx->status);
    return s == ORACLE_CUDA_OK ? ok(ctx) : s;
}

extern "C" oracle_cuda_status oracle_cuda_conv_step(oracle_cuda_context* ctx, const float* in_dev,
                                                    const float* weights_dev, float* history_dev, uint64_t channels,
                                                    uint32_t kernel, int apply_silu, float* out_dev, void* stream) {
    if (!ctx) return fail(nullptr, ORACLE_CUDA_INVALID_ARGUMENT, "context is null");
    if (channels == 0 || kernel == 0 || channels > 0xFFFFFFFFull)
        return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "depthwise convolution dimensions do not match SSM state");
    ORACLE_CUDA_TRY(ctx, cudaSetDevice(ctx->device), "cudaSetDevice");
    const oracle_cuda_status s = launch(ctx, conv_step_kernel, dim3(static_cast<uint32_t>((channels + 255) / 256)),
                                        dim3(256), 0, static_cast<cudaStream_t>(stream), false, in_dev, weights_dev,
                                        history_dev, static_cast<uint32_t>(channels), kernel, apply_silu, out_dev);
    return s == ORACLE_CUDA_OK ? ok(ctx) : s;
}

extern "C" oracle_cuda_status oracle_cuda_gated_delta_step(oracle_cuda_context* ctx, const float* q_dev,
                                                           const float* k_dev, const float* v_dev,
                                                           const float* beta_dev, const float* log_decay_dev,
                                                           float* state_dev, uint32_t heads, uint32_t qk_heads,
                                                           uint32_t key_dim, uint32_t value_dim, float eps,
                                                           float* out_dev, void* stream) {
    if (!ctx) return fail(nullptr, ORACLE_CUDA_INVALID_ARGUMENT, "context is null");
    if (!(eps > 0.0f)) return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "gated delta normalization epsilon must be positive");
    if (heads == 0 || key_dim == 0 || value_dim == 0)
        return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "gated_delta_step dimensions do not match SSM state");
    if (qk_heads == 0 || heads % qk_heads != 0)  // repeat_heads_tiled (qwen35_block.cpp:229-233)
        return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "Qwen3.5 repeated-head dimensions are incompatible");
    if (value_dim > 1024 || value_dim % 32 != 0 || key_dim > 4096)
        return fail(ctx, ORACLE_CUDA_UNSUPPORTED, "gated delta value dimension must be a multiple of 32 up to 1024");
    ORACLE_CUDA_TRY(ctx, cudaSetDevice(ctx->device), "cudaSetDevice");
    const oracle_cuda_status s =
        launch(ctx, gated_delta_kernel, dim3(heads), dim3(value_dim), 2 * key_dim * sizeof(float),
               static_cast<cudaStream_t>(stream), false, q_dev, k_dev, v_dev, beta_dev, log_decay_dev, state_dev,
               qk_heads, key_dim, value_dim, eps, out_dev);
    return s == ORACLE_CUDA_OK ? ok(ctx) : s;
}

extern "C" oracle_cuda_status oracle_cuda_swiglu(oracle_cuda_context* ctx, const float* gate_dev, const float* up_dev,
                                                 uint64_t n, float* out_dev, void* stream) {
    if (!ctx) return fail(nullptr, ORACLE_CUDA_INVALID_ARGUMENT, "context is null");
    if (n == 0) return ok(ctx);
    ORACLE_CUDA_TRY(ctx, cudaSetDevice(ctx->device), "cudaSetDevice");
    const oracle_cuda_status s = launch(ctx, swiglu_kernel, dim3(grid_for(n, ctx->sm_count)), dim3(256), 0,
                                        static_cast<cudaStream_t>(stream), false, gate_dev, up_dev, n, out_dev);
    return s == ORACLE_CUDA_OK ? ok(ctx) : s;
}

extern "C" oracle_cuda_status oracle_cuda_add(oracle_cuda_context* ctx, const float* a_dev, const float* b_dev,
                                              uint64_t n, float* out_dev, void* stream) {
    if (!ctx) return fail(nullptr, ORACLE_CUDA_INVALID_ARGUMENT, "context is null");
    if (n == 0) return ok(ctx);
    ORACLE_CUDA_TRY(ctx, cudaSetDevice(ctx->device), "cudaSetDevice");
    const oracle_cuda_status s = launch(ctx, add_kernel, dim3(grid_for(n, ctx->sm_count)), dim3(256), 0,
                                        static_cast<cudaStream_t>(stream), false, a_dev, b_dev, n, out_dev);
    return s == ORACLE_CUDA_OK ? ok(ctx) : s;
}

// ---------------------------------------------------------------- graph-replayable decode step

extern "C" oracle_cuda_status oracle_cuda_rope_table(oracle_cuda_context* ctx, uint64_t rotary_dim,
                                                     const int32_t* sections, float base, uint64_t positions,
                                                     float* table_dev) {
    if (!ctx) return fail(nullptr, ORACLE_CUDA_INVALID_ARGUMENT, "context is null");
    if (rotary_dim == 0 || rotary_dim % 2 != 0)
        return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "RoPE dimension must be non-zero, even, and within head width");
    if (!(base > 0.0f) || !std::isfinite(base))
        return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "RoPE frequency base must be positive and finite");
    if (!sections) return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "RoPE sections pointer is null");
    int64_t section_sum = 0;
    for (int i = 0; i < 4; ++i) {
        if (sections[i] < 0) return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "RoPE dimension sections must be non-negative");
        section_sum += sections[i];
    }
    if (section_sum != static_cast<int64_t>(rotary_dim / 2))
        return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "RoPE dimension sections must sum to half the rotary dimension");
    if (positions == 0 || positions > 0xFFFFFFFFull || rotary_dim / 2 > kRopeMaxHalf)
        return fail(ctx, ORACLE_CUDA_UNSUPPORTED, "RoPE table positions must be in [1, 2^32), rotary dimension <= 256");
    if (!table_dev) return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "RoPE table pointer is null");
    // apply_qwen35_rope's expressions (reference_kernels.cpp:104-113) for text
    // positions (RopePosition::text: every coordinate equals the position)
    const size_t half = rotary_dim / 2;
    std::vector<double> inverse_frequency(half);
    for (size_t f = 0; f < half; ++f) {
        const double exponent = (2.0 * static_cast<double>(f)) / static_cast<double>(rotary_dim);
        inverse_frequency[f] = 1.0 / std::pow(base, exponent);
    }
    std::vector<float> table(positions * half * 2);
    for (uint64_t p = 0; p < positions; ++p)
        for (size_t f = 0; f < half; ++f) {
            const uint64_t coordinate = rope_coordinate(f, p, p, p, sections);
            const double angle = static_cast<double>(coordinate) * inverse_frequency[f];
            table[(p * half + f) * 2] = static_cast<float>(std::cos(angle));
            table[(p * half + f) * 2 + 1] = static_cast<float>(std::sin(angle));
        }
    ORACLE_CUDA_TRY(ctx, cudaSetDevice(ctx->device), "cudaSetDevice");
    ORACLE_CUDA_TRY(ctx, cudaMemcpy(table_dev, table.data(), table.size() * sizeof(float), cudaMemcpyHostToDevice),
                    "cudaMemcpy(RoPE table)");
    return ok(ctx);
}

extern "C" oracle_cuda_status oracle_cuda_rope_at(oracle_cuda_context* ctx, float* heads_dev, uint64_t n_heads,
                                                  uint64_t head_dim, uint64_t rotary_dim, const float* table_dev,
                                                  uint64_t positions, const uint32_t* pos_dev, void* stream) {
    if (!ctx) return fail(nullptr, ORACLE_CUDA_INVALID_ARGUMENT, "context is null");
    if (rotary_dim == 0 || rotary_dim % 2 != 0 || rotary_dim > head_dim)
        return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "RoPE dimension must be non-zero, even, and within head width");
    if (!table_dev || !pos_dev) return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "RoPE table or position pointer is null");
    if (positions > 0xFFFFFFFFull || n_heads * (rotary_dim / 2) > 0xFFFFFFFFull || head_dim > 0xFFFFFFFFull)
        return fail(ctx, ORACLE_CUDA_UNSUPPORTED, "RoPE shape too large");
    ORACLE_CUDA_TRY(ctx, cudaSetDevice(ctx->device), "cudaSetDevice");
    const uint64_t n = n_heads * (rotary_dim / 2);
    const oracle_cuda_status s =
        launch(ctx, rope_pos_kernel, dim3(static_cast<uint32_t>((n + 255) / 256)), dim3(256), 0,
               static_cast<cudaStream_t>(stream), false, heads_dev, static_cast<uint32_t>(n_heads),
               static_cast<uint32_t>(head_dim), static_cast<uint32_t>(rotary_dim / 2), table_dev, pos_dev,
               static_cast<uint32_t>(positions), ctx->status);
    return s == ORACLE_CUDA_OK ? ok(ctx) : s;
}

namespace {
// The probabilities (attention_output_pos_kernel with no values: max, exp,
// double sum, normalisation, in place) then their weighted sum of the values
// (attention_values_pos_kernel), or the single output kernel where the
// shapes do not fit the staged kernel.
oracle_cuda_status launch_attention_output(oracle_cuda_context* ctx, cudaStream_t st, bool pdl, float* scores,
                                           const float* values, const uint32_t* pos, uint32_t cap,
                                           uint32_t q_heads, uint32_t kv_heads, uint32_t value_dim,
                                           const float* gate, uint32_t gate_stride, float* out) {
    const uint32_t group = q_heads / kv_heads;
    const bool staged = value_dim % kAttnDims == 0 && group * kAttnDims <= 1024 &&
                        reinterpret_cast<uintptr_t>(values) % 16 == 0 &&
                        attn_values_smem_floats(group) * sizeof(float) <= size_t(ctx->max_smem_optin);
    oracle_cuda_status s = launch(ctx, attention_output_pos_kernel, dim3(q_heads), dim3(256), 0, st, pdl, scores,
                                  staged ? static_cast<const float*>(nullptr) : values, pos, cap, q_heads, kv_heads,
                                  value_dim, gate, gate_stride, out, ctx->status);
    if (s != ORACLE_CUDA_OK || !staged) return s;
    const size_t smem = size_t(attn_values_smem_floats(group)) * sizeof(float);
    return launch(ctx, attention_values_pos_kernel, dim3(kv_heads, value_dim / kAttnDims), dim3(group * kAttnDims),
                  smem, st, pdl, static_cast<const float*>(scores), values, pos, cap, q_heads, kv_heads, value_dim,
                  gate, gate_stride, out);
}
}  // namespace

extern "C" oracle_cuda_status oracle_cuda_attention_step_at(oracle_cuda_context* ctx, const float* q_dev,
                                                            const float* k_new_dev, const float* v_new_dev,
                                                            float* keys_dev, float* values_dev, uint64_t capacity,
                                                            const uint32_t* pos_dev, uint32_t q_heads,
                                                            uint32_t kv_heads, uint32_t key_dim, uint32_t value_dim,
                                                            float* scores_dev, float* out_dev, void* stream) {
    if (!ctx) return fail(nullptr, ORACLE_CUDA_INVALID_ARGUMENT, "context is null");
    if (kv_heads == 0 || q_heads % kv_heads != 0 || key_dim == 0 || value_dim == 0)
        return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "causal_attention_step dimensions are incompatible");
    if (capacity == 0 || capacity > 0xFFFFFFFFull || !pos_dev)
        return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "KV cache capacity must be in [1, 2^32) with a position");
    ORACLE_CUDA_TRY(ctx, cudaSetDevice(ctx->device), "cudaSetDevice");
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    const uint32_t cap = static_cast<uint32_t>(capacity);
    const uint32_t nk = kv_heads * key_dim, nv = kv_heads * value_dim;
    oracle_cuda_status s = launch(ctx, attention_append_pos_kernel, dim3(grid_for(nk + nv, ctx->sm_count)), dim3(256),
                                  0, st, false, k_new_dev, v_new_dev, keys_dev, values_dev, pos_dev, cap, nk, nv,
                                  ctx->status);
    if (s != ORACLE_CUDA_OK) return s;
    const float scale = 1.0f / std::sqrt(static_cast<float>(key_dim));
    // enough warps per head that a full cache takes about 32 tokens per warp
    uint32_t chunks = static_cast<uint32_t>((capacity + 255) / 256);
    if (chunks > 64) chunks = 64;
    s = launch(ctx, attention_scores_pos_kernel, dim3(q_heads, chunks), dim3(256), 0, st, false, q_dev,
               static_cast<const float*>(keys_dev), pos_dev, cap, q_heads, kv_heads, key_dim, scale, scores_dev);
    if (s != ORACLE_CUDA_OK) return s;
    s = launch_attention_output(ctx, st, false, scores_dev, values_dev, pos_dev, cap, q_heads, kv_heads, value_dim,
                                nullptr, 0u, out_dev);
    return s == ORACLE_CUDA_OK ? ok(ctx) : s;
}


extern "C" oracle_cuda_status oracle_cuda_position_advance(oracle_cuda_context* ctx, uint32_t* pos_dev,
                                                           void* stream) {
    if (!ctx) return fail(nullptr, ORACLE_CUDA_INVALID_ARGUMENT, "context is null");
    if (!pos_dev) return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "position pointer is null");
    ORACLE_CUDA_TRY(ctx, cudaSetDevice(ctx->device), "cudaSetDevice");
    const oracle_cuda_status s =
        launch(ctx, step_advance_kernel, dim3(1), dim3(32), 0, static_cast<cudaStream_t>(stream), false, pos_dev);
    return s == ORACLE_CUDA_OK ? ok(ctx) : s;
}

extern "C" oracle_cuda_status oracle_cuda_split_query_gate(oracle_cuda_context* ctx, const float* full_dev,
                                                           uint32_t heads, uint32_t width, float* query_dev,
                                                           float* gate_dev, void* stream) {
    if (!ctx) return fail(nullptr, ORACLE_CUDA_INVALID_ARGUMENT, "context is null");
    if (heads == 0 || width == 0 || uint64_t(heads) * width > 0xFFFFFFFFull)
        return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "Qwen3.5 joint query/gate projection width mismatch");
    ORACLE_CUDA_TRY(ctx, cudaSetDevice(ctx->device), "cudaSetDevice");
    const uint64_t n = uint64_t(heads) * width;
    const oracle_cuda_status s = launch(ctx, split_query_gate_kernel, dim3(static_cast<uint32_t>((n + 255) / 256)),
                                        dim3(256), 0, static_cast<cudaStream_t>(stream), false, full_dev, heads,
                                        width, query_dev, gate_dev);
    return s == ORACLE_CUDA_OK ? ok(ctx) : s;
}

extern "C" oracle_cuda_status oracle_cuda_gate_sigmoid_mul(oracle_cuda_context* ctx, float* x_dev,
                                                           const float* gate_dev, uint64_t n, void* stream) {
    if (!ctx) return fail(nullptr, ORACLE_CUDA_INVALID_ARGUMENT, "context is null");
    if (n == 0) return ok(ctx);
    if (n > 0xFFFFFFFFull) return fail(ctx, ORACLE_CUDA_UNSUPPORTED, "vector too long");
    ORACLE_CUDA_TRY(ctx, cudaSetDevice(ctx->device), "cudaSetDevice");
    const oracle_cuda_status s = launch(ctx, gate_sigmoid_mul_kernel, dim3(static_cast<uint32_t>((n + 255) / 256)),
                                        dim3(256), 0, static_cast<cudaStream_t>(stream), false, x_dev, gate_dev,
                                        static_cast<uint32_t>(n));
    return s == ORACLE_CUDA_OK ? ok(ctx) : s;
}

extern "C" oracle_cuda_status oracle_cuda_mul_silu(oracle_cuda_context* ctx, float* x_dev, const float* z_dev,
                                                   uint64_t n, void* stream) {
    if (!ctx) return fail(nullptr, ORACLE_CUDA_INVALID_ARGUMENT, "context is null");
    if (n == 0) return ok(ctx);
    if (n > 0xFFFFFFFFull) return fail(ctx, ORACLE_CUDA_UNSUPPORTED, "vector too long");
    ORACLE_CUDA_TRY(ctx, cudaSetDevice(ctx->device), "cudaSetDevice");
    const oracle_cuda_status s = launch(ctx, mul_silu_kernel, dim3(static_cast<uint32_t>((n + 255) / 256)), dim3(256),
                                        0, static_cast<cudaStream_t>(stream), false, x_dev, z_dev,
                                        static_cast<uint32_t>(n));
    return s == ORACLE_CUDA_OK ? ok(ctx) : s;
}

extern "C" oracle_cuda_status oracle_cuda_gdn_gates(oracle_cuda_context* ctx, const float* beta_dev,
                                                    const float* alpha_dev, const float* time_step_bias_dev,
                                                    const float* decay_dev, uint32_t heads, float* beta_out_dev,
                                                    float* log_decay_dev, void* stream) {
    if (!ctx) return fail(nullptr, ORACLE_CUDA_INVALID_ARGUMENT, "context is null");
    if (heads == 0) return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "Qwen3.5 recurrent alpha/beta width mismatch");
    ORACLE_CUDA_TRY(ctx, cudaSetDevice(ctx->device), "cudaSetDevice");
    const oracle_cuda_status s = launch(ctx, gdn_gates_kernel, dim3((heads + 255) / 256), dim3(256), 0,
                                        static_cast<cudaStream_t>(stream), false, beta_dev, alpha_dev,
                                        time_step_bias_dev, decay_dev, heads, beta_out_dev, log_decay_dev);
    return s == ORACLE_CUDA_OK ? ok(ctx) : s;
}

extern "C" oracle_cuda_status oracle_cuda_argmax_rows(oracle_cuda_context* ctx, const float* x_dev, uint32_t rows,
                                                      uint64_t n, unsigned long long* keys_dev, void* stream) {
    if (!ctx) return fail(nullptr, ORACLE_CUDA_INVALID_ARGUMENT, "context is null");
    if (n == 0 || rows == 0) return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "cannot sample an empty logits vector");
    if (n > 0xFFFFFFFFull) return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "logits vector exceeds token-id range");
    if (rows > 65535) return fail(ctx, ORACLE_CUDA_UNSUPPORTED, "at most 65535 logits rows per call");
    if (!x_dev || !keys_dev) return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "null logits or key");
    ORACLE_CUDA_TRY(ctx, cudaSetDevice(ctx->device), "cudaSetDevice");
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    ORACLE_CUDA_TRY(ctx, cudaMemsetAsync(keys_dev, 0, rows * sizeof(unsigned long long), st), "cudaMemsetAsync");
    uint64_t blocks = (n + 255) / 256;
    const uint64_t cap = (uint64_t(ctx->sm_count) * 4 + rows - 1) / rows;
    if (blocks > cap) blocks = cap;
    const oracle_cuda_status s =
        launch(ctx, argmax_kernel, dim3(static_cast<uint32_t>(blocks), rows), dim3(256), 0, st,
               (ctx->flags & ORACLE_CUDA_FLAG_PDL) != 0, x_dev, n, 0u, keys_dev);
    return s == ORACLE_CUDA_OK ? ok(ctx) : s;
}

extern "C" oracle_cuda_status oracle_cuda_token_commit_rows(oracle_cuda_context* ctx, unsigned long long* keys_dev,
                                                            uint32_t rows, const uint32_t* prompt_dev,
                                                            uint32_t n_prompt, uint32_t* pos_dev,
                                                            uint32_t* next_id_dev, uint32_t* tokens_dev,
                                                            uint32_t tokens_capacity, void* stream) {
    if (!ctx) return fail(nullptr, ORACLE_CUDA_INVALID_ARGUMENT, "context is null");
    if (rows == 0) return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "no sequences to commit");
    if (!keys_dev || !pos_dev || !next_id_dev || (n_prompt > 0 && !prompt_dev) ||
        (tokens_capacity > 0 && !tokens_dev))
        return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "token commit pointer is null");
    ORACLE_CUDA_TRY(ctx, cudaSetDevice(ctx->device), "cudaSetDevice");
    const oracle_cuda_status s =
        launch(ctx, token_commit_rows_kernel, dim3(1), dim3(256), 0, static_cast<cudaStream_t>(stream),
               (ctx->flags & ORACLE_CUDA_FLAG_PDL) != 0, keys_dev, rows, prompt_dev, n_prompt, pos_dev, next_id_dev,
               tokens_dev, tokens_capacity, ctx->status);
    return s == ORACLE_CUDA_OK ? ok(ctx) : s;
}

extern "C" oracle_cuda_status oracle_cuda_token_commit(oracle_cuda_context* ctx, const unsigned long long* key_dev,
                                                       const uint32_t* prompt_dev, uint32_t n_prompt,
                                                       uint32_t* pos_dev, uint32_t* next_id_dev,
                                                       uint32_t* tokens_dev, uint32_t tokens_capacity,
                                                       void* stream) {
    if (!ctx) return fail(nullptr, ORACLE_CUDA_INVALID_ARGUMENT, "context is null");
    if (!key_dev || !pos_dev || !next_id_dev || (n_prompt > 0 && !prompt_dev) || (tokens_capacity > 0 && !tokens_dev))
        return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "token commit pointer is null");
    ORACLE_CUDA_TRY(ctx, cudaSetDevice(ctx->device), "cudaSetDevice");
    const oracle_cuda_status s =
        launch(ctx, token_commit_kernel, dim3(1), dim3(32), 0, static_cast<cudaStream_t>(stream),
               (ctx->flags & ORACLE_CUDA_FLAG_PDL) != 0, key_dev,
               prompt_dev, n_prompt, pos_dev, next_id_dev, tokens_dev, tokens_capacity, ctx->status);
    return s == ORACLE_CUDA_OK ? ok(ctx) : s;
}

// ---------------------------------------------------------------- fused block cores

extern "C" oracle_cuda_status oracle_cuda_gdn_core(oracle_cuda_context* ctx, const float* qkv_dev, const float* z_dev,
                                                   const float* beta_dev, const float* alpha_dev,
                                                   const float* time_step_bias_dev, const float* decay_dev,
                                                   const float* conv_weights_dev, float* history_dev,
                                                   float* state_dev, const float* norm_dev, uint32_t key_heads,
                                                   uint32_t value_heads, uint32_t head_dim, uint32_t conv_kernel,
                                                   float eps, const uint32_t* pos_dev, float* out_dev, void* stream) {
    return oracle_cuda_gdn_core_seqs(ctx, qkv_dev, z_dev, beta_dev, alpha_dev, time_step_bias_dev, decay_dev,
                                     conv_weights_dev, history_dev, state_dev, norm_dev, key_heads, value_heads,
                                     head_dim, conv_kernel, eps, pos_dev, 1, out_dev, stream);
}

extern "C" oracle_cuda_status oracle_cuda_gdn_core_seqs(oracle_cuda_context* ctx, const float* qkv_dev,
                                                        const float* z_dev, const float* beta_dev,
                                                        const float* alpha_dev, const float* time_step_bias_dev,
                                                        const float* decay_dev, const float* conv_weights_dev,
                                                        float* history_dev, float* state_dev, const float* norm_dev,
                                                        uint32_t key_heads, uint32_t value_heads, uint32_t head_dim,
                                                        uint32_t conv_kernel, float eps, const uint32_t* pos_dev,
                                                        uint32_t seqs, float* out_dev, void* stream) {
    if (!ctx) return fail(nullptr, ORACLE_CUDA_INVALID_ARGUMENT, "context is null");
    if (seqs == 0 || seqs > 65535) return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "sequence count must be in [1, 65535]");
    if (key_heads == 0 || value_heads == 0 || value_heads % key_heads != 0)
        return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "Qwen3.5 repeated-head dimensions are incompatible");
    if (conv_kernel == 0 || head_dim == 0)
        return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "Qwen3.5 recurrent state dimensions do not match the manifest");
    if (head_dim != 64 && head_dim != 128)
        return fail(ctx, ORACLE_CUDA_UNSUPPORTED, "fused recurrent block supports head widths 64 and 128");
    if (!(eps > 0.0f) || !std::isfinite(eps))
        return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "Qwen3.5 RMSNorm epsilon must be positive and finite");
    if (!pos_dev) return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "position pointer is null");
    ORACLE_CUDA_TRY(ctx, cudaSetDevice(ctx->device), "cudaSetDevice");
    const oracle_cuda_status s =
        launch(ctx, head_dim == 128 ? gdn_core_kernel<128> : gdn_core_kernel<64>, dim3(value_heads, seqs),
               dim3(4 * head_dim), 0,
               static_cast<cudaStream_t>(stream), (ctx->flags & ORACLE_CUDA_FLAG_PDL) != 0, qkv_dev, z_dev, beta_dev, alpha_dev, time_step_bias_dev,
               decay_dev, conv_weights_dev, history_dev, state_dev, norm_dev, key_heads, value_heads, conv_kernel,
               eps, pos_dev, out_dev);
    return s == ORACLE_CUDA_OK ? ok(ctx) : s;
}

extern "C" oracle_cuda_status oracle_cuda_attention_prep_at(oracle_cuda_context* ctx, const float* q_full_dev,
                                                            const float* k_dev, const float* v_dev,
                                                            const float* q_norm_dev, const float* k_norm_dev,
                                                            float eps, const float* table_dev, uint64_t rotary_dim,
                                                            uint32_t q_heads, uint32_t kv_heads, uint32_t head_dim,
                                                            float* keys_dev, float* values_dev, uint64_t capacity,
                                                            const uint32_t* pos_dev, float* q_out_dev, void* stream) {
    if (!ctx) return fail(nullptr, ORACLE_CUDA_INVALID_ARGUMENT, "context is null");
    if (kv_heads == 0 || q_heads % kv_heads != 0 || head_dim == 0)
        return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "causal_attention_step dimensions are incompatible");
    if (rotary_dim == 0 || rotary_dim % 2 != 0 || rotary_dim > head_dim)
        return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "RoPE dimension must be non-zero, even, and within head width");
    if (head_dim % 32 != 0 || head_dim > 1024)
        return fail(ctx, ORACLE_CUDA_UNSUPPORTED, "fused attention needs a head width that is a multiple of 32 up to 1024");
    if (!(eps > 0.0f) || !std::isfinite(eps))
        return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "Qwen3.5 RMSNorm epsilon must be positive and finite");
    if (capacity == 0 || capacity > 0xFFFFFFFFull || !pos_dev || !table_dev)
        return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "KV cache capacity must be in [1, 2^32) with a position and table");
    ORACLE_CUDA_TRY(ctx, cudaSetDevice(ctx->device), "cudaSetDevice");
    const oracle_cuda_status s =
        launch(ctx, attention_prep_kernel, dim3(q_heads), dim3(head_dim), 0, static_cast<cudaStream_t>(stream),
               (ctx->flags & ORACLE_CUDA_FLAG_PDL) != 0,
               q_full_dev, k_dev, v_dev, q_norm_dev, k_norm_dev, eps, table_dev,
               static_cast<uint32_t>(rotary_dim / 2), q_heads, kv_heads, keys_dev, values_dev,
               static_cast<uint32_t>(capacity), pos_dev, q_out_dev, ctx->status);
    return s == ORACLE_CUDA_OK ? ok(ctx) : s;
}

extern "C" oracle_cuda_status oracle_cuda_attention_core_at(oracle_cuda_context* ctx, const float* q_dev,
                                                            const float* keys_dev, const float* values_dev,
                                                            uint64_t capacity, const uint32_t* pos_dev,
                                                            uint32_t q_heads, uint32_t kv_heads, uint32_t key_dim,
                                                            uint32_t value_dim, const float* gate_dev,
                                                            uint32_t gate_stride, float* scores_dev, float* out_dev,
                                                            void* stream) {
    if (!ctx) return fail(nullptr, ORACLE_CUDA_INVALID_ARGUMENT, "context is null");
    if (kv_heads == 0 || q_heads % kv_heads != 0 || key_dim == 0 || value_dim == 0)
        return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "causal_attention_step dimensions are incompatible");
    if (capacity == 0 || capacity > 0xFFFFFFFFull || !pos_dev)
        return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "KV cache capacity must be in [1, 2^32) with a position");
    ORACLE_CUDA_TRY(ctx, cudaSetDevice(ctx->device), "cudaSetDevice");
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    const uint32_t cap = static_cast<uint32_t>(capacity);
    const float scale = 1.0f / std::sqrt(static_cast<float>(key_dim));
    uint32_t chunks = static_cast<uint32_t>((capacity + 255) / 256);
    if (chunks > 64) chunks = 64;
    const bool pdl = (ctx->flags & ORACLE_CUDA_FLAG_PDL) != 0;
    oracle_cuda_status s = launch(ctx, attention_scores_pos_kernel, dim3(q_heads, chunks), dim3(256), 0, st, pdl,
                                  q_dev, keys_dev, pos_dev, cap, q_heads, kv_heads, key_dim, scale, scores_dev);
    if (s != ORACLE_CUDA_OK) return s;
    s = launch_attention_output(ctx, st, pdl, scores_dev, values_dev, pos_dev, cap, q_heads, kv_heads, value_dim,
                                gate_dev, gate_stride, out_dev);
    return s == ORACLE_CUDA_OK ? ok(ctx) : s;
}

extern "C" oracle_cuda_status oracle_cuda_matvec_program_ex_allgather(oracle_cuda_context* ctx,
                                                                      oracle_cuda_peer_group* group,
                                                                      const oracle_cuda_matvec_op_ex* ops,
                                                                      uint32_t n_ops, void* stream) {
    if (!group) return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "peer group is null");
    return program_run(ctx, ops, n_ops, stream, group);
}

static_assert(kTraceWords == ORACLE_CUDA_TRACE_WORDS, "trace record size");

extern "C" oracle_cuda_status oracle_cuda_set_program_trace(oracle_cuda_context* ctx, unsigned long long* trace_dev,
                                                            uint32_t records) {
    if (!ctx) return fail(nullptr, ORACLE_CUDA_INVALID_ARGUMENT, "context is null");
    if (records > 0 && !trace_dev) return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "trace buffer is null");
    if (trace_dev && reinterpret_cast<uintptr_t>(trace_dev) % 8)
        return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "trace buffer must be 8-byte aligned");
    ctx->trace = records > 0 ? trace_dev : nullptr;
    ctx->trace_records = records;
    return ok(ctx);
}

extern "C" oracle_cuda_status oracle_cuda_matvec_program_sharded(oracle_cuda_context* ctx,
                                                                 oracle_cuda_peer_group* group,
                                                                 const oracle_cuda_sharded_op* ops, uint32_t n_ops,
                                                                 const oracle_cuda_sharded_step* step, void* stream) {
    if (!ctx) return fail(nullptr, ORACLE_CUDA_INVALID_ARGUMENT, "context is null");
    if (!group) return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "peer group is null");
    if (!ops || n_ops == 0 || n_ops > kProgramMaxOps)
        return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT,
                    "a matvec program holds 1 to " + std::to_string(kProgramMaxOps) + " ops");
    if (!step) return fail(ctx, ORACLE_CUDA_INVALID_ARGUMENT, "step information is null");
    oracle_cuda_matvec_op_ex ex[kProgramMaxOps] = {};
    for (uint32_t k = 0; k < n_ops; ++k) ex[k] = ops[k].ex;
    return program_run(ctx, ex, n_ops, stream, group, ops, step);
}
