// ref_shim.cpp -- C entry points over Oracle's OWN compiled hot-path sources.
//
// TEST INFRASTRUCTURE ONLY.  oracle/Makefile compiles this file together with
// the reference's unmodified sources, where they lie in the reference tree
// (src/model/{ggml_type,storage_decode,mapped_gguf,gguf}.cpp,
// src/backend/cpu/quantized_reference.cpp, src/core/{mapped_file,tensor}.cpp,
// src/runtime/{sampler,reference_kernels,hybrid_cache}.cpp,
// src/model/qwen35_manifest.cpp), into
// oracle/_ref/liboracle_ref.so.  Tests use it to pin the C restatement
// (quant_oracle.c) and the CUDA path against the reference itself, and
// bench.py's reference arm times reference_storage_matvec through it.
//
// Every function returns 0 on success or a code naming the C++ exception the
// reference threw, with its what() message copied into `err`:
//   1 std::invalid_argument, 2 std::out_of_range, 3 std::overflow_error,
//   4 std::runtime_error, 5 std::logic_error, 9 any other std::exception.
#include "oracle/backend/cpu/quantized_reference.hpp"
#include "oracle/model/ggml_type.hpp"
#include "oracle/model/gguf.hpp"
#include "oracle/model/mapped_gguf.hpp"
#include "oracle/model/storage_decode.hpp"
#include "oracle/runtime/reference_kernels.hpp"
#include "oracle/runtime/sampler.hpp"

#include <algorithm>
#include <cstddef>
#include <cstdint>
#include <cstring>
#include <span>
#include <stdexcept>
#include <string>

namespace {

int report(const std::exception& e, int code, char* err, std::size_t errlen) {
    if (err && errlen) {
        std::strncpy(err, e.what(), errlen - 1);
        err[errlen - 1] = '\0';
    }
    return code;
}

template <typename F>
int guarded(char* err, std::size_t errlen, F&& body) {
    try {
        body();
        return 0;
    } catch (const std::invalid_argument& e) {
        return report(e, 1, err, errlen);
    } catch (const std::out_of_range& e) {
        return report(e, 2, err, errlen);
    } catch (const std::overflow_error& e) {
        return report(e, 3, err, errlen);
    } catch (const std::runtime_error& e) {
        return report(e, 4, err, errlen);
    } catch (const std::logic_error& e) {
        return report(e, 5, err, errlen);
    } catch (const std::exception& e) {
        return report(e, 9, err, errlen);
    }
}

std::span<const std::byte> bytes_of(const void* p, std::uint64_t n) {
    return {static_cast<const std::byte*>(p), static_cast<std::size_t>(n)};
}

}  // namespace

extern "C" {

float oref_f16_to_f32(std::uint16_t bits) { return oracle::model::f16_to_f32(bits); }
float oref_bf16_to_f32(std::uint16_t bits) { return oracle::model::bf16_to_f32(bits); }

// ggml_type_layout (ggml_type.cpp:69-75): 1 when registered, 0 otherwise.
int oref_type_layout(std::uint32_t type, std::uint64_t* block_elements,
                     std::uint64_t* bytes_per_block, int* quantized, char* name,
                     std::size_t namelen) {
    const auto* layout = oracle::model::ggml_type_layout(type);
    if (!layout) return 0;
    *block_elements = layout->block_elements;
    *bytes_per_block = layout->bytes_per_block;
    *quantized = layout->quantized ? 1 : 0;
    if (name && namelen) {
        std::size_t n = layout->name.size() < namelen - 1 ? layout->name.size() : namelen - 1;
        std::memcpy(name, layout->name.data(), n);
        name[n] = '\0';
    }
    return 1;
}

// ggml_row_byte_size (ggml_type.cpp:77-94).
int oref_row_byte_size(std::uint64_t row_elements, std::uint32_t type, std::uint64_t* out,
                       char* err, std::size_t errlen) {
    return guarded(err, errlen, [&] { *out = oracle::model::ggml_row_byte_size(row_elements, type); });
}

// make_storage_row_view + decode_storage_row (storage_decode.cpp:182-198, :244-294).
int oref_decode_row(std::uint32_t type, std::uint64_t elements, const void* row,
                    std::uint64_t nbytes, float* out, std::uint64_t out_len, char* err,
                    std::size_t errlen) {
    return guarded(err, errlen, [&] {
        auto view = oracle::model::make_storage_row_view(type, elements, bytes_of(row, nbytes));
        oracle::model::decode_storage_row(view, std::span<float>(out, out_len));
    });
}

// reference_storage_dot (quantized_reference.cpp:24-82).
int oref_storage_dot(std::uint32_t type, std::uint64_t elements, const void* row,
                     std::uint64_t nbytes, const float* x, std::uint64_t x_len, float* out,
                     char* err, std::size_t errlen) {
    return guarded(err, errlen, [&] {
        auto view = oracle::model::make_storage_row_view(type, elements, bytes_of(row, nbytes));
        *out = oracle::backend::cpu::reference_storage_dot(view, std::span<const float>(x, x_len));
    });
}

// reference_storage_matvec (quantized_reference.cpp:128-162).
int oref_storage_matvec(std::uint32_t type, std::uint64_t rows, std::uint64_t cols,
                        const void* matrix, std::uint64_t nbytes, const float* x,
                        std::uint64_t x_len, float* y, std::uint64_t y_len, char* err,
                        std::size_t errlen) {
    return guarded(err, errlen, [&] {
        oracle::backend::cpu::reference_storage_matvec(
            type, rows, cols, bytes_of(matrix, nbytes), std::span<const float>(x, x_len),
            std::span<float>(y, y_len));
    });
}

// reference_mapped_tensor_matvec / reference_decode_mapped_tensor
// (quantized_reference.cpp:85-126) over an in-memory GgufTensorView, the way
// the reference's own tests build one (tests/test_phase2a.cpp:301-306).
int oref_mapped_tensor_matvec(std::uint32_t type, const std::uint64_t* dims, std::uint64_t ndims,
                              const void* data, std::uint64_t nbytes, const float* x,
                              std::uint64_t x_len, float* y, std::uint64_t y_len, char* err,
                              std::size_t errlen) {
    return guarded(err, errlen, [&] {
        oracle::model::GgufTensorInfo info{"shim.weight", {dims, dims + ndims}, type, 0};
        const auto* layout = oracle::model::ggml_type_layout(type);
        if (!layout) throw std::runtime_error("unsupported GGML tensor type");
        const oracle::model::GgufTensorView view(&info, layout,
                                                 static_cast<const std::byte*>(data),
                                                 static_cast<std::size_t>(nbytes), 0);
        oracle::backend::cpu::reference_mapped_tensor_matvec(
            view, std::span<const float>(x, x_len), std::span<float>(y, y_len));
    });
}

int oref_decode_mapped_tensor(std::uint32_t type, const std::uint64_t* dims, std::uint64_t ndims,
                              const void* data, std::uint64_t nbytes, float* out,
                              std::uint64_t out_len, char* err, std::size_t errlen) {
    return guarded(err, errlen, [&] {
        oracle::model::GgufTensorInfo info{"shim.weight", {dims, dims + ndims}, type, 0};
        const auto* layout = oracle::model::ggml_type_layout(type);
        if (!layout) throw std::runtime_error("unsupported GGML tensor type");
        const oracle::model::GgufTensorView view(&info, layout,
                                                 static_cast<const std::byte*>(data),
                                                 static_cast<std::size_t>(nbytes), 0);
        oracle::backend::cpu::reference_decode_mapped_tensor(view, std::span<float>(out, out_len));
    });
}

}  // extern "C"

// Sampler::sample with the default configuration (temperature 0: greedy),
// src/runtime/sampler.cpp:22-46.
extern "C" int oref_greedy_token(const float* logits, std::uint64_t n, std::uint32_t* token, char* err,
                                 std::size_t errlen) {
    return guarded(err, errlen, [&] {
        oracle::runtime::Sampler sampler{};
        *token = sampler.sample(std::span<const float>(logits, static_cast<std::size_t>(n))).token_id;
    });
}

// ---------------------------------------------------------------- decoder kernels (reference_kernels.cpp)

namespace {

oracle::core::Tensor tensor_from(const float* data, std::size_t rows, std::size_t cols) {
    oracle::core::Tensor t({rows, cols});
    std::copy(data, data + rows * cols, t.data().begin());
    return t;
}

}  // namespace

// apply_qwen35_rope (reference_kernels.cpp:74-123) on heads [n_heads x head_dim], in place.
extern "C" int oref_rope(float* heads, std::uint64_t n_heads, std::uint64_t head_dim, std::uint64_t rotary_dim,
                         const std::int32_t* sections, float base, std::uint64_t pos_t, std::uint64_t pos_h,
                         std::uint64_t pos_w, char* err, std::size_t errlen) {
    return guarded(err, errlen, [&] {
        auto t = tensor_from(heads, n_heads, head_dim);
        oracle::runtime::apply_qwen35_rope(t, {pos_t, pos_h, pos_w}, rotary_dim,
                                           {sections[0], sections[1], sections[2], sections[3]}, base);
        std::copy(t.data().begin(), t.data().end(), heads);
    });
}

// causal_attention_step (reference_kernels.cpp:125-190): a KV cache holding
// `length` earlier tokens (keys/values [length][kv_heads][dim]), one new token
// appended, attention of q [q_heads x key_dim] over all of them.
extern "C" int oref_attention_step(const float* q, const float* k_new, const float* v_new, const float* keys,
                                   const float* values, std::uint64_t length, std::uint64_t capacity,
                                   std::uint64_t q_heads, std::uint64_t kv_heads, std::uint64_t key_dim,
                                   std::uint64_t value_dim, float* out, char* err, std::size_t errlen) {
    return guarded(err, errlen, [&] {
        oracle::runtime::KvCache cache(capacity, kv_heads, key_dim, value_dim);
        for (std::uint64_t t = 0; t < length; ++t)
            cache.append(std::span<const float>(keys + t * kv_heads * key_dim, kv_heads * key_dim),
                         std::span<const float>(values + t * kv_heads * value_dim, kv_heads * value_dim));
        auto tq = tensor_from(q, q_heads, key_dim);
        auto tk = tensor_from(k_new, kv_heads, key_dim);
        auto tv = tensor_from(v_new, kv_heads, value_dim);
        oracle::core::Tensor to({q_heads, value_dim});
        oracle::runtime::causal_attention_step(tq, tk, tv, cache, to);
        std::copy(to.data().begin(), to.data().end(), out);
    });
}

// causal_depthwise_convolution_step (reference_kernels.cpp:192-219); history
// [channels][kernel] in and out.
extern "C" int oref_conv_step(const float* in, const float* weights, float* history, std::uint64_t channels,
                              std::uint64_t kernel, int apply_silu, float* out, char* err, std::size_t errlen) {
    return guarded(err, errlen, [&] {
        oracle::runtime::SsmState state(channels, kernel, 1, 1, 1);
        auto h = state.convolution_history();
        std::copy(history, history + channels * kernel, h.begin());
        oracle::runtime::causal_depthwise_convolution_step(std::span<const float>(in, channels),
                                                           std::span<const float>(weights, channels * kernel), state,
                                                           std::span<float>(out, channels), apply_silu != 0);
        std::copy(h.begin(), h.end(), history);
    });
}

// gated_delta_step (reference_kernels.cpp:221-335); recurrent state
// [heads][key_dim][value_dim] in and out.
extern "C" int oref_gated_delta_step(const float* q, const float* k, const float* v, const float* beta,
                                     const float* log_decay, float* state_io, std::uint64_t heads,
                                     std::uint64_t key_dim, std::uint64_t value_dim, float eps, float* out, char* err,
                                     std::size_t errlen) {
    return guarded(err, errlen, [&] {
        oracle::runtime::SsmState state(1, 1, heads, key_dim, value_dim);
        auto r = state.recurrent();
        std::copy(state_io, state_io + heads * key_dim * value_dim, r.begin());
        auto tq = tensor_from(q, heads, key_dim);
        auto tk = tensor_from(k, heads, key_dim);
        auto tv = tensor_from(v, heads, value_dim);
        oracle::core::Tensor to({heads, value_dim});
        oracle::runtime::gated_delta_step(tq, tk, tv, std::span<const float>(beta, heads),
                                          std::span<const float>(log_decay, heads), state, to, eps);
        std::copy(to.data().begin(), to.data().end(), out);
        std::copy(r.begin(), r.end(), state_io);
    });
}
