// ref_shim.cpp -- C entry points over Oracle's OWN compiled hot-path sources.
//
// TEST INFRASTRUCTURE ONLY.  oracle/Makefile compiles this file together with
// the reference's unmodified sources, where they lie in the reference tree
// (src/model/{ggml_type,storage_decode,mapped_gguf,gguf}.cpp,
// src/backend/cpu/quantized_reference.cpp, src/core/mapped_file.cpp,
// src/runtime/sampler.cpp), into
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
#include "oracle/runtime/sampler.hpp"

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
