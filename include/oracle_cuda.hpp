// oracle_cuda.hpp -- C++20 adapter over the C ABI, with Oracle's own signatures.
//
// Header-only.  Include it inside the Oracle tree (it uses Oracle's
// StorageRowView and GgufTensorView, include/oracle/model/storage_decode.hpp and
// mapped_gguf.hpp) and link liboracle_cuda.so.  Each member function has the
// signature and the error behaviour of the reference function it replaces:
//
//   reference (include/oracle/backend/cpu/quantized_reference.hpp:12-27)   here
//   reference_storage_dot(row, vector)                    -> Backend::storage_dot
//   reference_storage_matvec(type, rows, cols, m, x, y)   -> Backend::storage_matvec
//   reference_mapped_tensor_matvec(tensor, x, y)          -> Backend::mapped_tensor_matvec
//   reference_decode_mapped_tensor(tensor, out)           -> Backend::decode_mapped_tensor
//   decode_storage_row(row, out)  (storage_decode.hpp:41) -> Backend::decode_storage_row
//
// Failures throw the exception class the reference throws for the same input
// (std::invalid_argument, std::out_of_range, std::overflow_error,
// std::runtime_error, std::logic_error) with the reference's message; CUDA
// failures throw std::runtime_error.  Calls are synchronous, like the
// reference.  The GGUF-tensor forms register the tensor's bytes on first use
// (Oracle's weights are immutable mmap pages, so they stay resident in HBM);
// the span forms copy their bytes on every call, as the reference reads them
// on every call, unless the caller registered the span (register_span).
#pragma once

#include "oracle_cuda.h"

#include <cstddef>
#include <cstdint>
#include <span>
#include <stdexcept>
#include <string>

#if __has_include("oracle/model/mapped_gguf.hpp")
#include "oracle/model/mapped_gguf.hpp"
#include "oracle/model/storage_decode.hpp"
#define ORACLE_CUDA_HAVE_ORACLE_TYPES 1
#endif

namespace oracle::backend::cuda {

enum class Contract : int {
    F32 = ORACLE_CUDA_CONTRACT_F32,  // Oracle's: decode to f32, sequential f32 sum (bit-identical)
    Q8K = ORACLE_CUDA_CONTRACT_Q8K,  // GGML's: activations quantized to Q8_K, integer block dots
};

[[noreturn]] inline void throw_status(oracle_cuda_status status, const char* message) {
    const std::string m = message ? message : "";
    switch (status) {
        case ORACLE_CUDA_INVALID_ARGUMENT: throw std::invalid_argument(m);
        case ORACLE_CUDA_OUT_OF_RANGE: throw std::out_of_range(m);
        case ORACLE_CUDA_OVERFLOW: throw std::overflow_error(m);
        case ORACLE_CUDA_RUNTIME_ERROR: throw std::runtime_error(m);
        case ORACLE_CUDA_LOGIC_ERROR: throw std::logic_error(m);
        default: throw std::runtime_error(std::string(oracle_cuda_status_name(status)) + ": " + m);
    }
}

class Backend {
public:
    explicit Backend(int device = 0, Contract contract = Contract::F32, std::uint32_t flags = 0) : contract_(contract) {
        const oracle_cuda_status s = oracle_cuda_create(device, &ctx_);
        if (s != ORACLE_CUDA_OK) throw_status(s, oracle_cuda_last_error(nullptr));
        if (flags) check(oracle_cuda_set_flags(ctx_, flags));
    }
    ~Backend() { oracle_cuda_destroy(ctx_); }
    Backend(const Backend&) = delete;
    Backend& operator=(const Backend&) = delete;

    void set_contract(Contract c) noexcept { contract_ = c; }
    [[nodiscard]] Contract contract() const noexcept { return contract_; }
    [[nodiscard]] oracle_cuda_context* context() const noexcept { return ctx_; }

    // reference_storage_matvec (quantized_reference.cpp:128-162)
    void storage_matvec(std::uint32_t type, std::size_t rows, std::size_t cols, std::span<const std::byte> matrix,
                        std::span<const float> vector, std::span<float> output) {
        check(oracle_cuda_host_storage_matvec(ctx_, static_cast<int>(contract_), type, rows, cols, matrix.data(),
                                              matrix.size(), vector.data(), vector.size(), output.data(),
                                              output.size()));
    }

    // Make a span's bytes resident (the caller promises they never change
    // while registered); the calls above then read the resident copy.
    void register_span(std::uint32_t type, std::size_t rows, std::size_t cols, std::span<const std::byte> bytes) {
        check(oracle_cuda_register_host_weight(ctx_, type, rows, cols, bytes.data(), bytes.size()));
    }

    // decode_storage_row's row form and the GGUF-tensor form (rows x dims[0])
    void decode_rows(std::uint32_t type, std::size_t rows, std::size_t cols, std::span<const std::byte> bytes,
                     std::span<float> output) {
        check(oracle_cuda_host_decode_rows(ctx_, type, rows, cols, bytes.data(), bytes.size(), output.data(),
                                           output.size()));
    }

#ifdef ORACLE_CUDA_HAVE_ORACLE_TYPES
    // reference_storage_dot (quantized_reference.cpp:24-82)
    [[nodiscard]] float storage_dot(model::StorageRowView row, std::span<const float> vector) {
        float out = 0.0f;
        check(oracle_cuda_host_storage_dot(ctx_, static_cast<int>(contract_), row.type, row.element_count,
                                           row.bytes.data(), row.bytes.size(), vector.data(), vector.size(), &out));
        return out;
    }

    // decode_storage_row (storage_decode.cpp:244-294)
    void decode_storage_row(model::StorageRowView row, std::span<float> output) {
        // the reference validates the view first (make_storage_row_view), then the output length
        const auto view = model::make_storage_row_view(row.type, row.element_count, row.bytes);
        if (output.size() != view.element_count) throw std::invalid_argument("decoded row output size mismatch");
        decode_rows(view.type, 1, view.element_count, view.bytes, output);
    }

    // reference_mapped_tensor_matvec (quantized_reference.cpp:107-126): GGUF
    // dims[0] = columns, dims[1] = rows.
    void mapped_tensor_matvec(const model::GgufTensorView& tensor, std::span<const float> vector,
                              std::span<float> output) {
        const auto dims = tensor.dimensions();
        if (dims.size() != 2) throw std::invalid_argument("mapped tensor matvec requires a rank-2 tensor");
        const auto rows = static_cast<std::size_t>(dims[1]), cols = static_cast<std::size_t>(dims[0]);
        register_mapped(tensor.layout().type, rows, cols, tensor.bytes());
        storage_matvec(tensor.layout().type, rows, cols, tensor.bytes(), vector, output);
    }

    // reference_decode_mapped_tensor (quantized_reference.cpp:85-105)
    void decode_mapped_tensor(const model::GgufTensorView& tensor, std::span<float> output) {
        const std::size_t rows = model::gguf_tensor_row_count(tensor);
        const auto dims = tensor.dimensions();
        if (output.size() != rows * static_cast<std::size_t>(dims.front()))
            throw std::invalid_argument("mapped tensor decode output length mismatch");
        register_mapped(tensor.layout().type, rows, static_cast<std::size_t>(dims.front()), tensor.bytes());
        decode_rows(tensor.layout().type, rows, static_cast<std::size_t>(dims.front()), tensor.bytes(), output);
    }
#endif

private:
    // A mapped tensor's bytes are registered when its geometry is valid; an
    // invalid one is left to the call, which reports the reference's error.
    void register_mapped(std::uint32_t type, std::size_t rows, std::size_t cols, std::span<const std::byte> bytes) {
        (void)oracle_cuda_register_host_weight(ctx_, type, rows, cols, bytes.data(), bytes.size());
    }

    void check(oracle_cuda_status s) const {
        if (s != ORACLE_CUDA_OK) throw_status(s, oracle_cuda_last_error(ctx_));
    }

    oracle_cuda_context* ctx_ = nullptr;
    Contract contract_;
};

}  // namespace oracle::backend::cuda
