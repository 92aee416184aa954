// ref_q8k_projection.cpp -- GGML's Q8_K activation contract under Oracle's forward.
//
// TEST INFRASTRUCTURE ONLY.  oracle/Makefile compiles the reference's
// src/runtime/qwen35_block.cpp and src/runtime/qwen35_forward.cpp with
//   -Dreference_mapped_tensor_matvec=oracle_q8k_projection_matvec
//   -Dmake_storage_row_view=oracle_q8k_make_storage_row_view
//   -Ddecode_storage_row=oracle_q8k_decode_storage_row
// into oracle/_ref/liboracle_ref_q8k.so, so that every projection and the
// embedding row of the reference's own decode step land here.  Q4_K and Q6_K
// projections run GGML's contract as restated in quant_oracle.c: the input is
// quantized to Q8_K (quantize_row_q8_K) and each row is the integer block dot
// (ggml_vec_dot_q4_K_q8_K / ggml_vec_dot_q6_K_q8_K) -- the contract the GPU
// matvec program implements bit for bit.  Q4_K embedding rows decode with
// GGML's dequantize_row_q4_K (quant_oracle.c).  Every other type goes to the
// reference's own function unchanged.  The sources themselves are not edited.
#include "oracle/backend/cpu/quantized_reference.hpp"
#include "oracle/model/ggml_type.hpp"
#include "oracle/model/mapped_gguf.hpp"
#include "oracle/model/storage_decode.hpp"

extern "C" {
#include "quant_oracle.h"
}

#include <cstddef>
#include <cstdint>
#include <limits>
#include <span>
#include <stdexcept>
#include <string>
#include <vector>

namespace {
constexpr std::uint32_t kQ4K = 12, kQ6K = 14;
}

namespace oracle::backend::cpu {

void oracle_q8k_projection_matvec(const model::GgufTensorView& tensor, std::span<const float> vector,
                                  std::span<float> output);

void oracle_q8k_projection_matvec(const model::GgufTensorView& tensor, std::span<const float> vector,
                                  std::span<float> output) {
    const std::uint32_t type = tensor.layout().type;
    if (type != kQ4K && type != kQ6K) {
        reference_mapped_tensor_matvec(tensor, vector, output);
        return;
    }
    const auto dims = tensor.dimensions();
    if (dims.size() != 2) throw std::invalid_argument("Q8_K projection requires a rank-2 tensor");
    const std::uint64_t cols = dims[0], rows = dims[1];
    if (vector.size() != cols || output.size() != rows)
        throw std::invalid_argument("Q8_K projection vector lengths do not match the tensor");
    std::vector<std::uint8_t> q8k(cols / 256 * 292);
    if (oq_quantize_row_q8_k(vector.data(), cols, q8k.data()) != 0)
        throw std::invalid_argument("Q8_K quantization needs a multiple of 256 columns");
    const auto* w = reinterpret_cast<const std::uint8_t*>(tensor.bytes().data());
    if (oq_matvec_q8_k(type, rows, cols, w, q8k.data(), 1, output.data()) != 0)
        throw std::runtime_error("Q8_K projection failed");
}

}  // namespace oracle::backend::cpu

namespace oracle::model {

StorageRowView oracle_q8k_make_storage_row_view(std::uint32_t type, std::size_t element_count,
                                                std::span<const std::byte> bytes);
StorageRowView oracle_q8k_make_storage_row_view(const GgufTensorView& tensor, std::size_t row_index);
void oracle_q8k_decode_storage_row(StorageRowView row, std::span<float> output);

StorageRowView oracle_q8k_make_storage_row_view(std::uint32_t type, std::size_t element_count,
                                                std::span<const std::byte> bytes) {
    if (type != kQ4K) return make_storage_row_view(type, element_count, bytes);
    if (element_count % 256 != 0 || bytes.size() != element_count / 256 * 144)
        throw std::invalid_argument("storage row byte size mismatch");
    return StorageRowView{type, element_count, bytes};
}

StorageRowView oracle_q8k_make_storage_row_view(const GgufTensorView& tensor, std::size_t row_index) {
    if (tensor.layout().type != kQ4K) return make_storage_row_view(tensor, row_index);
    const auto dims = tensor.dimensions();
    const std::size_t cols = dims.front();
    const std::size_t rows = gguf_tensor_row_count(tensor);
    if (row_index >= rows) throw std::out_of_range("GGUF tensor row index exceeds row count");
    const std::size_t row_bytes = cols / 256 * 144;
    return oracle_q8k_make_storage_row_view(kQ4K, cols, tensor.bytes().subspan(row_index * row_bytes, row_bytes));
}

void oracle_q8k_decode_storage_row(StorageRowView row, std::span<float> output) {
    if (row.type != kQ4K) {
        decode_storage_row(row, output);
        return;
    }
    if (output.size() != row.element_count) throw std::invalid_argument("storage decode output length mismatch");
    if (oq_decode_row(kQ4K, row.element_count, reinterpret_cast<const std::uint8_t*>(row.bytes.data()),
                      output.data()) != 0)
        throw std::invalid_argument("Q4_K row decode failed");
}

}  // namespace oracle::model
