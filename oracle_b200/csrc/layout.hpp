// layout.hpp -- the GGML storage-layout registry and row geometry checks.
//
// The table lists every ggml_type id with (name, elements per block, bytes per
// block, quantized).  It is a format fact shared with GGML and with Oracle's
// registry (src/model/ggml_type.cpp:12-56), so the entries match those byte
// for byte; removed ids carry zero sizes and are rejected like Oracle does
// (ggml_type_layout, ggml_type.cpp:69-75).  Row sizing follows
// ggml_row_byte_size (ggml_type.cpp:77-94): overflow-checked, error on a zero
// or ragged row.
#pragma once

#include <cstdint>
#include <limits>
#include <string>

namespace oracle_cuda {

struct TypeLayout {
    uint32_t type;
    const char* name;
    uint64_t block_elements;
    uint64_t bytes_per_block;
    bool quantized;
};

inline constexpr uint32_t kTypeF32 = 0, kTypeF16 = 1, kTypeQ8_0 = 8, kTypeQ4_K = 12,
                          kTypeQ5_K = 13, kTypeQ6_K = 14, kTypeQ8_K = 15, kTypeBF16 = 30;

inline constexpr TypeLayout kLayouts[] = {
    {0, "f32", 1, 4, false},           {1, "f16", 1, 2, false},
    {2, "q4_0", 32, 18, true},         {3, "q4_1", 32, 20, true},
    {4, "deprecated_q4_2", 0, 0, false}, {5, "deprecated_q4_3", 0, 0, false},
    {6, "q5_0", 32, 22, true},         {7, "q5_1", 32, 24, true},
    {8, "q8_0", 32, 34, true},         {9, "q8_1", 32, 36, true},
    {10, "q2_K", 256, 84, true},       {11, "q3_K", 256, 110, true},
    {12, "q4_K", 256, 144, true},      {13, "q5_K", 256, 176, true},
    {14, "q6_K", 256, 210, true},      {15, "q8_K", 256, 292, true},
    {16, "iq2_xxs", 256, 66, true},    {17, "iq2_xs", 256, 74, true},
    {18, "iq3_xxs", 256, 98, true},    {19, "iq1_s", 256, 50, true},
    {20, "iq4_nl", 32, 18, true},      {21, "iq3_s", 256, 110, true},
    {22, "iq2_s", 256, 82, true},      {23, "iq4_xs", 256, 136, true},
    {24, "i8", 1, 1, false},           {25, "i16", 1, 2, false},
    {26, "i32", 1, 4, false},          {27, "i64", 1, 8, false},
    {28, "f64", 1, 8, false},          {29, "iq1_m", 256, 56, true},
    {30, "bf16", 1, 2, false},         {31, "removed_q4_0_4_4", 0, 0, false},
    {32, "removed_q4_0_4_8", 0, 0, false}, {33, "removed_q4_0_8_8", 0, 0, false},
    {34, "tq1_0", 256, 54, true},      {35, "tq2_0", 256, 66, true},
    {36, "removed_iq4_nl_4_4", 0, 0, false}, {37, "removed_iq4_nl_4_8", 0, 0, false},
    {38, "removed_iq4_nl_8_8", 0, 0, false}, {39, "mxfp4", 32, 17, true},
    {40, "nvfp4", 64, 36, true},       {41, "q1_0", 128, 18, true},
    {42, "q2_0", 64, 18, true},
};
inline constexpr uint32_t kLayoutCount = sizeof(kLayouts) / sizeof(kLayouts[0]);

inline const TypeLayout* type_layout(uint32_t type) {
    if (type >= kLayoutCount) return nullptr;
    const TypeLayout& l = kLayouts[type];
    return (l.block_elements == 0 || l.bytes_per_block == 0) ? nullptr : &l;
}

// Error classes mirror the C++ exceptions Oracle throws on this path.
enum class ErrorKind : int {
    None = 0,
    InvalidArgument = 1,  // std::invalid_argument
    OutOfRange = 2,       // std::out_of_range
    Overflow = 3,         // std::overflow_error
    Runtime = 4,          // std::runtime_error
    Logic = 5,            // std::logic_error
};

struct Error {
    ErrorKind kind = ErrorKind::None;
    std::string message;
    explicit operator bool() const { return kind != ErrorKind::None; }
};

inline Error make_error(ErrorKind k, std::string m) { return Error{k, std::move(m)}; }

inline bool checked_mul(uint64_t a, uint64_t b, uint64_t* out) {
    if (a != 0 && b > std::numeric_limits<uint64_t>::max() / a) return false;
    *out = a * b;
    return true;
}

// ggml_row_byte_size (ggml_type.cpp:77-94), same checks and messages.
inline Error row_byte_size(uint64_t row_elements, uint32_t type, uint64_t* out) {
    const TypeLayout* l = type_layout(type);
    if (!l) return make_error(ErrorKind::Runtime, "unsupported GGML tensor type: " + std::to_string(type));
    if (row_elements == 0)
        return make_error(ErrorKind::InvalidArgument, "GGML tensor row must contain at least one element");
    if (row_elements % l->block_elements != 0)
        return make_error(ErrorKind::Runtime, "GGML tensor row length " + std::to_string(row_elements) +
                                                  " is not divisible by block size " +
                                                  std::to_string(l->block_elements) + " for type " +
                                                  l->name);
    if (!checked_mul(row_elements / l->block_elements, l->bytes_per_block, out))
        return make_error(ErrorKind::Overflow, "GGML row byte size overflow");
    return {};
}

// The types this CUDA path decodes (Oracle's decoder set, storage_decode.cpp:192-196,
// widened by Q4_K, which the path exists to serve).
inline bool decodable(uint32_t type) {
    return type == kTypeF32 || type == kTypeF16 || type == kTypeBF16 || type == kTypeQ8_0 ||
           type == kTypeQ4_K || type == kTypeQ5_K || type == kTypeQ6_K;
}

// The weight types with a Q8_K integer dot on this path.
inline bool q8k_dot_type(uint32_t type) { return type == kTypeQ4_K || type == kTypeQ6_K; }

}  // namespace oracle_cuda
