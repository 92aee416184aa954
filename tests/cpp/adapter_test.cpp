// adapter_test.cpp -- the C++ adapter (include/oracle_cuda.hpp) against the
// reference's own compiled functions (oracle/_ref/liboracle_ref.so), driven
// the way the reference's tests drive them (tests/test_phase2a.cpp in the
// Oracle repository).  Exit status 0 when every check passes.
//
// TEST INFRASTRUCTURE: links the reference checker library.  Needs a B200.
#include "oracle_cuda.hpp"

#include "oracle/backend/cpu/quantized_reference.hpp"
#include "oracle/model/ggml_type.hpp"
#include "oracle/model/mapped_gguf.hpp"
#include "oracle/model/storage_decode.hpp"

#include <array>
#include <cstdio>
#include <cstring>
#include <exception>
#include <functional>
#include <random>
#include <string>
#include <typeinfo>
#include <vector>

namespace cuda = oracle::backend::cuda;
namespace ref = oracle::backend::cpu;
namespace model = oracle::model;

static int g_failures = 0;

static void check(bool ok, const std::string& what) {
    if (!ok) {
        std::fprintf(stderr, "FAIL: %s\n", what.c_str());
        ++g_failures;
    }
}

static bool same_bits(float a, float b) {
    std::uint32_t x, y;
    std::memcpy(&x, &a, 4);
    std::memcpy(&y, &b, 4);
    return x == y;
}

// Run both callables; both must throw the same exception type with the same message.
static void same_error(const std::function<void()>& mine, const std::function<void()>& theirs, const std::string& what) {
    std::string mt, mm, tt, tm;
    try { mine(); } catch (const std::exception& e) { mt = typeid(e).name(); mm = e.what(); }
    try { theirs(); } catch (const std::exception& e) { tt = typeid(e).name(); tm = e.what(); }
    check(!tt.empty(), what + ": the reference did not throw");
    check(mt == tt, what + ": exception type " + mt + " vs reference " + tt);
    check(mm == tm, what + ": message '" + mm + "' vs reference '" + tm + "'");
}

static void store_u16(std::vector<std::byte>& b, std::size_t off, std::uint16_t v) {
    b[off] = static_cast<std::byte>(v & 0xFF);
    b[off + 1] = static_cast<std::byte>(v >> 8);
}

static std::vector<std::byte> q5_fixture() {  // test_phase2a.cpp:50-62
    std::vector<std::byte> b(176);
    store_u16(b, 0, 0x3800);
    store_u16(b, 2, 0x3400);
    const std::uint8_t sc[12] = {2, 2, 2, 2, 3, 3, 3, 3, 0x32, 0x32, 0x32, 0x32};
    for (int i = 0; i < 12; ++i) b[4 + i] = static_cast<std::byte>(sc[i]);
    for (int i = 16; i < 48; ++i) b[i] = std::byte{0xFF};
    for (int i = 48; i < 176; ++i) b[i] = std::byte{0x21};
    return b;
}

static std::vector<std::byte> q6_fixture() {  // test_phase2a.cpp:64-71
    std::vector<std::byte> b(210);
    for (int i = 0; i < 128; ++i) b[i] = std::byte{0x21};
    for (int i = 128; i < 192; ++i) b[i] = std::byte{0xFF};
    for (int i = 192; i < 208; ++i) b[i] = std::byte{0x02};
    store_u16(b, 208, 0x3800);
    return b;
}

static std::vector<std::byte> q8_fixture(std::uint16_t d, const std::vector<int>& q) {  // :78-88
    std::vector<std::byte> b(34);
    store_u16(b, 0, d);
    for (int i = 0; i < 32; ++i) b[2 + i] = static_cast<std::byte>(static_cast<std::uint8_t>(q[i % q.size()]));
    return b;
}

int main() {
    cuda::Backend be(0, cuda::Contract::F32);
    const std::vector<int> ramp = {0, 1, -1, 127, -128, 2, -2, 3, -3, 4, -4, 5, -5, 6, -6, 7,
                                   -7, 8, -8, 9, -9, 10, -10, 11, -11, 12, -12, 13, -13, 14, -14, 15};
    std::vector<float> ones(512, 1.0f);

    // known answers of the reference's own tests, through the adapter
    auto q5 = q5_fixture();
    auto q6 = q6_fixture();
    auto q8 = q8_fixture(0x3C00, ramp);
    check(be.storage_dot(model::make_storage_row_view(13, 256, q5), std::span(ones).first(256)) == 4288.0f, "Q5_K dot 4288");
    check(be.storage_dot(model::make_storage_row_view(14, 256, q6), std::span(ones).first(256)) == 4480.0f, "Q6_K dot 4480");
    check(be.storage_dot(model::make_storage_row_view(8, 32, q8), std::span(ones).first(32)) == 14.0f, "Q8_0 dot 14");
    std::vector<std::byte> two(q5);
    two.insert(two.end(), q5.begin(), q5.end());
    check(be.storage_dot(model::make_storage_row_view(13, 512, two), ones) == 8576.0f, "Q5_K two-block dot 8576");
    auto second = q5;
    for (int i = 16; i < 176; ++i) second[i] = std::byte{0};
    std::vector<std::byte> mat(q5);
    mat.insert(mat.end(), second.begin(), second.end());
    std::array<float, 2> y2{};
    be.storage_matvec(13, 2, 256, mat, std::span(ones).first(256), y2);
    check(y2[0] == 4288.0f && y2[1] == -192.0f, "Q5_K matvec {4288, -192}");

    // mapped tensor views, as test_phase2a.cpp:342-392 builds them
    auto q8b = q8_fixture(0x3800, {4});
    std::vector<std::byte> m8(q8);
    m8.insert(m8.end(), q8b.begin(), q8b.end());
    model::GgufTensorInfo info{"adapter.q8_0.weight", {32, 2}, 8, 0};
    const model::GgufTensorView tensor(&info, model::ggml_type_layout(8), m8.data(), m8.size(), 8192);
    std::array<float, 2> ym{};
    be.mapped_tensor_matvec(tensor, std::span(ones).first(32), ym);
    check(ym[0] == 14.0f && ym[1] == 64.0f, "Q8_0 mapped matvec {14, 64}");
    std::vector<float> dec(64), dec_ref(64);
    be.decode_mapped_tensor(tensor, dec);
    ref::reference_decode_mapped_tensor(tensor, dec_ref);
    bool dsame = true;
    for (int i = 0; i < 64; ++i) dsame = dsame && same_bits(dec[i], dec_ref[i]);
    check(dsame, "decode_mapped_tensor == reference");

    // random rows of every reference-supported type: bit-identical to the reference
    std::mt19937_64 rng(5150);
    for (std::uint32_t type : {8u, 13u, 14u, 1u, 30u, 0u}) {
        const std::size_t rows = 33, cols = type == 8 ? 512 : (type == 13 || type == 14) ? 1024 : 250;
        const std::size_t rb = model::ggml_row_byte_size(cols, type);
        std::vector<std::byte> w(rows * rb);
        for (auto& v : w) v = static_cast<std::byte>(rng() & 0xFF);
        // keep f16 scales finite: clear exponent bits of the scale fields
        if (type == 8) for (std::size_t b = 0; b < w.size(); b += 34) w[b + 1] &= std::byte{0x3B};
        if (type == 13) for (std::size_t b = 0; b < w.size(); b += 176) { w[b + 1] &= std::byte{0x3B}; w[b + 3] &= std::byte{0x3B}; }
        if (type == 14) for (std::size_t b = 0; b < w.size(); b += 210) w[b + 209] &= std::byte{0x3B};
        if (type == 1) for (std::size_t b = 1; b < w.size(); b += 2) w[b] &= std::byte{0x3B};
        if (type == 30) for (std::size_t b = 1; b < w.size(); b += 2) w[b] &= std::byte{0x3F};
        if (type == 0) for (std::size_t b = 3; b < w.size(); b += 4) w[b] &= std::byte{0x3F};
        std::vector<float> x(cols);
        std::normal_distribution<float> nd;
        for (auto& v : x) v = nd(rng);
        std::vector<float> y(rows), yr(rows);
        be.storage_matvec(type, rows, cols, w, x, y);
        ref::reference_storage_matvec(type, rows, cols, w, x, yr);
        bool same = true;
        for (std::size_t r = 0; r < rows; ++r) same = same && same_bits(y[r], yr[r]);
        check(same, "storage_matvec == reference for type " + std::to_string(type));
        std::vector<float> drow(cols), drow_ref(cols);
        auto view = model::make_storage_row_view(type, cols, std::span(w).first(rb));
        be.decode_storage_row(view, drow);
        model::decode_storage_row(view, drow_ref);
        bool dsame2 = true;
        for (std::size_t i = 0; i < cols; ++i) dsame2 = dsame2 && same_bits(drow[i], drow_ref[i]);
        check(dsame2, "decode_storage_row == reference for type " + std::to_string(type));
    }

    // errors: same exception class and message as the reference
    std::array<float, 3> y3{};
    same_error([&] { be.storage_matvec(8, 0, 32, q8, std::span(ones).first(32), std::span(y3).first(2)); },
               [&] { ref::reference_storage_matvec(8, 0, 32, q8, std::span(ones).first(32), std::span(y3).first(2)); },
               "zero rows");
    same_error([&] { be.storage_matvec(8, 1, 32, q8, std::span(ones).first(31), std::span(y3).first(1)); },
               [&] { ref::reference_storage_matvec(8, 1, 32, q8, std::span(ones).first(31), std::span(y3).first(1)); },
               "vector length");
    same_error([&] { be.storage_matvec(8, 1, 32, q8, std::span(ones).first(32), std::span(y3).first(3)); },
               [&] { ref::reference_storage_matvec(8, 1, 32, q8, std::span(ones).first(32), std::span(y3).first(3)); },
               "output length");
    same_error([&] { be.storage_matvec(8, 1, 17, q8, std::span(ones).first(17), std::span(y3).first(1)); },
               [&] { ref::reference_storage_matvec(8, 1, 17, q8, std::span(ones).first(17), std::span(y3).first(1)); },
               "ragged row (not divisible by block size)");
    same_error([&] { be.storage_matvec(999, 1, 32, q8, std::span(ones).first(32), std::span(y3).first(1)); },
               [&] { ref::reference_storage_matvec(999, 1, 32, q8, std::span(ones).first(32), std::span(y3).first(1)); },
               "unknown type");
    same_error([&] { be.storage_matvec(8, 1, 32, std::span(q8).first(33), std::span(ones).first(32), std::span(y3).first(1)); },
               [&] { ref::reference_storage_matvec(8, 1, 32, std::span(q8).first(33), std::span(ones).first(32), std::span(y3).first(1)); },
               "matrix byte size");
    std::vector<std::byte> q40(18 * 2);
    same_error([&] { be.storage_matvec(2, 2, 32, q40, std::span(ones).first(32), std::span(y3).first(2)); },
               [&] { ref::reference_storage_matvec(2, 2, 32, q40, std::span(ones).first(32), std::span(y3).first(2)); },
               "registered type the decoder rejects (q4_0)");
    std::array<float, 1> short_out{};
    same_error([&] { be.decode_storage_row(model::make_storage_row_view(13, 256, q5), short_out); },
               [&] { model::decode_storage_row(model::make_storage_row_view(13, 256, q5), short_out); },
               "decode output length");
    const model::GgufTensorView malformed(&info, model::ggml_type_layout(8), m8.data(), m8.size() - 1, 8192);
    std::vector<float> dm(64);
    same_error([&] { be.decode_mapped_tensor(malformed, dm); }, [&] { ref::reference_decode_mapped_tensor(malformed, dm); },
               "mapped tensor with inconsistent byte geometry");

    // the Q8_K contract through the same adapter, on a Q4_K row (which Oracle itself rejects)
    be.set_contract(cuda::Contract::Q8K);
    std::vector<std::byte> q4(144);
    std::memcpy(q4.data(), q5.data(), 16);
    for (int i = 16; i < 144; ++i) q4[i] = std::byte{0x21};
    // Oracle's make_storage_row_view rejects type 12 (storage_decode.cpp:192-196); a Q4_K-enabled
    // caller builds the view directly
    const model::StorageRowView q4view{12, 256, std::span<const std::byte>(q4)};
    const float q4dot = be.storage_dot(q4view, std::span(ones).first(256));
    check(q4dot == 192.0f, "Q4_K x Q8_K dot of the Q4_K analogue fixture = 192 (ones quantize exactly)");

    if (g_failures == 0) std::printf("adapter_test: all checks passed\n");
    return g_failures == 0 ? 0 : 1;
}
