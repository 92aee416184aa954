// gguf_test.cpp -- Oracle's own MappedGgufModel views fed to the B200 path.
//
// Opens a GGUF file (written by tests/golden/make_gguf.py) with the
// reference's MappedGgufModel (mmap, zero-copy tensor views) and, for every
// tensor, checks the C++ adapter against the reference's compiled functions:
//   * 2-D tensors the reference decodes: Backend::mapped_tensor_matvec (f32
//     contract) bit-identical to reference_mapped_tensor_matvec;
//   * Q4_K (which the reference rejects, storage_decode.cpp:192-196): the
//     reference's exception is checked, and the GPU result (both contracts)
//     is compared bit for bit with the C restatement (oracle/quant_oracle.c);
//   * 1-D tensors: Backend::decode_mapped_tensor bit-identical to
//     reference_decode_mapped_tensor.
// Prints one line per tensor and exits non-zero on any mismatch.
#include "oracle/backend/cpu/quantized_reference.hpp"
#include "oracle/model/mapped_gguf.hpp"
#include "oracle/model/storage_decode.hpp"
#include "oracle_cuda.hpp"

extern "C" {
#include "../../oracle/quant_oracle.h"
}

#include <cmath>
#include <cstdio>
#include <cstring>
#include <stdexcept>
#include <vector>

namespace {

bool same_bits(const std::vector<float>& a, const std::vector<float>& b) {
    return a.size() == b.size() && std::memcmp(a.data(), b.data(), a.size() * sizeof(float)) == 0;
}

std::vector<float> activation(std::size_t n, unsigned seed) {
    std::vector<float> x(n);
    unsigned s = seed * 2654435761u + 1u;
    for (auto& v : x) {
        s = s * 1664525u + 1013904223u;
        v = static_cast<float>(static_cast<int>(s >> 9) % 2001 - 1000) / 357.0f;
    }
    return x;
}

}  // namespace

int main(int argc, char** argv) {
    if (argc < 2) {
        std::fprintf(stderr, "usage: gguf_test FILE.gguf\n");
        return 2;
    }
    namespace cuda = oracle::backend::cuda;
    oracle::model::MappedGgufModel model(argv[1]);
    cuda::Backend f32{0, cuda::Contract::F32};
    cuda::Backend q8k{0, cuda::Contract::Q8K};
    int failures = 0, checked = 0;
    for (const auto& t : model.tensors()) {
        const auto dims = t.dimensions();
        const uint32_t type = t.layout().type;
        std::string label(t.name());
        bool ok = true;
        if (dims.size() == 1) {
            std::vector<float> want(dims[0]), got(dims[0]);
            oracle::backend::cpu::reference_decode_mapped_tensor(t, want);
            f32.decode_mapped_tensor(t, got);
            ok = same_bits(want, got);
        } else if (dims.size() == 2) {
            const std::size_t cols = dims[0], rows = dims[1];
            const auto x = activation(cols, static_cast<unsigned>(rows));
            std::vector<float> got(rows);
            f32.mapped_tensor_matvec(t, x, got);
            if (type != 12) {
                std::vector<float> want(rows);
                oracle::backend::cpu::reference_mapped_tensor_matvec(t, x, want);
                ok = same_bits(want, got);
            } else {
                bool threw = false;
                try {
                    std::vector<float> want(rows);
                    oracle::backend::cpu::reference_mapped_tensor_matvec(t, x, want);
                } catch (const std::invalid_argument& e) {
                    threw = std::strstr(e.what(), "does not support GGML type 12") != nullptr;
                }
                const auto* w = reinterpret_cast<const uint8_t*>(t.bytes().data());
                std::vector<float> want(rows);
                oq_storage_matvec_f32(type, rows, cols, w, x.data(), 1, want.data());
                ok = threw && same_bits(want, got);
                // GGML's Q8_K contract through the same view
                std::vector<uint8_t> qx(cols / 256 * 292);
                oq_quantize_row_q8_k(x.data(), cols, qx.data());
                std::vector<float> want_q(rows), got_q(rows);
                oq_matvec_q8_k(type, rows, cols, w, qx.data(), 1, want_q.data());
                q8k.mapped_tensor_matvec(t, x, got_q);
                ok = ok && same_bits(want_q, got_q);
            }
        }
        ++checked;
        if (!ok) ++failures;
        std::printf("%-24s type %2u dims %zu: %s\n", label.c_str(), type, dims.size(), ok ? "ok" : "MISMATCH");
    }
    std::printf("%d tensors, %d failures\n", checked, failures);
    return failures == 0 && checked > 0 ? 0 : 1;
}
