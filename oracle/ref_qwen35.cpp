// ref_qwen35.cpp -- Oracle's own Qwen3.5 decode loop behind a C ABI.
//
// TEST INFRASTRUCTURE ONLY (the checker for the GPU decoder, never shipped).
// Compiled by oracle/Makefile together with the reference's unmodified
// sources into oracle/_ref/liboracle_ref.so and oracle/_ref/liboracle_ref_q8k.so.
// A model is either a GGUF file mapped by the reference's MappedGgufModel
// (src/model/mapped_gguf.cpp) or tensors in host buffers wrapped in the
// reference's GgufTensorView; a token step is the reference's
// execute_qwen35_reference_token (src/runtime/qwen35_forward.cpp) on its
// HybridCache at RopePosition::text(sequence_length()), and greedy decoding is
// Qwen35GenerationSession::generate_fresh's loop (qwen35_generation.cpp:
// 733-747, 846): every prompt token through the forward, then the reference's
// Sampler at temperature 0 picks each token, which is fed back.
//
// Binding: admit_q4k = 0 binds with the reference's own bind_qwen35_weights
// (src/model/qwen35_weights.cpp), which admits Q5_K / Q6_K / Q8_0 / float
// matrices only.  admit_q4k = 1 binds the same tensor names without the type
// gate, the one-line change a maintainer makes to run Q4_K_M models
// (allowed_storage_type, qwen35_weights.cpp:49-59); the reference's storage
// decoder still rejects Q4_K, so that mode is only useful in
// liboracle_ref_q8k.so, where the projections run GGML's Q8_K contract
// (ref_q8k_projection.cpp).
//
// liboracle_ref_gate.so (OREF_GATE_PATCHED) is the same Q8_K build whose
// qwen35_weights.cpp is a build-directory copy of the reference's with that
// one-line change applied (Q4_K admitted in allowed_storage_type's matrix
// branch, oracle/Makefile); there admit_q4k = 1 binds with the reference's
// own bind_qwen35_weights, so the binder's names, shapes, byte sizes and
// roles are checked by the reference itself.
#include "oracle/model/mapped_gguf.hpp"
#include "oracle/model/qwen35_manifest.hpp"
#include "oracle/model/qwen35_weights.hpp"
#include "oracle/runtime/hybrid_cache.hpp"
#include "oracle/runtime/qwen35_forward.hpp"
#include "oracle/runtime/sampler.hpp"

#include <cstddef>
#include <cstdint>
#include <cstring>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

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

namespace model = oracle::model;
namespace runtime = oracle::runtime;

// The reference binder's tensor names (qwen35_weights.cpp:131-380) without
// its storage-type gate.  Shapes are left to the forward's own checks.
model::Qwen35Weights bind_admitting_q4k(std::span<const model::GgufTensorView> tensors,
                                        const model::Qwen35Manifest& manifest) {
    auto find = [&](const std::string& name) -> const model::GgufTensorView* {
        for (const auto& t : tensors)
            if (t.name() == name) return &t;
        return nullptr;
    };
    auto need = [&](const std::string& name) {
        const model::GgufTensorView* t = find(name);
        if (!t) throw std::runtime_error("missing required Qwen3.5 tensor: " + name);
        return t;
    };
    model::Qwen35Weights w;
    w.token_embedding = need("token_embd.weight");
    w.output_norm = need("output_norm.weight");
    w.output = find("output.weight");
    if (!w.output) {
        w.output = w.token_embedding;
        w.output_is_tied = true;
    }
    for (std::uint32_t i = 0; i < manifest.backbone_block_count; ++i) {
        const std::string p = "blk." + std::to_string(i) + ".";
        model::Qwen35BackboneBlockWeights b;
        b.index = i;
        b.kind = manifest.is_full_attention_block(i) ? model::Qwen35BlockKind::full_attention
                                                     : model::Qwen35BlockKind::recurrent;
        b.input_norm = need(p + "attn_norm.weight");
        b.post_attention_norm = need(p + "post_attention_norm.weight");
        if (b.kind == model::Qwen35BlockKind::full_attention) {
            b.attention = model::Qwen35AttentionWeights{need(p + "attn_q.weight"),      need(p + "attn_k.weight"),
                                                        need(p + "attn_v.weight"),      need(p + "attn_output.weight"),
                                                        need(p + "attn_q_norm.weight"), need(p + "attn_k_norm.weight")};
        } else {
            b.recurrent = model::Qwen35RecurrentWeights{
                need(p + "attn_qkv.weight"),   need(p + "attn_gate.weight"),  need(p + "ssm_conv1d.weight"),
                need(p + "ssm_dt.bias"),       need(p + "ssm_a"),             need(p + "ssm_beta.weight"),
                need(p + "ssm_alpha.weight"),  need(p + "ssm_norm.weight"),   need(p + "ssm_out.weight")};
        }
        b.mlp = model::Qwen35MlpWeights{need(p + "ffn_gate.weight"), need(p + "ffn_down.weight"),
                                        need(p + "ffn_up.weight")};
        w.blocks.push_back(std::move(b));
    }
    // the block-family counts the forward cross-checks (qwen35_forward.cpp:233-254)
    w.report.backbone_block_count = manifest.backbone_block_count;
    w.report.tied_output = w.output_is_tied;
    for (const auto& b : w.blocks) {
        if (b.kind == model::Qwen35BlockKind::full_attention)
            ++w.report.attention_block_count;
        else
            ++w.report.recurrent_block_count;
    }
    return w;
}

}  // namespace

struct oref_qwen35 {
    std::unique_ptr<model::MappedGgufModel> mapped;
    std::vector<model::GgufTensorInfo> infos;  // buffer-backed models
    std::vector<model::GgufTensorView> views;
    model::Qwen35Manifest manifest;
    model::Qwen35Weights weights;
    std::unique_ptr<runtime::HybridCache> cache;
};

extern "C" {

// The manifest fields a buffer-backed model needs (Qwen35Manifest,
// include/oracle/model/qwen35_manifest.hpp:12-47).
typedef struct oref_qwen35_manifest {
    uint32_t block_count, context_length, embedding_length, feed_forward_length;
    uint32_t head_count, head_count_kv, key_length, value_length;
    float rms_epsilon;
    uint32_t rope_dimension_count;
    int32_t rope_sections[4];
    float rope_frequency_base;
    uint32_t conv_kernel, state_size, group_count, time_step_rank, inner_size, full_attention_interval;
    uint32_t vocabulary_size;
} oref_qwen35_manifest;

int oref_qwen35_open_gguf(const char* path, int admit_q4k, uint64_t max_tokens, oref_qwen35** out, char* err,
                          std::size_t errlen) {
    return guarded(err, errlen, [&] {
        auto m = std::make_unique<oref_qwen35>();
        m->mapped = std::make_unique<model::MappedGgufModel>(path);
        m->manifest = model::load_qwen35_manifest(m->mapped->file());
#ifdef OREF_GATE_PATCHED
        (void)admit_q4k;
        m->weights = model::bind_qwen35_weights(*m->mapped, m->manifest);
#else
        m->weights = admit_q4k ? bind_admitting_q4k(m->mapped->tensors(), m->manifest)
                               : model::bind_qwen35_weights(*m->mapped, m->manifest);
#endif
        m->cache = std::make_unique<runtime::HybridCache>(m->manifest, max_tokens);
        *out = m.release();
    });
}

int oref_qwen35_open_buffers(const oref_qwen35_manifest* mf, uint32_t n, const char* const* names,
                             const uint32_t* types, const uint32_t* n_dims, const uint64_t* dims,
                             const void* const* data, const uint64_t* sizes, int admit_q4k, uint64_t max_tokens,
                             oref_qwen35** out, char* err, std::size_t errlen) {
    return guarded(err, errlen, [&] {
        auto m = std::make_unique<oref_qwen35>();
        model::Qwen35Manifest& g = m->manifest;
        g.architecture = "qwen35";
        g.model_name = "synthetic";
        g.total_block_count = g.backbone_block_count = mf->block_count;
        g.context_length = mf->context_length;
        g.embedding_length = mf->embedding_length;
        g.feed_forward_length = mf->feed_forward_length;
        g.attention_head_count = mf->head_count;
        g.attention_head_count_kv = mf->head_count_kv;
        g.attention_key_length = mf->key_length;
        g.attention_value_length = mf->value_length;
        g.attention_rms_epsilon = mf->rms_epsilon;
        g.rope_dimension_count = mf->rope_dimension_count;
        for (int i = 0; i < 4; ++i) g.rope_dimension_sections[i] = mf->rope_sections[i];
        g.rope_frequency_base = mf->rope_frequency_base;
        g.ssm_convolution_kernel = mf->conv_kernel;
        g.ssm_state_size = mf->state_size;
        g.ssm_group_count = mf->group_count;
        g.ssm_time_step_rank = mf->time_step_rank;
        g.ssm_inner_size = mf->inner_size;
        g.full_attention_interval = mf->full_attention_interval;
        g.vocabulary_size = mf->vocabulary_size;
        m->infos.resize(n);
        for (uint32_t i = 0; i < n; ++i) {
            m->infos[i].name = names[i];
            m->infos[i].dimensions.assign(dims + 4 * i, dims + 4 * i + n_dims[i]);
            m->infos[i].ggml_type = types[i];
        }
        m->views.reserve(n);
        for (uint32_t i = 0; i < n; ++i) {
            const model::GgmlTypeLayout* layout = model::ggml_type_layout(types[i]);
            if (!layout) throw std::invalid_argument("unknown GGML type " + std::to_string(types[i]));
            m->views.emplace_back(&m->infos[i], layout, static_cast<const std::byte*>(data[i]),
                                  static_cast<std::size_t>(sizes[i]), 0);
        }
#ifdef OREF_GATE_PATCHED
        (void)admit_q4k;
        m->weights = model::bind_qwen35_weights(m->views, g);
#else
        m->weights = admit_q4k ? bind_admitting_q4k(m->views, g) : model::bind_qwen35_weights(m->views, g);
#endif
        m->cache = std::make_unique<runtime::HybridCache>(g, max_tokens);
        *out = m.release();
    });
}

uint32_t oref_qwen35_vocab(const oref_qwen35* m) { return m ? m->manifest.vocabulary_size : 0; }

void oref_qwen35_reset(oref_qwen35* m) {
    if (m) m->cache->reset();
}

// One token through the reference's forward at the cache's current length;
// logits (vocabulary_size floats) may be null.
int oref_qwen35_forward(oref_qwen35* m, uint32_t token, float* logits, char* err, std::size_t errlen) {
    return guarded(err, errlen, [&] {
        const std::size_t position = m->cache->sequence_length();
        runtime::Qwen35ForwardResult r = runtime::execute_qwen35_reference_token(
            m->manifest, m->weights, token, *m->cache, runtime::RopePosition::text(position), false);
        if (logits) std::memcpy(logits, r.logits.data(), r.logits.size() * sizeof(float));
    });
}

// Fresh greedy generation: n_new tokens after the prompt.
int oref_qwen35_greedy(oref_qwen35* m, const uint32_t* prompt, uint64_t n_prompt, uint64_t n_new, uint32_t* tokens,
                       char* err, std::size_t errlen) {
    return guarded(err, errlen, [&] {
        if (n_prompt == 0) throw std::invalid_argument("greedy decoding needs a prompt");
        m->cache->reset();
        runtime::Sampler sampler(runtime::SamplingConfig{});
        runtime::Qwen35ForwardResult current;
        for (uint64_t i = 0; i < n_prompt; ++i) {
            const std::size_t position = m->cache->sequence_length();
            current = runtime::execute_qwen35_reference_token(m->manifest, m->weights, prompt[i], *m->cache,
                                                              runtime::RopePosition::text(position), false);
        }
        for (uint64_t g = 0; g < n_new; ++g) {
            tokens[g] = sampler.sample(current.logits).token_id;
            if (g + 1 == n_new) break;
            const std::size_t position = m->cache->sequence_length();
            current = runtime::execute_qwen35_reference_token(m->manifest, m->weights, tokens[g], *m->cache,
                                                              runtime::RopePosition::text(position), false);
        }
    });
}

void oref_qwen35_close(oref_qwen35* m) { delete m; }

}  // extern "C"
