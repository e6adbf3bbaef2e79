// Synthetic model construction for the reference harnesses (test
// infrastructure): builds mini_llama's own MiniLlamaModel from the seeded
// generator of synth.h and quantizes it with the reference's
// QuantizeModelToQ80/Q40 (src/model.cpp:454-493).
#pragma once

#include <string>
#include <vector>

#include "include/model.h"
#include "include/quantized_tensor.h"
#include "synth.h"

namespace mini_llama {
namespace harness {

inline Tensor Synth(const std::vector<int>& shape, uint64_t seed, uint64_t stream, double sigma) {
    Tensor t(shape, 0.0f);
    uint64_t key = synth_key(seed, stream);
    for (size_t i = 0; i < t.data.size(); ++i) t.data[i] = synth_normal(key, i, sigma);
    return t;
}

struct ModelSpec {
    const char* name;
    int vocab, dim, hidden, layers, heads, kv_heads, head_dim, max_seq;
    float theta, eps;
    RopeType rope;
    bool bias, tied;
    int quant;  // 8 = Q8_0, 4 = Q4_0
    uint64_t seed, prompt_seed;
};

inline ModelSpec GetSpec(const std::string& name) {
    if (name == "tiny")
        return {"tiny", 256, 64, 176, 2, 4, 2, 16, 128, 1e4f, 1e-5f, RopeType::kNormal,
                false, false, 8, 0, 1};
    if (name == "qwen2")
        return {"qwen2", 151936, 896, 4864, 24, 14, 2, 64, 256, 1e6f, 1e-6f, RopeType::kNeoX,
                true, true, 8, 3, 3};
    if (name == "llama2_l2")
        return {"llama2_l2", 32000, 4096, 11008, 2, 32, 32, 128, 64, 1e4f, 1e-5f,
                RopeType::kNormal, false, false, 4, 5, 5};
    throw std::runtime_error("unknown model " + name);
}

inline QuantizedTensor SynthLinear(int rows, int cols, uint64_t seed, uint64_t stream) {
    return ToQuantizedTensor(Synth({rows, cols}, seed, stream, 0.02));
}

inline MiniLlamaModel BuildModel(const ModelSpec& s) {
    MiniLlamaModel m;
    ModelConfig& c = m.config;
    c.vocab_size = s.vocab;
    c.dim = s.dim;
    c.hidden_dim = s.hidden;
    c.n_layers = s.layers;
    c.n_heads = s.heads;
    c.n_kv_heads = s.kv_heads;
    c.head_dim = s.head_dim;
    c.max_seq_len = s.max_seq;
    c.rope_theta = s.theta;
    c.rms_norm_eps = s.eps;
    c.rope_type = s.rope;
    int qd = s.heads * s.head_dim, kd = s.kv_heads * s.head_dim;
    m.token_embedding = Synth({s.vocab, s.dim}, s.seed, SYNTH_STREAM_EMBEDDING, 0.02);
    m.layers.resize(s.layers);
    for (int l = 0; l < s.layers; ++l) {
        LayerWeights& w = m.layers[l];
        w.attention_norm = Tensor({s.dim}, 1.0f);
        w.ffn_norm = Tensor({s.dim}, 1.0f);
        w.wq = SynthLinear(qd, s.dim, s.seed, synth_stream_layer(l, SYNTH_KIND_WQ));
        w.wk = SynthLinear(kd, s.dim, s.seed, synth_stream_layer(l, SYNTH_KIND_WK));
        w.wv = SynthLinear(kd, s.dim, s.seed, synth_stream_layer(l, SYNTH_KIND_WV));
        w.wo = SynthLinear(s.dim, qd, s.seed, synth_stream_layer(l, SYNTH_KIND_WO));
        w.w_gate = SynthLinear(s.hidden, s.dim, s.seed, synth_stream_layer(l, SYNTH_KIND_GATE));
        w.w_up = SynthLinear(s.hidden, s.dim, s.seed, synth_stream_layer(l, SYNTH_KIND_UP));
        w.w_down = SynthLinear(s.dim, s.hidden, s.seed, synth_stream_layer(l, SYNTH_KIND_DOWN));
        if (s.bias) {
            w.bq = Synth({qd}, s.seed, synth_stream_layer(l, SYNTH_KIND_BQ), 0.02);
            w.bk = Synth({kd}, s.seed, synth_stream_layer(l, SYNTH_KIND_BK), 0.02);
            w.bv = Synth({kd}, s.seed, synth_stream_layer(l, SYNTH_KIND_BV), 0.02);
        }
    }
    m.final_norm = Tensor({s.dim}, 1.0f);
    m.lm_head = s.tied ? ToQuantizedTensor(m.token_embedding)
                       : SynthLinear(s.vocab, s.dim, s.seed, SYNTH_STREAM_LM_HEAD);
    m.is_loaded = true;
    if (s.quant == 8) QuantizeModelToQ80(m);
    else QuantizeModelToQ40(m);
    return m;
}

inline std::vector<int> PromptTokens(const ModelSpec& s, int n) {
    std::vector<int> ids(n);
    uint64_t key = synth_key(s.prompt_seed, SYNTH_STREAM_PROMPT);
    for (int i = 0; i < n; ++i) ids[i] = static_cast<int>(synth_index(key, i, s.vocab));
    return ids;
}


}  // namespace harness
}  // namespace mini_llama
