// A GGUF file through the reference's own loader (LoadGgufModel,
// src/gguf_loader.cpp:327-399) and forward pass (ForwardBatch over the prompt,
// then one token at a time, greedy GetArgMax; src/forward.cpp, src/ops.cpp:199-212).
// TEST INFRASTRUCTURE: used by ref_harness (reference CPU path) and
// forward_on_b200 (the same model on this library) for the GGUF round trip.
#pragma once

#include <stdexcept>
#include <string>
#include <vector>

#include "include/batch.h"
#include "include/context.h"
#include "include/forward.h"
#include "include/gguf_loader.h"
#include "include/model.h"
#include "include/ops.h"
#include "synth.h"

namespace mini_llama {
namespace harness {

struct GgufRun {
    std::vector<int> tokens;                // greedy ids
    std::vector<std::vector<float>> logits; // logits that chose each id
};

inline MiniLlamaModel LoadGgufOrThrow(const std::string& path) {
    MiniLlamaModel model = LoadGgufModel(path);
    if (!model.is_loaded) throw std::runtime_error("LoadGgufModel: " + model.load_error);
    return model;
}

// Prompt ids: the seeded uniform stream of synth.h over the model's vocabulary.
inline std::vector<int> GgufPrompt(const MiniLlamaModel& model, int n, uint64_t seed) {
    std::vector<int> ids(n);
    const uint64_t key = synth_key(seed, SYNTH_STREAM_PROMPT);
    for (int i = 0; i < n; ++i)
        ids[i] = static_cast<int>(synth_index(key, static_cast<uint64_t>(i), model.config.vocab_size));
    return ids;
}

inline GgufRun RunGguf(MiniLlamaModel& model, std::vector<int> tokens, int n_new) {
    GgufRun r;
    MiniLlamaContext ctx(&model);
    Tensor logits = ForwardBatch(ctx, model, MiniBatch::GetMultiMiniBatch(tokens, 0));
    for (int i = 0; i < n_new; ++i) {
        const int next = GetArgMax(logits);
        r.tokens.push_back(next);
        r.logits.push_back(logits.data);
        if (i + 1 == n_new) break;
        tokens.push_back(next);
        logits = ForwardBatch(ctx, model, MiniBatch::GetSingleMiniBatch(next, static_cast<int>(tokens.size()) - 1));
    }
    return r;
}

}  // namespace harness
}  // namespace mini_llama
