// Drives the reference's own, unchanged device path (src/forward.cpp
// ForwardToken/ForwardBatch with model.cuda_weights set by
// UploadModelWeightsToCuda, src/model.cpp:255-286) linked against the
// mini_llama_b200 adapter instead of the reference CUDA sources.  TEST
// INFRASTRUCTURE: shows that forward.cpp, model.cpp and the sampler drop in
// unchanged, and measures that path.
//
//   forward_on_b200 <model> <prompt_len> <n_new>
// prints one JSON line: generated tokens, per-step top-1 logit, timings.
//
//   forward_on_b200 --gguf <file> <prompt_len> <n_new> <seed>
// loads a GGUF file with the reference loader, runs the reference CPU path,
// then uploads the same model (UploadModelWeightsToCuda) and runs it on this
// library; prints both token lists and the largest logit difference.
#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <string>
#include <vector>

#include "include/batch.h"
#include "include/context.h"
#include "include/forward.h"
#include "include/model.h"
#include "include/ops.h"
#include "ref_gguf_run.h"
#include "ref_models.h"

using namespace mini_llama;
using namespace mini_llama::harness;

namespace {

int GgufRoundTrip(const std::string& path, int prompt_len, int n_new, uint64_t seed) {
    MiniLlamaModel model = LoadGgufOrThrow(path);
    const std::vector<int> prompt = GgufPrompt(model, prompt_len, seed);
    const GgufRun cpu = RunGguf(model, prompt, n_new);
    UploadModelWeightsToCuda(model, 0);
    const GgufRun dev = RunGguf(model, prompt, n_new);
    double err = 0.0, scale = 0.0, gap = 1e30;  // gap: smallest top-2 margin of the CPU logits
    for (size_t i = 0; i < cpu.logits.size() && i < dev.logits.size(); ++i) {
        float b1 = -1e30f, b2 = -1e30f;
        for (size_t j = 0; j < cpu.logits[i].size() && j < dev.logits[i].size(); ++j) {
            const float v = cpu.logits[i][j];
            err = std::max(err, static_cast<double>(std::fabs(v - dev.logits[i][j])));
            scale = std::max(scale, static_cast<double>(std::fabs(v)));
            if (v > b1) {
                b2 = b1;
                b1 = v;
            } else if (v > b2) {
                b2 = v;
            }
        }
        gap = std::min(gap, static_cast<double>(b1) - b2);
    }
    auto list = [](const std::vector<int>& v) {
        std::string o = "[";
        for (size_t i = 0; i < v.size(); ++i) o += (i ? ", " : "") + std::to_string(v[i]);
        return o + "]";
    };
    std::printf("{\"cpu\": %s, \"b200\": %s, \"logit_err\": %.9g, \"logit_scale\": %.9g, \"cpu_min_gap\": %.9g, "
                "\"neox\": %d, \"vocab\": %d, \"linear_calls\": %zu}\n",
                list(cpu.tokens).c_str(), list(dev.tokens).c_str(), err, scale, gap,
                model.config.rope_type == RopeType::kNeoX ? 1 : 0, model.config.vocab_size,
                ModelCudaLinearCalls(model));
    return 0;
}

}  // namespace

int main(int argc, char** argv) {
    if (argc == 6 && std::string(argv[1]) == "--gguf") {
        try {
            return GgufRoundTrip(argv[2], std::atoi(argv[3]), std::atoi(argv[4]),
                                 std::strtoull(argv[5], nullptr, 10));
        } catch (const std::exception& e) {
            std::fprintf(stderr, "forward_on_b200: %s\n", e.what());
            return 1;
        }
    }
    if (argc != 4) {
        std::fprintf(stderr, "usage: forward_on_b200 <model> <prompt_len> <n_new>\n");
        return 2;
    }
    try {
        ModelSpec spec = GetSpec(argv[1]);
        const int prompt_len = std::atoi(argv[2]), n_new = std::atoi(argv[3]);
        MiniLlamaModel model = BuildModel(spec);
        UploadModelWeightsToCuda(model, 0);
        MiniLlamaContext ctx(&model);
        std::vector<int> tokens = PromptTokens(spec, prompt_len);
        std::vector<int> generated;
        std::vector<float> top1;
        auto t0 = std::chrono::steady_clock::now();
        Tensor logits = ForwardBatch(ctx, model, MiniBatch::GetMultiMiniBatch(tokens, 0));
        auto t1 = std::chrono::steady_clock::now();
        for (int i = 0; i < n_new; ++i) {
            const int next = GetArgMax(logits);
            generated.push_back(next);
            top1.push_back(logits.data[next]);
            if (i + 1 == n_new) break;
            tokens.push_back(next);
            logits = ForwardBatch(ctx, model,
                                  MiniBatch::GetSingleMiniBatch(next, static_cast<int>(tokens.size()) - 1));
        }
        auto t2 = std::chrono::steady_clock::now();
        const double prefill_ms = std::chrono::duration<double, std::milli>(t1 - t0).count();
        const double decode_ms = std::chrono::duration<double, std::milli>(t2 - t1).count();
        std::printf("{\"model\": \"%s\", \"prefill_ms\": %.3f, \"decode_ms\": %.3f, "
                    "\"decode_tokens\": %d, \"generated\": [",
                    spec.name, prefill_ms, decode_ms, n_new - 1);
        for (size_t i = 0; i < generated.size(); ++i)
            std::printf("%s%d", i ? ", " : "", generated[i]);
        std::printf("], \"top1\": [");
        for (size_t i = 0; i < top1.size(); ++i) std::printf("%s%.9g", i ? ", " : "", top1[i]);
        std::printf("], \"linear_calls\": %zu}\n", ModelCudaLinearCalls(model));
        return 0;
    } catch (const std::exception& e) {
        std::fprintf(stderr, "forward_on_b200: %s\n", e.what());
        return 1;
    }
}
