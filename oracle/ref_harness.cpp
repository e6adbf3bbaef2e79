// Reference harness: drives the reference mini_llama CPU implementation, built
// from its own sources by oracle/Makefile, on the seeded synthetic inputs of
// oracle/synth.h.  TEST INFRASTRUCTURE ONLY.
//
//   ref_harness golden <outdir> [case ...]   write golden vectors (raw little-
//                                            endian files) for tests/golden/
//   ref_harness bench <model> <threads> <prompt_len> <n_predict> <steps> <warmup>
//                                            time the reference RunBenchmark
//                                            (src/debug.cpp:79-143); one JSON
//                                            line per step on stdout
//   ref_harness decode <model> <threads> <prompt_len> <tokens> <steps> <warmup>
//                                            prefill the prompt once (untimed,
//                                            ForwardBatch), then time steps of
//                                            <tokens> greedy decode tokens each,
//                                            continuing the sequence: the decode
//                                            loop of RunBenchmark (src/debug.cpp:
//                                            112-127); one JSON line per step
//   ref_harness gguf <file> <prompt_len> <n_new> <seed>
//                                            load a GGUF file (LoadGgufModel)
//                                            and decode greedily; one JSON line
//
// Every numeric result comes from the reference's own functions: QuantizeToQ80/
// Q40 and DeQuantize* (src/quant.cpp), LinearQ80/Q40/Q41 (src/quant.cpp:409-418),
// RmsNorm/RoPE/Silu/Swiglu/Softmax/GetArgMax (src/ops.cpp), the RoPE tables of
// MiniLlamaContext (src/context.cpp:16-25), QuantizeModelToQ80/Q40
// (src/model.cpp:454-493), ForwardToken (src/forward.cpp:642-666) and
// RunBenchmark.  The Q4_1 quantizer and the attention reference come from the
// reference GPU unit test through ref_gpu_test_shim.cpp.
#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <set>
#include <stdexcept>
#include <string>
#include <vector>

#include "include/batch.h"
#include "include/context.h"
#include "include/sampler.h"
#include "include/debug.h"
#include "include/forward.h"
#include "include/kv_cache.h"
#include "include/model.h"
#include "include/ops.h"
#include "include/quant.h"
#include "include/thread_pool.h"
#include "ref_gguf_run.h"
#include "ref_models.h"
#include "synth.h"

namespace mini_llama {
std::vector<BlockQ41> HarnessQuantizeQ41(const Tensor& t);
Tensor HarnessAttentionReference(const Tensor& q, const KVCache& cache, int layer, int pos,
                                 int n_heads, int n_kv_heads, int head_dim);
}  // namespace mini_llama

using namespace mini_llama;
using namespace mini_llama::harness;

namespace {

std::string g_out;

void WriteBin(const std::string& name, const void* data, size_t bytes) {
    std::string path = g_out + "/" + name;
    FILE* f = std::fopen(path.c_str(), "wb");
    if (!f) throw std::runtime_error("cannot write " + path);
    if (bytes && std::fwrite(data, 1, bytes, f) != bytes) throw std::runtime_error("short write");
    std::fclose(f);
}

void WriteF32(const std::string& name, const Tensor& t) {
    WriteBin(name + ".f32", t.data.data(), t.data.size() * sizeof(float));
}

template <typename T>
void WriteVec(const std::string& name, const std::vector<T>& v, const char* ext) {
    WriteBin(name + ext, v.data(), v.size() * sizeof(T));
}

// ---------------------------------------------------------------- fp16
void CaseFp16() {
    // Fp16ToFloat over every bit pattern, observed through DeQuantizeFromQ80 of
    // blocks whose only element is q = 1.
    std::vector<BlockQ80> blocks(65536);
    for (int i = 0; i < 65536; ++i) {
        std::memset(&blocks[i], 0, sizeof(BlockQ80));
        blocks[i].d = static_cast<u_int16_t>(i);
        blocks[i].qs[0] = 1;
    }
    WriteF32("fp16_to_f32", DeQuantizeFromQ80(blocks, {65536, 1}));

    // FloatToFp16 observed through the scale QuantizeToQ80/Q40 store for a
    // block whose largest magnitude is the probe.
    std::vector<float> probes = {127.0f / 65536.0f, 190.5f, 7.0f / 65536.0f, 10.5f,
                                 1.0f, 65504.0f * 127.0f, 1e-12f, 3.0e-8f * 127.0f};
    uint64_t key = synth_key(11, 1);
    for (int i = 0; i < 4096; ++i) {
        // log-uniform magnitudes from 2^-40 to 2^24, random sign
        uint64_t r = synth_u64(key, static_cast<uint64_t>(i));
        double e = -40.0 + 64.0 * static_cast<double>(r >> 11) * (1.0 / 9007199254740992.0);
        float v = static_cast<float>(std::ldexp(1.0 + (r & 0x3ff) / 1024.0, static_cast<int>(e)));
        probes.push_back((r >> 63) ? -v : v);
    }
    std::vector<u_int16_t> d80, d40;
    for (float p : probes) {
        Tensor t({32}, 0.0f);
        t.data[0] = p;
        t.data[7] = p * 0.25f;
        d80.push_back(QuantizeToQ80(t)[0].d);
        d40.push_back(QuantizeToQ40(t)[0].d);
    }
    WriteBin("fp16_probes.f32", probes.data(), probes.size() * sizeof(float));
    WriteVec("fp16_q80_d", d80, ".u16");
    WriteVec("fp16_q40_d", d40, ".u16");
}

// ---------------------------------------------------------------- quant + linear
const int kLinearShapes[][2] = {{5, 13}, {5, 32}, {5, 33}, {5, 64}, {5, 129},
                                {7, 176}, {16, 896}, {3, 4864}};

void CaseQuantLinear() {
    int idx = 0;
    for (const auto& s : kLinearShapes) {
        int n = s[0], k = s[1];
        std::string tag = std::to_string(n) + "x" + std::to_string(k);
        Tensor w = Synth({n, k}, 2, SYNTH_STREAM_W + 16ULL * idx, 0.02);
        Tensor x = Synth({3, k}, 2, SYNTH_STREAM_X + 16ULL * idx, 1.0);
        Tensor x1 = Synth({k}, 2, SYNTH_STREAM_X + 16ULL * idx + 1, 1.0);
        std::vector<BlockQ80> q80 = QuantizeToQ80(w);
        std::vector<BlockQ40> q40 = QuantizeToQ40(w);
        std::vector<BlockQ41> q41 = HarnessQuantizeQ41(w);
        WriteBin("q80_" + tag + ".u8", q80.data(), q80.size() * sizeof(BlockQ80));
        WriteBin("q40_" + tag + ".u8", q40.data(), q40.size() * sizeof(BlockQ40));
        WriteBin("q41_" + tag + ".u8", q41.data(), q41.size() * sizeof(BlockQ41));
        WriteF32("deq80_" + tag, DeQuantizeFromQ80(q80, w.shape));
        WriteF32("deq40_" + tag, DeQuantizeFromQ40(q40, w.shape));
        WriteF32("deq41_" + tag, DequantizeFromQ41(q41, w.shape));
        WriteF32("lin80_" + tag, LinearQ80(x, q80, w.shape));
        WriteF32("lin40_" + tag, LinearQ40(x, q40, w.shape));
        WriteF32("lin41_" + tag, LinearQ41(x, q41, w.shape));
        WriteF32("lin80v_" + tag, LinearQ80(x1, q80, w.shape));
        WriteF32("lin40v_" + tag, LinearQ40(x1, q40, w.shape));
        WriteF32("lin41v_" + tag, LinearQ41(x1, q41, w.shape));
        ++idx;
    }
    // zero blocks stay all-zero (test/core_cpu_test.cpp:182-196)
    Tensor zero({2, 64}, 0.0f);
    std::vector<BlockQ80> z80 = QuantizeToQ80(zero);
    std::vector<BlockQ40> z40 = QuantizeToQ40(zero);
    WriteBin("zero_q80.u8", z80.data(), z80.size() * sizeof(BlockQ80));
    WriteBin("zero_q40.u8", z40.data(), z40.size() * sizeof(BlockQ40));
}

// ---------------------------------------------------------------- rmsnorm / activations
void CaseNormAct() {
    int idx = 0;
    for (int n : {129, 896, 4096}) {
        Tensor x = Synth({n}, 2, 100 + idx, 1.0);
        Tensor w = Synth({n}, 2, 200 + idx, 0.1);
        for (float& v : w.data) v = 1.0f + v;
        for (float eps : {1e-5f, 1e-6f}) {
            std::string tag = std::to_string(n) + (eps == 1e-5f ? "_e5" : "_e6");
            WriteF32("rmsnorm_" + tag, RmsNorm(x, w, eps));
        }
        ++idx;
    }
    Tensor g = Synth({4864}, 2, 300, 2.0);
    Tensor u = Synth({4864}, 2, 301, 1.0);
    WriteF32("silu", Silu(g));
    WriteF32("swiglu", Swiglu(g, u));
    WriteF32("softmax", Softmax(g));
    Tensor ties({9}, 0.0f);
    ties.data = {0.5f, 2.0f, -1.0f, 2.0f, 1.0f, 2.0f, 0.0f, -3.0f, 1.5f};
    std::vector<int> am = {GetArgMax(ties), GetArgMax(g), GetArgMax(u)};
    WriteVec("argmax", am, ".i32");
}

// ---------------------------------------------------------------- rope
struct RopeCase {
    const char* tag;
    int head_dim, n_heads, n_kv_heads, max_seq_len;
    float theta;
    RopeType type;
    std::vector<int> positions;
};

void CaseRope() {
    std::vector<RopeCase> cases = {
        {"qwen2", 64, 14, 2, 32768, 1e6f, RopeType::kNeoX, {0, 1, 63, 191, 8191, 32767}},
        {"llama", 128, 32, 8, 768, 1e4f, RopeType::kNormal, {0, 5, 511, 767}},
        {"tiny", 16, 4, 2, 128, 1e4f, RopeType::kNormal, {0, 3, 11, 127}},
        {"gputest_normal", 14, 4, 2, 64, 1e4f, RopeType::kNormal, {3, 11}},
        {"gputest_neox", 14, 4, 2, 64, 1e4f, RopeType::kNeoX, {3, 11}},
    };
    int idx = 0;
    for (const RopeCase& c : cases) {
        MiniLlamaModel model;
        model.config.head_dim = c.head_dim;
        model.config.max_seq_len = c.max_seq_len;
        model.config.rope_theta = c.theta;
        model.config.n_layers = 1;
        model.config.n_kv_heads = 1;
        model.config.n_heads = 1;
        MiniLlamaContext ctx(&model);
        for (int pos : c.positions) {
            Tensor q = Synth({c.n_heads, c.head_dim}, 4, 400 + idx, 1.0);
            Tensor k = Synth({c.n_kv_heads, c.head_dim}, 4, 500 + idx, 1.0);
            RoPE(q, k, pos, ctx.rope_cos, ctx.rope_sin, c.type);
            std::string tag = std::string(c.tag) + "_p" + std::to_string(pos);
            WriteF32("rope_q_" + tag, q);
            WriteF32("rope_k_" + tag, k);
            ++idx;
        }
    }
}

// ---------------------------------------------------------------- attention
void AttentionOne(const std::string& tag, int layers, int layer, int pos, int n_heads,
                  int n_kv_heads, int head_dim, uint64_t stream) {
    int max_seq_len = pos + 1;
    KVCache cache(layers, max_seq_len, n_kv_heads, head_dim);
    size_t per_layer = static_cast<size_t>(max_seq_len) * n_kv_heads * head_dim;
    uint64_t kkey = synth_key(4, stream + 1), vkey = synth_key(4, stream + 2);
    for (size_t i = 0; i < per_layer; ++i) {
        cache.keys.data[layer * per_layer + i] = synth_normal(kkey, i, 1.0);
        cache.values.data[layer * per_layer + i] = synth_normal(vkey, i, 1.0);
    }
    Tensor q = Synth({n_heads, head_dim}, 4, stream, 1.0);
    WriteF32("attn_" + tag,
             HarnessAttentionReference(q, cache, layer, pos, n_heads, n_kv_heads, head_dim));
}

void CaseAttention() {
    uint64_t stream = 1000;
    // grid of the reference GPU unit test (test/gpu_core_test.cpp:463-467)
    for (int hd : {7, 128, 129})
        for (int pos : {0, 4, 126, 127, 128, 256}) {
            AttentionOne("grid_hd" + std::to_string(hd) + "_p" + std::to_string(pos), 2, 1, pos,
                         4, 2, hd, stream);
            stream += 8;
        }
    // tile geometries of the split-K kernel: (heads, KV heads, head_dim, pos),
    // 2 layers, layer 1, stream 5000 + 16 heads + head_dim
    const int geo[6][4] = {{32, 1, 64, 300}, {12, 4, 96, 257}, {8, 8, 256, 100},
                           {6, 2, 20, 70},   {4, 1, 8, 40},    {7, 7, 30, 33}};
    for (const auto& g : geo)
        AttentionOne("geo_" + std::to_string(g[0]) + "x" + std::to_string(g[1]) + "x" + std::to_string(g[2]) +
                         "_p" + std::to_string(g[3]),
                     2, 1, g[3], g[0], g[1], g[2], 5000 + 16 * g[0] + g[2]);
    // decode-attention sweep shapes
    for (int shape = 0; shape < 2; ++shape) {
        int nh = shape == 0 ? 14 : 32, nkv = shape == 0 ? 2 : 8, hd = shape == 0 ? 64 : 128;
        for (int pos : {127, 1023, 8191, 32767}) {
            AttentionOne("sweep_" + std::to_string(nh) + "x" + std::to_string(hd) + "_p" +
                             std::to_string(pos),
                         1, 0, pos, nh, nkv, hd, stream);
            stream += 8;
        }
    }
}

// Greedy generation through ForwardToken, recording every step's logits
// summary.  Step i is the forward of the token at position i.
void CaseModel(const std::string& name, int prompt_len, int n_new, bool full_logits) {
    ModelSpec s = GetSpec(name);
    MiniLlamaModel model = BuildModel(s);
    MiniLlamaContext ctx(&model);
    std::vector<int> tokens = PromptTokens(s, prompt_len);
    std::vector<float> top_val, all_logits, moments;
    std::vector<int> top_idx, generated;
    int steps = prompt_len + n_new - 1;
    const int kTop = 8;
    for (int step = 0; step < steps; ++step) {
        ctx.pos = step;
        Tensor logits = ForwardToken(ctx, model, tokens[step]);
        ctx.token_history.push_back(tokens[step]);
        std::vector<int> order(logits.data.size());
        for (size_t i = 0; i < order.size(); ++i) order[i] = static_cast<int>(i);
        std::partial_sort(order.begin(), order.begin() + kTop, order.end(), [&](int a, int b) {
            if (logits.data[a] != logits.data[b]) return logits.data[a] > logits.data[b];
            return a < b;
        });
        for (int t = 0; t < kTop; ++t) {
            top_idx.push_back(order[t]);
            top_val.push_back(logits.data[order[t]]);
        }
        double sum = 0.0, sq = 0.0, amax = 0.0;
        for (float v : logits.data) {
            sum += v;
            sq += static_cast<double>(v) * v;
            amax = std::max(amax, std::fabs(static_cast<double>(v)));
        }
        moments.push_back(static_cast<float>(sum));
        moments.push_back(static_cast<float>(sq));
        moments.push_back(static_cast<float>(amax));
        if (full_logits || step == prompt_len - 1)
            all_logits.insert(all_logits.end(), logits.data.begin(), logits.data.end());
        if (step >= prompt_len - 1) {
            int next = GetArgMax(logits);
            generated.push_back(next);
            if (static_cast<int>(tokens.size()) == step + 1) tokens.push_back(next);
        }
    }
    WriteVec("model_" + name + "_prompt", PromptTokens(s, prompt_len), ".i32");
    WriteVec("model_" + name + "_generated", generated, ".i32");
    WriteVec("model_" + name + "_top_idx", top_idx, ".i32");
    WriteVec("model_" + name + "_top_val", top_val, ".f32");
    WriteVec("model_" + name + "_moments", moments, ".f32");
    WriteVec("model_" + name + "_logits", all_logits, ".f32");
}

// ---------------------------------------------------------------- bench
int Bench(const std::string& name, int threads, int prompt_len, int n_predict, int steps,
          int warmup) {
    ModelSpec s = GetSpec(name);
    SetThreadCount(threads);
    auto t0 = std::chrono::steady_clock::now();
    MiniLlamaModel model = BuildModel(s);
    auto t1 = std::chrono::steady_clock::now();
    std::vector<int> prompt = PromptTokens(s, prompt_len);
    std::printf("{\"event\": \"built\", \"model\": \"%s\", \"build_s\": %.3f, \"threads\": %d}\n",
                s.name, std::chrono::duration<double>(t1 - t0).count(), GetThreadCount());
    std::fflush(stdout);
    for (int i = 0; i < warmup + steps; ++i) {
        BenchmarkResult r = RunBenchmark(model, prompt, n_predict, 0, false);
        std::printf(
            "{\"event\": \"step\", \"timed\": %s, \"decode_tokens\": %d, \"decode_ms\": %.4f, "
            "\"decode_tok_s\": %.6f, \"prefill_tokens\": %d, \"prefill_ms\": %.4f}\n",
            i >= warmup ? "true" : "false", r.n_decode_tokens, r.decode_ms,
            r.decode_tokens_per_sec(), r.n_prompt_tokens, r.prefill_ms);
        std::fflush(stdout);
    }
    return 0;
}

// ---------------------------------------------------------------- decode sample
// The decode loop of RunBenchmark (src/debug.cpp:112-127) split into timed
// steps: greedy sampling with seed 0, one single-token batch per position.
int DecodeSample(const std::string& name, int threads, int prompt_len, int tokens, int steps, int warmup) {
    ModelSpec s = GetSpec(name);
    SetThreadCount(threads);
    auto t0 = std::chrono::steady_clock::now();
    MiniLlamaModel model = BuildModel(s);
    std::vector<int> seq = PromptTokens(s, prompt_len);
    MiniLlamaContext ctx(&model);
    MiniSampler sampler(0);
    SamplerParams params;
    params.seed = 0;
    auto t1 = std::chrono::steady_clock::now();
    Tensor logits = ForwardBatch(ctx, model, MiniBatch::GetMultiMiniBatch(seq, 0));
    seq.push_back(sampler.Sample(logits, params));
    auto t2 = std::chrono::steady_clock::now();
    std::printf(
        "{\"event\": \"built\", \"model\": \"%s\", \"build_s\": %.3f, \"prefill_ms\": %.3f, "
        "\"threads\": %d}\n",
        s.name, std::chrono::duration<double>(t1 - t0).count(),
        std::chrono::duration<double, std::milli>(t2 - t1).count(), GetThreadCount());
    std::fflush(stdout);
    for (int i = 0; i < warmup + steps; ++i) {
        const int first = static_cast<int>(seq.size()) - 1;
        if (first + tokens > model.config.max_seq_len) throw std::runtime_error("decode sample passes max_seq_len");
        auto a = std::chrono::steady_clock::now();
        for (int j = 0; j < tokens; ++j) {
            logits = ForwardBatch(ctx, model, MiniBatch::GetSingleMiniBatch(seq.back(), static_cast<int>(seq.size()) - 1));
            seq.push_back(sampler.Sample(logits, params));
        }
        auto b = std::chrono::steady_clock::now();
        const double ms = std::chrono::duration<double, std::milli>(b - a).count();
        std::printf(
            "{\"event\": \"step\", \"timed\": %s, \"first_pos\": %d, \"decode_tokens\": %d, "
            "\"decode_ms\": %.4f, \"decode_tok_s\": %.6f}\n",
            i >= warmup ? "true" : "false", first, tokens, ms, tokens * 1000.0 / ms);
        std::fflush(stdout);
    }
    return 0;
}

}  // namespace

int main(int argc, char** argv) {
    try {
        if (argc >= 3 && std::string(argv[1]) == "golden") {
            g_out = argv[2];
            std::set<std::string> want;
            for (int i = 3; i < argc; ++i) want.insert(argv[i]);
            auto on = [&](const char* c) { return want.empty() || want.count(c); };
            if (on("fp16")) CaseFp16();
            if (on("quant")) CaseQuantLinear();
            if (on("normact")) CaseNormAct();
            if (on("rope")) CaseRope();
            if (on("attention")) CaseAttention();
            if (on("tiny")) CaseModel("tiny", 4, 8, true);
            if (on("llama2_l2")) CaseModel("llama2_l2", 6, 6, false);
            if (on("qwen2")) CaseModel("qwen2", 64, 128, false);
            return 0;
        }
        if (argc == 6 && std::string(argv[1]) == "gguf") {
            MiniLlamaModel model = LoadGgufOrThrow(argv[2]);
            const GgufRun r = RunGguf(model, GgufPrompt(model, std::atoi(argv[3]), std::strtoull(argv[5], nullptr, 10)),
                                      std::atoi(argv[4]));
            std::printf("{\"tokens\": [");
            for (size_t i = 0; i < r.tokens.size(); ++i) std::printf("%s%d", i ? ", " : "", r.tokens[i]);
            std::printf("], \"neox\": %d, \"vocab\": %d, \"dim\": %d, \"head_dim\": %d, \"lm_head_f32\": %d}\n",
                        model.config.rope_type == RopeType::kNeoX ? 1 : 0, model.config.vocab_size,
                        model.config.dim, model.config.head_dim, model.lm_head.type == QuantType::kF32 ? 1 : 0);
            return 0;
        }
        if (argc == 8 && std::string(argv[1]) == "decode") {
            return DecodeSample(argv[2], std::atoi(argv[3]), std::atoi(argv[4]), std::atoi(argv[5]),
                                std::atoi(argv[6]), std::atoi(argv[7]));
        }
        if (argc == 8 && std::string(argv[1]) == "bench") {
            return Bench(argv[2], std::atoi(argv[3]), std::atoi(argv[4]), std::atoi(argv[5]),
                         std::atoi(argv[6]), std::atoi(argv[7]));
        }
        std::fprintf(stderr,
                     "usage: ref_harness golden <outdir> [case...] | bench <model> <threads> "
                     "<prompt_len> <n_predict> <steps> <warmup> | decode <model> <threads> <prompt_len> "
                     "<tokens> <steps> <warmup>\n");
        return 2;
    } catch (const std::exception& e) {
        std::fprintf(stderr, "ref_harness: %s\n", e.what());
        return 1;
    }
}
