// Decode session: the whole-token device path of mini_llama (device branch of
// ForwardToken, src/forward.cpp:292-333 and :642-666, plus the greedy GetArgMax
// of src/ops.cpp:199-212) as one CUDA graph per token.
//
// Per layer the graph holds five kernels, each a fused step:
//   1. RMSNorm(x) -> [wq|wk|wv] GEMV + bias                      -> qkv
//   2. RoPE(q, k) from the reference CPU tables, KV-cache write,
//      split-K GQA attention                                      -> partials
//   3. merge partials -> wo GEMV + residual                        -> x_mid
//   4. RMSNorm(x_mid) -> [gate|up] GEMV -> SwiGLU                  -> ff
//   5. down GEMV + residual                                        -> x
// then RMSNorm -> lm_head GEMV -> arg-max (token and position stay on the
// device).  Kernels are launched with programmatic dependent launch, so each
// one streams its weights into shared memory while the previous one finishes.
//
// Q8_0 models whose shapes fit run instead the persistent decode kernel of
// megakernel.cu: every step of a whole generate / decode call in one
// cooperative launch.  The graph stays captured and can be selected with
// mlb_session_use_persistent(session, 0).
#include <algorithm>
#include <array>
#include <climits>
#include <cmath>
#include <memory>
#include <vector>

#include "attention.cuh"
#include "megakernel.cuh"
#include "model.cuh"
#include "qgemv.cuh"
#include "qmma.cuh"
#include "rows.cuh"

namespace mlb {

namespace {

constexpr int kKinds = 15;
constexpr int kRingBudget = 96 * 1024;

// x = embedding[hist[pos]]; an out-of-range token sets the status flag and
// leaves zeros rather than reading outside the table.
__global__ void DecodeEmbedKernel(const float* table, int vocab, int dim, const int* hist,
                                  const int* pos, float* x, int* status) {
    GridDepWait();
    GridDepLaunch();
    const int tok = hist[*pos];
    const bool ok = tok >= 0 && tok < vocab;
    if (!ok && threadIdx.x == 0 && blockIdx.x == 0) atomicExch(status, MLB_ERR_OUT_OF_RANGE);
    const float* row = table + size_t(ok ? tok : 0) * dim;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < dim; i += gridDim.x * blockDim.x)
        x[i] = ok ? row[i] : 0.0f;
}

size_t Align256(size_t v) { return (v + 255) & ~size_t(255); }

size_t LinearBytes(int qtype, int rows, int cols) {
    return size_t(rows) * ((cols + 31) / 32) * BlockBytes(qtype);
}

}  // namespace
}  // namespace mlb

struct mlb_session {
    mlb_model* model = nullptr;
    float* kc = nullptr;
    float* vc = nullptr;
    float* x = nullptr;
    float* xmid = nullptr;
    float* qkv = nullptr;
    float* attn = nullptr;
    float* ff = nullptr;
    float* logits = nullptr;
    float* part_ml = nullptr;
    float* part_o = nullptr;
    float* am_val = nullptr;
    int* am_idx = nullptr;
    unsigned* am_counter = nullptr;
    int* state = nullptr;  // [0] pos, [1] gen_from, [2] next token, [3] status
    int* hist = nullptr;   // [max_seq_len + 1]
    int chunks = 1;
    bool merge_in_oproj = true;  // the O-projection's prologue merges the attention partials
    size_t cache_floats = 0;
    // persistent decode kernel
    bool mega_ok = false;  // the model's shapes fit it
    std::string mega_reason;
    bool mega = false;     // selected for generate / decode_device / forward
    mlb::MegaParams mp = {};
    size_t mega_smem = 0;
    unsigned* counters = nullptr;
    size_t counter_bytes = 0;
    unsigned long long* qkvt = nullptr;  // tagged q, k, v words (never match a stale tag)
    size_t qkvt_bytes = 0;
    unsigned tag_base = 1;               // next (step 0, layer 0) tag; 0 marks never written
    unsigned long long wait_ns = 2000000000ull;  // bound of one wait in the persistent kernel
    int withhold = -1;                   // test hook: a phase counter never signalled
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    // prompt pass: all prompt tokens through each layer at once (row buffers
    // for max_seq_len tokens, allocated on first use)
    int prefill_min = 16;  // prompts of at least this many tokens take it (0: never)
    bool pf_ready = false;
    float *pf_x = nullptr, *pf_xn = nullptr, *pf_q = nullptr, *pf_k = nullptr, *pf_v = nullptr;
    float *pf_attn = nullptr, *pf_o = nullptr, *pf_xmid = nullptr, *pf_gate = nullptr, *pf_up = nullptr;
    float *pf_sw = nullptr, *pf_d = nullptr, *pf_part_ml = nullptr, *pf_part_o = nullptr;
    int* pf_pos = nullptr;
    std::vector<void*> allocations;
};

namespace mlb {
namespace {

void* DevAlloc(mlb_session* s, DeviceContext& c, size_t bytes) {
    void* p = nullptr;
    CheckCuda(cudaMallocFromPoolAsync(&p, bytes, c.pool, c.stream), "cudaMallocFromPoolAsync");
    s->allocations.push_back(p);
    return p;
}

void ValidateConfig(const mlb_model_config& c) {
    const char* w = "mlb_model_create";
    Require(c.vocab_size > 0 && c.dim > 0 && c.hidden_dim > 0 && c.n_layers > 0, w,
            "model dimensions must be positive");
    Require(c.n_heads > 0 && c.n_kv_heads > 0 && c.head_dim > 0 && c.max_seq_len > 0, w,
            "head shape must be positive");
    Require(c.n_heads % c.n_kv_heads == 0, w, "n_heads must be divisible by n_kv_heads");
    Require(c.head_dim % 2 == 0, w, "head_dim must be positive and even");
    Require(c.head_dim <= 256, w, "head_dim above 256 is not supported", MLB_ERR_UNSUPPORTED);
    Require(c.weight_type == MLB_Q8_0 || c.weight_type == MLB_Q4_0 || c.weight_type == MLB_Q4_1, w,
            "weight_type must be Q8_0, Q4_0 or Q4_1");
    Require(std::isfinite(c.rms_norm_eps) && c.rms_norm_eps > 0.0f, w,
            "eps must be positive and finite");
    Require(std::isfinite(c.rope_theta) && c.rope_theta > 0.0f, w, "theta must be positive");
}

size_t KindBytes(const mlb_model_config& c, int kind) {
    const int qd = c.n_heads * c.head_dim, kd = c.n_kv_heads * c.head_dim;
    const int qt = c.weight_type;
    switch (kind) {
        case MLB_W_EMBEDDING: return size_t(c.vocab_size) * c.dim * 4;
        case MLB_W_FINAL_NORM: return size_t(c.dim) * 4;
        case MLB_W_LM_HEAD: return LinearBytes(qt, c.vocab_size, c.dim);
        case MLB_W_ATTN_NORM: return size_t(c.dim) * 4;
        case MLB_W_WQ: return LinearBytes(qt, qd, c.dim);
        case MLB_W_WK: return LinearBytes(qt, kd, c.dim);
        case MLB_W_WV: return LinearBytes(qt, kd, c.dim);
        case MLB_W_BQ: return c.qkv_bias ? size_t(qd) * 4 : 0;
        case MLB_W_BK: return c.qkv_bias ? size_t(kd) * 4 : 0;
        case MLB_W_BV: return c.qkv_bias ? size_t(kd) * 4 : 0;
        case MLB_W_WO: return LinearBytes(qt, c.dim, qd);
        case MLB_W_FFN_NORM: return size_t(c.dim) * 4;
        case MLB_W_GATE: return LinearBytes(qt, c.hidden_dim, c.dim);
        case MLB_W_UP: return LinearBytes(qt, c.hidden_dim, c.dim);
        case MLB_W_DOWN: return LinearBytes(qt, c.dim, c.hidden_dim);
    }
    return 0;
}

bool IsLinear(int kind) {
    return kind == MLB_W_LM_HEAD || kind == MLB_W_WQ || kind == MLB_W_WK || kind == MLB_W_WV ||
           kind == MLB_W_WO || kind == MLB_W_GATE || kind == MLB_W_UP || kind == MLB_W_DOWN;
}

void LinearShape(const mlb_model_config& c, int kind, int& rows, int& cols) {
    const int qd = c.n_heads * c.head_dim, kd = c.n_kv_heads * c.head_dim;
    switch (kind) {
        case MLB_W_LM_HEAD: rows = c.vocab_size; cols = c.dim; break;
        case MLB_W_WQ: rows = qd; cols = c.dim; break;
        case MLB_W_WK: case MLB_W_WV: rows = kd; cols = c.dim; break;
        case MLB_W_WO: rows = c.dim; cols = qd; break;
        case MLB_W_GATE: case MLB_W_UP: rows = c.hidden_dim; cols = c.dim; break;
        default: rows = c.dim; cols = c.hidden_dim; break;  // MLB_W_DOWN
    }
}

void RepackOne(mlb_model* m, DeviceContext& c, int l, int kind) {
    int rows = 0, cols = 0;
    LinearShape(m->cfg, kind, rows, cols);
    const auto& src = m->Get(l, kind);
    LaunchRepackQ80R16(c, m->Ptr(src), rows, cols, const_cast<uint8_t*>(m->R16(l, kind)));
    if (m->r16c && (kind == MLB_W_WO || kind == MLB_W_DOWN))
        LaunchRepackQ80R16(c, m->Ptr(src), rows, cols, const_cast<uint8_t*>(m->R16C(l, kind)), true);
}

// Shapes the persistent decode kernel handles: whole 32-blocks everywhere,
// head_dim 32, 64 or 128 (a K/V row is 8, 16 or 32 float4 lanes), and its
// six-stage ring of the largest
// item (two row tiles of a dim-wide weight, or one dim-tall block column)
// plus its vectors within the shared-memory limit.
// Empty when it fits, else the reason.
std::string MegaShapeOk(const mlb_model_config& cf, const DeviceContext& c, int& stage_bytes) {
    if (cf.weight_type != MLB_Q8_0) return "weights are not Q8_0";
    if (cf.dim % 32 || cf.hidden_dim % 32) return "dim and hidden_dim must be multiples of 32";
    if (cf.head_dim != 32 && cf.head_dim != 64 && cf.head_dim != 128)
        return "head_dim must be 32, 64 or 128";
    const int tile_b = (cf.dim / 32) * kR16Chunk;
    const int col_b = ((cf.dim + 15) / 16) * kR16Chunk;
    stage_bytes = std::max(2 * tile_b, col_b);
    MegaParams p = {};
    p.n_layers = cf.n_layers;
    p.dim = cf.dim;
    p.hidden = cf.hidden_dim;
    p.vocab = cf.vocab_size;
    p.n_heads = cf.n_heads;
    p.hd = cf.head_dim;
    p.qd = cf.n_heads * cf.head_dim;
    p.kd = cf.n_kv_heads * cf.head_dim;
    p.stage_bytes = stage_bytes;
    p.list_cap = MegaListCap(p, c.sm_count);
    int coop = 0;
    cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, c.device);
    if (!coop) return "the device has no cooperative launch";
    if (MegaSmemBytes(p) > static_cast<size_t>(c.max_smem_optin))
        return "needs " + std::to_string(MegaSmemBytes(p)) + " B of shared memory, the device has " +
               std::to_string(c.max_smem_optin);
    return "";
}

// Q8_0 models keep an R16 copy of every linear weight for the integer-MMA GEMV.
void PrepareR16(mlb_model* m, DeviceContext& c, int chunks) {
    if (m->cfg.weight_type != MLB_Q8_0 || m->r16) return;
    // Every GEMV step must leave room for a two-stage ring of whole 16-row
    // tiles (gate/up hold two tiles per stage).
    auto need = [](int k, int tiles_per_stage, int aux) {
        const int nb = (k + 31) / 32;
        return QmmaSmem::Bytes(1, nb, tiles_per_stage * nb * kR16Chunk, 2, aux);
    };
    const mlb_model_config& cf = m->cfg;
    // (the O-projection's merge prologue is optional: when the attention
    // partials do not fit it, the step merges them in a separate kernel)
    (void)chunks;
    const size_t worst = std::max({need(cf.dim, 2, cf.dim), need(cf.hidden_dim, 1, 0),
                                   need(cf.n_heads * cf.head_dim, 1, 0)});
    if (worst + 4096 > static_cast<size_t>(c.max_smem_optin)) return;
    size_t off = 0;
    auto slot = [&](int kind) {
        int rows = 0, cols = 0;
        LinearShape(m->cfg, kind, rows, cols);
        mlb_model::Slot s;
        s.offset = off;
        s.bytes = R16Bytes(rows, cols);
        off += Align256(s.bytes);
        return s;
    };
    m->r16_lm_head = slot(MLB_W_LM_HEAD);
    m->r16_layer.resize(m->cfg.n_layers);
    const int kinds[] = {MLB_W_WQ, MLB_W_WK, MLB_W_WV, MLB_W_WO, MLB_W_GATE, MLB_W_UP, MLB_W_DOWN};
    for (int l = 0; l < m->cfg.n_layers; ++l)
        for (int k : kinds) m->r16_layer[l][k] = slot(k);
    int stage_bytes = 0;
    m->mega_reason = MegaShapeOk(cf, c, stage_bytes);
    m->r16c = m->mega_reason.empty();
    if (m->r16c) {
        m->r16c_layer.resize(m->cfg.n_layers);
        for (int l = 0; l < m->cfg.n_layers; ++l) {
            m->r16c_layer[l][0] = slot(MLB_W_WO);
            m->r16c_layer[l][1] = slot(MLB_W_DOWN);
        }
    }
    m->r16_bytes = off;
    CheckCuda(cudaMallocAsync(&m->r16, off, c.stream), "cudaMallocAsync(R16 weights)");
    RepackOne(m, c, -1, MLB_W_LM_HEAD);
    for (int l = 0; l < m->cfg.n_layers; ++l)
        for (int k : kinds) RepackOne(m, c, l, k);
}

// Captures one token step on the library stream.
void CaptureStep(mlb_session* s, DeviceContext& c) {
    mlb_model* m = s->model;
    const mlb_model_config& cf = m->cfg;
    const int qt = cf.weight_type;
    const int qd = cf.n_heads * cf.head_dim, kd = cf.n_kv_heads * cf.head_dim;
    int* pos = s->state;
    int* gen_from = s->state + 1;
    int* next = s->state + 2;
    int* status = s->state + 3;
    cudaStream_t st = c.stream;
    const bool r16 = m->r16 != nullptr;
    // Plans and launches one GEMV step: integer-MMA over R16 weights for Q8_0
    // models, the bulk-copy SIMT GEMV over GGUF blocks otherwise.
    auto gemv = [&](GemvParams& p, bool dual, int pro, int epi, const char* what) {
        GemvPlan plan = r16 ? PlanQmma(p, 1, dual, c.sm_count, c.max_smem_optin, 1, kRingBudget)
                            : PlanGemv(p, qt, 1, dual, c.sm_count, c.max_smem_optin, 1, kRingBudget);
        Require(plan.ok, "mlb_session", std::string(what) + " shape not supported by the GEMV",
                MLB_ERR_UNSUPPORTED);
        if (epi == kEpiArgmax)
            Require(plan.grid <= 4 * c.sm_count, "mlb_session", "arg-max partial buffer too small");
        if (r16) LaunchQmmaDecode(pro, epi, p, plan, st);
        else LaunchGemvDecode(qt, pro, epi, p, plan, st);
    };
    auto WL = [&](int l, int kind) {
        return r16 ? m->R16(l, kind) : static_cast<const uint8_t*>(m->Ptr(m->Get(l, kind)));
    };
    // The O-projection merges the step's attention partials in its prologue
    // when they fit its shared memory, else a merge kernel runs first.
    if (s->chunks > 1) {
        GemvParams p = {};
        p.K = qd;
        p.nseg = 1;
        p.seg[0] = GemvSeg{WL(0, MLB_W_WO), nullptr, cf.dim, 0, 0, 0};
        p.part_ml = s->part_ml;
        p.part_o = s->part_o;
        p.n_heads = cf.n_heads;
        p.head_dim = cf.head_dim;
        p.chunks = s->chunks;
        const GemvPlan plan = r16 ? PlanQmma(p, 1, false, c.sm_count, c.max_smem_optin, 1, kRingBudget)
                                  : PlanGemv(p, qt, 1, false, c.sm_count, c.max_smem_optin, 1, kRingBudget);
        s->merge_in_oproj = plan.ok;
    }

    CheckCuda(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal), "cudaStreamBeginCapture");
    try {
        Launch("DecodeEmbedKernel", DecodeEmbedKernel, dim3(4), dim3(256), 0, st, true,
               static_cast<const float*>(m->Ptr(m->global[MLB_W_EMBEDDING])), cf.vocab_size,
               cf.dim, const_cast<const int*>(s->hist), const_cast<const int*>(pos), s->x, status);
        for (int l = 0; l < cf.n_layers; ++l) {
            auto W = [&](int kind) { return WL(l, kind); };
            auto F = [&](int kind) { return static_cast<const float*>(m->Ptr(m->Get(l, kind))); };
            // 1. RMSNorm + QKV + bias
            {
                GemvParams p = {};
                p.K = cf.dim;
                p.nseg = 3;
                p.seg[0] = GemvSeg{W(MLB_W_WQ), F(MLB_W_BQ), qd, 0, 0, 0};
                p.seg[1] = GemvSeg{W(MLB_W_WK), F(MLB_W_BK), kd, qd, 0, 0};
                p.seg[2] = GemvSeg{W(MLB_W_WV), F(MLB_W_BV), kd, qd + kd, 0, 0};
                p.x = s->x;
                p.y = s->qkv;
                p.y_stride = qd + 2 * kd;
                p.norm_w = F(MLB_W_ATTN_NORM);
                p.eps = cf.rms_norm_eps;
                p.status = status;
                gemv(p, false, kProRmsNorm, kEpiStore, "QKV");
            }
            // 2. RoPE + KV write + split-K attention
            {
                AttnParams a = {};
                a.q = s->qkv;
                a.q_batch_stride = 0;
                a.kc = s->kc;
                a.vc = s->vc;
                a.seq_stride = 0;
                a.layer = l;
                a.max_seq_len = cf.max_seq_len;
                a.n_heads = cf.n_heads;
                a.n_kv = cf.n_kv_heads;
                a.hd = cf.head_dim;
                a.group = cf.n_heads / cf.n_kv_heads;
                a.hgroups = (a.group + kAttnGmax - 1) / kAttnGmax;
                a.chunks = s->chunks;
                a.scale = 1.0f / std::sqrt(static_cast<float>(cf.head_dim));
                a.pos_dev = pos;
                a.pos_stride = 0;
                a.out = s->attn;
                a.part_ml = s->part_ml;
                a.part_o = s->part_o;
                a.fused_rope = 1;
                a.kv_new = s->qkv + qd;
                a.rope_cos = m->rope_cos;
                a.rope_sin = m->rope_sin;
                a.neox = cf.rope_type == MLB_ROPE_NEOX;
                a.status = status;
                LaunchAttention(a, 1, st, true);
            }
            // 3. O projection + residual
            {
                GemvParams p = {};
                p.K = qd;
                p.nseg = 1;
                p.seg[0] = GemvSeg{W(MLB_W_WO), nullptr, cf.dim, 0, 0, 0};
                p.x = s->attn;
                p.y = s->xmid;
                p.y_stride = cf.dim;
                p.residual = s->x;
                p.res_stride = cf.dim;
                p.status = status;
                if (s->chunks > 1 && s->merge_in_oproj) {
                    p.part_ml = s->part_ml;
                    p.part_o = s->part_o;
                    p.n_heads = cf.n_heads;
                    p.head_dim = cf.head_dim;
                    p.chunks = s->chunks;
                    gemv(p, false, kProAttnMerge, kEpiResidual, "O-projection");
                } else {
                    // long caches: more partials than the prologue holds; the
                    // merge kernel writes the attention rows first
                    if (s->chunks > 1)
                        LaunchAttnMerge(s->part_ml, s->part_o, s->chunks, cf.head_dim, s->attn, cf.n_heads, st);
                    gemv(p, false, kProPlain, kEpiResidual, "O-projection");
                }
            }
            // 4. RMSNorm + gate/up + SwiGLU
            {
                GemvParams p = {};
                p.K = cf.dim;
                p.nseg = 2;
                p.seg[0] = GemvSeg{W(MLB_W_GATE), nullptr, cf.hidden_dim, 0, 0, 0};
                p.seg[1] = GemvSeg{W(MLB_W_UP), nullptr, cf.hidden_dim, 0, 0, 0};
                p.x = s->xmid;
                p.y = s->ff;
                p.y_stride = cf.hidden_dim;
                p.norm_w = F(MLB_W_FFN_NORM);
                p.eps = cf.rms_norm_eps;
                p.status = status;
                gemv(p, true, kProRmsNorm, kEpiSwiglu, "FFN");
            }
            // 5. down + residual
            {
                GemvParams p = {};
                p.K = cf.hidden_dim;
                p.nseg = 1;
                p.seg[0] = GemvSeg{W(MLB_W_DOWN), nullptr, cf.dim, 0, 0, 0};
                p.x = s->ff;
                p.y = s->x;
                p.y_stride = cf.dim;
                p.residual = s->xmid;
                p.res_stride = cf.dim;
                p.status = status;
                gemv(p, false, kProPlain, kEpiResidual, "down-projection");
            }
        }
        // final RMSNorm + lm_head + arg-max
        {
            GemvParams p = {};
            p.K = cf.dim;
            p.nseg = 1;
            p.seg[0] = GemvSeg{WL(-1, MLB_W_LM_HEAD), nullptr, cf.vocab_size, 0, 0, 0};
            p.x = s->x;
            p.y = s->logits;
            p.y_stride = cf.vocab_size;
            p.norm_w = static_cast<const float*>(m->Ptr(m->global[MLB_W_FINAL_NORM]));
            p.eps = cf.rms_norm_eps;
            p.am_val = s->am_val;
            p.am_idx = s->am_idx;
            p.am_counter = s->am_counter;
            p.am_token = next;
            p.am_pos = pos;
            p.am_hist = s->hist;
            p.am_gen_from = gen_from;
            p.status = status;
            gemv(p, false, kProRmsNorm, kEpiArgmax, "lm_head");
        }
    } catch (...) {
        cudaGraph_t g = nullptr;
        cudaStreamEndCapture(st, &g);
        if (g) cudaGraphDestroy(g);
        throw;
    }
    CheckCuda(cudaStreamEndCapture(st, &s->graph), "cudaStreamEndCapture");
    CheckCuda(cudaGraphInstantiate(&s->exec, s->graph, 0), "cudaGraphInstantiate");
}

// Sets up the persistent decode kernel for a session (when the model has its
// R16C weights): the per-layer weight table on the device, a second
// activation buffer, the phase counters and the launch parameters.
void PrepareMega(mlb_session* s, DeviceContext& c) {
    mlb_model* m = s->model;
    if (!m->r16 || !m->r16c) {
        s->mega_reason = m->r16 ? m->mega_reason : "no R16 weights (Q8_0 models only)";
        return;
    }
    const mlb_model_config& cf = m->cfg;
    int stage_bytes = 0;
    s->mega_reason = MegaShapeOk(cf, c, stage_bytes);
    if (!s->mega_reason.empty()) return;
    std::vector<MegaLayer> layers(cf.n_layers);
    for (int l = 0; l < cf.n_layers; ++l) {
        auto F = [&](int kind) { return static_cast<const float*>(m->Ptr(m->Get(l, kind))); };
        MegaLayer& L = layers[l];
        L.wqkv[0] = m->R16(l, MLB_W_WQ);
        L.wqkv[1] = m->R16(l, MLB_W_WK);
        L.wqkv[2] = m->R16(l, MLB_W_WV);
        L.bias[0] = F(MLB_W_BQ);
        L.bias[1] = F(MLB_W_BK);
        L.bias[2] = F(MLB_W_BV);
        L.attn_norm = F(MLB_W_ATTN_NORM);
        L.ffn_norm = F(MLB_W_FFN_NORM);
        L.wo = m->R16C(l, MLB_W_WO);
        L.gate = m->R16(l, MLB_W_GATE);
        L.up = m->R16(l, MLB_W_UP);
        L.down = m->R16C(l, MLB_W_DOWN);
    }
    MegaLayer* dl = static_cast<MegaLayer*>(DevAlloc(s, c, layers.size() * sizeof(MegaLayer)));
    CheckCuda(cudaMemcpyAsync(dl, layers.data(), layers.size() * sizeof(MegaLayer),
                              cudaMemcpyHostToDevice, c.stream),
              "cudaMemcpyAsync(layer table)");
    s->counter_bytes = size_t(kMkPhases * cf.n_layers + 2) * sizeof(unsigned);
    s->qkvt_bytes = size_t(cf.n_heads + 2 * cf.n_kv_heads) * cf.head_dim * 8;
    s->qkvt = static_cast<unsigned long long*>(DevAlloc(s, c, s->qkvt_bytes));
    CheckCuda(cudaMemsetAsync(s->qkvt, 0, s->qkvt_bytes, c.stream), "cudaMemsetAsync(qkv words)");
    s->counters = static_cast<unsigned*>(DevAlloc(s, c, s->counter_bytes));
    float* x2 = static_cast<float*>(DevAlloc(s, c, size_t(cf.dim) * 4));
    MegaParams& p = s->mp;
    p.n_layers = cf.n_layers;
    p.dim = cf.dim;
    p.hidden = cf.hidden_dim;
    p.vocab = cf.vocab_size;
    p.n_heads = cf.n_heads;
    p.n_kv = cf.n_kv_heads;
    p.hd = cf.head_dim;
    p.max_seq = cf.max_seq_len;
    p.qd = cf.n_heads * cf.head_dim;
    p.kd = cf.n_kv_heads * cf.head_dim;
    p.group = cf.n_heads / cf.n_kv_heads;
    p.eps = cf.rms_norm_eps;
    p.scale = 1.0f / std::sqrt(static_cast<float>(cf.head_dim));
    p.neox = cf.rope_type == MLB_ROPE_NEOX;
    p.embedding = static_cast<const float*>(m->Ptr(m->global[MLB_W_EMBEDDING]));
    p.final_norm = static_cast<const float*>(m->Ptr(m->global[MLB_W_FINAL_NORM]));
    p.lm_head = m->R16(-1, MLB_W_LM_HEAD);
    p.layers = dl;
    p.rope_cos = m->rope_cos;
    p.rope_sin = m->rope_sin;
    p.kc = s->kc;
    p.vc = s->vc;
    p.xbuf[0] = s->x;
    p.xbuf[1] = x2;
    p.xmid = s->xmid;
    p.qkvt = s->qkvt;
    p.logits = s->logits;
    p.am_val = s->am_val;
    p.am_idx = s->am_idx;
    p.counters = s->counters;
    p.hist = s->hist;
    p.next_token = s->state + 2;
    p.status = s->state + 3;
    p.stage_bytes = stage_bytes;
    p.list_cap = MegaListCap(p, c.sm_count);
    // cached K rows of the first attention pass in shared memory, as many as
    // the limit leaves room for (a multiple of 8, at most one pass)
    p.kst_rows = 0;
    const size_t smem0 = MegaSmemBytes(p), optin = static_cast<size_t>(c.max_smem_optin);
    if (smem0 < optin) {
        size_t rows = (optin - smem0) / (4 * size_t(p.hd));
        rows = std::min<size_t>({rows, size_t(kMkAttnChunk), size_t(p.max_seq)});
        p.kst_rows = static_cast<int>(rows & ~size_t(7));
    }
    s->mega_smem = MegaSmemBytes(p);
    s->mega_reason = MegaFits(p, s->mega_smem, c.sm_count);
    s->mega_ok = s->mega_reason.empty();
    s->mega = s->mega_ok;
}

// n_steps decode steps from start_pos in one launch of the persistent kernel;
// hist[pos + 1] receives the arg-max when pos + 1 >= gen_from.
void RunMega(mlb_session* s, DeviceContext& c, int start_pos, int n_steps, int gen_from) {
    CheckCuda(cudaMemsetAsync(s->counters, 0, s->counter_bytes, c.stream), "cudaMemsetAsync(counters)");
    const unsigned span = static_cast<unsigned>(n_steps) * static_cast<unsigned>(s->mp.n_layers);
    if (s->tag_base > 0xF0000000u - span) {  // tags would wrap: start over on a cleared buffer
        s->tag_base = 1;
        CheckCuda(cudaMemsetAsync(s->qkvt, 0, s->qkvt_bytes, c.stream), "cudaMemsetAsync(qkv words)");
    }
    MegaParams p = s->mp;
    p.wait_ns = s->wait_ns;
    p.withhold = s->withhold;
    p.tag_base = s->tag_base;
    s->tag_base += span;
    p.start_pos = start_pos;
    p.n_steps = n_steps;
    p.gen_from = gen_from;
    LaunchMegaDecode(p, c.sm_count, s->mega_smem, c.stream);
}

// First maximum of x[0..n) (src/ops.cpp:199-212) into hist[slot] (when slot
// >= 0) and *token; one CTA.
__global__ void PrefillArgmaxKernel(const float* x, int n, int* hist, int slot, int* token) {
    __shared__ float sv[1024];
    __shared__ int si[1024];
    GridDepWait();
    GridDepLaunch();
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int i = threadIdx.x; i < n; i += blockDim.x)
        if (x[i] > bv || (x[i] == bv && i < bi)) {
            bv = x[i];
            bi = i;
        }
    sv[threadIdx.x] = bv;
    si[threadIdx.x] = bi;
    __syncthreads();
    for (int o = blockDim.x / 2; o > 0; o >>= 1) {
        if (threadIdx.x < o) {
            const float ov = sv[threadIdx.x + o];
            const int oi = si[threadIdx.x + o];
            if (ov > sv[threadIdx.x] || (ov == sv[threadIdx.x] && oi < si[threadIdx.x])) {
                sv[threadIdx.x] = ov;
                si[threadIdx.x] = oi;
            }
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        const int tok = si[0] == 0x7fffffff ? 0 : si[0];
        *token = tok;
        if (slot >= 0) hist[slot] = tok;
    }
}

void EnsurePrefill(mlb_session* s, DeviceContext& c) {
    if (s->pf_ready) return;
    const mlb_model_config& cf = s->model->cfg;
    const size_t R = size_t(cf.max_seq_len);
    const int qd = cf.n_heads * cf.head_dim, kd = cf.n_kv_heads * cf.head_dim;
    auto A = [&](size_t floats) { return static_cast<float*>(DevAlloc(s, c, std::max<size_t>(floats, 1) * 4)); };
    s->pf_x = A(R * cf.dim);
    s->pf_xn = A(R * cf.dim);
    s->pf_xmid = A(R * cf.dim);
    s->pf_o = A(R * cf.dim);
    s->pf_d = A(R * cf.dim);
    s->pf_q = A(R * qd);
    s->pf_attn = A(R * qd);
    s->pf_k = A(R * kd);
    s->pf_v = A(R * kd);
    s->pf_gate = A(R * cf.hidden_dim);
    s->pf_up = A(R * cf.hidden_dim);
    s->pf_sw = A(R * cf.hidden_dim);
    s->pf_part_ml = A(R * cf.n_heads * s->chunks * 2);
    s->pf_part_o = A(R * cf.n_heads * s->chunks * cf.head_dim);
    s->pf_pos = static_cast<int*>(DevAlloc(s, c, R * 4));
    s->pf_ready = true;
}

// Tokens hist[start .. start + n) through every layer at once: each linear is
// one call on n rows (the tcgen05 path from 9 rows), RoPE and the KV write
// for all n positions first, then causal attention as a batch of n queries
// over the session's cache (query i sees positions 0 .. start + i).  The last
// row's logits land in s->logits and their first arg-max in hist[start + n]
// (and state[2]).  The work per sequence position is the decode step's.
void Prefill(mlb_session* s, DeviceContext& c, int start, int n) {
    mlb_model* m = s->model;
    const mlb_model_config& cf = m->cfg;
    const int qt = cf.weight_type, hd = cf.head_dim, D = cf.dim, F = cf.hidden_dim;
    const int qd = cf.n_heads * hd, kd = cf.n_kv_heads * hd;
    cudaStream_t st = c.stream;
    int* status = s->state + 3;
    auto W = [&](int l, int kind) { return static_cast<const uint8_t*>(m->Ptr(m->Get(l, kind))); };
    auto Fv = [&](int l, int kind) { return static_cast<const float*>(m->Ptr(m->Get(l, kind))); };
    // (not captured into a graph: the tensor-core linears use the context's workspace)
    // same_x: x is the previous linear's input, unchanged (its x images are reused)
    auto linear = [&](const float* x, const uint8_t* w, int rows, int K, int N, const float* bias, float* y,
                      bool same_x = false) {
        LinearRows(c, qt, x, w, rows, K, N, bias, y, nullptr, same_x);
    };
    // linears that read the same x (q / k / v, gate / up): one launch of the
    // integer-MMA linear for all of them where that path takes each one, else
    // one call each
    auto linears = [&](const float* x, int rows, int K, const WideSeg* segs, int nseg) {
        bool one = rows >= kTcMinRows && rows <= kWideMaxRows;
        for (int i = 0; i < nseg && one; ++i) one = WidePreferred(rows, K, segs[i].N);
        if (one && LaunchWideLinearSegs(c, qt, x, rows, K, segs, nseg, c.status, nullptr, false)) return;
        for (int i = 0; i < nseg; ++i) linear(x, segs[i].w, rows, K, segs[i].N, segs[i].bias, segs[i].y, i > 0);
    };
    auto rms = [&](const float* x, const float* w, float* y, int rows) {
        Launch("RowsRmsNormKernel", RowsRmsNormKernel, dim3(rows), dim3(256), 0, st, true, x, w, y, D,
               cf.rms_norm_eps);
    };
    auto add = [&](const float* a, const float* b, float* y, size_t cnt) {
        Launch("RowsAddKernel", RowsAddKernel, dim3(RowsGrid(cnt, 256, c.sm_count)), dim3(256), 0, st, true, a, b,
               cnt, y);
    };
    const int hgroups = (cf.n_heads / cf.n_kv_heads + kAttnGmax - 1) / kAttnGmax;
    const int chunks = std::min(s->chunks, AttnChunks(start + n, n, cf.n_kv_heads, hgroups, c.sm_count));
    Launch("RowsEmbedKernel", RowsEmbedKernel, dim3(n), dim3(256), 0, st, true,
           static_cast<const float*>(m->Ptr(m->global[MLB_W_EMBEDDING])), cf.vocab_size, D,
           const_cast<const int*>(s->hist + start), s->pf_x, status);
    for (int l = 0; l < cf.n_layers; ++l) {
        rms(s->pf_x, Fv(l, MLB_W_ATTN_NORM), s->pf_xn, n);
        {
            const WideSeg qkv[3] = {{W(l, MLB_W_WQ), cf.qkv_bias ? Fv(l, MLB_W_BQ) : nullptr, s->pf_q, qd},
                                    {W(l, MLB_W_WK), cf.qkv_bias ? Fv(l, MLB_W_BK) : nullptr, s->pf_k, kd},
                                    {W(l, MLB_W_WV), cf.qkv_bias ? Fv(l, MLB_W_BV) : nullptr, s->pf_v, kd}};
            linears(s->pf_xn, n, D, qkv, 3);
        }
        Launch("RowsRopeKvKernel", RowsRopeKvKernel, dim3(n), dim3(256), 0, st, true, s->pf_q,
               const_cast<const float*>(s->pf_k), const_cast<const float*>(s->pf_v), cf.n_heads, cf.n_kv_heads, hd,
               start, const_cast<const float*>(m->rope_cos), const_cast<const float*>(m->rope_sin),
               cf.rope_type == MLB_ROPE_NEOX ? 1 : 0, s->kc, s->vc, l, cf.max_seq_len, s->pf_pos);
        AttnParams a = {};
        a.q = s->pf_q;
        a.q_batch_stride = size_t(qd);
        a.kc = s->kc;
        a.vc = s->vc;
        a.seq_stride = 0;  // every query reads the session's one cache
        a.layer = l;
        a.max_seq_len = cf.max_seq_len;
        a.n_heads = cf.n_heads;
        a.n_kv = cf.n_kv_heads;
        a.hd = hd;
        a.group = cf.n_heads / cf.n_kv_heads;
        a.hgroups = hgroups;
        a.chunks = chunks;
        a.scale = 1.0f / std::sqrt(static_cast<float>(hd));
        a.pos_dev = s->pf_pos;
        a.pos_stride = 1;
        a.out = s->pf_attn;
        a.part_ml = s->pf_part_ml;
        a.part_o = s->pf_part_o;
        a.fused_rope = 0;
        a.status = status;
        LaunchAttention(a, n, st, true);
        if (chunks > 1) {
            LaunchAttnMerge(s->pf_part_ml, s->pf_part_o, chunks, hd, s->pf_attn, n * cf.n_heads, st);
        }
        linear(s->pf_attn, W(l, MLB_W_WO), n, qd, D, nullptr, s->pf_o);
        add(s->pf_x, s->pf_o, s->pf_xmid, size_t(n) * D);
        rms(s->pf_xmid, Fv(l, MLB_W_FFN_NORM), s->pf_xn, n);
        {
            const WideSeg gu[2] = {{W(l, MLB_W_GATE), nullptr, s->pf_gate, F}, {W(l, MLB_W_UP), nullptr, s->pf_up, F}};
            linears(s->pf_xn, n, D, gu, 2);
        }
        Launch("RowsSwigluKernel", RowsSwigluKernel, dim3(RowsGrid(size_t(n) * F, 256, c.sm_count)), dim3(256), 0,
               st, true, const_cast<const float*>(s->pf_gate), const_cast<const float*>(s->pf_up), size_t(n) * F,
               s->pf_sw);
        linear(s->pf_sw, W(l, MLB_W_DOWN), n, F, D, nullptr, s->pf_d);
        add(s->pf_xmid, s->pf_d, s->pf_x, size_t(n) * D);
    }
    // the last token: final RMSNorm, lm_head, arg-max
    rms(s->pf_x + size_t(n - 1) * D, static_cast<const float*>(m->Ptr(m->global[MLB_W_FINAL_NORM])), s->pf_xn, 1);
    linear(s->pf_xn, W(-1, MLB_W_LM_HEAD), 1, D, cf.vocab_size, nullptr, s->logits);
    Launch("PrefillArgmaxKernel", PrefillArgmaxKernel, dim3(1), dim3(1024), 0, st, true,
           const_cast<const float*>(s->logits), cf.vocab_size, s->hist, start + n <= cf.max_seq_len ? start + n : -1,
           s->state + 2);
}

void CheckStatus(mlb_session* s, DeviceContext& c) {
    int status = 0;
    CheckCuda(cudaMemcpyAsync(&status, s->state + 3, sizeof(int), cudaMemcpyDeviceToHost, c.stream),
              "cudaMemcpyAsync(status)");
    CheckCuda(cudaStreamSynchronize(c.stream), "cudaStreamSynchronize");
    if (status == 0) {  // the tensor-core linears of the prompt pass report into the context's word
        CheckCuda(cudaMemcpyAsync(&status, c.status, sizeof(int), cudaMemcpyDeviceToHost, c.stream),
                  "cudaMemcpyAsync(status)");
        CheckCuda(cudaStreamSynchronize(c.stream), "cudaStreamSynchronize");
        if (status != 0) CheckCuda(cudaMemsetAsync(c.status, 0, sizeof(int), c.stream), "cudaMemsetAsync");
    }
    if (status != 0) {
        CheckCuda(cudaMemsetAsync(s->state + 3, 0, sizeof(int), c.stream), "cudaMemsetAsync");
        Fail(status, status == MLB_ERR_DEVICE_TIMEOUT
                         ? "mlb_session: a bounded device wait expired"
                         : status == MLB_ERR_UNSUPPORTED
                               ? "mlb_session: persistent kernel schedule exceeds its list"
                               : "mlb_session: token id out of range on the device");
    }
}

void SetState(mlb_session* s, DeviceContext& c, int pos, int gen_from) {
    int* h = static_cast<int*>(PinnedStaging(c, 16));
    CheckCuda(cudaStreamSynchronize(c.stream), "cudaStreamSynchronize");
    h[0] = pos;
    h[1] = gen_from;
    CheckCuda(cudaMemcpyAsync(s->state, h, 2 * sizeof(int), cudaMemcpyHostToDevice, c.stream),
              "cudaMemcpyAsync(state)");
}

}  // namespace
}  // namespace mlb

using namespace mlb;

extern "C" {

int mlb_model_create(int device, const mlb_model_config* config, mlb_model** model) {
    return Guard([&] {
        Require(config && model, "mlb_model_create", "null argument");
        *model = nullptr;
        ValidateConfig(*config);
        DeviceContext& c = Ctx(device);
        auto m = std::make_unique<mlb_model>();
        m->device = device;
        m->cfg = *config;
        size_t off = 0;
        for (int k = 0; k < 3; ++k) {
            m->global[k].offset = off;
            m->global[k].bytes = KindBytes(*config, k);
            off += Align256(m->global[k].bytes);
        }
        m->layer.resize(config->n_layers);
        for (int l = 0; l < config->n_layers; ++l)
            for (int k = MLB_W_ATTN_NORM; k < kKinds; ++k) {
                m->layer[l][k].offset = off;
                m->layer[l][k].bytes = KindBytes(*config, k);
                off += Align256(m->layer[l][k].bytes);
            }
        const int half = config->head_dim / 2;
        const size_t table = size_t(config->max_seq_len) * half * 4;
        m->arena_bytes = off + 2 * Align256(table);
        CheckCuda(cudaMallocAsync(&m->arena, m->arena_bytes, c.stream), "cudaMallocAsync(weights)");
        CheckCuda(cudaMemsetAsync(m->arena, 0, m->arena_bytes, c.stream), "cudaMemsetAsync(weights)");
        m->rope_cos = reinterpret_cast<float*>(static_cast<char*>(m->arena) + off);
        m->rope_sin = reinterpret_cast<float*>(static_cast<char*>(m->arena) + off + Align256(table));
        // RoPE tables exactly as the reference CPU builds them (src/context.cpp:16-25)
        std::vector<float> cs(size_t(config->max_seq_len) * half), sn(cs.size());
        for (int pos = 0; pos < config->max_seq_len; ++pos)
            for (int i = 0; i < half; ++i) {
                float freq = 1.0f / std::pow(config->rope_theta,
                                             static_cast<float>(2 * i) / static_cast<float>(config->head_dim));
                cs[size_t(pos) * half + i] = std::cos(static_cast<float>(pos) * freq);
                sn[size_t(pos) * half + i] = std::sin(static_cast<float>(pos) * freq);
            }
        CheckCuda(cudaMemcpyAsync(m->rope_cos, cs.data(), table, cudaMemcpyHostToDevice, c.stream),
                  "cudaMemcpyAsync(rope)");
        CheckCuda(cudaMemcpyAsync(m->rope_sin, sn.data(), table, cudaMemcpyHostToDevice, c.stream),
                  "cudaMemcpyAsync(rope)");
        CheckCuda(cudaStreamSynchronize(c.stream), "cudaStreamSynchronize");
        *model = m.release();
    });
}

int mlb_model_destroy(mlb_model* model) {
    return Guard([&] {
        if (!model) return;
        DeviceContext& c = Ctx(model->device);
        CheckCuda(cudaStreamSynchronize(c.stream), "cudaStreamSynchronize");
        if (model->arena) CheckCuda(cudaFreeAsync(model->arena, c.stream), "cudaFreeAsync");
        if (model->r16) CheckCuda(cudaFreeAsync(model->r16, c.stream), "cudaFreeAsync");
        delete model;
    });
}

int mlb_model_weight(mlb_model* model, int layer, int kind, void** dev_ptr, size_t* bytes) {
    return Guard([&] {
        Require(model && dev_ptr && bytes, "mlb_model_weight", "null argument");
        Require(kind >= 0 && kind < kKinds, "mlb_model_weight", "unknown weight kind");
        if (kind >= MLB_W_ATTN_NORM)
            Require(layer >= 0 && layer < model->cfg.n_layers, "mlb_model_weight",
                    "layer out of range", MLB_ERR_OUT_OF_RANGE);
        const auto& slot = model->Get(layer, kind);
        *dev_ptr = model->Ptr(slot);
        *bytes = slot.bytes;
    });
}

int mlb_model_set_weight(mlb_model* model, int layer, int kind, const void* src, size_t bytes,
                         int src_is_host) {
    return Guard([&] {
        Require(model && src, "mlb_model_set_weight", "null argument");
        Require(kind >= 0 && kind < kKinds, "mlb_model_set_weight", "unknown weight kind");
        if (kind >= MLB_W_ATTN_NORM)
            Require(layer >= 0 && layer < model->cfg.n_layers, "mlb_model_set_weight",
                    "layer out of range", MLB_ERR_OUT_OF_RANGE);
        const auto& slot = model->Get(layer, kind);
        Require(bytes == slot.bytes, "mlb_model_set_weight",
                "weight shape is not match: expected " + std::to_string(slot.bytes) +
                    " bytes, got " + std::to_string(bytes));
        DeviceContext& c = Ctx(model->device);
        CheckCuda(cudaMemcpyAsync(model->Ptr(slot), src, bytes,
                                  src_is_host ? cudaMemcpyHostToDevice : cudaMemcpyDeviceToDevice,
                                  c.stream),
                  "cudaMemcpyAsync(weight)");
        if (model->r16 && IsLinear(kind)) RepackOne(model, c, layer, kind);
        if (src_is_host) CheckCuda(cudaStreamSynchronize(c.stream), "cudaStreamSynchronize");
    });
}

int mlb_model_bytes(mlb_model* model, size_t* bytes) {
    return Guard([&] {
        Require(model && bytes, "mlb_model_bytes", "null argument");
        *bytes = model->arena_bytes;
    });
}

int mlb_session_create(mlb_model* model, mlb_session** session) {
    return Guard([&] {
        Require(model && session, "mlb_session_create", "null argument");
        *session = nullptr;
        DeviceContext& c = Ctx(model->device);
        const mlb_model_config& cf = model->cfg;
        auto s = std::make_unique<mlb_session>();
        s->model = model;
        const int qd = cf.n_heads * cf.head_dim, kd = cf.n_kv_heads * cf.head_dim;
        s->cache_floats = size_t(cf.n_layers) * cf.max_seq_len * kd;
        const int hgroups = (cf.n_heads / cf.n_kv_heads + kAttnGmax - 1) / kAttnGmax;
        s->chunks = AttnChunks(cf.max_seq_len, 1, cf.n_kv_heads, hgroups, c.sm_count);
        s->kc = static_cast<float*>(DevAlloc(s.get(), c, s->cache_floats * 4));
        s->vc = static_cast<float*>(DevAlloc(s.get(), c, s->cache_floats * 4));
        s->x = static_cast<float*>(DevAlloc(s.get(), c, size_t(cf.dim) * 4));
        s->xmid = static_cast<float*>(DevAlloc(s.get(), c, size_t(cf.dim) * 4));
        s->qkv = static_cast<float*>(DevAlloc(s.get(), c, size_t(qd + 2 * kd) * 4));
        s->attn = static_cast<float*>(DevAlloc(s.get(), c, size_t(qd) * 4));
        s->ff = static_cast<float*>(DevAlloc(s.get(), c, size_t(cf.hidden_dim) * 4));
        s->logits = static_cast<float*>(DevAlloc(s.get(), c, size_t(cf.vocab_size) * 4));
        const size_t prow = size_t(cf.n_heads) * s->chunks;
        s->part_ml = static_cast<float*>(DevAlloc(s.get(), c, prow * 2 * 4));
        s->part_o = static_cast<float*>(DevAlloc(s.get(), c, prow * cf.head_dim * 4));
        s->am_val = static_cast<float*>(DevAlloc(s.get(), c, size_t(4) * c.sm_count * 4));
        s->am_idx = static_cast<int*>(DevAlloc(s.get(), c, size_t(4) * c.sm_count * 4));
        s->am_counter = static_cast<unsigned*>(DevAlloc(s.get(), c, 256));
        s->state = static_cast<int*>(DevAlloc(s.get(), c, 256));
        s->hist = static_cast<int*>(DevAlloc(s.get(), c, size_t(cf.max_seq_len + 1) * 4));
        CheckCuda(cudaMemsetAsync(s->kc, 0, s->cache_floats * 4, c.stream), "cudaMemsetAsync");
        CheckCuda(cudaMemsetAsync(s->vc, 0, s->cache_floats * 4, c.stream), "cudaMemsetAsync");
        CheckCuda(cudaMemsetAsync(s->am_counter, 0, 256, c.stream), "cudaMemsetAsync");
        CheckCuda(cudaMemsetAsync(s->state, 0, 256, c.stream), "cudaMemsetAsync");
        CheckCuda(cudaMemsetAsync(s->hist, 0, size_t(cf.max_seq_len + 1) * 4, c.stream),
                  "cudaMemsetAsync");
        PrepareR16(model, c, s->chunks);
        PrepareMega(s.get(), c);
        CheckCuda(cudaStreamSynchronize(c.stream), "cudaStreamSynchronize");
        CaptureStep(s.get(), c);
        *session = s.release();
    });
}

int mlb_session_destroy(mlb_session* session) {
    return Guard([&] {
        if (!session) return;
        DeviceContext& c = Ctx(session->model->device);
        CheckCuda(cudaStreamSynchronize(c.stream), "cudaStreamSynchronize");
        if (session->exec) cudaGraphExecDestroy(session->exec);
        if (session->graph) cudaGraphDestroy(session->graph);
        for (void* p : session->allocations) CheckCuda(cudaFreeAsync(p, c.stream), "cudaFreeAsync");
        delete session;
    });
}

int mlb_session_reset(mlb_session* session) {
    return Guard([&] {
        Require(session != nullptr, "mlb_session_reset", "null session");
        DeviceContext& c = Ctx(session->model->device);
        CheckCuda(cudaMemsetAsync(session->kc, 0, session->cache_floats * 4, c.stream), "cudaMemsetAsync");
        CheckCuda(cudaMemsetAsync(session->vc, 0, session->cache_floats * 4, c.stream), "cudaMemsetAsync");
    });
}

int mlb_session_forward(mlb_session* session, int token, int pos, float* logits, int* next_token) {
    return Guard([&] {
        Require(session != nullptr, "ForwardToken", "null session");
        const mlb_model_config& cf = session->model->cfg;
        Require(token >= 0 && token < cf.vocab_size, "ForwardToken", "token id out of range",
                MLB_ERR_OUT_OF_RANGE);
        Require(pos >= 0 && pos < cf.max_seq_len, "ForwardToken", "position out of range",
                MLB_ERR_OUT_OF_RANGE);
        DeviceContext& c = Ctx(session->model->device);
        int* h = static_cast<int*>(PinnedStaging(c, 16));
        CheckCuda(cudaStreamSynchronize(c.stream), "cudaStreamSynchronize");
        h[0] = pos;
        h[1] = INT_MAX;
        h[2] = token;
        CheckCuda(cudaMemcpyAsync(session->state, h, 2 * sizeof(int), cudaMemcpyHostToDevice, c.stream),
                  "cudaMemcpyAsync(state)");
        CheckCuda(cudaMemcpyAsync(session->hist + pos, h + 2, sizeof(int), cudaMemcpyHostToDevice,
                                  c.stream),
                  "cudaMemcpyAsync(token)");
        if (session->mega) RunMega(session, c, pos, 1, INT_MAX);
        else CheckCuda(cudaGraphLaunch(session->exec, c.stream), "cudaGraphLaunch");
        if (logits)
            CheckCuda(cudaMemcpyAsync(logits, session->logits, size_t(cf.vocab_size) * 4,
                                      cudaMemcpyDeviceToHost, c.stream),
                      "cudaMemcpyAsync(logits)");
        if (next_token)
            CheckCuda(cudaMemcpyAsync(h + 3, session->state + 2, sizeof(int), cudaMemcpyDeviceToHost,
                                      c.stream),
                      "cudaMemcpyAsync(next)");
        CheckStatus(session, c);
        if (next_token) *next_token = h[3];
    });
}

int mlb_session_generate(mlb_session* session, const int* prompt, int n_prompt, int start_pos,
                         int n_new, int* out_tokens) {
    return Guard([&] {
        const char* w = "mlb_session_generate";
        Require(session && prompt && out_tokens, w, "null argument");
        Require(n_prompt > 0 && n_new > 0, w, "prompt and generation must be non-empty");
        const mlb_model_config& cf = session->model->cfg;
        Require(start_pos >= 0 && start_pos + n_prompt + n_new - 1 <= cf.max_seq_len, w,
                "position out of range", MLB_ERR_OUT_OF_RANGE);
        for (int i = 0; i < n_prompt; ++i)
            Require(prompt[i] >= 0 && prompt[i] < cf.vocab_size, w, "token id out of range",
                    MLB_ERR_OUT_OF_RANGE);
        DeviceContext& c = Ctx(session->model->device);
        CheckCuda(cudaMemcpyAsync(session->hist + start_pos, prompt, size_t(n_prompt) * 4,
                                  cudaMemcpyHostToDevice, c.stream),
                  "cudaMemcpyAsync(prompt)");
        if (session->prefill_min > 0 && n_prompt >= session->prefill_min) {
            // the prompt in one pass, then the remaining n_new - 1 decode steps
            EnsurePrefill(session, c);
            Prefill(session, c, start_pos, n_prompt);
            const int from = start_pos + n_prompt;
            if (n_new > 1) {
                SetState(session, c, from, from);
                if (session->mega) {
                    RunMega(session, c, from, n_new - 1, from);
                } else {
                    for (int i = 0; i < n_new - 1; ++i)
                        CheckCuda(cudaGraphLaunch(session->exec, c.stream), "cudaGraphLaunch");
                }
            }
        } else {
            SetState(session, c, start_pos, start_pos + n_prompt);
            const int steps = n_prompt + n_new - 1;
            if (session->mega) {
                RunMega(session, c, start_pos, steps, start_pos + n_prompt);
            } else {
                for (int i = 0; i < steps; ++i)
                    CheckCuda(cudaGraphLaunch(session->exec, c.stream), "cudaGraphLaunch");
            }
        }
        CheckCuda(cudaMemcpyAsync(out_tokens, session->hist + start_pos + n_prompt, size_t(n_new) * 4,
                                  cudaMemcpyDeviceToHost, c.stream),
                  "cudaMemcpyAsync(tokens)");
        CheckStatus(session, c);
    });
}

int mlb_session_decode_device(mlb_session* session, int* tokens, int start_pos, int n_steps) {
    return Guard([&] {
        const char* w = "mlb_session_decode_device";
        Require(session && tokens, w, "null argument");
        Require(n_steps > 0, w, "n_steps must be positive");
        const mlb_model_config& cf = session->model->cfg;
        Require(start_pos >= 0 && start_pos + n_steps <= cf.max_seq_len, w,
                "position out of range", MLB_ERR_OUT_OF_RANGE);
        DeviceContext& c = Ctx(session->model->device);
        CheckCuda(cudaMemcpyAsync(session->hist + start_pos, tokens, sizeof(int),
                                  cudaMemcpyDeviceToDevice, c.stream),
                  "cudaMemcpyAsync(token)");
        SetState(session, c, start_pos, start_pos + 1);
        if (session->mega) {
            RunMega(session, c, start_pos, n_steps, start_pos + 1);
        } else {
            for (int i = 0; i < n_steps; ++i)
                CheckCuda(cudaGraphLaunch(session->exec, c.stream), "cudaGraphLaunch");
        }
        CheckCuda(cudaMemcpyAsync(tokens + 1, session->hist + start_pos + 1, size_t(n_steps) * 4,
                                  cudaMemcpyDeviceToDevice, c.stream),
                  "cudaMemcpyAsync(tokens)");
    });
}

int mlb_session_logits(mlb_session* session, const float** logits) {
    return Guard([&] {
        Require(session && logits, "mlb_session_logits", "null argument");
        *logits = session->logits;
    });
}

int mlb_session_gemv_path(mlb_session* session, int* path) {
    return Guard([&] {
        Require(session && path, "mlb_session_gemv_path", "null argument");
        *path = session->mega ? 2 : (session->model->r16 ? 1 : 0);
    });
}

int mlb_session_trace(mlb_session* session, unsigned long long* device_buffer, size_t entries) {
    return Guard([&] {
        Require(session != nullptr, "mlb_session_trace", "null session");
        Require(device_buffer != nullptr || entries == 0, "mlb_session_trace", "null buffer");
        session->mp.trace = device_buffer;
        session->mp.trace_cap = device_buffer ? entries : 0;
    });
}

int mlb_session_wait_limit(mlb_session* session, unsigned long long nanoseconds) {
    return Guard([&] {
        Require(session != nullptr, "mlb_session_wait_limit", "null session");
        Require(nanoseconds > 0, "mlb_session_wait_limit", "the wait limit must be positive");
        session->wait_ns = nanoseconds;
    });
}

int mlb_session_test_withhold_signal(mlb_session* session, int counter) {
    return Guard([&] {
        Require(session != nullptr, "mlb_session_test_withhold_signal", "null session");
        Require(counter >= -1, "mlb_session_test_withhold_signal", "counter must be -1 or a phase counter");
        session->withhold = counter;
    });
}

int mlb_session_use_persistent(mlb_session* session, int enable) {
    return Guard([&] {
        Require(session != nullptr, "mlb_session_use_persistent", "null session");
        Require(!enable || session->mega_ok, "mlb_session_use_persistent",
                "the persistent decode kernel does not support this model: " + session->mega_reason,
                MLB_ERR_UNSUPPORTED);
        DeviceContext& c = Ctx(session->model->device);
        CheckCuda(cudaStreamSynchronize(c.stream), "cudaStreamSynchronize");
        session->mega = enable != 0;
    });
}

int mlb_session_prefill_min(mlb_session* session, int min_tokens) {
    return Guard([&] {
        Require(session != nullptr, "mlb_session_prefill_min", "null argument");
        Require(min_tokens >= 0, "mlb_session_prefill_min", "min_tokens must not be negative");
        session->prefill_min = min_tokens;
    });
}

int mlb_session_kv_cache(mlb_session* session, float** key_cache, float** value_cache) {
    return Guard([&] {
        Require(session && key_cache && value_cache, "mlb_session_kv_cache", "null argument");
        *key_cache = session->kc;
        *value_cache = session->vc;
    });
}

}  // extern "C"
