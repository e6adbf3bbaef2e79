// Batched decode driver (include/mlb.h, mlb_batch_*): B independent sequences
// decoded in lockstep, optionally tensor-parallel over NCCL.  Per sequence it
// computes what ForwardToken does (src/forward.cpp:292-333, :642-666) followed
// by the greedy GetArgMax (src/ops.cpp:199-212); the reference itself has no
// batched path (ForwardBatch, src/forward.cpp:668-684, loops one token of one
// sequence at a time).
//
// One step, captured once as a CUDA graph (position and prompt length in
// device memory):
//   x[b] = embedding[hist[b][pos]]
//   per layer:
//     xn = RMSNorm(x)                                    (rows of `batch`)
//     q, k, v = xn . [wq|wk|wv]^T + bias                 this rank's heads
//     RoPE + KV write + split-K attention (+ merge)      this rank's KV heads
//     all-gather attention rows -> x_mid = x + attn . wo^T   (wo rows sliced,
//                                                        all-gathered, added)
//     xn = RMSNorm(x_mid)
//     s = silu(xn . w_gate^T) * (xn . w_up^T)            hidden rows sliced
//     all-gather s -> x = x_mid + s . w_down^T           (rows sliced, gathered)
//   logits = RMSNorm(x) . lm_head^T                      vocabulary sliced
//   per-rank first arg-max, all-gathered and merged -> hist[b][pos + 1]
//   pos += 1
// A rank's slices are contiguous row ranges of the model's GGUF weights (a
// pointer offset: no copy).  NCCL all-gathers concatenate rank-major
// ([rank][b][slice]); GatherKernel reorders them into rows.
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <string>
#include <vector>

#include "attention.cuh"
#include "model.cuh"
#include "qgemv.cuh"
#include "rows.cuh"

struct mlb_batch {
    mlb_model* model = nullptr;
    int batch = 0;
    int rank = 0, size = 1;
    ncclComm_t comm = nullptr;
    // this rank's slices (half-open)
    int h0 = 0, h1 = 0, k0 = 0, k1 = 0, d0 = 0, d1 = 0, f0 = 0, f1 = 0, v0 = 0, v1 = 0;
    int chunks = 1;
    // device buffers
    float *x = nullptr, *xmid = nullptr, *xn = nullptr;
    float *q = nullptr, *k = nullptr, *v = nullptr;
    float *attn_l = nullptr, *attn = nullptr;
    float *o_l = nullptr;
    float *gate = nullptr, *up = nullptr, *sw_l = nullptr, *sw = nullptr;
    float *d_l = nullptr, *logits = nullptr;
    float *gbuf = nullptr;  // all-gather receive buffer
    float *part_ml = nullptr, *part_o = nullptr;
    float *kc = nullptr, *vc = nullptr;
    int* hist = nullptr;   // [batch][max_seq_len + 1]
    int* state = nullptr;  // [0] pos, [1] gen_from, [2] status
    unsigned long long* pairs = nullptr;  // per-row (value, index) of this rank, then all ranks'
    void* tc_ws = nullptr;
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    cudaEvent_t ev[3] = {nullptr, nullptr, nullptr};
    std::vector<void*> allocations;
};

namespace mlb {
namespace {

constexpr int kRowThreads = 256;

// NCCL is opened on first use, not linked: a process that imports PyTorch
// after loading this library must still resolve PyTorch's own NCCL, and most
// uses of the library never need a collective.  An NCCL already loaded in
// the process (PyTorch's) is reused; otherwise the system's libnccl.so.2.
struct NcclApi {
    ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
    ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
    const char* (*error_string)(ncclResult_t) = nullptr;
};

const NcclApi& Nccl() {
    static NcclApi api;
    static bool loaded = false;
    if (!loaded) {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
        if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) {
            const char* e = dlerror();
            Fail(MLB_ERR_UNSUPPORTED, std::string("NCCL: libnccl.so.2 could not be loaded: ") + (e ? e : "unknown"));
        }
        auto sym = [&](const char* name) {
            void* f = dlsym(h, name);
            Require(f != nullptr, "NCCL", std::string("symbol missing: ") + name, MLB_ERR_UNSUPPORTED);
            return f;
        };
        api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(sym("ncclGetUniqueId"));
        api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(sym("ncclCommInitRank"));
        api.all_gather = reinterpret_cast<decltype(api.all_gather)>(sym("ncclAllGather"));
        api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(sym("ncclCommDestroy"));
        api.error_string = reinterpret_cast<decltype(api.error_string)>(sym("ncclGetErrorString"));
        loaded = true;
    }
    return api;
}

void CheckNccl(ncclResult_t r, const char* what) {
    if (r != ncclSuccess)
        Fail(MLB_ERR_CUDA, std::string(what) + ": " + Nccl().error_string(r));
}

// x[b] = table[hist[b][pos]]; an out-of-range token records the status and
// leaves zeros.
__global__ void BatchEmbedKernel(const float* table, int vocab, int dim, const int* hist, int hist_stride,
                                 const int* state, float* x, int* status) {
    GridDepWait();
    GridDepLaunch();
    const int b = blockIdx.x;
    const int tok = hist[size_t(b) * hist_stride + state[0]];
    const bool ok = tok >= 0 && tok < vocab;
    if (!ok && threadIdx.x == 0) atomicExch(status, MLB_ERR_OUT_OF_RANGE);
    const float* row = table + size_t(ok ? tok : 0) * dim;
    for (int i = threadIdx.x; i < dim; i += blockDim.x) x[size_t(b) * dim + i] = ok ? row[i] : 0.0f;
}

// dst[b][r * n + j] = src[r][b][j] (+ add[b][r * n + j]): all-gathered slices
// back into rows.
__global__ void GatherKernel(const float* src, int ranks, int batch, int n, const float* add, float* dst) {
    GridDepWait();
    GridDepLaunch();
    const size_t row = size_t(ranks) * n, total = size_t(batch) * row;
    for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < total; i += size_t(gridDim.x) * blockDim.x) {
        const size_t b = i / row, c = i - b * row;
        const size_t r = c / n, j = c - r * n;
        const float v = src[(r * batch + b) * n + j];
        dst[i] = add ? add[i] + v : v;
    }
}

__device__ __forceinline__ unsigned long long PackPair(float v, int i) {
    return (static_cast<unsigned long long>(__float_as_uint(v)) << 32) | static_cast<unsigned>(i);
}
__device__ __forceinline__ float PairVal(unsigned long long p) { return __uint_as_float(unsigned(p >> 32)); }
__device__ __forceinline__ int PairIdx(unsigned long long p) { return static_cast<int>(unsigned(p)); }

// First maximum: larger value, or equal value at a smaller index.
__device__ __forceinline__ bool Better(float v, int i, float bv, int bi) {
    return v > bv || (v == bv && i < bi);
}

// Per row b: the first maximum of logits[b][0..n) as (value, col0 + index).
__global__ void RowArgmaxKernel(const float* logits, int n, int col0, unsigned long long* pairs) {
    __shared__ float sv[kRowThreads];
    __shared__ int si[kRowThreads];
    GridDepWait();
    GridDepLaunch();
    const float* row = logits + size_t(blockIdx.x) * n;
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float v = row[i];
        if (Better(v, col0 + i, bv, bi)) {
            bv = v;
            bi = col0 + i;
        }
    }
    sv[threadIdx.x] = bv;
    si[threadIdx.x] = bi;
    __syncthreads();
    for (int o = blockDim.x / 2; o > 0; o >>= 1) {
        if (threadIdx.x < o && Better(sv[threadIdx.x + o], si[threadIdx.x + o], sv[threadIdx.x], si[threadIdx.x])) {
            sv[threadIdx.x] = sv[threadIdx.x + o];
            si[threadIdx.x] = si[threadIdx.x + o];
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) pairs[blockIdx.x] = PackPair(sv[0], si[0]);
}

// Merges the ranks' pairs ([rank][batch]) per row, appends the token to the
// row's history when generating, and advances the position.  One CTA.
__global__ void MergeArgmaxKernel(const unsigned long long* pairs, int ranks, int batch, int* hist, int hist_stride,
                                  int max_seq_len, int* state) {
    GridDepWait();
    GridDepLaunch();
    const int pos = state[0], gen_from = state[1];
    for (int b = threadIdx.x; b < batch; b += blockDim.x) {
        float bv = -INFINITY;
        int bi = 0x7fffffff;
        for (int r = 0; r < ranks; ++r) {
            const unsigned long long p = pairs[size_t(r) * batch + b];
            if (Better(PairVal(p), PairIdx(p), bv, bi)) {
                bv = PairVal(p);
                bi = PairIdx(p);
            }
        }
        const int tok = bi == 0x7fffffff ? 0 : bi;
        if (pos + 1 >= gen_from && pos + 1 <= max_seq_len) hist[size_t(b) * hist_stride + pos + 1] = tok;
    }
    __syncthreads();
    if (threadIdx.x == 0) state[0] = pos + 1;
}

int GridFor(size_t n, int threads, int sms) {
    return static_cast<int>(std::max<size_t>(1, std::min<size_t>((n + threads - 1) / threads, size_t(4) * sms)));
}

void Shard(const mlb_model_config& cf, int rank, int size, int* r) {
    const char* w = "mlb_batch_shard";
    Require(size >= 1 && rank >= 0 && rank < size, w, "tp_rank must lie in [0, tp_size)");
    Require(cf.n_kv_heads % size == 0, w,
            "tp_size must divide n_kv_heads (attention is split by KV-head group)", MLB_ERR_UNSUPPORTED);
    Require(cf.dim % size == 0 && cf.hidden_dim % size == 0 && cf.vocab_size % size == 0, w,
            "tp_size must divide dim, hidden_dim and vocab_size", MLB_ERR_UNSUPPORTED);
    const int nkv = cf.n_kv_heads / size, nh = cf.n_heads / size;
    const int dl = cf.dim / size, fl = cf.hidden_dim / size, vl = cf.vocab_size / size;
    const int v[10] = {rank * nh, (rank + 1) * nh, rank * nkv, (rank + 1) * nkv, rank * dl,
                       (rank + 1) * dl, rank * fl, (rank + 1) * fl, rank * vl, (rank + 1) * vl};
    std::memcpy(r, v, sizeof(v));
}

template <typename T>
T* Alloc(mlb_batch* b, size_t count) {
    void* p = nullptr;
    CheckCuda(cudaMalloc(&p, std::max<size_t>(count, 1) * sizeof(T)), "cudaMalloc(batch)");
    b->allocations.push_back(p);
    return static_cast<T*>(p);
}

// Rows [r0, r1) of a GGUF-block weight with `cols` columns.
const uint8_t* Rows(const mlb_model* m, int l, int kind, int r0, int cols) {
    const int nb = (cols + 31) / 32;
    return static_cast<const uint8_t*>(m->Ptr(m->Get(l, kind))) + size_t(r0) * nb * BlockBytes(m->cfg.weight_type);
}

void CaptureBatchStep(mlb_batch* s, DeviceContext& c) {
    mlb_model* m = s->model;
    const mlb_model_config& cf = m->cfg;
    const int qt = cf.weight_type, B = s->batch, G = s->size, hd = cf.head_dim;
    const int nh = s->h1 - s->h0, nkv = s->k1 - s->k0;
    const int qd_l = nh * hd, kd_l = nkv * hd, qd = cf.n_heads * hd;
    const int dl = s->d1 - s->d0, fl = s->f1 - s->f0, vl = s->v1 - s->v0;
    const int hist_stride = cf.max_seq_len + 1;
    int* status = s->state + 2;
    cudaStream_t st = c.stream;
    auto F = [&](int l, int kind) { return static_cast<const float*>(m->Ptr(m->Get(l, kind))); };
    // same_x: x is the previous linear's input, unchanged (its x images are reused)
    auto linear = [&](const float* x, const uint8_t* w, int K, int N, const float* bias, float* y,
                      bool same_x = false) {
        LinearRows(c, qt, x, w, B, K, N, bias, y, s->tc_ws, same_x);
    };
    // rank-sliced rows -> whole rows on every rank (plus `add` when given)
    auto gather = [&](const float* local, int n_local, const float* add, float* dst) {
        const float* src = local;
        if (G > 1) {
            CheckNccl(Nccl().all_gather(local, s->gbuf, size_t(B) * n_local, ncclFloat, s->comm, st), "ncclAllGather");
            src = s->gbuf;
        }
        const size_t n = size_t(B) * G * n_local;
        Launch("GatherKernel", GatherKernel, dim3(GridFor(n, 256, c.sm_count)), dim3(256), 0, st, true, src, G, B,
               n_local, add, dst);
    };

    CheckCuda(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal), "cudaStreamBeginCapture");
    try {
        Launch("BatchEmbedKernel", BatchEmbedKernel, dim3(B), dim3(kRowThreads), 0, st, true,
               static_cast<const float*>(m->Ptr(m->global[MLB_W_EMBEDDING])), cf.vocab_size, cf.dim,
               const_cast<const int*>(s->hist), hist_stride, const_cast<const int*>(s->state), s->x, status);
        for (int l = 0; l < cf.n_layers; ++l) {
            // 1. RMSNorm, this rank's q / k / v rows (+ bias)
            Launch("RowsRmsNormKernel", RowsRmsNormKernel, dim3(B), dim3(kRowThreads), 0, st, true,
                   const_cast<const float*>(s->x), F(l, MLB_W_ATTN_NORM), s->xn, cf.dim, cf.rms_norm_eps);
            const float* bq = cf.qkv_bias ? F(l, MLB_W_BQ) + size_t(s->h0) * hd : nullptr;
            const float* bk = cf.qkv_bias ? F(l, MLB_W_BK) + size_t(s->k0) * hd : nullptr;
            const float* bv = cf.qkv_bias ? F(l, MLB_W_BV) + size_t(s->k0) * hd : nullptr;
            linear(s->xn, Rows(m, l, MLB_W_WQ, s->h0 * hd, cf.dim), cf.dim, qd_l, bq, s->q);
            linear(s->xn, Rows(m, l, MLB_W_WK, s->k0 * hd, cf.dim), cf.dim, kd_l, bk, s->k, true);
            linear(s->xn, Rows(m, l, MLB_W_WV, s->k0 * hd, cf.dim), cf.dim, kd_l, bv, s->v, true);
            // 2. RoPE + KV write + split-K attention over this rank's KV heads
            {
                AttnParams a = {};
                a.q = s->q;
                a.q_batch_stride = size_t(qd_l);
                a.kc = s->kc;
                a.vc = s->vc;
                a.seq_stride = size_t(cf.n_layers) * cf.max_seq_len * kd_l;
                a.layer = l;
                a.max_seq_len = cf.max_seq_len;
                a.n_heads = nh;
                a.n_kv = nkv;
                a.hd = hd;
                a.group = cf.n_heads / cf.n_kv_heads;
                a.hgroups = (a.group + kAttnGmax - 1) / kAttnGmax;
                a.chunks = s->chunks;
                a.scale = 1.0f / std::sqrt(static_cast<float>(hd));
                a.pos_dev = s->state;
                a.pos_stride = 0;
                a.out = s->attn_l;
                a.part_ml = s->part_ml;
                a.part_o = s->part_o;
                a.fused_rope = 1;
                a.kv_new = s->k;
                a.v_new = s->v;
                a.kv_batch_stride = size_t(kd_l);
                a.rope_cos = m->rope_cos;
                a.rope_sin = m->rope_sin;
                a.neox = cf.rope_type == MLB_ROPE_NEOX;
                a.status = status;
                LaunchAttention(a, B, st, true);
                if (s->chunks > 1) {
                    LaunchAttnMerge(s->part_ml, s->part_o, s->chunks, hd, s->attn_l, B * nh, st);
                }
            }
            // 3. whole attention rows -> this rank's wo rows -> x_mid = x + all rows
            if (G > 1) gather(s->attn_l, qd_l, nullptr, s->attn);
            linear(s->attn, Rows(m, l, MLB_W_WO, s->d0, qd), qd, dl, nullptr, s->o_l);
            gather(s->o_l, dl, s->x, s->xmid);
            // 4. RMSNorm, this rank's gate / up rows, SwiGLU
            Launch("RowsRmsNormKernel", RowsRmsNormKernel, dim3(B), dim3(kRowThreads), 0, st, true,
                   const_cast<const float*>(s->xmid), F(l, MLB_W_FFN_NORM), s->xn, cf.dim, cf.rms_norm_eps);
            linear(s->xn, Rows(m, l, MLB_W_GATE, s->f0, cf.dim), cf.dim, fl, nullptr, s->gate);
            linear(s->xn, Rows(m, l, MLB_W_UP, s->f0, cf.dim), cf.dim, fl, nullptr, s->up, true);
            Launch("RowsSwigluKernel", RowsSwigluKernel, dim3(GridFor(size_t(B) * fl, 256, c.sm_count)), dim3(256), 0, st,
                   true, const_cast<const float*>(s->gate), const_cast<const float*>(s->up), size_t(B) * fl,
                   s->sw_l);
            // 5. whole SwiGLU rows -> this rank's down rows -> x = x_mid + all rows
            if (G > 1) gather(s->sw_l, fl, nullptr, s->sw);
            linear(s->sw, Rows(m, l, MLB_W_DOWN, s->d0, cf.hidden_dim), cf.hidden_dim, dl, nullptr, s->d_l);
            gather(s->d_l, dl, s->xmid, s->x);
        }
        // final RMSNorm, this rank's vocabulary rows, arg-max merged over ranks
        Launch("RowsRmsNormKernel", RowsRmsNormKernel, dim3(B), dim3(kRowThreads), 0, st, true,
               const_cast<const float*>(s->x), static_cast<const float*>(m->Ptr(m->global[MLB_W_FINAL_NORM])), s->xn,
               cf.dim, cf.rms_norm_eps);
        linear(s->xn, Rows(m, -1, MLB_W_LM_HEAD, s->v0, cf.dim), cf.dim, vl, nullptr, s->logits);
        Launch("RowArgmaxKernel", RowArgmaxKernel, dim3(B), dim3(kRowThreads), 0, st, true,
               const_cast<const float*>(s->logits), vl, s->v0, s->pairs);
        const unsigned long long* all = s->pairs;
        if (G > 1) {
            CheckNccl(Nccl().all_gather(s->pairs, s->pairs + B, size_t(B), ncclUint64, s->comm, st), "ncclAllGather");
            all = s->pairs + B;
        }
        Launch("MergeArgmaxKernel", MergeArgmaxKernel, dim3(1), dim3(std::min(1024, std::max(32, B))), 0, st, true,
               all, G, B, s->hist, hist_stride, cf.max_seq_len, s->state);
    } catch (...) {
        cudaGraph_t g = nullptr;
        cudaStreamEndCapture(st, &g);
        if (g) cudaGraphDestroy(g);
        throw;
    }
    CheckCuda(cudaStreamEndCapture(st, &s->graph), "cudaStreamEndCapture");
    CheckCuda(cudaGraphInstantiate(&s->exec, s->graph, 0), "cudaGraphInstantiate");
}

void DestroyBatch(mlb_batch* b) {
    if (!b) return;
    if (b->exec) cudaGraphExecDestroy(b->exec);
    if (b->graph) cudaGraphDestroy(b->graph);
    for (cudaEvent_t e : b->ev)
        if (e) cudaEventDestroy(e);
    if (b->comm) Nccl().comm_destroy(b->comm);
    for (void* p : b->allocations) cudaFree(p);
    delete b;
}

}  // namespace
}  // namespace mlb

using namespace mlb;

extern "C" {

int mlb_nccl_unique_id(void* id) {
    return Guard([&] {
        Require(id != nullptr, "mlb_nccl_unique_id", "null argument");
        static_assert(sizeof(ncclUniqueId) == MLB_NCCL_ID_BYTES, "NCCL id size");
        int n = 0;
        Require(cudaGetDeviceCount(&n) == cudaSuccess && n > 0, "mlb_nccl_unique_id", "no CUDA device",
                MLB_ERR_UNSUPPORTED);
        ncclUniqueId u;
        CheckNccl(Nccl().get_unique_id(&u), "ncclGetUniqueId");
        std::memcpy(id, &u, sizeof(u));
    });
}

int mlb_batch_shard(const mlb_model_config* config, int tp_rank, int tp_size, int* ranges) {
    return Guard([&] {
        Require(config && ranges, "mlb_batch_shard", "null argument");
        Shard(*config, tp_rank, tp_size, ranges);
    });
}

int mlb_batch_create(mlb_model* model, int batch, int tp_rank, int tp_size, const void* nccl_id,
                     mlb_batch** out) {
    return Guard([&] {
        const char* w = "mlb_batch_create";
        Require(model && out, w, "null argument");
        *out = nullptr;
        Require(batch >= 1 && batch <= 1024, w, "batch must lie in [1, 1024]");
        Require(tp_size == 1 || nccl_id != nullptr, w, "tensor parallelism needs an NCCL id");
        const mlb_model_config& cf = model->cfg;
        int r[10];
        Shard(cf, tp_rank, tp_size, r);
        Require(cf.head_dim <= 256 && cf.head_dim % 2 == 0, w, "head_dim must be even and at most 256",
                MLB_ERR_UNSUPPORTED);
        DeviceContext& c = Ctx(model->device);
        mlb_batch* b = new mlb_batch();
        try {
            b->model = model;
            b->batch = batch;
            b->rank = tp_rank;
            b->size = tp_size;
            b->h0 = r[0], b->h1 = r[1], b->k0 = r[2], b->k1 = r[3], b->d0 = r[4], b->d1 = r[5];
            b->f0 = r[6], b->f1 = r[7], b->v0 = r[8], b->v1 = r[9];
            const int hd = cf.head_dim, nh = b->h1 - b->h0, nkv = b->k1 - b->k0;
            const size_t B = size_t(batch);
            const int dl = b->d1 - b->d0, fl = b->f1 - b->f0, vl = b->v1 - b->v0;
            b->x = Alloc<float>(b, B * cf.dim);
            b->xmid = Alloc<float>(b, B * cf.dim);
            b->xn = Alloc<float>(b, B * cf.dim);
            b->q = Alloc<float>(b, B * nh * hd);
            b->k = Alloc<float>(b, B * nkv * hd);
            b->v = Alloc<float>(b, B * nkv * hd);
            b->attn_l = Alloc<float>(b, B * nh * hd);
            b->attn = tp_size > 1 ? Alloc<float>(b, B * cf.n_heads * hd) : b->attn_l;
            b->o_l = Alloc<float>(b, B * dl);
            b->gate = Alloc<float>(b, B * fl);
            b->up = Alloc<float>(b, B * fl);
            b->sw_l = Alloc<float>(b, B * fl);
            b->sw = tp_size > 1 ? Alloc<float>(b, B * cf.hidden_dim) : b->sw_l;
            b->d_l = Alloc<float>(b, B * dl);
            b->logits = Alloc<float>(b, B * vl);
            const size_t gmax = std::max({size_t(cf.n_heads) * hd, size_t(cf.dim), size_t(cf.hidden_dim)});
            b->gbuf = tp_size > 1 ? Alloc<float>(b, B * gmax) : nullptr;
            const int hgroups = (cf.n_heads / cf.n_kv_heads + kAttnGmax - 1) / kAttnGmax;
            b->chunks = AttnChunks(cf.max_seq_len, batch, nkv, hgroups, c.sm_count);
            b->part_ml = Alloc<float>(b, B * nh * b->chunks * 2);
            b->part_o = Alloc<float>(b, B * nh * b->chunks * hd);
            const size_t cache = B * cf.n_layers * size_t(cf.max_seq_len) * nkv * hd;
            b->kc = Alloc<float>(b, cache);
            b->vc = Alloc<float>(b, cache);
            CheckCuda(cudaMemset(b->kc, 0, cache * 4), "cudaMemset(kc)");
            CheckCuda(cudaMemset(b->vc, 0, cache * 4), "cudaMemset(vc)");
            b->hist = Alloc<int>(b, B * (cf.max_seq_len + 1));
            CheckCuda(cudaMemset(b->hist, 0, B * (cf.max_seq_len + 1) * 4), "cudaMemset(hist)");
            b->state = Alloc<int>(b, 4);
            CheckCuda(cudaMemset(b->state, 0, 16), "cudaMemset(state)");
            b->pairs = Alloc<unsigned long long>(b, B * (tp_size + 1));
            if (batch >= kTcMinRows) {
                const int K[6] = {cf.dim, cf.dim, cf.n_heads * hd, cf.dim, cf.hidden_dim, cf.dim};
                const int N[6] = {nh * hd, nkv * hd, dl, fl, dl, vl};
                size_t ws = 0;
                for (int i = 0; i < 6; ++i) ws = std::max(ws, TcWorkspaceBytes(batch, K[i], N[i], c.sm_count));
                b->tc_ws = Alloc<uint8_t>(b, ws);
            }
            for (cudaEvent_t& e : b->ev) CheckCuda(cudaEventCreate(&e), "cudaEventCreate");
            if (tp_size > 1) {
                ncclUniqueId id;
                std::memcpy(&id, nccl_id, sizeof(id));
                CheckNccl(Nccl().comm_init_rank(&b->comm, tp_size, id, tp_rank), "ncclCommInitRank");
            }
            CheckCuda(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
            CaptureBatchStep(b, c);
        } catch (...) {
            DestroyBatch(b);
            throw;
        }
        *out = b;
    });
}

int mlb_batch_destroy(mlb_batch* batch) {
    return Guard([&] {
        if (!batch) return;
        Ctx(batch->model->device);
        cudaStreamSynchronize(Ctx(batch->model->device).stream);
        DestroyBatch(batch);
    });
}

int mlb_batch_generate(mlb_batch* b, const int* prompts, int n_prompt, int n_new, int* out_tokens,
                       float* prefill_ms, float* decode_ms) {
    return Guard([&] {
        const char* w = "mlb_batch_generate";
        Require(b && prompts && out_tokens, w, "null argument");
        Require(n_prompt > 0 && n_new > 0, w, "prompt and generation must be non-empty");
        const mlb_model_config& cf = b->model->cfg;
        Require(n_prompt + n_new - 1 <= cf.max_seq_len, w, "position out of range", MLB_ERR_OUT_OF_RANGE);
        for (size_t i = 0; i < size_t(b->batch) * n_prompt; ++i)
            Require(prompts[i] >= 0 && prompts[i] < cf.vocab_size, w, "token id out of range",
                    MLB_ERR_OUT_OF_RANGE);
        DeviceContext& c = Ctx(b->model->device);
        const size_t hs = size_t(cf.max_seq_len + 1) * 4;
        CheckCuda(cudaMemcpy2DAsync(b->hist, hs, prompts, size_t(n_prompt) * 4, size_t(n_prompt) * 4, b->batch,
                                    cudaMemcpyHostToDevice, c.stream),
                  "cudaMemcpy2DAsync(prompts)");
        int* h = static_cast<int*>(PinnedStaging(c, 16));
        CheckCuda(cudaStreamSynchronize(c.stream), "cudaStreamSynchronize");
        h[0] = 0;
        h[1] = n_prompt;
        h[2] = 0;
        CheckCuda(cudaMemcpyAsync(b->state, h, 3 * sizeof(int), cudaMemcpyHostToDevice, c.stream),
                  "cudaMemcpyAsync(state)");
        CheckCuda(cudaEventRecord(b->ev[0], c.stream), "cudaEventRecord");
        for (int i = 0; i < n_prompt; ++i) CheckCuda(cudaGraphLaunch(b->exec, c.stream), "cudaGraphLaunch");
        CheckCuda(cudaEventRecord(b->ev[1], c.stream), "cudaEventRecord");
        for (int i = 1; i < n_new; ++i) CheckCuda(cudaGraphLaunch(b->exec, c.stream), "cudaGraphLaunch");
        CheckCuda(cudaEventRecord(b->ev[2], c.stream), "cudaEventRecord");
        CheckCuda(cudaMemcpy2DAsync(out_tokens, size_t(n_new) * 4, b->hist + n_prompt, hs, size_t(n_new) * 4,
                                    b->batch, cudaMemcpyDeviceToHost, c.stream),
                  "cudaMemcpy2DAsync(tokens)");
        CheckCuda(cudaMemcpyAsync(h, b->state, 3 * sizeof(int), cudaMemcpyDeviceToHost, c.stream),
                  "cudaMemcpyAsync(state)");
        CheckCuda(cudaStreamSynchronize(c.stream), "cudaStreamSynchronize");
        if (h[2] != 0) Fail(h[2], "mlb_batch_generate: a token id was out of range");
        int st = 0;
        CheckCuda(cudaMemcpy(&st, c.status, sizeof(int), cudaMemcpyDeviceToHost), "cudaMemcpy(status)");
        if (st != 0) {
            CheckCuda(cudaMemset(c.status, 0, sizeof(int)), "cudaMemset(status)");
            Fail(st, "mlb_batch_generate: a bounded device wait expired");
        }
        float t = 0.0f;
        if (prefill_ms) {
            CheckCuda(cudaEventElapsedTime(&t, b->ev[0], b->ev[1]), "cudaEventElapsedTime");
            *prefill_ms = t;
        }
        if (decode_ms) {
            CheckCuda(cudaEventElapsedTime(&t, b->ev[1], b->ev[2]), "cudaEventElapsedTime");
            *decode_ms = t;
        }
    });
}

int mlb_batch_logits(mlb_batch* b, const float** logits, int* cols, int* col0) {
    return Guard([&] {
        Require(b && logits && cols && col0, "mlb_batch_logits", "null argument");
        *logits = b->logits;
        *cols = b->v1 - b->v0;
        *col0 = b->v0;
    });
}

}  // extern "C"
