// Decode-attention entry points (replace mini_llama include/cuda_attention.h:10-14).
#include <algorithm>
#include <cmath>
#include <cstring>
#include <mutex>
#include <string>

#include "attention.cuh"

namespace mlb {

int AttnChunks(int max_npos, int batch, int n_kv, int hgroups, int sm_count) {
    const long long base = 1LL * batch * n_kv * std::max(1, hgroups);  // CTAs per chunk
    const long long slots = 1LL * kAttnCtasPerSm * sm_count;            // resident CTAs
    // short contexts: 64-position chunks, halved while the grid is below
    // two waves of SMs (down to 16 positions)
    long long c = (max_npos + 63) / 64;
    while (c * 2 * base <= 2LL * sm_count && c * 2 * 16 <= max_npos) c *= 2;
    if (c * base <= slots) return static_cast<int>(std::max(1LL, c));
    // long contexts: each CTA loops over the tiles of its chunk, so the grid
    // needs only the resident CTAs; the first count from there whose waves are
    // at least 95 % full (else the fullest one tried)
    const long long c0 = std::max(1LL, slots / base);
    long long best = c0;
    double best_eff = 0.0;
    for (long long k = c0; k <= std::min(c, 8 * c0); ++k) {
        const long long ctas = k * base, waves = (ctas + slots - 1) / slots;
        const double eff = static_cast<double>(ctas) / static_cast<double>(waves * slots);
        if (eff > best_eff + 1e-9) {
            best = k;
            best_eff = eff;
        }
        if (eff >= 0.95) break;
    }
    return static_cast<int>(best);
}

namespace {

// out[b][h][d] = sum_c e^(m_c - M) o_c[d] / sum_c e^(m_c - M) l_c, one CTA of
// kAttnMergeThreads per (sequence, head, 32 dimensions): the chunk weights
// once into shared memory (kAttnMergeBatch at a time), then a warp per chunk
// slice, a lane per dimension, over the unnormalised outputs (eight rows in
// flight per thread); the slices summed at the end.
constexpr int kAttnMergeThreads = 256;
constexpr int kAttnMergeBatch = 1024;

__global__ void __launch_bounds__(kAttnMergeThreads) AttnMergeKernel(const float* part_ml, const float* part_o,
                                                                    int chunks, int hd, float* out) {
    constexpr int nsl = kAttnWarps;  // chunk slices
    __shared__ float wt[kAttnMergeBatch];
    __shared__ float sred[kAttnMergeThreads];
    __shared__ float sden[kAttnWarps];
    GridDepWait();
    GridDepLaunch();
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const size_t bh = blockIdx.x;  // b * n_heads + h
    const int d = blockIdx.y * 32 + lane;
    const bool dok = d < hd;
    const float* ml = part_ml + bh * chunks * 2;
    const float* po = part_o + bh * chunks * hd;
    float mx = -INFINITY;
    for (int c = tid; c < chunks; c += kAttnMergeThreads) mx = fmaxf(mx, ml[2 * c]);
    mx = WarpMax(mx);
    if (lane == 0) sden[warp] = mx;
    __syncthreads();
    mx = sden[0];
    for (int w = 1; w < kAttnWarps; ++w) mx = fmaxf(mx, sden[w]);
    float num = 0.0f, den = 0.0f;
    for (int c0 = 0; c0 < chunks; c0 += kAttnMergeBatch) {
        const int cn = min(kAttnMergeBatch, chunks - c0);
        __syncthreads();  // wt of the previous batch (and sden) fully read
        for (int c = tid; c < cn; c += kAttnMergeThreads) {
            const float mc = ml[2 * (c0 + c)];
            const float w = mc == -INFINITY ? 0.0f : expf(mc - mx);
            wt[c] = w;
            den = fmaf(w, ml[2 * (c0 + c) + 1], den);
        }
        __syncthreads();
        if (dok) {
            int c = warp;
            for (; c + 7 * nsl < cn; c += 8 * nsl) {
                float v[8];
#pragma unroll
                for (int k = 0; k < 8; ++k) v[k] = po[size_t(c0 + c + k * nsl) * hd + d];
#pragma unroll
                for (int k = 0; k < 8; ++k) num = fmaf(wt[c + k * nsl], v[k], num);
            }
            for (; c < cn; c += nsl) num = fmaf(wt[c], po[size_t(c0 + c) * hd + d], num);
        }
    }
    den = WarpSum(den);
    __syncthreads();
    if (lane == 0) sden[warp] = den;
    sred[tid] = num;
    __syncthreads();
    if (warp == 0 && dok) {
        float tden = 0.0f;
        for (int w = 0; w < kAttnWarps; ++w) tden += sden[w];
        float t = 0.0f;
        for (int sl = 0; sl < nsl; ++sl) t += sred[sl * 32 + lane];
        out[bh * hd + d] = tden > 0.0f ? t / tden : 0.0f;
    }
}

// A cache as a [rows][n_kv][hd] fp32 tensor map (no swizzle, no multicast)
// whose boxes are T rows of one KV head.  False when it cannot be encoded.
bool CacheMap(const float* base, int hd, int n_kv, long long rows, int T, CUtensorMap& map) {
    std::memset(&map, 0, sizeof(map));
    const PFN_cuTensorMapEncodeTiled_v12000 encode = TensorMapEncoder();
    if (!encode) return false;
    const cuuint64_t gdim[3] = {cuuint64_t(hd), cuuint64_t(n_kv), cuuint64_t(rows)};
    const cuuint64_t gstride[2] = {cuuint64_t(hd) * 4, cuuint64_t(n_kv) * hd * 4};
    const cuuint32_t box[3] = {cuuint32_t(hd), 1, cuuint32_t(T)};
    const cuuint32_t estride[3] = {1, 1, 1};
    return encode(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(base), gdim, gstride, box, estride,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int GM, bool TMA>
void LaunchAttnT(const AttnParams& p, int batch, cudaStream_t stream, bool pdl, const CUtensorMap& km,
                 const CUtensorMap& vm) {
    const size_t smem = AttnSmemBytes(p.hd, GM);
    static int configured[64] = {};
    int dev = 0;
    CheckCuda(cudaGetDevice(&dev), "cudaGetDevice");
    if (dev >= 64 || configured[dev] < static_cast<int>(smem)) {
        CheckCuda(cudaFuncSetAttribute(AttnSplitKernel<GM, TMA>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem)),
                  "cudaFuncSetAttribute(AttnSplitKernel)");
        if (dev < 64) configured[dev] = static_cast<int>(smem);
    }
    dim3 grid(p.n_kv * p.hgroups, p.chunks, batch);
    Launch("AttnSplitKernel", AttnSplitKernel<GM, TMA>, grid, dim3(kAttnThreads), smem, stream, pdl, p, km, vm);
}

template <bool TMA>
void LaunchAttnG(const AttnParams& p, int batch, cudaStream_t stream, bool pdl, const CUtensorMap& km,
                 const CUtensorMap& vm) {
    const int g = std::min(p.group, kAttnGmax);
    if (g <= 1) return LaunchAttnT<1, TMA>(p, batch, stream, pdl, km, vm);
    if (g <= 2) return LaunchAttnT<2, TMA>(p, batch, stream, pdl, km, vm);
    if (g <= 4) return LaunchAttnT<4, TMA>(p, batch, stream, pdl, km, vm);
    if (g <= 8) return LaunchAttnT<8, TMA>(p, batch, stream, pdl, km, vm);
    return LaunchAttnT<16, TMA>(p, batch, stream, pdl, km, vm);
}

}  // namespace

void LaunchAttention(const AttnParams& p, int batch, cudaStream_t stream, bool pdl) {
    if (p.hd < 1 || p.hd > 256) Fail(MLB_ERR_UNSUPPORTED, "attention: head_dim above 256 is not supported");
    AttnParams a = p;
    const AttnGeom G = AttnGeometry(p.hd);
    const size_t pstride = size_t(p.n_kv) * p.hd;
    // Tile copies as tensor-map boxes when rows are whole 16-byte pieces and
    // the caches are 16-byte aligned; the maps span the rows this launch can
    // reach: every sequence's layers up to `layer`.
    bool tma = (p.hd & 3) == 0 &&
               ((reinterpret_cast<uintptr_t>(p.kc) | reinterpret_cast<uintptr_t>(p.vc)) & 15) == 0 &&
               p.seq_stride % pstride == 0;
    CUtensorMap km, vm;
    std::memset(&km, 0, sizeof(km));
    std::memset(&vm, 0, sizeof(vm));
    if (tma) {
        const long long seq_rows = static_cast<long long>(p.seq_stride / pstride);
        const long long rows = (p.seq_stride ? (batch - 1) * seq_rows : 0) + (p.layer + 1LL) * p.max_seq_len;
        tma = seq_rows < (1LL << 30) && rows + G.T < (1LL << 31) && CacheMap(p.kc, p.hd, p.n_kv, rows, G.T, km) &&
              CacheMap(p.vc, p.hd, p.n_kv, rows, G.T, vm);
        a.seq_rows = static_cast<int>(seq_rows);
    }
    if (tma) LaunchAttnG<true>(a, batch, stream, pdl, km, vm);
    else LaunchAttnG<false>(a, batch, stream, pdl, km, vm);
}

void LaunchAttnMerge(const float* part_ml, const float* part_o, int chunks, int hd, float* out, int rows,
                     cudaStream_t stream) {
    AttnMergeKernel<<<dim3(rows, (hd + 31) / 32), kAttnMergeThreads, 0, stream>>>(part_ml, part_o, chunks, hd, out);
    CheckCuda(cudaGetLastError(), "AttnMergeKernel");
}

namespace {

void AttentionDecode(const char* caller, int device, int batch, const float* q, const float* kc,
                     const float* vc, int n_layers, int max_seq_len, int layer,
                     const int* positions, int pos, int n_heads, int n_kv_heads, int head_dim,
                     float* out) {
    Require(q && kc && vc && out, caller, "CUDA KV cache is empty");
    Require(batch > 0, caller, "batch must be positive");
    Require(n_layers > 0 && max_seq_len > 0, caller, "cache shape must be positive");
    Require(layer >= 0 && layer < n_layers, caller, "layer out of range", MLB_ERR_OUT_OF_RANGE);
    Require(pos >= 0 && pos < max_seq_len, caller, "position out of range", MLB_ERR_OUT_OF_RANGE);
    Require(n_heads > 0 && n_kv_heads > 0 && head_dim > 0, caller,
            "head counts and head_dim must be positive");
    Require(n_heads % n_kv_heads == 0, caller, "n_heads must be divisible by n_kv_heads");
    Require(head_dim <= 256, caller, "head_dim above 256 is not supported", MLB_ERR_UNSUPPORTED);
    DeviceContext& c = Ctx(device);
    AttnParams p = {};
    p.q = q;
    p.q_batch_stride = size_t(n_heads) * head_dim;
    p.kc = const_cast<float*>(kc);
    p.vc = const_cast<float*>(vc);
    p.seq_stride = size_t(n_layers) * max_seq_len * n_kv_heads * head_dim;
    p.layer = layer;
    p.max_seq_len = max_seq_len;
    p.n_heads = n_heads;
    p.n_kv = n_kv_heads;
    p.hd = head_dim;
    p.group = n_heads / n_kv_heads;
    p.hgroups = (p.group + kAttnGmax - 1) / kAttnGmax;
    p.scale = 1.0f / std::sqrt(static_cast<float>(head_dim));
    p.pos_dev = positions;
    p.pos_stride = positions ? 1 : 0;
    p.pos_host = pos;
    p.chunks = AttnChunks(pos + 1, batch, n_kv_heads, p.hgroups, c.sm_count);
    p.out = out;
    p.status = c.status;
    if (p.chunks > 1) {
        const size_t rows = size_t(batch) * n_heads * p.chunks;
        float* ws = static_cast<float*>(Workspace(c, rows * (head_dim + 2) * sizeof(float)));
        p.part_ml = ws;
        p.part_o = ws + rows * 2;
    }
    LaunchAttention(p, batch, c.stream, false);
    if (p.chunks > 1) {
        LaunchAttnMerge(p.part_ml, p.part_o, p.chunks, head_dim, out, batch * n_heads, c.stream);
    }
}

}  // namespace
}  // namespace mlb

using namespace mlb;

extern "C" {

int mlb_attention_decode(int device, const float* q, const float* key_cache,
                         const float* value_cache, int n_layers, int max_seq_len, int layer,
                         int pos, int n_heads, int n_kv_heads, int head_dim, float* out) {
    return Guard([&] {
        AttentionDecode("CudaAttentionDecodeDeviceInput", device, 1, q, key_cache, value_cache,
                        n_layers, max_seq_len, layer, nullptr, pos, n_heads, n_kv_heads,
                        head_dim, out);
    });
}

int mlb_attention_decode_batched(int device, int batch, const float* q, const float* key_cache,
                                 const float* value_cache, int n_layers, int max_seq_len,
                                 int layer, const int* positions, int max_pos, int n_heads,
                                 int n_kv_heads, int head_dim, float* out) {
    return Guard([&] {
        Require(positions != nullptr, "mlb_attention_decode_batched", "positions is null");
        AttentionDecode("mlb_attention_decode_batched", device, batch, q, key_cache, value_cache,
                        n_layers, max_seq_len, layer, positions, max_pos, n_heads, n_kv_heads,
                        head_dim, out);
    });
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Decode attention without any device allocation.
//
// Some callers cannot allocate device memory while they decode: an
// application whose other framework has already reserved all free device
// memory, or a host thread that must not take the allocator's locks or risk
// the implicit device synchronisation that freeing memory can cause.  For
// them this entry point keeps the split-K partials in one fixed array that is
// part of the library image (kNoAllocScratchFloats floats = 4 MiB on every
// device that loads the library, held until the process exits).
namespace {

constexpr size_t kNoAllocScratchFloats = size_t(1) << 20;  // 4 MiB
__device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchFloats];

std::mutex g_noalloc_mutex;
float* g_noalloc_ptr[64] = {};

// Device address of the array for `device` (which Ctx() has made current).
// Host code must not use g_noalloc_scratch itself: on the host that name is
// only a stand-in symbol, not device memory.
float* NoAllocScratch(int device) {
    std::lock_guard<std::mutex> lock(g_noalloc_mutex);
    Require(device >= 0 && device < 64, "mlb_attention_decode_noalloc", "device index above 63",
            MLB_ERR_UNSUPPORTED);
    if (g_noalloc_ptr[device] == nullptr) {
        void* ptr = nullptr;
        CheckCuda(cudaGetSymbolAddress(&ptr, g_noalloc_scratch), "cudaGetSymbolAddress");
        g_noalloc_ptr[device] = static_cast<float*>(ptr);
    }
    return g_noalloc_ptr[device];
}

}  // namespace

extern "C" int mlb_attention_decode_noalloc(int device, const float* q, const float* key_cache,
                                            const float* value_cache, int n_layers,
                                            int max_seq_len, int layer, int pos, int n_heads,
                                            int n_kv_heads, int head_dim, float* out) {
    return Guard([&] {
        const char* caller = "mlb_attention_decode_noalloc";
        Require(q && key_cache && value_cache && out, caller, "CUDA KV cache is empty");
        Require(n_layers > 0 && max_seq_len > 0, caller, "cache shape must be positive");
        Require(layer >= 0 && layer < n_layers, caller, "layer out of range", MLB_ERR_OUT_OF_RANGE);
        Require(pos >= 0 && pos < max_seq_len, caller, "position out of range",
                MLB_ERR_OUT_OF_RANGE);
        Require(n_heads > 0 && n_kv_heads > 0 && head_dim > 0, caller,
                "head counts and head_dim must be positive");
        Require(n_heads % n_kv_heads == 0, caller, "n_heads must be divisible by n_kv_heads");
        Require(head_dim <= 256, caller, "head_dim above 256 is not supported",
                MLB_ERR_UNSUPPORTED);
        DeviceContext& c = Ctx(device);
        AttnParams p = {};
        p.q = q;
        p.q_batch_stride = size_t(n_heads) * head_dim;
        p.kc = const_cast<float*>(key_cache);
        p.vc = const_cast<float*>(value_cache);
        p.seq_stride = size_t(n_layers) * max_seq_len * n_kv_heads * head_dim;
        p.layer = layer;
        p.max_seq_len = max_seq_len;
        p.n_heads = n_heads;
        p.n_kv = n_kv_heads;
        p.hd = head_dim;
        p.group = n_heads / n_kv_heads;
        p.hgroups = (p.group + kAttnGmax - 1) / kAttnGmax;
        p.scale = 1.0f / std::sqrt(static_cast<float>(head_dim));
        p.pos_host = pos;
        p.chunks = AttnChunks(pos + 1, 1, n_kv_heads, p.hgroups, c.sm_count);
        p.out = out;
        p.status = c.status;
        if (p.chunks > 1) {
            const size_t rows = size_t(n_heads) * p.chunks;
            const size_t need = rows * (head_dim + 2);
            Require(need <= kNoAllocScratchFloats, caller,
                    "attention needs " + std::to_string(need * 4) +
                        " bytes of split-K scratch; the fixed array holds " +
                        std::to_string(kNoAllocScratchFloats * 4) +
                        " (use mlb_attention_decode for this shape)",
                    MLB_ERR_UNSUPPORTED);
            // Every (head, chunk) slot the merge reads is written by this
            // call's attention kernel first, so nothing needs clearing.
            float* ws = NoAllocScratch(device);
            p.part_ml = ws;
            p.part_o = ws + rows * 2;
        }
        LaunchAttention(p, 1, c.stream, false);
        if (p.chunks > 1) {
            LaunchAttnMerge(p.part_ml, p.part_o, p.chunks, head_dim, out, n_heads, c.stream);
        }
    });
}
