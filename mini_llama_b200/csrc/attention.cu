// Decode-attention entry points (replace mini_llama include/cuda_attention.h:10-14).
#include <algorithm>
#include <cmath>
#include <mutex>
#include <string>

#include "attention.cuh"

namespace mlb {

int AttnChunks(int max_npos, int batch, int n_kv, int hgroups, int sm_count) {
    // at most kAttnChunk positions per CTA (K and V of a chunk fit in shared
    // memory); more chunks while the grid is below about two waves of SMs
    (void)hgroups;
    long long c = (max_npos + kAttnChunk - 1) / kAttnChunk;
    long long base = 1LL * batch * n_kv;
    while (c * 2 * base <= 2LL * sm_count && c * 2 * 16 <= max_npos) c *= 2;
    return static_cast<int>(std::max(1LL, c));
}

template <int DPL>
void LaunchAttnT(const AttnParams& p, int batch, cudaStream_t stream, bool pdl) {
    const size_t smem = AttnSmemBytes(p.hd);
    static int configured[64] = {};
    int dev = 0;
    CheckCuda(cudaGetDevice(&dev), "cudaGetDevice");
    if (dev >= 64 || configured[dev] < static_cast<int>(smem)) {
        CheckCuda(cudaFuncSetAttribute(AttnSplitKernel<DPL>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem)),
                  "cudaFuncSetAttribute(AttnSplitKernel)");
        if (dev < 64) configured[dev] = static_cast<int>(smem);
    }
    dim3 grid(p.n_kv * p.hgroups, p.chunks, batch);
    Launch("AttnSplitKernel", AttnSplitKernel<DPL>, grid, dim3(kAttnThreads), smem, stream, pdl, p);
}

void LaunchAttention(const AttnParams& p, int batch, cudaStream_t stream, bool pdl) {
    const int dpl = (p.hd + 31) / 32;
    if (dpl <= 1) return LaunchAttnT<1>(p, batch, stream, pdl);
    if (dpl <= 2) return LaunchAttnT<2>(p, batch, stream, pdl);
    if (dpl <= 4) return LaunchAttnT<4>(p, batch, stream, pdl);
    if (dpl <= 8) return LaunchAttnT<8>(p, batch, stream, pdl);
    Fail(MLB_ERR_UNSUPPORTED, "attention: head_dim above 256 is not supported");
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
    if (p.chunks > 1) {
        const size_t rows = size_t(batch) * n_heads * p.chunks;
        float* ws = static_cast<float*>(Workspace(c, rows * (head_dim + 2) * sizeof(float)));
        p.part_ml = ws;
        p.part_o = ws + rows * 2;
    }
    LaunchAttention(p, batch, c.stream, false);
    if (p.chunks > 1) {
        AttnMergeKernel<<<batch * n_heads, 128, 0, c.stream>>>(p.part_ml, p.part_o, p.chunks,
                                                               head_dim, out);
        CheckCuda(cudaGetLastError(), "AttnMergeKernel");
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
// part of the library image (kNoAllocScratchFloats floats = 16 MiB on every
// device that loads the library, held until the process exits).
namespace {

constexpr size_t kNoAllocScratchFloats = size_t(4) << 20;  // 16 MiB
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
            AttnMergeKernel<<<n_heads, 128, 0, c.stream>>>(p.part_ml, p.part_o, p.chunks, head_dim,
                                                            out);
            CheckCuda(cudaGetLastError(), "AttnMergeKernel");
        }
    });
}
