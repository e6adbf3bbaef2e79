// Split-K GQA decode attention over the fp32 KV cache.
//
// One CTA = (KV head, group of <= kAttnGmax query heads sharing it, chunk of
// positions, sequence).  The chunk is streamed through shared memory in tiles
// of T rows (T x padded head_dim = kAttnStageFloats, e.g. 32 rows of 128
// floats: 16 KB of K and 16 KB of V a tile) by a ring of kAttnStages stages,
// kAttnStages - 1 tiles ahead of the one being computed, so a CTA keeps two
// tiles in flight while it works.  A tile is two tensor-map boxes (TMA, one
// for K and one for V, completing on the stage's mbarrier) when head_dim is a
// multiple of 4 and the caches are 16-byte aligned; otherwise single-float
// cp.async copies.  Per tile:
//   scores   256 / T threads per position (consecutive lanes), each over a
//            quarter or less of the row's 16-byte pieces, every query head of
//            the group at once (q in shared memory, one dot per head in
//            registers), summed over the position's lanes by shuffles
//   softmax  a warp per head: the tile's maximum, the running maximum and sum
//            (online softmax across tiles), the tile's weights in place
//   values   a thread per (16-byte column, row group): o[head] += w x V row
//            for every head (V read once for all heads), scaled by the
//            running-maximum correction first
// Each row of K is read once for all query heads of its group and each tile
// costs three CTA barriers.  At the end the row groups' partial outputs are
// summed in shared memory: with one chunk the CTA writes the normalised
// output, otherwise (m, l, o) partials that a merge step (AttnMergeKernel, or
// the O-projection GEMV prologue in the decode graph) combines.
//
// The grid is sized by AttnChunks: short contexts split into chunks of at
// least 16 positions while the grid is below two waves; long contexts into as
// few chunks as fill kAttnCtasPerSm CTAs per SM, so the K/V bytes stream
// through long-running CTAs and the partials stay small.
//
// Replaces AttentionScoresKernel + AttentionReduceKernel (mini_llama
// src/cuda_attention.cu:87-181): one CTA per (head, position), a global score
// scratch, expf recomputed per (dim, position) and two device syncs.
#pragma once

#include <cuda.h>

#include "common.cuh"

namespace mlb {

constexpr int kAttnThreads = 256;
constexpr int kAttnWarps = kAttnThreads / 32;
constexpr int kAttnGmax = 16;           // query heads of one KV group handled by one CTA
constexpr int kAttnStages = 3;          // K/V tiles in the shared-memory ring
constexpr int kAttnStageFloats = 4096;  // tile rows x padded head_dim (rounded up to a power of two)
constexpr int kAttnCtasPerSm = 2;       // resident CTAs per SM the long-context grid is sized for
constexpr int kAttnPieces = 4;          // 16-byte pieces of a row one score thread covers at most

struct AttnParams {
    // query source: q[b][h][hd] (stride q_batch_stride per sequence)
    const float* q;
    size_t q_batch_stride;
    float* kc;  // caches [batch][n_layers][max_seq_len][n_kv][hd]
    float* vc;
    size_t seq_stride;  // floats per sequence in the caches
    int layer;
    int max_seq_len;
    int n_heads;
    int n_kv;
    int hd;
    int group;    // n_heads / n_kv
    int hgroups;  // ceil(group / kAttnGmax)
    int chunks;   // position chunks (any count >= 1; a CTA loops over its chunk's tiles)
    float scale;
    // positions: pos_dev ? pos_dev[b * pos_stride] : pos_host
    const int* pos_dev;
    int pos_stride;
    int pos_host;
    // outputs
    float* out;      // chunks == 1: [b][h][hd]
    float* part_ml;  // chunks > 1: [b][h][chunk][2]
    float* part_o;   // [b][h][chunk][hd]
    // decode-graph mode: q/k/v raw from the QKV GEMV, RoPE here, KV write here
    int fused_rope;
    const float* kv_new;    // k at kv_new[kvh*hd], v at kv_new[n_kv*hd + kvh*hd]
    const float* v_new;     // when set, v at v_new[kvh*hd] instead
    size_t kv_batch_stride; // floats between sequences' kv_new (and v_new) rows
    const float* rope_cos;  // [max_seq_len][hd/2]
    const float* rope_sin;
    int neox;
    // device status word: a tile copy that does not arrive within
    // kAttnWaitNs records MLB_ERR_DEVICE_TIMEOUT here (tensor-map path)
    int* status;
    // tensor-map path: cache rows of sequence b, layer `layer` start at row
    // b * seq_rows + layer * max_seq_len of the [rows][n_kv][hd] maps
    int seq_rows;
};

constexpr uint64_t kAttnWaitNs = 2000000000ull;  // bound of one tile wait

// Tile geometry of a head_dim (the same on host and device).
struct AttnGeom {
    int hdp;  // head_dim rounded up to a multiple of 4 (row stride in shared memory)
    int lpr;  // 16-byte pieces per row (hdp / 4)
    int T;    // rows per tile
    int tpp;  // score threads per position (kAttnThreads / T)
    int R;    // row groups of the value pass (kAttnThreads / lpr)
    // K rows are stored as they are; the score thread of row r takes its
    // pieces ssub + tpp i in the order i ^ (((r >> ksh) & kmk) * kml / tpp),
    // which puts the eight threads of a shared-memory phase on eight distinct
    // bank groups
    int ksh, kmk, kml;
};

__host__ __device__ inline AttnGeom AttnGeometry(int hd) {
    AttnGeom g;
    g.hdp = (hd + 3) & ~3;
    g.lpr = g.hdp / 4;
    int p2 = 4;
    while (p2 < g.hdp) p2 <<= 1;
    g.T = kAttnStageFloats / p2 < kAttnThreads ? kAttnStageFloats / p2 : kAttnThreads;
    g.tpp = kAttnThreads / g.T;
    g.R = kAttnThreads / g.lpr;
    g.ksh = g.kmk = g.kml = 0;
    if ((g.lpr & (g.lpr - 1)) == 0) {
        if (g.lpr >= 8 && g.tpp < 8) {  // rows of 8+ pieces: a phase spans 8 / tpp rows
            g.kmk = 8 / g.tpp - 1;
            g.kml = g.tpp;
        } else if (g.lpr < 8) {  // one thread per row, 8 / lpr rows per 128 bytes
            g.ksh = g.lpr == 4 ? 1 : (g.lpr == 2 ? 2 : 3);
            g.kmk = g.lpr - 1;
            g.kml = 1;
        }
    }
    return g;
}

// Shared memory of the kernel for (head_dim, heads per CTA GM): a 128-byte
// header (the stages' mbarriers, the abort flag), then floats: the ring (its
// space holds the row groups' partial outputs after the loop), q of the
// group, this token's k and v rows, the tile's scores, three per-head
// scalars.
constexpr int kAttnHeader = 128;

__host__ __device__ inline size_t AttnSmemBytes(int hd, int gm) {
    const AttnGeom g = AttnGeometry(hd);
    const size_t ring = size_t(2) * kAttnStages * g.T * g.hdp;
    const size_t red = size_t(g.R) * gm * g.hdp;
    return kAttnHeader + ((ring > red ? ring : red) + size_t(gm) * g.hdp + 2 * size_t(g.hdp) +
                          size_t(gm) * g.T + 3 * size_t(gm)) * 4;
}

__device__ __forceinline__ void CpAsyncCommit() { asm volatile("cp.async.commit_group;" ::: "memory"); }

template <int N>
__device__ __forceinline__ void CpAsyncWaitGroup() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ float4 Lds4(const float* p) { return *reinterpret_cast<const float4*>(p); }

// One 3-D tensor-map box (no multicast) into shared memory, completing on bar.
__device__ __forceinline__ void TmaLoad3D(void* dst, const CUtensorMap* map, int x, int y, int z, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
        "[%5];" ::"r"(SmemAddr(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(SmemAddr(bar))
        : "memory");
}

}  // namespace mlb

#include "attention_kernel.cuh"
