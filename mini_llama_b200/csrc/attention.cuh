// Split-K GQA decode attention.
//
// One CTA = (KV head, group of <= kAttnGmax query heads sharing it, chunk of
// positions, sequence).  Each of the four warps walks 32-position tiles of the
// chunk: the K tile goes to warp-private shared memory (row stride hd+1, so a
// lane per position reads conflict-free), every lane scores its position for
// all query heads of the group, the warp keeps an online softmax (m, l) per
// head, then the V tile replaces K in shared memory and each lane accumulates
// its slice of the head dimension.  K and V of a position are read once for
// all query heads of the group.  The four warps merge in shared memory; with
// one chunk the CTA writes the normalised output, otherwise (m, l, o) partials
// that a merge step (a small kernel, or the O-projection GEMV prologue in the
// decode graph) combines.
//
// Replaces AttentionScoresKernel + AttentionReduceKernel (mini_llama
// src/cuda_attention.cu:87-181): one CTA per (head, position), a global score
// scratch, expf recomputed per (dim, position) and two device syncs.
#pragma once

#include "common.cuh"

namespace mlb {

constexpr int kAttnThreads = 128;
constexpr int kAttnWarps = kAttnThreads / 32;
constexpr int kAttnGmax = 8;
constexpr int kAttnTile = 32;

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
    int chunks;
    float scale;
    // positions: pos_dev ? pos_dev[b * pos_stride] : pos_host
    const int* pos_dev;
    int pos_stride;
    int pos_host;
    // outputs
    float* out;  // chunks == 1: [b][h][hd]
    float* part_ml;  // chunks > 1: [b][h][chunk][2]
    float* part_o;   // [b][h][chunk][hd]
    // decode-graph mode: q/k/v raw from the QKV GEMV, RoPE here, KV write here
    int fused_rope;
    const float* kv_new;   // k at kv_new[kvh*hd], v at kv_new[n_kv*hd + kvh*hd]
    const float* rope_cos;  // [max_seq_len][hd/2]
    const float* rope_sin;
    int neox;
};

// K and V tiles are fetched together (two buffers per warp) for head_dim <=
// 128; above that one buffer is reused (K, then V) to fit shared memory.
__host__ __device__ inline int AttnTileBuffers(int hd) { return hd <= 128 ? 2 : 1; }

__host__ __device__ inline size_t AttnSmemBytes(int hd) {
    const size_t row = size_t(hd) + 1;
    return (size_t(kAttnGmax) * hd +                      // q
            size_t(AttnTileBuffers(hd)) * kAttnWarps * kAttnTile * row +  // K/V tiles
            size_t(kAttnWarps) * kAttnGmax * kAttnTile +  // probabilities per warp
            size_t(kAttnWarps) * kAttnGmax * 2 +          // (m, l) per warp
            size_t(kAttnWarps) * kAttnGmax * hd) * 4;     // o per warp
}

template <int DPL>
__global__ void __launch_bounds__(kAttnThreads) AttnSplitKernel(const AttnParams p) {
    extern __shared__ __align__(16) float asmem[];
    const int hd = p.hd;
    const int row = hd + 1;
    const int nbuf = AttnTileBuffers(hd);
    float* qs = asmem;                                         // [G][hd]
    float* tiles = qs + kAttnGmax * hd;                        // [nbuf][W][32][row]
    float* probs = tiles + nbuf * kAttnWarps * kAttnTile * row;  // [W][G][32]
    float* mls = probs + kAttnWarps * kAttnGmax * kAttnTile;   // [W][G][2]
    float* os = mls + kAttnWarps * kAttnGmax * 2;              // [W][G][hd]

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int kvh = blockIdx.x / p.hgroups, hg = blockIdx.x % p.hgroups;
    const int chunk = blockIdx.y, b = blockIdx.z;
    const int h0 = kvh * p.group + hg * kAttnGmax;
    const int gcnt = min(kAttnGmax, p.group - hg * kAttnGmax);

    GridDepWait();
    GridDepLaunch();

    // A position outside the cache (possible only through a device array)
    // attends to nothing and yields zeros instead of reading out of bounds.
    const int pos_raw = p.pos_dev ? p.pos_dev[size_t(b) * p.pos_stride] : p.pos_host;
    const bool valid = pos_raw >= 0 && pos_raw < p.max_seq_len;
    const int pos = valid ? pos_raw : 0;
    const int npos = valid ? pos_raw + 1 : 0;
    const int clen = (npos + p.chunks - 1) / p.chunks;
    const int p0 = chunk * clen, p1 = min(npos, p0 + clen);

    const size_t pos_stride = size_t(p.n_kv) * hd;
    float* kbase = p.kc + size_t(b) * p.seq_stride + size_t(p.layer) * p.max_seq_len * pos_stride +
                   size_t(kvh) * hd;
    float* vbase = p.vc + size_t(b) * p.seq_stride + size_t(p.layer) * p.max_seq_len * pos_stride +
                   size_t(kvh) * hd;

    // ---- q of the group into shared memory (rotated in decode-graph mode)
    const float* qsrc = p.q + size_t(b) * p.q_batch_stride;
    for (int i = threadIdx.x; i < gcnt * hd; i += kAttnThreads) {
        int g = i / hd, d = i - g * hd;
        qs[g * hd + d] = qsrc[size_t(h0 + g) * hd + d];
    }
    if (p.fused_rope && valid) {
        __syncthreads();
        const int half = hd / 2;
        const float* ct = p.rope_cos + size_t(pos) * half;
        const float* st = p.rope_sin + size_t(pos) * half;
        for (int i = threadIdx.x; i < gcnt * half; i += kAttnThreads) {
            int g = i / half, j = i - g * half;
            int a = p.neox ? j : 2 * j, c2 = p.neox ? j + half : 2 * j + 1;
            float x0 = qs[g * hd + a], x1 = qs[g * hd + c2], cs = ct[j], sn = st[j];
            qs[g * hd + a] = __fsub_rn(__fmul_rn(x0, cs), __fmul_rn(x1, sn));
            qs[g * hd + c2] = __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, cs));
        }
        // the chunk holding `pos` stores the rotated k and v of this token
        if (pos >= p0 && pos < p1) {
            const float* kn = p.kv_new + size_t(kvh) * hd;
            const float* vn = p.kv_new + size_t(p.n_kv) * hd + size_t(kvh) * hd;
            float* kd = kbase + size_t(pos) * pos_stride;
            float* vd = vbase + size_t(pos) * pos_stride;
            for (int j = threadIdx.x; j < half; j += kAttnThreads) {
                int a = p.neox ? j : 2 * j, c2 = p.neox ? j + half : 2 * j + 1;
                float x0 = kn[a], x1 = kn[c2], cs = ct[j], sn = st[j];
                kd[a] = __fsub_rn(__fmul_rn(x0, cs), __fmul_rn(x1, sn));
                kd[c2] = __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, cs));
            }
            for (int d = threadIdx.x; d < hd; d += kAttnThreads) vd[d] = vn[d];
        }
    }
    __syncthreads();

    float m[kAttnGmax], l[kAttnGmax], o[kAttnGmax][DPL];
#pragma unroll
    for (int g = 0; g < kAttnGmax; ++g) {
        m[g] = -INFINITY;
        l[g] = 0.0f;
#pragma unroll
        for (int j = 0; j < DPL; ++j) o[g][j] = 0.0f;
    }
    float* tile = tiles + warp * kAttnTile * row;
    float* vtile = nbuf == 2 ? tiles + (kAttnWarps + warp) * kAttnTile * row : tile;
    float* pr = probs + warp * kAttnGmax * kAttnTile;

    for (int t0 = p0 + warp * kAttnTile; t0 < p1; t0 += kAttnWarps * kAttnTile) {
        const int tn = min(kAttnTile, p1 - t0);
        // K (and V) tile -> shared with asynchronous copies, all in flight
        for (int r = 0; r < tn; ++r) {
            const float* src = kbase + size_t(t0 + r) * pos_stride;
            for (int d = lane; d < hd; d += 32) CpAsync4(tile + r * row + d, src + d);
        }
        if (nbuf == 2) {
            for (int r = 0; r < tn; ++r) {
                const float* src = vbase + size_t(t0 + r) * pos_stride;
                for (int d = lane; d < hd; d += 32) CpAsync4(vtile + r * row + d, src + d);
            }
        }
        CpAsyncWaitAll();
        __syncwarp();
        float s[kAttnGmax];
#pragma unroll
        for (int g = 0; g < kAttnGmax; ++g) s[g] = 0.0f;
        if (lane < tn) {
            const float* kr = tile + lane * row;
            for (int d = 0; d < hd; ++d) {
                float kv = kr[d];
#pragma unroll
                for (int g = 0; g < kAttnGmax; ++g)
                    if (g < gcnt) s[g] = fmaf(qs[g * hd + d], kv, s[g]);
            }
        }
#pragma unroll
        for (int g = 0; g < kAttnGmax; ++g) {
            if (g >= gcnt) break;
            float sc = lane < tn ? s[g] * p.scale : -INFINITY;
            float mt = WarpMax(sc);
            float mn = fmaxf(m[g], mt);
            float pv = lane < tn ? expf(sc - mn) : 0.0f;
            float corr = (m[g] == -INFINITY) ? 0.0f : expf(m[g] - mn);
            l[g] = l[g] * corr + WarpSum(pv);
            m[g] = mn;
#pragma unroll
            for (int j = 0; j < DPL; ++j) o[g][j] *= corr;
            pr[g * kAttnTile + lane] = pv;
        }
        __syncwarp();
        if (nbuf == 1) {  // V tile replaces K
            for (int r = 0; r < tn; ++r) {
                const float* src = vbase + size_t(t0 + r) * pos_stride;
                for (int d = lane; d < hd; d += 32) CpAsync4(vtile + r * row + d, src + d);
            }
            CpAsyncWaitAll();
            __syncwarp();
        }
        for (int r = 0; r < tn; ++r) {
#pragma unroll
            for (int j = 0; j < DPL; ++j) {
                const int d = lane + 32 * j;
                if (d < hd) {
                    float vv = vtile[r * row + d];
#pragma unroll
                    for (int g = 0; g < kAttnGmax; ++g)
                        if (g < gcnt) o[g][j] = fmaf(pr[g * kAttnTile + r], vv, o[g][j]);
                }
            }
        }
        __syncwarp();
    }

    // ---- merge the warps
    float* mw = mls + warp * kAttnGmax * 2;
    float* ow = os + warp * kAttnGmax * hd;
#pragma unroll
    for (int g = 0; g < kAttnGmax; ++g) {
        if (g >= gcnt) break;
        if (lane == 0) {
            mw[2 * g] = m[g];
            mw[2 * g + 1] = l[g];
        }
#pragma unroll
        for (int j = 0; j < DPL; ++j) {
            const int d = lane + 32 * j;
            if (d < hd) ow[g * hd + d] = o[g][j];
        }
    }
    __syncthreads();
    for (int i = threadIdx.x; i < gcnt * hd; i += kAttnThreads) {
        const int g = i / hd, d = i - g * hd;
        float mx = -INFINITY;
        for (int w = 0; w < kAttnWarps; ++w) mx = fmaxf(mx, mls[(w * kAttnGmax + g) * 2]);
        float num = 0.0f, den = 0.0f;
        for (int w = 0; w < kAttnWarps; ++w) {
            float mw2 = mls[(w * kAttnGmax + g) * 2];
            if (mw2 == -INFINITY) continue;
            float wt = expf(mw2 - mx);
            den = fmaf(wt, mls[(w * kAttnGmax + g) * 2 + 1], den);
            num = fmaf(wt, os[(w * kAttnGmax + g) * hd + d], num);
        }
        const int h = h0 + g;
        if (p.chunks == 1) {
            p.out[(size_t(b) * p.n_heads + h) * hd + d] = den > 0.0f ? num / den : 0.0f;
        } else {
            const size_t pc = (size_t(b) * p.n_heads + h) * p.chunks + chunk;
            p.part_o[pc * hd + d] = num;
            if (d == 0) {
                p.part_ml[pc * 2] = mx;
                p.part_ml[pc * 2 + 1] = den;
            }
        }
    }
}

// out[b][h][d] = sum_c e^(m_c - M) o_c[d] / sum_c e^(m_c - M) l_c
static __global__ void AttnMergeKernel(const float* part_ml, const float* part_o, int chunks, int hd,
                                float* out) {
    GridDepWait();
    GridDepLaunch();
    const size_t bh = blockIdx.x;  // b * n_heads + h
    const float* ml = part_ml + bh * chunks * 2;
    float mx = -INFINITY;
    for (int c = 0; c < chunks; ++c) mx = fmaxf(mx, ml[2 * c]);
    for (int d = threadIdx.x; d < hd; d += blockDim.x) {
        float num = 0.0f, den = 0.0f;
        for (int c = 0; c < chunks; ++c) {
            float mc = ml[2 * c];
            if (mc == -INFINITY) continue;
            float wt = expf(mc - mx);
            den = fmaf(wt, ml[2 * c + 1], den);
            num = fmaf(wt, part_o[(bh * chunks + c) * hd + d], num);
        }
        out[bh * hd + d] = den > 0.0f ? num / den : 0.0f;
    }
}

void LaunchAttention(const AttnParams& p, int batch, cudaStream_t stream, bool pdl);
int AttnChunks(int max_npos, int batch, int n_kv, int hgroups, int sm_count);

}  // namespace mlb
