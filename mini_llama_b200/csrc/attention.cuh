// Split-K GQA decode attention.
//
// One CTA = (KV head, group of <= kAttnGmax query heads sharing it, chunk of
// <= kAttnChunk positions, sequence).  The CTA stages q of its heads and the K
// and V rows of its chunk in shared memory with asynchronous copies (one
// memory round trip; each K/V row is read once for all query heads of the
// group).  Warps then take (query head, 32-position tile) items: a lane per
// position scores its key (K rows at stride hd+1, conflict-free), the warp
// forms the tile's softmax (max, sum), and a lane per head dimension
// accumulates the probability-weighted V rows.  The tiles of a head merge in
// shared memory; with one chunk the CTA writes the normalised output,
// otherwise (m, l, o) partials that a merge step (a small kernel, or the
// O-projection GEMV prologue in the decode graph) combines.
//
// Replaces AttentionScoresKernel + AttentionReduceKernel (mini_llama
// src/cuda_attention.cu:87-181): one CTA per (head, position), a global score
// scratch, expf recomputed per (dim, position) and two device syncs.
#pragma once

#include "common.cuh"

namespace mlb {

constexpr int kAttnThreads = 256;
constexpr int kAttnWarps = kAttnThreads / 32;
constexpr int kAttnGmax = 16;   // query heads of one KV group handled by one CTA
constexpr int kAttnTile = 32;   // positions per warp item (one per lane)
constexpr int kAttnChunk = 64;  // positions per CTA (K and V of the chunk sit in shared memory)

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
    int chunks;   // position chunks; chunks * kAttnChunk >= positions + 1
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
};

__host__ __device__ inline size_t AttnSmemBytes(int hd) {
    const int items = kAttnGmax * (kAttnChunk / kAttnTile);
    return (size_t(kAttnGmax) * hd +                  // q
            size_t(kAttnChunk) * (hd + 1) +            // K rows (stride hd+1: lane per position)
            size_t(kAttnChunk) * hd +                  // V rows
            size_t(items) * (hd + 2)) * 4;             // per-item (m, l, o)
}

template <int DPL>
__global__ void __launch_bounds__(kAttnThreads) AttnSplitKernel(const AttnParams p) {
    extern __shared__ __align__(16) float asmem[];
    const int hd = p.hd;
    const int krow = hd + 1;
    float* qs = asmem;                         // [G][hd]
    float* ks = qs + kAttnGmax * hd;           // [chunk][hd+1]
    float* vs = ks + kAttnChunk * krow;        // [chunk][hd]
    float* res = vs + kAttnChunk * hd;         // [items][hd+2]: m, l, o[hd]

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
    const int clen = min(kAttnChunk, (npos + p.chunks - 1) / p.chunks);
    const int p0 = min(npos, chunk * clen), p1 = min(npos, p0 + clen);
    const int len = p1 - p0;
    const bool own_new = p.fused_rope && valid && pos >= p0 && pos < p1;

    const size_t pos_stride = size_t(p.n_kv) * hd;
    float* kbase = p.kc + size_t(b) * p.seq_stride + size_t(p.layer) * p.max_seq_len * pos_stride +
                   size_t(kvh) * hd;
    float* vbase = p.vc + size_t(b) * p.seq_stride + size_t(p.layer) * p.max_seq_len * pos_stride +
                   size_t(kvh) * hd;

    // ---- q of the group, and K/V of the chunk, into shared memory
    const float* qsrc = p.q + size_t(b) * p.q_batch_stride + size_t(h0) * hd;
    for (int i = threadIdx.x; i < gcnt * hd; i += kAttnThreads) CpAsync4(qs + i, qsrc + i);
    for (int i = threadIdx.x; i < len * hd; i += kAttnThreads) {
        const int r = i / hd, d = i - r * hd;
        if (own_new && p0 + r == pos) continue;  // this token's row comes from kv_new below
        CpAsync4(ks + r * krow + d, kbase + size_t(p0 + r) * pos_stride + d);
        CpAsync4(vs + r * hd + d, vbase + size_t(p0 + r) * pos_stride + d);
    }
    CpAsyncWaitAll();
    __syncthreads();
    if (p.fused_rope && valid) {
        // RoPE with the reference CPU tables; the chunk holding `pos` also
        // rotates this token's k and stores k, v into the cache.
        const int half = hd / 2;
        const float* ct = p.rope_cos + size_t(pos) * half;
        const float* st = p.rope_sin + size_t(pos) * half;
        for (int i = threadIdx.x; i < gcnt * half; i += kAttnThreads) {
            const int g = i / half, j = i - g * half;
            const int a = p.neox ? j : 2 * j, c2 = p.neox ? j + half : 2 * j + 1;
            const float x0 = qs[g * hd + a], x1 = qs[g * hd + c2], cs = ct[j], sn = st[j];
            qs[g * hd + a] = __fsub_rn(__fmul_rn(x0, cs), __fmul_rn(x1, sn));
            qs[g * hd + c2] = __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, cs));
        }
        if (own_new) {
            const float* kn = p.kv_new + size_t(b) * p.kv_batch_stride + size_t(kvh) * hd;
            const float* vn = (p.v_new ? p.v_new + size_t(b) * p.kv_batch_stride
                                       : p.kv_new + size_t(b) * p.kv_batch_stride + size_t(p.n_kv) * hd) +
                              size_t(kvh) * hd;
            float* kd = kbase + size_t(pos) * pos_stride;
            float* vd = vbase + size_t(pos) * pos_stride;
            const int r = pos - p0;
            for (int j = threadIdx.x; j < half; j += kAttnThreads) {
                const int a = p.neox ? j : 2 * j, c2 = p.neox ? j + half : 2 * j + 1;
                const float x0 = kn[a], x1 = kn[c2], cs = ct[j], sn = st[j];
                const float ka = __fsub_rn(__fmul_rn(x0, cs), __fmul_rn(x1, sn));
                const float kb = __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, cs));
                kd[a] = ka;
                kd[c2] = kb;
                ks[r * krow + a] = ka;
                ks[r * krow + c2] = kb;
            }
            for (int d = threadIdx.x; d < hd; d += kAttnThreads) {
                const float v = vn[d];
                vd[d] = v;
                vs[r * hd + d] = v;
            }
        }
        __syncthreads();
    }

    // ---- items: (query head, 32-position tile); lane = position for the
    // scores, lane = head dimension for the weighted sum of V
    const int ntile = (len + kAttnTile - 1) / kAttnTile;
    for (int item = warp; item < gcnt * ntile; item += kAttnWarps) {
        const int g = item / ntile, tile = item - g * ntile;
        const int r0 = tile * kAttnTile;
        const int tn = min(kAttnTile, len - r0);
        const float* qh = qs + g * hd;
        float s = -INFINITY;
        if (lane < tn) {
            const float* kr = ks + (r0 + lane) * krow;
            float acc = 0.0f;
            for (int d = 0; d < hd; ++d) acc = fmaf(qh[d], kr[d], acc);
            s = acc * p.scale;
        }
        const float mt = WarpMax(s);
        const float pv = lane < tn ? expf(s - mt) : 0.0f;
        const float lt = WarpSum(pv);
        float o[DPL];
#pragma unroll
        for (int j = 0; j < DPL; ++j) o[j] = 0.0f;
        for (int r = 0; r < tn; ++r) {
            const float pr = __shfl_sync(0xffffffffu, pv, r);
            const float* vr = vs + (r0 + r) * hd;
#pragma unroll
            for (int j = 0; j < DPL; ++j) {
                const int d = lane + 32 * j;
                if (d < hd) o[j] = fmaf(pr, vr[d], o[j]);
            }
        }
        float* rr = res + item * (hd + 2);
        if (lane == 0) {
            rr[0] = mt;
            rr[1] = lt;
        }
#pragma unroll
        for (int j = 0; j < DPL; ++j) {
            const int d = lane + 32 * j;
            if (d < hd) rr[2 + d] = o[j];
        }
    }
    __syncthreads();

    // ---- merge the tiles of each head: final output or the chunk's partial
    for (int i = threadIdx.x; i < gcnt * hd; i += kAttnThreads) {
        const int g = i / hd, d = i - g * hd;
        float mx = -INFINITY;
        for (int tl = 0; tl < ntile; ++tl) mx = fmaxf(mx, res[(g * ntile + tl) * (hd + 2)]);
        float num = 0.0f, den = 0.0f;
        for (int tl = 0; tl < ntile; ++tl) {
            const float* rr = res + (g * ntile + tl) * (hd + 2);
            const float wt = expf(rr[0] - mx);
            den = fmaf(wt, rr[1], den);
            num = fmaf(wt, rr[2 + d], num);
        }
        const int h = h0 + g;
        if (p.chunks == 1) {
            p.out[(size_t(b) * p.n_heads + h) * hd + d] = den > 0.0f ? num / den : 0.0f;
        } else {
            const size_t pc = (size_t(b) * p.n_heads + h) * p.chunks + chunk;
            p.part_o[pc * hd + d] = num;
            if (d == 0) {
                p.part_ml[pc * 2] = ntile ? mx : -INFINITY;
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
