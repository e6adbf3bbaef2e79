// Dequant-fused GEMV for GGUF Q8_0 / Q4_0 / Q4_1 blocks (rows <= 8).
//
// y[m, n] = sum_k x[m, k] * dequant(W[n, k])  for m < M, n < N.
//
// The weight matrix is streamed once from HBM: each CTA walks a strided list
// of row tiles; one elected thread moves a whole tile (contiguous rows of
// blocks) into a shared-memory ring with a single cp.async.bulk (TMA bulk
// copy, no multicast) completing on an mbarrier, several tiles ahead of the
// compute.  x (fp32) sits in shared memory for the whole kernel.  Eight lanes
// cooperate on one 32-element block (4 elements each), four blocks per warp
// step; the int8 -> fp32 conversion uses the exponent-splice trick and the
// products run on the sm_100 packed f32x2 FMA.
//
// Replaces the reference kernels Q80LinearKernel / Q40LinearKernel /
// Q41LinearKernel (mini_llama src/cuda_quant.cu:40-135), which read the blocks
// with one thread per output row and uncoalesced byte loads.
#pragma once

#include "common.cuh"

namespace mlb {

constexpr int kGemvThreads = 256;
constexpr int kGemvWarps = kGemvThreads / 32;
constexpr int kGemvMaxM = 8;
constexpr int kGemvMaxTileRows = 64;
constexpr int kGemvStages = 4;
constexpr int kGemvMaxWarps = 16;

template <int QT>
struct QTraits;
template <>
struct QTraits<MLB_Q8_0> {
    static constexpr int kBytes = 34;
    static constexpr int kAlignRows = 8;  // rows * 34 * nb % 16 == 0 when rows*nb % 8 == 0
};
template <>
struct QTraits<MLB_Q4_0> {
    static constexpr int kBytes = 18;
    static constexpr int kAlignRows = 8;
};
template <>
struct QTraits<MLB_Q4_1> {
    static constexpr int kBytes = 20;
    static constexpr int kAlignRows = 4;
};

inline int BlockBytes(int qtype) {
    return qtype == MLB_Q8_0 ? 34 : qtype == MLB_Q4_0 ? 18 : qtype == MLB_Q4_1 ? 20 : 0;
}

enum GemvPrologue { kProPlain = 0, kProRmsNorm = 1, kProAttnMerge = 2 };
enum GemvEpilogue {
    kEpiStore = 0,     // y = acc (+ bias)
    kEpiResidual = 1,  // y = acc + residual (residual may alias y)
    kEpiSwiglu = 2,    // y = silu(acc_gate) * acc_up   (two weight matrices)
    kEpiArgmax = 3     // y = acc, plus the first arg-max over all rows
};

// One weight matrix (segment) of the launch.  Segments share K and qtype.
struct GemvSeg {
    const uint8_t* w;
    const float* bias;  // [rows] or null
    int rows;
    int out_offset;  // column offset of this segment in y
    int tile_rows;   // rows per tile
    int tiles;       // tiles of this segment
};

struct GemvParams {
    int K;
    int nb;
    int rowbytes;
    int M;
    const float* x;   // [M, K]
    float* y;         // [M, y_stride]
    int y_stride;
    int nseg;
    GemvSeg seg[3];   // kEpiSwiglu: seg[0] = gate, seg[1] = up (same tiling)
    int total_tiles;
    int stage_bytes;
    int aux_floats;   // shared floats for norm weights or attention partials
    int nstages;      // integer-MMA kernel: ring stages
    // prologue
    const float* norm_w;
    float eps;
    // attention-merge prologue: partials [n_heads][chunks] (m, l) and
    // [n_heads][chunks][head_dim] unnormalised outputs
    const float* part_ml;
    const float* part_o;
    int n_heads;
    int head_dim;
    int chunks;
    // residual epilogue
    const float* residual;
    int res_stride;
    // argmax epilogue
    float* am_val;
    int* am_idx;
    unsigned int* am_counter;
    int* am_token;       // written by the last CTA
    int* am_pos;         // incremented by the last CTA when non-null
    int* am_hist;        // token history: hist[pos + 1] = token when pos + 1 >= *am_gen_from
    const int* am_gen_from;
    int* status;         // device error flag (bounded waits)
};

__device__ __forceinline__ float2 F2(float a, float b) { return make_float2(a, b); }

// int8x4 (as uint32) -> 4 floats, exact: splice each byte (biased by 128)
// into the mantissa of 2^23 and subtract 2^23 + 128.
__device__ __forceinline__ void I8x4ToF(uint32_t w, float2& lo, float2& hi) {
    uint32_t u = w ^ 0x80808080u;
    const float2 bias = make_float2(8388736.0f, 8388736.0f);
    float a = __int_as_float(__byte_perm(u, 0x4B000000u, 0x7440));
    float b = __int_as_float(__byte_perm(u, 0x4B000000u, 0x7441));
    float c = __int_as_float(__byte_perm(u, 0x4B000000u, 0x7442));
    float d = __int_as_float(__byte_perm(u, 0x4B000000u, 0x7443));
    lo = __fadd2_rn(F2(a, b), make_float2(-bias.x, -bias.y));
    hi = __fadd2_rn(F2(c, d), make_float2(-bias.x, -bias.y));
}

// Unsigned nibble pair extraction for Q4: bytes b0 b1 (in the low 16 bits of
// w) -> low nibbles (elements j, j+1) and high nibbles (elements j+16, j+17).
__device__ __forceinline__ void U4x4ToF(uint32_t w, float2& lo, float2& hi) {
    uint32_t lo4 = w & 0x0F0Fu;         // bytes: n0, n1 (low nibbles)
    uint32_t hi4 = (w >> 4) & 0x0F0Fu;  // high nibbles
    const float m = 8388608.0f;
    float a = __int_as_float(0x4B000000u | (lo4 & 0xFFu));
    float b = __int_as_float(0x4B000000u | (lo4 >> 8));
    float c = __int_as_float(0x4B000000u | (hi4 & 0xFFu));
    float d = __int_as_float(0x4B000000u | (hi4 >> 8));
    lo = __fadd2_rn(F2(a, b), make_float2(-m, -m));
    hi = __fadd2_rn(F2(c, d), make_float2(-m, -m));
}

__device__ __forceinline__ uint32_t Lds16x2(const uint8_t* p) {
    uint32_t a = *reinterpret_cast<const uint16_t*>(p);
    uint32_t b = *reinterpret_cast<const uint16_t*>(p + 2);
    return a | (b << 16);
}

// One lane's share of one block: 4 of the 32 elements (sub = 0..7), for M
// rows of x.  xk points at x_s[0][k0] (row stride kpad floats).
template <int QT, int M>
__device__ __forceinline__ void BlockDot(const uint8_t* blk, const float* xk, int kpad, int sub,
                                         float (&acc)[M]) {
    if constexpr (QT == MLB_Q8_0) {
        float d = HalfBits(*reinterpret_cast<const uint16_t*>(blk));
        float2 q01, q23;
        I8x4ToF(Lds16x2(blk + 2 + 4 * sub), q01, q23);
#pragma unroll
        for (int m = 0; m < M; ++m) {
            float4 xv = *reinterpret_cast<const float4*>(xk + m * kpad + 4 * sub);
            float2 s = __fmul2_rn(q01, F2(xv.x, xv.y));
            s = __ffma2_rn(q23, F2(xv.z, xv.w), s);
            acc[m] = fmaf(d, s.x + s.y, acc[m]);
        }
    } else {
        constexpr int kQs = (QT == MLB_Q4_0) ? 2 : 4;
        float d = HalfBits(*reinterpret_cast<const uint16_t*>(blk));
        uint32_t w = *reinterpret_cast<const uint16_t*>(blk + kQs + 2 * sub);
        float2 lo, hi;
        U4x4ToF(w, lo, hi);
        if constexpr (QT == MLB_Q4_0) {
            lo = __fadd2_rn(lo, make_float2(-8.0f, -8.0f));
            hi = __fadd2_rn(hi, make_float2(-8.0f, -8.0f));
        }
#pragma unroll
        for (int m = 0; m < M; ++m) {
            float2 xl = *reinterpret_cast<const float2*>(xk + m * kpad + 2 * sub);
            float2 xh = *reinterpret_cast<const float2*>(xk + m * kpad + 16 + 2 * sub);
            float2 s = __fmul2_rn(lo, xl);
            s = __ffma2_rn(hi, xh, s);
            float dot = s.x + s.y;
            if constexpr (QT == MLB_Q4_1) {
                float mn = HalfBits(*reinterpret_cast<const uint16_t*>(blk + 2));
                float xs = (xl.x + xl.y) + (xh.x + xh.y);
                acc[m] = fmaf(mn, xs, fmaf(d, dot, acc[m]));
            } else {
                acc[m] = fmaf(d, dot, acc[m]);
            }
        }
    }
}

}  // namespace mlb

namespace mlb {

// Shared-memory carve-up of the GEMV kernel: weight ring | mbarriers | x rows
// [M][kpad] | aux (norm weights or attention partials) | partial sums.
struct GemvSmem {
    static __host__ __device__ int XFloats(int M, int nb) { return M * nb * 32; }
    static __host__ __device__ size_t RedBytes() { return 2ull * kGemvMaxTileRows * kGemvMaxM * 2 * 4; }
    static __host__ __device__ size_t Bytes(int M, int nb, int stage_bytes, int aux_floats) {
        return size_t(kGemvStages) * stage_bytes + 16 * kGemvStages + size_t(XFloats(M, nb)) * 4 +
               size_t((aux_floats + 3) & ~3) * 4 + RedBytes() + 64;
    }
};

struct TileRef {
    int seg;
    int row0;
    int rows;
};

__device__ __forceinline__ TileRef LocateTile(const GemvParams& p, int t, bool dual) {
    TileRef r{0, 0, 0};
    int nseg = dual ? 1 : p.nseg;
    for (int s = 0; s < nseg; ++s) {
        if (t < p.seg[s].tiles) {
            r.seg = s;
            r.row0 = t * p.seg[s].tile_rows;
            int left = p.seg[s].rows - r.row0;
            r.rows = left < p.seg[s].tile_rows ? left : p.seg[s].tile_rows;
            return r;
        }
        t -= p.seg[s].tiles;
    }
    return r;
}

// Issue the bulk copy of one tile into a stage (called by one thread).  The
// copied range is 16-byte aligned at both ends; the last tile of a segment may
// leave a ragged tail of < 16 bytes that CopyTail() fetches after the wait.
__device__ __forceinline__ void IssueTile(const GemvParams& p, const TileRef& tr, bool dual,
                                          uint8_t* stage, uint64_t* bar) {
    uint32_t total = 0;
    const int parts = dual ? 2 : 1;
    size_t seg_bytes = size_t(tr.rows) * p.rowbytes;
    uint32_t body = static_cast<uint32_t>(seg_bytes & ~size_t(15));
    total = body * parts;
    if (total) MbarExpectTx(bar, total);
    else asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(SmemAddr(bar)) : "memory");
    for (int part = 0; part < parts; ++part) {
        const GemvSeg& s = p.seg[dual ? part : tr.seg];
        const uint8_t* src = s.w + size_t(tr.row0) * p.rowbytes;
        if (body) BulkLoad(stage + part * (p.stage_bytes / 2), src, body, bar);
    }
}

__device__ __forceinline__ void CopyTail(const GemvParams& p, const TileRef& tr, bool dual,
                                         uint8_t* stage) {
    size_t seg_bytes = size_t(tr.rows) * p.rowbytes;
    int tail = static_cast<int>(seg_bytes & 15);
    size_t body = seg_bytes - tail;
    const int parts = dual ? 2 : 1;
    if (threadIdx.x < tail * parts) {
        int part = threadIdx.x / tail, i = threadIdx.x % tail;
        const GemvSeg& s = p.seg[dual ? part : tr.seg];
        const uint8_t* src = s.w + size_t(tr.row0) * p.rowbytes + body;
        stage[part * (p.stage_bytes / 2) + body + i] = src[i];
    }
}

// First arg-max over the rows of all CTAs: each CTA reduces its candidates,
// the last CTA to arrive reduces the CTAs' results and writes the token (and
// the token history / position when given).  No CTA waits on another.
__device__ __forceinline__ void ArgmaxFinish(const GemvParams& p, float best_val, int best_idx) {
    const int tid = threadIdx.x;
    // CTA-level first-max, then the last CTA to finish reduces all CTAs.
    __shared__ float sval[512];
    __shared__ int sidx[512];
    __shared__ bool last;
    sval[tid] = best_val;
    sidx[tid] = best_idx;
    __syncthreads();
    for (int o = blockDim.x / 2; o > 0; o >>= 1) {
        if (tid < o) {
            float ov = sval[tid + o];
            int oi = sidx[tid + o];
            if (ov > sval[tid] || (ov == sval[tid] && oi < sidx[tid])) {
                sval[tid] = ov;
                sidx[tid] = oi;
            }
        }
        __syncthreads();
    }
    if (tid == 0) {
        p.am_val[blockIdx.x] = sval[0];
        p.am_idx[blockIdx.x] = sidx[0];
        __threadfence();
        unsigned prev = atomicAdd(p.am_counter, 1u);
        last = (prev == gridDim.x - 1);
    }
    __syncthreads();
    if (last) {
        __threadfence();
        float bv = -INFINITY;
        int bi = 0x7fffffff;
        for (int c = tid; c < gridDim.x; c += blockDim.x) {
            float v = __ldcg(&p.am_val[c]);
            int i = __ldcg(&p.am_idx[c]);
            if (v > bv || (v == bv && i < bi)) {
                bv = v;
                bi = i;
            }
        }
        sval[tid] = bv;
        sidx[tid] = bi;
        __syncthreads();
        for (int o = blockDim.x / 2; o > 0; o >>= 1) {
            if (tid < o) {
                float ov = sval[tid + o];
                int oi = sidx[tid + o];
                if (ov > sval[tid] || (ov == sval[tid] && oi < sidx[tid])) {
                    sval[tid] = ov;
                    sidx[tid] = oi;
                }
            }
            __syncthreads();
        }
        if (tid == 0) {
            const int tok = sidx[0] == 0x7fffffff ? 0 : sidx[0];
            *p.am_token = tok;
            if (p.am_pos) {
                const int ps = *p.am_pos;
                if (p.am_hist && ps + 1 >= *p.am_gen_from) p.am_hist[ps + 1] = tok;
                *p.am_pos = ps + 1;
            }
            *p.am_counter = 0;
        }
    }
}

// Stages x (M rows, RMS-normalised or merged from attention partials) into
// shared memory as rows of kpad floats, zero padded.  Every global read is an
// asynchronous copy issued before any is waited on, so the prologue costs one
// memory round trip.  Ends with a CTA barrier.
template <int M, int PRO>
__device__ __forceinline__ void StageGemvX(const GemvParams& p, float* xs, float* aux, int kpad) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if constexpr (PRO == kProAttnMerge) {
        const int nml = p.n_heads * p.chunks * 2;
        StageFloats(aux, p.part_ml, nml);
        StageFloats(aux + nml, p.part_o, p.n_heads * p.chunks * p.head_dim);
        CpAsyncWaitAll();
        __syncthreads();
        // x[k] for k = h*head_dim + d: merge of the split-K partial softmax.
        for (int k = tid; k < kpad; k += blockDim.x) {
            float v = 0.0f;
            if (k < p.K) {
                const int h = k / p.head_dim, d = k - h * p.head_dim;
                const float* ml = aux + h * p.chunks * 2;
                const float* po = aux + nml + h * p.chunks * p.head_dim + d;
                float mx = -INFINITY;
                for (int c = 0; c < p.chunks; ++c) mx = fmaxf(mx, ml[2 * c]);
                float num = 0.0f, den = 0.0f;
                for (int c = 0; c < p.chunks; ++c) {
                    const float mc = ml[2 * c];
                    if (mc == -INFINITY) continue;
                    const float wgt = expf(mc - mx);
                    den = fmaf(wgt, ml[2 * c + 1], den);
                    num = fmaf(wgt, po[c * p.head_dim], num);
                }
                v = den > 0.0f ? num / den : 0.0f;
            }
            xs[k] = v;
        }
    } else {
        for (int m = 0; m < M; ++m) StageFloats(xs + m * kpad, p.x + size_t(m) * p.K, p.K);
        if constexpr (PRO == kProRmsNorm) StageFloats(aux, p.norm_w, p.K);
        for (int m = 0; m < M; ++m)
            for (int k = p.K + tid; k < kpad; k += blockDim.x) xs[m * kpad + k] = 0.0f;
        CpAsyncWaitAll();
        __syncthreads();
        if constexpr (PRO == kProRmsNorm) {
            __shared__ float wsum[kGemvMaxWarps];
            for (int m = 0; m < M; ++m) {
                float* xr = xs + m * kpad;
                float ss = 0.0f;
                for (int k = tid; k < p.K; k += blockDim.x) ss = fmaf(xr[k], xr[k], ss);
                ss = WarpSum(ss);
                if (lane == 0) wsum[warp] = ss;
                __syncthreads();
                float tot = 0.0f;
#pragma unroll
                for (int w = 0; w < (blockDim.x >> 5); ++w) tot += wsum[w];
                __syncthreads();
                const float scale = 1.0f / sqrtf(tot / static_cast<float>(p.K) + p.eps);
                for (int k = tid; k < p.K; k += blockDim.x) xr[k] = xr[k] * scale * aux[k];
            }
        }
    }
    __syncthreads();

}

template <int QT, int M, int PRO, int EPI>
__global__ void __launch_bounds__(kGemvThreads) GemvKernel(const GemvParams p) {
    constexpr bool kDual = (EPI == kEpiSwiglu);
    constexpr int kBB = QTraits<QT>::kBytes;
    extern __shared__ __align__(128) uint8_t smem[];
    uint8_t* stages = smem;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + size_t(kGemvStages) * p.stage_bytes);
    float* xs = reinterpret_cast<float*>(smem + size_t(kGemvStages) * p.stage_bytes +
                                         16 * kGemvStages);
    const int kpad = p.nb * 32;
    float* aux = xs + M * kpad;
    float* red = aux + ((p.aux_floats + 3) & ~3);  // [2][kGemvMaxTileRows][M][2]

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int ntiles = p.total_tiles;

    __shared__ int s_abort;
    if (tid == 0) {
        s_abort = 0;
        for (int s = 0; s < kGemvStages; ++s) MbarInit(&bars[s], 1);
        FenceMbarInit();
    }
    __syncthreads();
    // Weights do not depend on the previous kernel: start streaming them
    // before waiting on it.
    if (tid == 0) {
        for (int s = 0; s < kGemvStages; ++s) {
            int t = blockIdx.x + s * gridDim.x;
            if (t < ntiles) IssueTile(p, LocateTile(p, t, kDual), kDual,
                                      stages + size_t(s) * p.stage_bytes, &bars[s]);
        }
    }
    GridDepWait();
    GridDepLaunch();

    StageGemvX<M, PRO>(p, xs, aux, kpad);

    float best_val = -INFINITY;
    int best_idx = 0x7fffffff;
    const int groups = (p.nb + 3) >> 2;
    const int blk_in_group = lane >> 3, sub = lane & 7;

    int it = 0;
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++it) {
        const int s = it % kGemvStages;
        const uint32_t parity = (it / kGemvStages) & 1;
        uint8_t* stage = stages + size_t(s) * p.stage_bytes;
        TileRef tr = LocateTile(p, t, kDual);
        // A wait that gives up marks the CTA; every thread leaves the loop
        // together after the barrier below, so no thread is left waiting.
        if (!MbarWait(&bars[s], parity)) s_abort = 1;
        if ((size_t(tr.rows) * p.rowbytes) & 15) {
            CopyTail(p, tr, kDual, stage);
            __syncthreads();
        }
        // ---- compute partial sums: items = rows x parts
        const int P = tr.rows >= kGemvWarps ? 1 : kGemvWarps / tr.rows;
        const int items = tr.rows * P;
        float* rbuf = red + (it & 1) * (kGemvMaxTileRows * M * 2);
        for (int item = warp; item < items; item += kGemvWarps) {
            const int r = item / P, part = item - r * P;
            float acc[M], acc2[M];
#pragma unroll
            for (int m = 0; m < M; ++m) acc[m] = acc2[m] = 0.0f;
            const uint8_t* row = stage + size_t(r) * p.rowbytes;
            const uint8_t* row2 = row + p.stage_bytes / 2;
            // two block groups per iteration: independent loads in flight
            for (int g = part; g < groups; g += 2 * P) {
                const int b0 = g * 4 + blk_in_group;
                const int b1 = b0 + 4 * P;
                if (b0 < p.nb) {
                    BlockDot<QT, M>(row + b0 * kBB, xs + b0 * 32, kpad, sub, acc);
                    if constexpr (kDual) BlockDot<QT, M>(row2 + b0 * kBB, xs + b0 * 32, kpad, sub, acc2);
                }
                if (b1 < p.nb) {
                    BlockDot<QT, M>(row + b1 * kBB, xs + b1 * 32, kpad, sub, acc);
                    if constexpr (kDual) BlockDot<QT, M>(row2 + b1 * kBB, xs + b1 * 32, kpad, sub, acc2);
                }
            }
#pragma unroll
            for (int m = 0; m < M; ++m) {
                float v = WarpSum(acc[m]);
                float v2 = 0.0f;
                if constexpr (kDual) v2 = WarpSum(acc2[m]);
                if (lane == 0) {
                    // deterministic: partials of a row are combined in part order below
                    rbuf[(item * M + m) * 2] = v;
                    rbuf[(item * M + m) * 2 + 1] = v2;
                }
            }
        }
        __syncthreads();
        if (s_abort) {
            // Leave no bulk copy in flight into this CTA's shared memory: wait
            // (bounded) for the fills already issued for the next stages.
            if (tid == 0) {
                if (p.status) atomicExch(p.status, MLB_ERR_DEVICE_TIMEOUT);
                for (int k = 0; k < kGemvStages; ++k) {
                    const int tk = t + k * gridDim.x;
                    if (tk >= ntiles) break;
                    const int ik = it + k;
                    MbarWait(&bars[ik % kGemvStages], (ik / kGemvStages) & 1);
                }
            }
            break;
        }
        // stage s is free again: refill it with the tile kGemvStages ahead
        if (tid == 0) {
            int tn = t + kGemvStages * gridDim.x;
            if (tn < ntiles) IssueTile(p, LocateTile(p, tn, kDual), kDual, stage, &bars[s]);
        }
        // ---- epilogue: one thread per (row, m)
        const GemvSeg& sg = p.seg[tr.seg];
        for (int e = tid; e < tr.rows * M; e += kGemvThreads) {
            const int r = e / M, m = e - r * M;
            float v = 0.0f, v2 = 0.0f;
            for (int part = 0; part < P; ++part) {
                v += rbuf[((r * P + part) * M + m) * 2];
                if constexpr (kDual) v2 += rbuf[((r * P + part) * M + m) * 2 + 1];
            }
            const int n = tr.row0 + r;
            const size_t out = size_t(m) * p.y_stride + sg.out_offset + n;
            if constexpr (EPI == kEpiStore) {
                if (sg.bias) v += sg.bias[n];
                p.y[out] = v;
            } else if constexpr (EPI == kEpiResidual) {
                p.y[out] = v + p.residual[size_t(m) * p.res_stride + sg.out_offset + n];
            } else if constexpr (EPI == kEpiSwiglu) {
                float sig = 1.0f / (1.0f + expf(-v));
                p.y[out] = v * sig * v2;
            } else {  // kEpiArgmax (M == 1)
                p.y[out] = v;
                if (v > best_val || (v == best_val && n < best_idx)) {
                    best_val = v;
                    best_idx = n;
                }
            }
        }
    }

    if constexpr (EPI == kEpiArgmax) ArgmaxFinish(p, best_val, best_idx);
}

// Host-side planning of a GEMV launch: tile sizes, stage size and grid.
struct GemvPlan {
    bool ok = false;  // false: shape needs the fallback kernel
    int grid = 0;
    size_t smem = 0;
};

// Quantized linear for rows >= kTcMinRows on the tcgen05 tensor cores
// (tc05.cu); status receives MLB_ERR_DEVICE_TIMEOUT if a bounded wait expires.
// Up to kGemvMaxM rows one GEMV pass is faster; beyond, the GEMV would stream
// the weights once per kGemvMaxM rows while the tensor-core kernel's time
// hardly depends on the row count below 64.
// workspace: TcWorkspaceBytes(M, K, N, sm_count) bytes of device memory (a
// caller that captures the launch into a CUDA graph owns it), or null for the
// context's grow-only workspace.
constexpr int kTcMinRows = kGemvMaxM + 1;
// reuse_x: x and the workspace are those of the previous call on this stream
// and x has not changed since, so that call's x images are reused when the
// shapes match (the pre-pass is skipped); any mismatch runs the pre-pass.
void LaunchTcLinear(DeviceContext& c, int qtype, const float* x, const uint8_t* w, int M, int K, int N,
                    const float* bias, float* y, int* status, void* workspace = nullptr, bool reuse_x = false);
size_t TcWorkspaceBytes(int M, int K, int N, int sm_count);

// LaunchTcLinear first tries the integer-MMA linear (wide.cu: x's digit
// tables from one pre-pass, GGUF blocks straight from a bulk-copy ring,
// split-K sums in a deterministic pass) where it measured faster
// (WidePreferred: up to 32 rows, or up to kWideMaxRows rows on weights of at
// most 8 M elements); LaunchWideLinear returns false when the shape does not
// suit it (odd block count of Q8_0 / Q4_0, misaligned weights).  Its
// workspace (tables, partial sums) is part of TcWorkspaceBytes.
constexpr int kWideMaxRows = 64;
bool WidePreferred(int M, int K, int N);
bool LaunchWideLinear(DeviceContext& c, int qtype, const float* x, const uint8_t* w, int M, int K, int N,
                      const float* bias, float* y, int* status, void* workspace, bool reuse_x);
size_t WideWorkspaceBytes(int M, int K, int N, int sm_count, int max_smem);
// Several weight matrices (up to 3) that read the same x, same K and block
// type, in one launch of the integer-MMA linear (the x pre-pass once, the
// matrices' row groups side by side in the grid); false when the shape does
// not suit it.  Workspace: null for the context's grow-only workspace.
struct WideSeg {
    const uint8_t* w;
    const float* bias;
    float* y;
    int N;
};
bool LaunchWideLinearSegs(DeviceContext& c, int qtype, const float* x, int M, int K, const WideSeg* segs, int nseg,
                          int* status, void* workspace, bool reuse_x);

// Quantized linear over GGUF blocks for any row count (the GEMV up to
// kGemvMaxM rows at a time below kTcMinRows, the tensor cores above), on the
// context's stream; tc_workspace as for LaunchTcLinear.
void LinearRows(DeviceContext& c, int qtype, const float* x, const uint8_t* w, int rows, int K, int N,
                const float* bias, float* y, void* tc_workspace = nullptr, bool reuse_x = false);

// M = 1 launch of a decode-graph variant (pro/epi are GemvPrologue/GemvEpilogue).
void LaunchGemvDecode(int qtype, int pro, int epi, const GemvParams& p, const GemvPlan& plan,
                      cudaStream_t stream);

// ring_budget caps the bytes of the shared-memory weight ring (all stages).
GemvPlan PlanGemv(GemvParams& p, int qtype, int M, bool dual, int sm_count, int max_smem,
                  int ctas_per_sm, int ring_budget = 1 << 30);

// Fallback for shapes the bulk-copy kernel cannot take (unaligned weight
// base, rows longer than a stage): one warp per output row, direct loads.
template <int QT>
__global__ void GemvFallbackKernel(const float* x, const uint8_t* w, const float* bias, float* y,
                                   int M, int K, int N, int nb) {
    constexpr int kBB = QTraits<QT>::kBytes;
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= N * M) return;
    const int n = warp % N, m = warp / N;
    const float* xr = x + size_t(m) * K;
    const uint8_t* row = w + size_t(n) * nb * kBB;
    float acc = 0.0f;
    for (int k = lane; k < nb * 32; k += 32) {
        if (k >= K) break;
        const uint8_t* blk = row + (k >> 5) * kBB;
        int e = k & 31;
        float d = HalfBits(uint16_t(blk[0] | (blk[1] << 8)));
        float wv;
        if constexpr (QT == MLB_Q8_0) {
            wv = d * float(int8_t(blk[2 + e]));
        } else {
            constexpr int off = (QT == MLB_Q4_0) ? 2 : 4;
            int q = e < 16 ? (blk[off + e] & 15) : (blk[off + e - 16] >> 4);
            if constexpr (QT == MLB_Q4_0) wv = d * float(q - 8);
            else wv = d * float(q) + HalfBits(uint16_t(blk[2] | (blk[3] << 8)));
        }
        acc = fmaf(wv, xr[k], acc);
    }
    acc = WarpSum(acc);
    if (lane == 0) y[size_t(m) * N + n] = acc + (bias ? bias[n] : 0.0f);
}

}  // namespace mlb
