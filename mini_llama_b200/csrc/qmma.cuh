// Q8_0 GEMV on the tensor cores with exact integer arithmetic, over weights
// repacked into 16-row tiles ("R16 layout").
//
// R16 layout of a Q8_0 matrix [N, K] (nb = ceil(K/32) blocks per row, rows
// padded with zero rows to a multiple of 16):
//   row tile t = rows 16t..16t+15 is nb consecutive 544-byte chunks; chunk b
//   holds the 16 x 32 int8 quants of block column b (row i at byte 32*i, its
//   two 16-byte halves swapped when bit 2 of i is set, so ldmatrix reads are
//   bank-conflict free) followed by the 16 fp16 scales d[i] (bytes 512..543).
//   Same byte count as the GGUF blocks; every chunk is 16-byte aligned, so a
//   tile moves with one bulk copy and feeds ldmatrix directly.
//
// x is decomposed per 32-element block b into three signed int8 digit planes:
// with E the exponent of max|x_b| (max|x_b| < 2^E), X = rint(x * 2^(22-E))
// (|X| < 2^22) and X = D2*2^16 + D1*2^8 + D0, digits in [-128, 127].  One
// mma.m16n8k32.s8 per (16-row tile, block) yields the exact int32 sums
// S_j = sum_k q[r,k] * D_j[k]; the block's contribution to row r is
// d[r] * 2^(E-22) * (65536*S2 + 256*S1 + S0).  The only roundings are the
// rint of x (relative 2^-23 of the block maximum) and the fp32 combine, so the
// result is at least as accurate as an fp32 FMA chain.
//
// Digit columns of the MMA: column 4m+j holds digit plane j (j = 0: D2, 1: D1,
// 2: D0, 3: zero) of x row m; ceil(M/2) MMAs per block cover M <= 8 rows of x.
#pragma once

#include "qgemv.cuh"

namespace mlb {

constexpr int kR16Chunk = 544;

__host__ __device__ inline size_t R16Bytes(int rows, int cols) {
    return size_t((rows + 15) / 16) * ((cols + 31) / 32) * kR16Chunk;
}

// GGUF Q8_0 [N, nb] -> R16.  One thread per (row, block) of the padded rows.
// column_major = 1 orders the chunks by block column instead ("R16C": chunk
// (t, b) at b * ntiles + t), so one block column of every row tile -- the
// weights a split-K partial over 32 inputs needs -- is contiguous.
static __global__ void RepackQ80R16Kernel(const uint8_t* src, int rows, int cols, uint8_t* dst,
                                          int column_major) {
    const int nb = (cols + 31) / 32;
    const long long prow = (rows + 15) / 16 * 16LL;
    const long long total = prow * nb;
    for (long long idx = blockIdx.x * 1LL * blockDim.x + threadIdx.x; idx < total;
         idx += 1LL * gridDim.x * blockDim.x) {
        const int r = static_cast<int>(idx / nb), b = static_cast<int>(idx % nb);
        const int t = r >> 4, i = r & 15;
        const size_t ntiles = static_cast<size_t>((rows + 15) / 16);
        uint8_t* chunk = dst + (column_major ? size_t(b) * ntiles + t : size_t(t) * nb + b) * kR16Chunk;
        uint8_t q[32];
        uint16_t d = 0;
        if (r < rows) {
            const uint8_t* blk = src + (size_t(r) * nb + b) * 34;
            d = static_cast<uint16_t>(blk[0] | (blk[1] << 8));
            for (int k = 0; k < 32; ++k) q[k] = blk[2 + k];
        } else {
            for (int k = 0; k < 32; ++k) q[k] = 0;
        }
        const int swz = (i >> 2) & 1;
        for (int h = 0; h < 2; ++h)
            for (int k = 0; k < 16; ++k) chunk[32 * i + 16 * (h ^ swz) + k] = q[16 * h + k];
        chunk[512 + 2 * i] = d & 0xff;
        chunk[512 + 2 * i + 1] = d >> 8;
    }
}

__device__ __forceinline__ void LdMatrixX4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                           uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

__device__ __forceinline__ void MmaS8(int& d0, int& d1, int& d2, int& d3, uint32_t a0, uint32_t a1,
                                      uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
        "{%8, %9}, {%10, %11, %12, %13};"
        : "=r"(d0), "=r"(d1), "=r"(d2), "=r"(d3)
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0), "r"(0), "r"(0), "r"(0));
}

// Digit planes of x in shared memory: plane row (4m + j) of stride dstride
// bytes (a multiple of 16 plus 16, so the 8 column rows of a B-fragment load
// fall in different banks), and the per-block scale 2^(E-22) in sx[m][b].
__host__ __device__ inline int DigitStride(int nb) { return nb * 32 + 16; }

// Builds the digit planes of M rows of x (fp32 in shared memory, rows of
// kpad floats, zero padded) with one warp per (m, block).
template <int M>
__device__ __forceinline__ void BuildDigits(const float* xs, int kpad, int nb, int8_t* dig,
                                            float* sx) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nwarps = blockDim.x >> 5;
    const int dstride = DigitStride(nb);
    for (int item = warp; item < M * nb; item += nwarps) {
        const int m = item / nb, b = item - m * nb;
        const float v = xs[m * kpad + b * 32 + lane];
        const float mx = WarpMax(fabsf(v));
        const uint32_t mb = __float_as_uint(mx);
        int e = static_cast<int>((mb >> 23) & 0xff) - 126;  // mx < 2^e for normal mx
        int x = 0;
        float s = 0.0f;
        if (mx > 0.0f && e >= -104) {
            // 2^(22 - e) and 2^(e - 22) built from exponent bits (both normal)
            const float up = __uint_as_float(static_cast<uint32_t>(127 + 22 - e) << 23);
            s = __uint_as_float(static_cast<uint32_t>(127 + e - 22) << 23);
            x = __float2int_rn(v * up);
        }
        const int d0 = (x << 24) >> 24;
        const int x1 = (x - d0) >> 8;
        const int d1 = (x1 << 24) >> 24;
        const int d2 = (x1 - d1) >> 8;
        int8_t* base = dig + (4 * m) * dstride + b * 32 + lane;
        base[0] = static_cast<int8_t>(d2);
        base[dstride] = static_cast<int8_t>(d1);
        base[2 * dstride] = static_cast<int8_t>(d0);
        base[3 * dstride] = 0;
        if (lane == 0) sx[m * nb + b] = s;
    }
}

// Partial sums of one 16-row tile over the blocks b = first, first + step, ...
// acc[j][0..3]: rows (g, g) cols (2t, 2t+1) and rows (g+8, g+8) of MMA j.
template <int NJ>
__device__ __forceinline__ void TileDot(const uint8_t* tile, int nb, int first, int step,
                                        const int8_t* dig, int dstride, const float* sx, int M,
                                        float (&acc)[NJ][4]) {
    const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    // ldmatrix row address of this lane inside a chunk
    const int mi = lane >> 3;
    const int row = (lane & 7) + 8 * (mi & 1);
    const int half = mi >> 1;
    const uint32_t lrow = 32 * row + 16 * (half ^ ((row >> 2) & 1));
    const uint32_t tile_s = SmemAddr(tile);
    // digit weights of this lane's two columns
    float cw[NJ][2];
    int mrow[NJ];
#pragma unroll
    for (int j = 0; j < NJ; ++j) {
        const int c0 = 8 * j + 2 * t;
        mrow[j] = c0 >> 2;
        const int dg = c0 & 3;  // 0 or 2
        const bool live = mrow[j] < M;
        cw[j][0] = live ? (dg == 0 ? 65536.0f : 1.0f) : 0.0f;
        cw[j][1] = live ? (dg == 0 ? 256.0f : 0.0f) : 0.0f;
    }
    for (int b = first; b < nb; b += step) {
        const uint8_t* chunk = tile + size_t(b) * kR16Chunk;
        uint32_t a0, a1, a2, a3;
        LdMatrixX4(tile_s + b * kR16Chunk + lrow, a0, a1, a2, a3);
        const float dg = HalfBits(*reinterpret_cast<const uint16_t*>(chunk + 512 + 2 * g));
        const float dg8 = HalfBits(*reinterpret_cast<const uint16_t*>(chunk + 512 + 2 * (g + 8)));
#pragma unroll
        for (int j = 0; j < NJ; ++j) {
            const int col = 8 * j + g;  // B column this lane loads
            uint32_t b0 = 0, b1 = 0;
            if (col < 4 * M) {
                const int8_t* dp = dig + col * dstride + b * 32 + 4 * t;
                b0 = *reinterpret_cast<const uint32_t*>(dp);
                b1 = *reinterpret_cast<const uint32_t*>(dp + 16);
            }
            int c0, c1, c2, c3;
            MmaS8(c0, c1, c2, c3, a0, a1, a2, a3, b0, b1);
            const float s = mrow[j] < M ? sx[mrow[j] * nb + b] : 0.0f;
            const float vg = fmaf(static_cast<float>(c1), cw[j][1], static_cast<float>(c0) * cw[j][0]);
            const float vg8 = fmaf(static_cast<float>(c3), cw[j][1], static_cast<float>(c2) * cw[j][0]);
            acc[j][0] = fmaf(vg, dg * s, acc[j][0]);
            acc[j][2] = fmaf(vg8, dg8 * s, acc[j][2]);
        }
    }
}

}  // namespace mlb

namespace mlb {

// y[m, n] epilogue shared by the GEMV kernels.
template <int EPI>
__device__ __forceinline__ void GemvStoreOut(const GemvParams& p, const GemvSeg& sg, int m, int n,
                                             float v, float v2, float& best_val, int& best_idx) {
    const size_t out = size_t(m) * p.y_stride + sg.out_offset + n;
    if constexpr (EPI == kEpiStore) {
        if (sg.bias) v += sg.bias[n];
        p.y[out] = v;
    } else if constexpr (EPI == kEpiResidual) {
        p.y[out] = v + p.residual[size_t(m) * p.res_stride + sg.out_offset + n];
    } else if constexpr (EPI == kEpiSwiglu) {
        const float sig = 1.0f / (1.0f + expf(-v));
        p.y[out] = v * sig * v2;
    } else {  // kEpiArgmax (M == 1)
        p.y[out] = v;
        if (v > best_val || (v == best_val && n < best_idx)) {
            best_val = v;
            best_idx = n;
        }
    }
}

struct QmmaSmem {
    static __host__ __device__ size_t Bytes(int M, int nb, int stage_bytes, int nstages,
                                            int aux_floats) {
        const size_t kpad = size_t(nb) * 32;
        return size_t(nstages) * stage_bytes + 64 + M * kpad * 4 +
               size_t((aux_floats + 3) & ~3) * 4 + size_t(4 * M) * DigitStride(nb) +
               size_t((M * nb + 3) & ~3) * 4 + 2ull * 8 * 16 * M * 2 * 4 + 64;
    }
};

// Integer-MMA GEMV over R16 weights.  One work item = one 16-row tile (of
// every segment in turn; with kEpiSwiglu one tile of gate and the same tile of
// up).  Items stream through a shared-memory ring, one bulk copy each; the
// eight warps split the tile's K blocks and combine in shared memory.
template <int M, int PRO, int EPI>
__global__ void __launch_bounds__(256) QmmaGemvKernel(const GemvParams p) {
    constexpr bool kDual = (EPI == kEpiSwiglu);
    constexpr int NJ = (M + 1) / 2;
    constexpr int kWarps = 8;
    extern __shared__ __align__(128) uint8_t smem[];
    const int nst = p.nstages;
    const int kpad = p.nb * 32;
    const int dstride = DigitStride(p.nb);
    uint8_t* stages = smem;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + size_t(nst) * p.stage_bytes);
    float* xs = reinterpret_cast<float*>(smem + size_t(nst) * p.stage_bytes + 64);
    float* aux = xs + M * kpad;
    int8_t* dig = reinterpret_cast<int8_t*>(aux + ((p.aux_floats + 3) & ~3));
    float* sx = reinterpret_cast<float*>(dig + size_t(4 * M) * dstride);
    float* red = sx + ((M * p.nb + 3) & ~3);  // [2][kWarps][16][M][2]

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, t4 = lane & 3;
    const int ntiles = p.total_tiles;
    const uint32_t tile_bytes = static_cast<uint32_t>(p.nb) * kR16Chunk;

    auto locate = [&](int t, int& seg, int& ti) {
        seg = 0;
        const int nseg = kDual ? 1 : p.nseg;
        for (int s = 0; s < nseg; ++s) {
            if (t < p.seg[s].tiles) {
                seg = s;
                ti = t;
                return;
            }
            t -= p.seg[s].tiles;
        }
        ti = 0;
    };
    auto issue = [&](int t, int slot) {
        int seg, ti;
        locate(t, seg, ti);
        uint8_t* st = stages + size_t(slot) * p.stage_bytes;
        MbarExpectTx(&bars[slot], tile_bytes * (kDual ? 2 : 1));
        BulkLoad(st, p.seg[seg].w + size_t(ti) * tile_bytes, tile_bytes, &bars[slot]);
        if (kDual) BulkLoad(st + p.stage_bytes / 2, p.seg[1].w + size_t(ti) * tile_bytes, tile_bytes,
                            &bars[slot]);
    };

    __shared__ int s_abort;
    if (tid == 0) {
        s_abort = 0;
        for (int s = 0; s < nst; ++s) MbarInit(&bars[s], 1);
        FenceMbarInit();
    }
    __syncthreads();
    if (tid == 0)
        for (int s = 0; s < nst; ++s) {
            const int t = blockIdx.x + s * gridDim.x;
            if (t < ntiles) issue(t, s);
        }
    GridDepWait();
    GridDepLaunch();

    StageGemvX<M, PRO>(p, xs, aux, kpad);
    BuildDigits<M>(xs, kpad, p.nb, dig, sx);
    __syncthreads();

    float best_val = -INFINITY;
    int best_idx = 0x7fffffff;
    int it = 0;
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++it) {
        const int slot = it % nst;
        const uint32_t parity = (it / nst) & 1;
        uint8_t* st = stages + size_t(slot) * p.stage_bytes;
        int seg, ti;
        locate(t, seg, ti);
        if (!MbarWait(&bars[slot], parity)) s_abort = 1;

        float acc[NJ][4], acc2[NJ][4];
#pragma unroll
        for (int j = 0; j < NJ; ++j)
#pragma unroll
            for (int k = 0; k < 4; ++k) acc[j][k] = acc2[j][k] = 0.0f;
        TileDot<NJ>(st, p.nb, warp, kWarps, dig, dstride, sx, M, acc);
        if constexpr (kDual) TileDot<NJ>(st + p.stage_bytes / 2, p.nb, warp, kWarps, dig, dstride, sx, M, acc2);
        float* rb = red + (it & 1) * (kWarps * 16 * M * 2);
#pragma unroll
        for (int j = 0; j < NJ; ++j) {
            // columns 2t, 2t+1 of lanes t and t^1 belong to the same x row
            acc[j][0] += __shfl_xor_sync(0xffffffffu, acc[j][0], 1);
            acc[j][2] += __shfl_xor_sync(0xffffffffu, acc[j][2], 1);
            if constexpr (kDual) {
                acc2[j][0] += __shfl_xor_sync(0xffffffffu, acc2[j][0], 1);
                acc2[j][2] += __shfl_xor_sync(0xffffffffu, acc2[j][2], 1);
            }
            const int m = 2 * j + (t4 >> 1);
            if ((t4 & 1) == 0 && m < M) {
                rb[((warp * 16 + g) * M + m) * 2] = acc[j][0];
                rb[((warp * 16 + g + 8) * M + m) * 2] = acc[j][2];
                if constexpr (kDual) {
                    rb[((warp * 16 + g) * M + m) * 2 + 1] = acc2[j][0];
                    rb[((warp * 16 + g + 8) * M + m) * 2 + 1] = acc2[j][2];
                }
            }
        }
        __syncthreads();
        if (s_abort) {
            if (tid == 0) {
                if (p.status) atomicExch(p.status, MLB_ERR_DEVICE_TIMEOUT);
                for (int k = 0; k < nst; ++k) {
                    const int tk = t + k * gridDim.x;
                    if (tk >= ntiles) break;
                    MbarWait(&bars[(it + k) % nst], ((it + k) / nst) & 1);
                }
            }
            break;
        }
        if (tid == 0) {
            const int tn = t + nst * gridDim.x;
            if (tn < ntiles) issue(tn, slot);
        }
        const GemvSeg& sg = p.seg[seg];
        for (int e = tid; e < 16 * M; e += blockDim.x) {
            const int r = e / M, m = e - r * M;
            const int n = ti * 16 + r;
            if (n >= sg.rows) continue;
            float v = 0.0f, v2 = 0.0f;
#pragma unroll
            for (int w = 0; w < kWarps; ++w) {
                v += rb[((w * 16 + r) * M + m) * 2];
                if constexpr (kDual) v2 += rb[((w * 16 + r) * M + m) * 2 + 1];
            }
            GemvStoreOut<EPI>(p, sg, m, n, v, v2, best_val, best_idx);
        }
    }
    if constexpr (EPI == kEpiArgmax) ArgmaxFinish(p, best_val, best_idx);
}

GemvPlan PlanQmma(GemvParams& p, int M, bool dual, int sm_count, int max_smem, int ctas_per_sm,
                  int ring_budget);
void LaunchQmmaDecode(int pro, int epi, const GemvParams& p, const GemvPlan& plan,
                      cudaStream_t stream);
void LaunchQmmaStore(const GemvParams& p, const GemvPlan& plan, cudaStream_t stream);
void LaunchRepackQ80R16(DeviceContext& c, const void* src, int rows, int cols, void* dst,
                        bool column_major = false);

}  // namespace mlb
