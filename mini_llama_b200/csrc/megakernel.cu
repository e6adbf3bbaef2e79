// Persistent decode kernel (see megakernel.cuh for the design).
#include <algorithm>
#include <cmath>
#include <string>

#include "megakernel.cuh"

namespace mlb {
namespace {

constexpr int kMkSpin = 1 << 22;                    // poll bound of one dependency wait
constexpr uint64_t kMkWaitNs = 2000000000ull;       // bound of one shared-memory stage wait

__device__ __forceinline__ void ConsumerBar() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

__device__ __forceinline__ unsigned LdAcquire(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ int LdRelaxedInt(const int* p) {
    int v;
    asm volatile("ld.relaxed.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void RedAdd(float* p, float v) {
    asm volatile("red.global.add.f32 [%0], %1;" ::"l"(p), "f"(v) : "memory");
}

struct MkSmem {  // flags[0] is the CTA's abort flag (read by the producer warp too)
    uint8_t* ring;
    uint64_t* full;
    uint64_t* empty;
    float* xs;      // [dim] activation (then normalised)
    float* nw;      // [dim] norm weights
    int8_t* dig;    // 4 digit planes of xs, stride DigitStride(nb_dim)
    float* sx;      // [nb_dim] block scales of xs
    int8_t* vdig;   // 4 digit planes of a short vector (o of a head or ff of a block)
    float* vsx;     // [4] its block scales
    float* red;     // [8 warps][32 rows]
    float* vec;     // [4 * 128] small vectors (g, u / q, k, v, o)
    float* att;     // [8 warps][hd] attention partials
    float* sc;      // [kMkAttnChunk] scores / weights of a chunk of positions
    float* scratch; // [32]
    int* flags;     // [0] abort, [1] token
};

__device__ __forceinline__ int WorkerCount(int G, int T) { return T < G ? T : G; }

// Optional phase timeline: thread 0 stamps %globaltimer at the phase events of
// (step, layer) (layer n_layers = lm_head); skipped past the buffer's end.
__device__ __forceinline__ void Trace(const MegaParams& p, int step, int l, int ev) {
    if (p.trace == nullptr || threadIdx.x != 0) return;
    const size_t i =
        ((size_t(step) * (p.n_layers + 1) + l) * kMkTraceEvents + ev) * gridDim.x + blockIdx.x;
    if (i < p.trace_cap) p.trace[i] = GlobalTimerNs();
}

// ---------------------------------------------------------------- waits
// Consumer side: thread 0 polls the counter (acquire) until it reaches
// `target`; everybody then learns whether to go on.  Returns false on abort.
__device__ bool WaitCounter(const MegaParams& p, const MkSmem& s, int ctr, unsigned target) {
    if (threadIdx.x == 0) {
        bool ok = false;
        for (int it = 0; it < kMkSpin; ++it) {
            if (LdAcquire(p.counters + ctr) >= target) {
                ok = true;
                break;
            }
            if ((it & 255) == 255 && LdRelaxedInt(p.status) != 0) break;
        }
        if (!ok) {
            atomicCAS(p.status, 0, MLB_ERR_DEVICE_TIMEOUT);
            s.flags[0] = 1;
        }
    }
    ConsumerBar();
    return s.flags[0] == 0;
}

// Publishes this CTA's writes of the phase and increments the counter: the
// barrier orders every consumer thread's writes before thread 0's fence, which
// is cumulative over them, then the increment.
__device__ void Signal(const MegaParams& p, int ctr) {
    ConsumerBar();
    if (threadIdx.x == 0) {
        __threadfence();
        atomicAdd(p.counters + ctr, 1u);
    }
}

// Waits for the stage of chunk n (every consumer thread observes the phase),
// bounded; the barrier after it makes the go/abort decision uniform.
__device__ bool WaitChunk(const MegaParams& p, const MkSmem& s, unsigned n) {
    const int slot = n % kMkStages;
    const bool ok = MbarWaitFor(&s.full[slot], (n / kMkStages) & 1, kMkWaitNs, s.flags);
    if (!ok) {
        atomicCAS(p.status, 0, MLB_ERR_DEVICE_TIMEOUT);
        s.flags[0] = 1;
    }
    ConsumerBar();
    return s.flags[0] == 0;
}

// After every consumer thread is done with chunk n's stage.
__device__ void ReleaseChunk(const MkSmem& s, unsigned n) {
    ConsumerBar();
    if (threadIdx.x == 0)
        asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(SmemAddr(&s.empty[n % kMkStages]))
                     : "memory");
}

// ---------------------------------------------------------------- vectors
// n floats global -> shared (n % 4 == 0, both 16-byte aligned), L2 only.
__device__ void LoadVecCg(float* dst, const float* src, int n) {
    for (int i = threadIdx.x * 4; i < n; i += 256 * 4) CpAsync16(dst + i, src + i);
}

__device__ float ConsumerSum(float v, float* scratch) {
    v = WarpSum(v);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) scratch[warp] = v;
    ConsumerBar();
    float t = 0.0f;
#pragma unroll
    for (int w = 0; w < kMkConsumerWarps; ++w) t += scratch[w];
    ConsumerBar();
    return t;
}

__device__ float ConsumerMax(float v, float* scratch) {
    v = WarpMax(v);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) scratch[warp] = v;
    ConsumerBar();
    float t = -INFINITY;
#pragma unroll
    for (int w = 0; w < kMkConsumerWarps; ++w) t = fmaxf(t, scratch[w]);
    ConsumerBar();
    return t;
}

// In place x = x * rsqrt(mean(x^2) + eps) * w (the reference's product order).
__device__ void RmsNormSmem(float* x, const float* w, int n, float eps, float* scratch) {
    float ss = 0.0f;
    for (int i = threadIdx.x; i < n; i += 256) ss = fmaf(x[i], x[i], ss);
    const float tot = ConsumerSum(ss, scratch);
    const float scale = 1.0f / sqrtf(tot / static_cast<float>(n) + eps);
    for (int i = threadIdx.x; i < n; i += 256) x[i] = x[i] * scale * w[i];
    ConsumerBar();
}

// Digit planes (qmma.cuh) of nb blocks of x, one warp per block.
__device__ void DigitsMk(const float* x, int nb, int8_t* dig, int dstride, float* sx) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int b = warp; b < nb; b += kMkConsumerWarps) {
        const float v = x[b * 32 + lane];
        const float mx = WarpMax(fabsf(v));
        const int e = static_cast<int>((__float_as_uint(mx) >> 23) & 0xff) - 126;
        int xi = 0;
        float sc = 0.0f;
        if (mx > 0.0f && e >= -104) {
            const float up = __uint_as_float(static_cast<uint32_t>(127 + 22 - e) << 23);
            sc = __uint_as_float(static_cast<uint32_t>(127 + e - 22) << 23);
            xi = __float2int_rn(v * up);
        }
        const int d0 = (xi << 24) >> 24;
        const int x1 = (xi - d0) >> 8;
        const int d1 = (x1 << 24) >> 24;
        const int d2 = (x1 - d1) >> 8;
        int8_t* base = dig + b * 32 + lane;
        base[0] = static_cast<int8_t>(d2);
        base[dstride] = static_cast<int8_t>(d1);
        base[2 * dstride] = static_cast<int8_t>(d0);
        base[3 * dstride] = 0;
        if (lane == 0) sx[b] = sc;
    }
    ConsumerBar();
}

// ---------------------------------------------------------------- MMA pieces
struct LaneMma {
    uint32_t lrow;  // ldmatrix row offset inside a chunk
    float cw0, cw1; // digit weights of this lane's two columns (M = 1)
    int g, t;
};

__device__ __forceinline__ LaneMma MakeLane() {
    LaneMma l;
    const int lane = threadIdx.x & 31;
    l.g = lane >> 2;
    l.t = lane & 3;
    const int mi = lane >> 3;
    const int row = (lane & 7) + 8 * (mi & 1);
    const int half = mi >> 1;
    l.lrow = 32 * row + 16 * (half ^ ((row >> 2) & 1));
    l.cw0 = l.t == 0 ? 65536.0f : (l.t == 1 ? 1.0f : 0.0f);
    l.cw1 = l.t == 0 ? 256.0f : 0.0f;
    return l;
}

// One chunk (16 rows x 32 inputs) times one block of digits: adds the scaled
// contributions of rows g and g + 8 (before the lane-pair combine).
__device__ __forceinline__ void ChunkMma(const LaneMma& L, const uint8_t* chunk, const int8_t* dblk,
                                         int dstride, float sxb, float& vg, float& vg8) {
    uint32_t a0, a1, a2, a3;
    LdMatrixX4(SmemAddr(chunk) + L.lrow, a0, a1, a2, a3);
    uint32_t b0 = 0, b1 = 0;
    if (L.g < 4) {
        const int8_t* dp = dblk + L.g * dstride + 4 * L.t;
        b0 = *reinterpret_cast<const uint32_t*>(dp);
        b1 = *reinterpret_cast<const uint32_t*>(dp + 16);
    }
    int c0, c1, c2, c3;
    MmaS8(c0, c1, c2, c3, a0, a1, a2, a3, b0, b1);
    const float dg = HalfBits(*reinterpret_cast<const uint16_t*>(chunk + 512 + 2 * L.g));
    const float dg8 = HalfBits(*reinterpret_cast<const uint16_t*>(chunk + 512 + 2 * (L.g + 8)));
    const float v0 = fmaf(static_cast<float>(c1), L.cw1, static_cast<float>(c0) * L.cw0);
    const float v1 = fmaf(static_cast<float>(c3), L.cw1, static_cast<float>(c2) * L.cw0);
    vg = fmaf(v0, dg * sxb, vg);
    vg8 = fmaf(v1, dg8 * sxb, vg8);
}

// Row tiles of a stage (tiles_in_stage x nb chunks, row-tile major) against
// the digits of xs; the eight warps split the work by (tile, block); results
// (one value per row) land in s.red as [warp][tile * 16 + row].  Returns with
// the partials written (no barrier).
__device__ void RowTilesDot(const MkSmem& s, const LaneMma& L, const uint8_t* stage, int ntile, int nb,
                            int dstride) {
    const int warp = threadIdx.x >> 5;
    const int wpt = kMkConsumerWarps / ntile;  // warps per tile (ntile in {1, 2})
    const int tile = warp / wpt, part = warp % wpt;
    float vg = 0.0f, vg8 = 0.0f;
    const uint8_t* tb = stage + size_t(tile) * nb * kR16Chunk;
    for (int b = part; b < nb; b += wpt)
        ChunkMma(L, tb + size_t(b) * kR16Chunk, s.dig + b * 32, dstride, s.sx[b], vg, vg8);
    vg += __shfl_xor_sync(0xffffffffu, vg, 1);
    vg8 += __shfl_xor_sync(0xffffffffu, vg8, 1);
    if (L.t == 0) {
        s.red[warp * 32 + tile * 16 + L.g] = vg;
        s.red[warp * 32 + tile * 16 + L.g + 8] = vg8;
    }
}

// Sum of the partials of row r of tile `tile` (after a barrier).
__device__ __forceinline__ float RowTotal(const MkSmem& s, int ntile, int tile, int r) {
    const int wpt = kMkConsumerWarps / ntile;
    float v = 0.0f;
    for (int w = tile * wpt; w < (tile + 1) * wpt; ++w) v += s.red[w * 32 + tile * 16 + r];
    return v;
}

// A block column (ntiles chunks of 16 rows x 32 inputs) times one block of
// digits: out[row] += value (+ addend[row]) by red.add; a warp per row tile.
__device__ void ColumnDotAdd(const LaneMma& L, const uint8_t* column, int ntiles, int nrows,
                             const int8_t* dblk, int dstride, float sxb, float* out,
                             const float* addend) {
    const int warp = threadIdx.x >> 5;
    for (int t = warp; t < ntiles; t += kMkConsumerWarps) {
        float vg = 0.0f, vg8 = 0.0f;
        ChunkMma(L, column + size_t(t) * kR16Chunk, dblk, dstride, sxb, vg, vg8);
        vg += __shfl_xor_sync(0xffffffffu, vg, 1);
        vg8 += __shfl_xor_sync(0xffffffffu, vg8, 1);
        if (L.t == 0) {
            const int r0 = t * 16 + L.g, r1 = r0 + 8;
            if (r0 < nrows) RedAdd(out + r0, vg + (addend ? __ldcg(addend + r0) : 0.0f));
            if (r1 < nrows) RedAdd(out + r1, vg8 + (addend ? __ldcg(addend + r1) : 0.0f));
        }
    }
}

// ---------------------------------------------------------------- schedule
// The chunk sequence of one CTA for one step; the producer issues it, the
// consumers consume it, in the same order.
struct Chunk {
    const uint8_t* src;
    uint32_t bytes;
};

template <typename F>
__device__ void ForEachChunk(const MegaParams& p, int c, int G, F&& f) {
    const int nb_dim = p.dim / 32;
    const uint32_t tile_b = static_cast<uint32_t>(nb_dim) * kR16Chunk;
    const int tq = (p.qd + 15) / 16, tk = (p.kd + 15) / 16;
    const int t_qkv = tq + 2 * tk;
    const int ntiles_dim = (p.dim + 15) / 16;
    const uint32_t col_b = static_cast<uint32_t>(ntiles_dim) * kR16Chunk;
    const int nj = p.hidden / 32;
    const int t_lm = (p.vocab + 15) / 16;
    const int bph = p.hd / 32;  // wo block columns per head
    for (int l = 0; l < p.n_layers; ++l) {
        const MegaLayer& L = p.layers[l];
        for (int t = c; t < t_qkv; t += G) {
            const int seg = t < tq ? 0 : (t < tq + tk ? 1 : 2);
            const int ti = seg == 0 ? t : (seg == 1 ? t - tq : t - tq - tk);
            f(Chunk{L.wqkv[seg] + size_t(ti) * tile_b, tile_b});
        }
        for (int h = G - 1 - c; h < p.n_heads; h += G)
            for (int j = 0; j < bph; ++j)
                f(Chunk{L.wo + size_t(h * bph + j) * col_b, col_b});
        for (int j = c; j < nj; j += G) {
            f(Chunk{L.gate + size_t(2 * j) * tile_b, 2 * tile_b});
            f(Chunk{L.up + size_t(2 * j) * tile_b, 2 * tile_b});
            f(Chunk{L.down + size_t(j) * col_b, col_b});
        }
    }
    // lm_head: two row tiles per stage
    for (int t2 = c; 2 * t2 < t_lm; t2 += G)
        f(Chunk{p.lm_head + size_t(2 * t2) * tile_b, (2 * t2 + 1 < t_lm ? 2u : 1u) * tile_b});
}

__device__ void Producer(const MegaParams& p, const MkSmem& s) {
    if ((threadIdx.x & 31) != 0) return;
    const int G = gridDim.x, c = blockIdx.x;
    unsigned n = 0;
    bool abort = false;
    for (int step = 0; step < p.n_steps && !abort; ++step) {
        ForEachChunk(p, c, G, [&](const Chunk& ch) {
            if (abort) return;
            const int slot = n % kMkStages;
            if (n >= static_cast<unsigned>(kMkStages)) {
                if (!MbarWaitFor(&s.empty[slot], ((n / kMkStages) - 1) & 1, kMkWaitNs, s.flags)) {
                    abort = true;
                    atomicCAS(p.status, 0, MLB_ERR_DEVICE_TIMEOUT);
                    return;
                }
            }
            MbarExpectTx(&s.full[slot], ch.bytes);
            BulkLoad(s.ring + size_t(slot) * p.stage_bytes, ch.src, ch.bytes, &s.full[slot]);
            ++n;
        });
    }
    // Drain: wait (bounded) until every stage issued has landed, so no copy
    // into this CTA's shared memory is in flight when it exits.
    const unsigned first = n > static_cast<unsigned>(kMkStages) ? n - kMkStages : 0;
    for (unsigned k = first; k < n; ++k)
        MbarWaitFor(&s.full[k % kMkStages], (k / kMkStages) & 1, kMkWaitNs, nullptr);
}

// ---------------------------------------------------------------- consumers
__device__ void Consumers(const MegaParams& p, const MkSmem& s) {
    const int G = gridDim.x, c = blockIdx.x;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const LaneMma L = MakeLane();
    const int nb_dim = p.dim / 32;
    const int dstride = DigitStride(nb_dim);
    const int vstride = DigitStride(p.hd / 32 > 1 ? p.hd / 32 : 1);
    const int tq = (p.qd + 15) / 16, tk = (p.kd + 15) / 16;
    const int t_qkv = tq + 2 * tk;
    const int ntiles_dim = (p.dim + 15) / 16;
    const int nj = p.hidden / 32;
    const int t_lm = (p.vocab + 15) / 16;
    const int bph = p.hd / 32;
    // signals per step: one per QKV worker CTA, one per head, one per FFN
    // worker CTA; every CTA takes one LM ticket
    const unsigned w_qkv = WorkerCount(G, t_qkv), w_att = p.n_heads, w_ffn = WorkerCount(G, nj),
                   w_lm = G;
    const int ctr_lm_ticket = 3 * p.n_layers, ctr_token = 3 * p.n_layers + 1;
    unsigned n = 0;  // chunk counter (same sequence as the producer)

    for (int step = 0; step < p.n_steps; ++step) {
        const int pos = p.start_pos + step;
        const unsigned k1 = static_cast<unsigned>(step + 1);
        for (int l = 0; l < p.n_layers; ++l) {
            const MegaLayer& Lw = p.layers[l];
            float* xin = p.xbuf[l & 1];
            float* xout = p.xbuf[(l + 1) & 1];
            // ---------------- QKV
            if (c < t_qkv) {
                // independent of the wait: norm weights and the bias rows of
                // this CTA's first 32 tiles (s.vec[16 * i + r])
                LoadVecCg(s.nw, Lw.attn_norm, p.dim);
                for (int t = c, i = 0; t < t_qkv && i < 32; t += G, ++i) {
                    const int seg = t < tq ? 0 : (t < tq + tk ? 1 : 2);
                    const int ti = seg == 0 ? t : (seg == 1 ? t - tq : t - tq - tk);
                    if (Lw.bias[seg] && tid < 4) CpAsync16(s.vec + 16 * i + 4 * tid, Lw.bias[seg] + ti * 16 + 4 * tid);
                }
                if (l == 0) {
                    if (step > 0 && !WaitCounter(p, s, ctr_token, k1 - 1)) return;
                } else if (!WaitCounter(p, s, 3 * (l - 1) + 2, k1 * w_ffn)) {
                    return;
                }
                Trace(p, step, l, 0);
                if (l == 0) {
                    if (tid == 0) s.flags[1] = __ldcg(p.hist + pos);
                    ConsumerBar();
                    int tok = s.flags[1];
                    if (tok < 0 || tok >= p.vocab) {
                        if (tid == 0) atomicCAS(p.status, 0, MLB_ERR_OUT_OF_RANGE);
                        tok = 0;
                    }
                    LoadVecCg(s.xs, p.embedding + size_t(tok) * p.dim, p.dim);
                } else {
                    LoadVecCg(s.xs, xin, p.dim);
                }
                CpAsyncWaitAll();
                ConsumerBar();
                if (c == 0) {  // x_mid starts as x; the next x starts at zero
                    for (int i = tid; i < p.dim; i += 256) {
                        p.xmid[i] = s.xs[i];
                        xout[i] = 0.0f;
                    }
                }
                RmsNormSmem(s.xs, s.nw, p.dim, p.eps, s.scratch);
                DigitsMk(s.xs, nb_dim, s.dig, dstride, s.sx);
                Trace(p, step, l, 11);
                for (int t = c, i = 0; t < t_qkv; t += G, ++i) {
                    const int seg = t < tq ? 0 : (t < tq + tk ? 1 : 2);
                    const int ti = seg == 0 ? t : (seg == 1 ? t - tq : t - tq - tk);
                    const int rows = seg == 0 ? p.qd : p.kd;
                    const int off = seg == 0 ? 0 : (seg == 1 ? p.qd : p.qd + p.kd);
                    if (!WaitChunk(p, s, n)) return;
                    RowTilesDot(s, L, s.ring + size_t(n % kMkStages) * p.stage_bytes, 1, nb_dim, dstride);
                    ReleaseChunk(s, n);
                    ++n;
                    if (tid < 16) {
                        const int r = ti * 16 + tid;
                        if (r < rows) {
                            float v = RowTotal(s, 1, 0, tid);
                            if (Lw.bias[seg]) v += i < 32 ? s.vec[16 * i + tid] : Lw.bias[seg][r];
                            p.qkv[off + r] = v;
                        }
                    }
                    ConsumerBar();
                }
                Trace(p, step, l, 10);
                Signal(p, 3 * l + 0);
                Trace(p, step, l, 1);
            }
            // ---------------- attention + O projection, one query head
            for (int h = G - 1 - c; h < p.n_heads; h += G) {
                const int hd = p.hd, half = hd / 2, kvh = h / p.group;
                const size_t pstride = size_t(p.n_kv) * hd;
                const size_t lbase = size_t(l) * p.max_seq * pstride + size_t(kvh) * hd;
                // pull this head's cached K and V rows into L2 while QKV runs
                for (int pp = tid; pp < 2 * pos; pp += 256) {
                    const float* row = (pp < pos ? p.kc : p.vc) + lbase + size_t(pp < pos ? pp : pp - pos) * pstride;
                    BulkPrefetchL2(row, static_cast<uint32_t>(hd) * 4);
                }
                // RoPE rows of this position (s.att is free until the values pass)
                float* ct = s.att;
                float* st = s.att + half;
                LoadVecCg(ct, p.rope_cos + size_t(pos) * half, half);
                LoadVecCg(st, p.rope_sin + size_t(pos) * half, half);
                if (!WaitCounter(p, s, 3 * l + 0, k1 * w_qkv)) return;
                Trace(p, step, l, 2);
                float* q = s.vec;
                float* kn = s.vec + 128;
                float* vn = s.vec + 256;
                float* o = s.vec + 384;
                LoadVecCg(q, p.qkv + h * hd, hd);
                LoadVecCg(kn, p.qkv + p.qd + kvh * hd, hd);
                LoadVecCg(vn, p.qkv + p.qd + p.kd + kvh * hd, hd);
                for (int i = tid; i < hd; i += 256) o[i] = 0.0f;
                CpAsyncWaitAll();
                ConsumerBar();
                // RoPE with the reference CPU tables (bit-exact with them)
                for (int j = tid; j < half; j += 256) {
                    const int a = p.neox ? j : 2 * j, b2 = p.neox ? j + half : 2 * j + 1;
                    const float cs = ct[j], sn = st[j];
                    float x0 = q[a], x1 = q[b2];
                    q[a] = __fsub_rn(__fmul_rn(x0, cs), __fmul_rn(x1, sn));
                    q[b2] = __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, cs));
                    x0 = kn[a];
                    x1 = kn[b2];
                    kn[a] = __fsub_rn(__fmul_rn(x0, cs), __fmul_rn(x1, sn));
                    kn[b2] = __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, cs));
                }
                ConsumerBar();
                if (h % p.group == 0)  // the group's first head stores this token's k, v
                    for (int i = tid; i < hd; i += 256) {
                        p.kc[lbase + size_t(pos) * pstride + i] = kn[i];
                        p.vc[lbase + size_t(pos) * pstride + i] = vn[i];
                    }
                // Positions 0..pos in chunks of 256 with a running max and sum.
                // Scores: a thread per position (its K row as float4 loads, all
                // in flight together).  Values: a warp per 32 positions, lanes
                // over (row, float4 column), every row load in flight together.
                const int lpr = hd / 4, rpi = 32 / lpr;  // lanes per row, rows per pass
                const int rsub = lane / lpr, col = lane % lpr;
                float m_run = -INFINITY, l_run = 0.0f;
                for (int base = 0; base <= pos; base += kMkAttnChunk) {
                    const int pp = base + tid;
                    float sc = -INFINITY;
                    if (pp <= pos) {
                        const float4* kr = reinterpret_cast<const float4*>(
                            pp == pos ? kn : p.kc + lbase + size_t(pp) * pstride);
                        const float4* q4 = reinterpret_cast<const float4*>(q);
                        float dot = 0.0f;
                        if (pp == pos) {
                            for (int i = 0; i < lpr; ++i) {
                                const float4 kv = kr[i], qv = q4[i];
                                dot = fmaf(qv.x, kv.x, dot);
                                dot = fmaf(qv.y, kv.y, dot);
                                dot = fmaf(qv.z, kv.z, dot);
                                dot = fmaf(qv.w, kv.w, dot);
                            }
                        } else {
                            for (int i0 = 0; i0 < lpr; i0 += 8) {  // 8 loads in flight
                                float4 kv[8];
#pragma unroll
                                for (int i = 0; i < 8; ++i)
                                    if (i0 + i < lpr) kv[i] = __ldcg(kr + i0 + i);
#pragma unroll
                                for (int i = 0; i < 8; ++i)
                                    if (i0 + i < lpr) {
                                        const float4 qv = q4[i0 + i];
                                        dot = fmaf(qv.x, kv[i].x, dot);
                                        dot = fmaf(qv.y, kv[i].y, dot);
                                        dot = fmaf(qv.z, kv[i].z, dot);
                                        dot = fmaf(qv.w, kv[i].w, dot);
                                    }
                            }
                        }
                        sc = dot * p.scale;
                    }
                    // this warp's first 16 V row pieces, loaded before the
                    // softmax reductions so their latency overlaps them
                    const int r0 = base + warp * 32;
                    float4 vpre[16];
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        const int r = r0 + i * rpi + rsub;
                        vpre[i] = make_float4(0.f, 0.f, 0.f, 0.f);
                        if (i < lpr && r < pos)
                            vpre[i] = __ldcg(reinterpret_cast<const float4*>(p.vc + lbase + size_t(r) * pstride) + col);
                        else if (i < lpr && r == pos)
                            vpre[i] = reinterpret_cast<const float4*>(vn)[col];
                    }
                    const float mc = ConsumerMax(sc, s.scratch);
                    const float mnew = fmaxf(m_run, mc);
                    const float corr = m_run == -INFINITY ? 0.0f : expf(m_run - mnew);
                    const float wgt = pp <= pos ? expf(sc - mnew) : 0.0f;
                    s.sc[tid] = wgt;
                    const float lc = ConsumerSum(wgt, s.scratch);  // barriers publish s.sc
                    l_run = fmaf(l_run, corr, lc);
                    m_run = mnew;
                    // weighted V rows of this warp's 32 positions
                    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        const int r = r0 + i * rpi + rsub;
                        if (i < lpr && r <= pos) {
                            const float w = s.sc[r - base];
                            acc.x = fmaf(w, vpre[i].x, acc.x);
                            acc.y = fmaf(w, vpre[i].y, acc.y);
                            acc.z = fmaf(w, vpre[i].z, acc.z);
                            acc.w = fmaf(w, vpre[i].w, acc.w);
                        }
                    }
                    for (int i0 = 16; i0 < lpr; i0 += 8) {  // rows r0 + i * rpi + rsub, 16 <= i < lpr
                        float4 vv[8];
#pragma unroll
                        for (int i = 0; i < 8; ++i) {
                            const int r = r0 + (i0 + i) * rpi + rsub;
                            vv[i] = make_float4(0.f, 0.f, 0.f, 0.f);
                            if (i0 + i < lpr && r < pos)
                                vv[i] = __ldcg(reinterpret_cast<const float4*>(p.vc + lbase + size_t(r) * pstride) + col);
                            else if (i0 + i < lpr && r == pos)
                                vv[i] = reinterpret_cast<const float4*>(vn)[col];
                        }
#pragma unroll
                        for (int i = 0; i < 8; ++i) {
                            const int r = r0 + (i0 + i) * rpi + rsub;
                            if (i0 + i < lpr && r <= pos) {
                                const float w = s.sc[r - base];
                                acc.x = fmaf(w, vv[i].x, acc.x);
                                acc.y = fmaf(w, vv[i].y, acc.y);
                                acc.z = fmaf(w, vv[i].z, acc.z);
                                acc.w = fmaf(w, vv[i].w, acc.w);
                            }
                        }
                    }
                    for (int off = lpr; off < 32; off <<= 1) {
                        acc.x += __shfl_xor_sync(0xffffffffu, acc.x, off);
                        acc.y += __shfl_xor_sync(0xffffffffu, acc.y, off);
                        acc.z += __shfl_xor_sync(0xffffffffu, acc.z, off);
                        acc.w += __shfl_xor_sync(0xffffffffu, acc.w, off);
                    }
                    if (rsub == 0) reinterpret_cast<float4*>(s.att + warp * hd)[col] = acc;
                    ConsumerBar();
                    for (int d = tid; d < hd; d += 256) {
                        float t = 0.0f;
#pragma unroll
                        for (int w = 0; w < kMkConsumerWarps; ++w) t += s.att[w * hd + d];
                        o[d] = fmaf(o[d], corr, t);
                    }
                    ConsumerBar();
                }
                for (int d = tid; d < hd; d += 256) o[d] = o[d] / l_run;
                Trace(p, step, l, 8);
                ConsumerBar();
                DigitsMk(o, bph, s.vdig, vstride, s.vsx);
                for (int j = 0; j < bph; ++j) {
                    if (!WaitChunk(p, s, n)) return;
                    ColumnDotAdd(L, s.ring + size_t(n % kMkStages) * p.stage_bytes, ntiles_dim, p.dim,
                                 s.vdig + j * 32, vstride, s.vsx[j], p.xmid, nullptr);
                    ReleaseChunk(s, n);
                    ++n;
                }
                Trace(p, step, l, 9);
                Signal(p, 3 * l + 1);
                Trace(p, step, l, 3);
            }
            // ---------------- FFN: gate/up rows of a hidden block, SwiGLU, w_down column
            if (c < nj) {
                LoadVecCg(s.nw, Lw.ffn_norm, p.dim);  // independent of the wait
                if (!WaitCounter(p, s, 3 * l + 1, k1 * w_att)) return;
                Trace(p, step, l, 4);
                LoadVecCg(s.xs, p.xmid, p.dim);
                CpAsyncWaitAll();
                ConsumerBar();
                RmsNormSmem(s.xs, s.nw, p.dim, p.eps, s.scratch);
                DigitsMk(s.xs, nb_dim, s.dig, dstride, s.sx);
                Trace(p, step, l, 7);
                float* gv = s.vec;
                float* uv = s.vec + 32;
                float* ff = s.vec + 64;
                for (int j = c; j < nj; j += G) {
                    for (int part = 0; part < 2; ++part) {
                        if (!WaitChunk(p, s, n)) return;
                        RowTilesDot(s, L, s.ring + size_t(n % kMkStages) * p.stage_bytes, 2, nb_dim, dstride);
                        ReleaseChunk(s, n);
                        ++n;
                        if (tid < 32) (part == 0 ? gv : uv)[tid] = RowTotal(s, 2, tid >> 4, tid & 15);
                        ConsumerBar();
                    }
                    if (tid < 32) {
                        const float v = gv[tid];
                        const float sig = 1.0f / (1.0f + expf(-v));
                        ff[tid] = v * sig * uv[tid];
                    }
                    ConsumerBar();
                    DigitsMk(ff, 1, s.vdig, vstride, s.vsx);
                    if (!WaitChunk(p, s, n)) return;
                    ColumnDotAdd(L, s.ring + size_t(n % kMkStages) * p.stage_bytes, ntiles_dim, p.dim,
                                 s.vdig, vstride, s.vsx[0], xout, j == 0 ? p.xmid : nullptr);
                    ReleaseChunk(s, n);
                    ++n;
                }
                Trace(p, step, l, 6);
                Signal(p, 3 * l + 2);
                Trace(p, step, l, 5);
            }
        }
        // ---------------- lm_head + arg-max
        LoadVecCg(s.nw, p.final_norm, p.dim);  // independent of the wait
        if (!WaitCounter(p, s, 3 * (p.n_layers - 1) + 2, k1 * w_ffn)) return;
        Trace(p, step, p.n_layers, 0);
        float* xfin = p.xbuf[p.n_layers & 1];
        LoadVecCg(s.xs, xfin, p.dim);
        CpAsyncWaitAll();
        ConsumerBar();
        RmsNormSmem(s.xs, s.nw, p.dim, p.eps, s.scratch);
        DigitsMk(s.xs, nb_dim, s.dig, dstride, s.sx);
        float best = -INFINITY;
        int besti = 0x7fffffff;
        for (int t2 = c; 2 * t2 < t_lm; t2 += G) {
            // a lone last tile leaves stale bytes in the stage's second half;
            // its rows are past the vocabulary and skipped
            if (!WaitChunk(p, s, n)) return;
            RowTilesDot(s, L, s.ring + size_t(n % kMkStages) * p.stage_bytes, 2, nb_dim, dstride);
            ReleaseChunk(s, n);
            ++n;
            if (tid < 32) {
                const int r = (2 * t2 + (tid >> 4)) * 16 + (tid & 15);
                if (r < p.vocab) {
                    const float v = RowTotal(s, 2, tid >> 4, tid & 15);
                    p.logits[r] = v;
                    if (v > best || (v == best && r < besti)) {
                        best = v;
                        besti = r;
                    }
                }
            }
            ConsumerBar();
        }
        // CTA arg-max (first maximum) over the 32 candidate threads
        if (warp == 0) {
            for (int o = 16; o > 0; o >>= 1) {
                const float ov = __shfl_xor_sync(0xffffffffu, best, o);
                const int oi = __shfl_xor_sync(0xffffffffu, besti, o);
                if (ov > best || (ov == best && oi < besti)) {
                    best = ov;
                    besti = oi;
                }
            }
            if (lane == 0) {
                p.am_val[c] = best;
                p.am_idx[c] = besti;
            }
        }
        __threadfence();
        ConsumerBar();
        if (tid == 0) {
            const unsigned ticket = atomicAdd(p.counters + ctr_lm_ticket, 1u);
            s.flags[1] = ticket == k1 * w_lm - 1;
        }
        ConsumerBar();
        Trace(p, step, p.n_layers, 1);
        if (s.flags[1] && warp == 0) {  // last CTA of the step: pick the token
            __threadfence();
            float bv = -INFINITY;
            int bi = 0x7fffffff;
            for (int cc = lane; cc < static_cast<int>(w_lm); cc += 32) {
                const float v = __ldcg(p.am_val + cc);
                const int i = __ldcg(p.am_idx + cc);
                if (v > bv || (v == bv && i < bi)) {
                    bv = v;
                    bi = i;
                }
            }
            for (int o = 16; o > 0; o >>= 1) {
                const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                if (ov > bv || (ov == bv && oi < bi)) {
                    bv = ov;
                    bi = oi;
                }
            }
            if (lane == 0) {
                const int tok = bi == 0x7fffffff ? 0 : bi;
                if (pos + 1 >= p.gen_from && pos + 1 <= p.max_seq) p.hist[pos + 1] = tok;
                *p.next_token = tok;
                __threadfence();
                atomicAdd(p.counters + ctr_token, 1u);
            }
        }
        ConsumerBar();
    }
}

// 9 warps: one SM sub-partition holds 3 of them, so 168 registers a thread
// at most (16384 / 96, in steps of 8)
__global__ void __launch_bounds__(kMkThreads, 1) MegaDecodeKernel(const MegaParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int nb_dim = p.dim / 32;
    MkSmem s;
    size_t off = 0;
    auto take = [&](size_t bytes) {
        uint8_t* ptr = smem + off;
        off += (bytes + 127) & ~size_t(127);
        return ptr;
    };
    s.ring = take(size_t(kMkStages) * p.stage_bytes);
    s.full = reinterpret_cast<uint64_t*>(take(8 * kMkStages));
    s.empty = reinterpret_cast<uint64_t*>(take(8 * kMkStages));
    s.xs = reinterpret_cast<float*>(take(4 * size_t(p.dim)));
    s.nw = reinterpret_cast<float*>(take(4 * size_t(p.dim)));
    s.dig = reinterpret_cast<int8_t*>(take(4 * size_t(DigitStride(nb_dim))));
    s.sx = reinterpret_cast<float*>(take(4 * size_t(nb_dim)));
    s.vdig = reinterpret_cast<int8_t*>(take(4 * size_t(DigitStride(4))));
    s.vsx = reinterpret_cast<float*>(take(16));
    s.red = reinterpret_cast<float*>(take(4 * 8 * 32));
    s.vec = reinterpret_cast<float*>(take(4 * 512));
    s.att = reinterpret_cast<float*>(take(4 * 8 * 128));
    s.sc = reinterpret_cast<float*>(take(4 * kMkAttnChunk));
    s.scratch = reinterpret_cast<float*>(take(4 * 32));
    s.flags = reinterpret_cast<int*>(take(16));
    if (threadIdx.x == 0) {
        for (int i = 0; i < kMkStages; ++i) {
            MbarInit(&s.full[i], 1);
            MbarInit(&s.empty[i], 1);
        }
        FenceMbarInit();
        s.flags[0] = 0;
        s.flags[1] = 0;
    }
    __syncthreads();
    if (threadIdx.x >= kMkConsumerWarps * 32) {
        Producer(p, s);  // stops early when the consumers set flags[0]
    } else {
        Consumers(p, s);
    }
}

}  // namespace

size_t MegaSmemBytes(const MegaParams& p) {
    auto r = [](size_t b) { return (b + 127) & ~size_t(127); };
    const int nb_dim = p.dim / 32;
    return r(size_t(kMkStages) * p.stage_bytes) + r(8 * kMkStages) * 2 + r(4 * size_t(p.dim)) * 2 +
           r(4 * size_t(DigitStride(nb_dim))) + r(4 * size_t(nb_dim)) + r(4 * size_t(DigitStride(4))) +
           r(16) + r(4 * 8 * 32) + r(4 * 512) + r(4 * 8 * 128) + r(4 * kMkAttnChunk) + r(4 * 32) + r(16) + 128;
}

std::string MegaFits(const MegaParams& p, size_t smem, int sm_count) {
    (void)p;
    if (sm_count < 1) return "no SMs";
    cudaError_t e = cudaFuncSetAttribute(MegaDecodeKernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) {
        cudaGetLastError();
        return std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e);
    }
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, MegaDecodeKernel, kMkThreads, smem);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return std::string("cudaOccupancyMaxActiveBlocksPerMultiprocessor: ") + cudaGetErrorString(e);
    }
    if (per_sm < 1)
        return "one CTA (" + std::to_string(kMkThreads) + " threads, " + std::to_string(smem) +
               " B shared memory) does not fit on an SM";
    return "";
}

void LaunchMegaDecode(const MegaParams& p, int sm_count, size_t smem, cudaStream_t stream) {
    MegaParams args = p;
    void* kargs[] = {&args};
    CheckCuda(cudaLaunchCooperativeKernel(reinterpret_cast<void*>(MegaDecodeKernel), dim3(sm_count),
                                          dim3(kMkThreads), kargs, smem, stream),
              "cudaLaunchCooperativeKernel(MegaDecodeKernel)");
}

}  // namespace mlb
