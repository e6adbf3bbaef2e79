// Persistent decode kernel (see megakernel.cuh for the design).
#include <algorithm>
#include <cmath>
#include <string>

#include "megakernel.cuh"

namespace mlb {
namespace {

constexpr int kMkSpin = 1 << 26;  // backstop poll count of one dependency wait (the time bound p.wait_ns comes first)

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

// Tagged hand-over words: (tag << 32) | float bits, one single-copy-atomic
// 64-bit store; a reader polls the word until its tag is the expected one.
__device__ __forceinline__ void StTagged(unsigned long long* p, unsigned tag, float v) {
    const unsigned long long w = (static_cast<unsigned long long>(tag) << 32) | __float_as_uint(v);
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}

__device__ __forceinline__ unsigned long long LdTagged(const unsigned long long* p) {
    unsigned long long w;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    return w;
}

// A 16-byte L2 load as a volatile asm statement: it keeps its place among the
// other volatile statements (issued before a polling loop, not sunk past it).
__device__ __forceinline__ float4 LdCgF4(const float* p) {
    float4 v;
    asm volatile("ld.global.cg.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "l"(p));
    return v;
}

__device__ __forceinline__ void RedAdd(float* p, float v) {
    asm volatile("red.global.add.f32 [%0], %1;" ::"l"(p), "f"(v) : "memory");
}

// Four consecutive floats in one 16-byte vector reduction (p 16-byte aligned).
__device__ __forceinline__ void RedAdd4(float* p, float4 v) {
    asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w)
                 : "memory");
}

__host__ __device__ constexpr size_t Round128(size_t b) { return (b + 127) & ~size_t(127); }

struct Chunk {  // one ring stage of the schedule: one or two bulk copies, back to back
    const uint8_t* src;
    const uint8_t* src2;  // null, or the second copy (placed at bytes)
    uint32_t bytes;
    uint32_t bytes2;
};

// Shared-memory layout: fixed-size buffers at constant offsets, then
// xs, nw [dim], the digit planes and block scales of xs, then the ring.
constexpr size_t kOffFull = 0;                                            // kMkStages mbarriers
constexpr size_t kOffFlags = kOffFull + Round128(8 * kMkStages);          // 8 ints
constexpr size_t kOffScratch = kOffFlags + 128;                           // 32 floats
constexpr size_t kOffVsx = kOffScratch + 128;                             // 4 floats
constexpr size_t kOffVdig = kOffVsx + 128;                                // 4 planes of 4 blocks
constexpr size_t kOffRed = kOffVdig + Round128(4 * (4 * 32 + 16));        // 2 x 8 warps x 32
constexpr size_t kOffVec = kOffRed + 2 * 4 * 8 * 32;                      // 512 floats
constexpr size_t kOffAtt = kOffVec + 4 * 512;                             // 8 warps x 128
constexpr size_t kOffSc = kOffAtt + 4 * 8 * 128;                          // kMkAttnChunk floats
constexpr size_t kOffFixedEnd = kOffSc + Round128(4 * kMkAttnChunk);

struct MkSmem {  // flags[0] is the CTA's abort flag (read by the producer warp too)
    uint8_t* ring;
    uint64_t* full;
    struct Chunk* list;  // the CTA's chunk sequence of one step
    float* xs;      // [dim] activation (then normalised)
    float* nw;      // [dim] norm weights
    int8_t* dig;    // 4 digit planes of xs, stride DigitStride(nb_dim)
    float* sx;      // [nb_dim] block scales of xs
    int8_t* vdig;   // 4 digit planes of a short vector (o of a head or ff of a block)
    float* vsx;     // [4] its block scales
    float* red;     // [2][8 warps][32 rows], alternating by chunk (RedBuf)
    float* vec;     // [4 * 128] small vectors (g, u / q, k, v, o)
    float* att;     // [8 warps][hd] attention partials
    float* sc;      // [kMkAttnChunk] scores / weights of a chunk of positions
    float* acc;     // [dim] block-column products of the CTA, flushed by red.add
    float* kst;     // [kst_rows][hd] cached K rows of the attention item's KV head (swizzled)
    float* scratch; // [32]
    int* flags;     // [0] abort, [1] token, [2] chunks per step, [4] decision, [5] chunks issued
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
// Ring state of the consumers (identical in every thread): chunk n is the
// next to consume; chunk n + kMkStages, list entry li, is the next to issue.
struct Ring {
    unsigned n;
    unsigned li;
    unsigned len;    // chunks per step (list length)
    unsigned total;  // chunks of the launch
    uint64_t pol;    // L2 evict-first policy of the weight copies
};

// Uniform go / abort decision at a phase wait: thread 0 polls the counter
// (acquire; bounded, and it gives up when the status word is set), writes the
// decision between two barriers, and every thread reads it.  flags[0] is the
// CTA's sticky abort flag (any thread may set it), flags[4] the decision.
__device__ __forceinline__ bool WaitCounter(const MegaParams& p, const MkSmem& s, int ctr, unsigned target) {
    ConsumerBar();
    if (threadIdx.x == 0) {
        bool ok = s.flags[0] == 0;
        if (ok) {
            ok = false;
            uint64_t t0 = 0;
            for (int it = 0; it < kMkSpin; ++it) {
                if (LdAcquire(p.counters + ctr) >= target) {
                    ok = true;
                    break;
                }
                if ((it & 255) == 255) {
                    if (LdRelaxedInt(p.status) != 0) break;
                    const uint64_t now = GlobalTimerNs();
                    if (t0 == 0) t0 = now;
                    else if (now - t0 > p.wait_ns) break;
                }
            }
            if (!ok) atomicCAS(p.status, 0, MLB_ERR_DEVICE_TIMEOUT);
        }
        if (!ok) s.flags[0] = 1;
        s.flags[4] = ok ? 1 : 0;
    }
    ConsumerBar();
    return s.flags[4] != 0;
}

// Publishes this CTA's writes of the phase and increments the counter: the
// barrier orders every thread's writes before thread 0's release add, whose
// release semantics are cumulative over them (no separate fence, no return
// value to wait for).
__device__ __forceinline__ void RedRelease(unsigned* ctr) {
    asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(ctr) : "memory");
}

// (A counter equal to p.withhold is never signalled: the test hook that makes
// the waits on it expire.)
__device__ __forceinline__ void Signal(const MegaParams& p, int ctr) {
    ConsumerBar();
    if (threadIdx.x == 0 && ctr != p.withhold) RedRelease(p.counters + ctr);
}

// Waits (every thread) for the stage of chunk rg.n; bounded, and it gives up
// as soon as the status word is set.  A wait that gives up records the error
// and sets the sticky abort flag but returns normally: every thread still
// reaches every barrier, and the CTA leaves at its next phase wait.
__device__ __forceinline__ void WaitChunk(const MegaParams& p, const MkSmem& s, const Ring& rg) {
    if (!MbarWaitFor(&s.full[rg.n % kMkStages], (rg.n / kMkStages) & 1, p.wait_ns, p.status)) {
        atomicCAS(p.status, 0, MLB_ERR_DEVICE_TIMEOUT);
        s.flags[0] = 1;
    }
}

__device__ __forceinline__ uint8_t* StagePtr(const MegaParams& p, const MkSmem& s, const Ring& rg) {
    return s.ring + size_t(rg.n % kMkStages) * p.stage_bytes;
}

// List entry li into ring slot k % kMkStages; one thread at a time (thread 0
// in the prologue, then lane 0 of the last warp).
__device__ __forceinline__ void IssueChunk(const MegaParams& p, const MkSmem& s, unsigned k, unsigned li,
                                           uint64_t pol) {
    const Chunk ch = s.list[li];
    const int slot = k % kMkStages;
    uint8_t* dst = s.ring + size_t(slot) * p.stage_bytes;
    MbarExpectTx(&s.full[slot], ch.bytes + ch.bytes2);
    BulkLoadHint(dst, ch.src, ch.bytes, &s.full[slot], pol);
    if (ch.src2) BulkLoadHint(dst + ch.bytes, ch.src2, ch.bytes2, &s.full[slot], pol);
    ++s.flags[5];  // chunks issued
}

// After every thread is done with chunk rg.n's stage (the barrier): the slot
// takes chunk rg.n + kMkStages (unless the CTA is aborting), and the ring
// moves on.  The issuing thread's count of issued chunks (flags[5]) is read
// by thread 0 only after a barrier.
__device__ __forceinline__ void ReleaseChunk(const MegaParams& p, const MkSmem& s, Ring& rg) {
    ConsumerBar();
    const unsigned k = rg.n + kMkStages;
    // the last warp issues: warp 0 carries the per-chunk totals and digits
    if (threadIdx.x == kMkThreads - 32 && k < rg.total && s.flags[0] == 0) IssueChunk(p, s, k, rg.li, rg.pol);
    ++rg.n;
    rg.li = rg.li + 1 == rg.len ? 0 : rg.li + 1;
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

// Round to nearest even for |v| < 2^22 (the digit scaling guarantees it):
// adding 1.5 * 2^23 leaves the rounded integer in the low mantissa bits.
__device__ __forceinline__ int RoundSmall(float v) {
    return __float_as_int(v + 12582912.0f) - 0x4B400000;
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

// RMSNorm of x (n % 32 == 0, in shared memory) straight into the digit planes
// and block scales of the normalised vector, which is not stored: a thread
// per four elements, eight threads per 32-block (the block max by three
// shuffles).  Each normalised value is x * rsqrt(mean(x^2) + eps) * w in the
// reference's product order.
__device__ __forceinline__ float4 LdsF32x4(uint32_t a) {
    float4 v;
    asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(a));
    return v;
}

__device__ __forceinline__ void StsU32(uint32_t a, uint32_t v) {
    asm volatile("st.shared.u32 [%0], %1;" ::"r"(a), "r"(v) : "memory");
}

// Digits of four elements y[0..3] of a 32-block whose eight holders are the
// aligned eight lanes of this thread (block max by three shuffles; every lane
// takes part); when `on`, the four digit bytes of each plane go to dq +
// plane * dstride.  Returns the block scale.
__device__ __forceinline__ float QuadDigits(const float (&y)[4], bool on, uint32_t dq, int dstride) {
    float mx = fmaxf(fmaxf(fabsf(y[0]), fabsf(y[1])), fmaxf(fabsf(y[2]), fabsf(y[3])));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
    const int e = static_cast<int>((__float_as_uint(mx) >> 23) & 0xff) - 126;
    uint32_t p2 = 0, p1 = 0, p0 = 0;
    float sc = 0.0f;
    if (mx > 0.0f && e >= -104) {
        const float up = __uint_as_float(static_cast<uint32_t>(127 + 22 - e) << 23);
        sc = __uint_as_float(static_cast<uint32_t>(127 + e - 22) << 23);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int xi = RoundSmall(y[k] * up);
            const int d0 = (xi << 24) >> 24;
            const int x1 = (xi - d0) >> 8;
            const int d1 = (x1 << 24) >> 24;
            const int d2 = (x1 - d1) >> 8;
            p2 |= (static_cast<uint32_t>(d2) & 0xffu) << (8 * k);
            p1 |= (static_cast<uint32_t>(d1) & 0xffu) << (8 * k);
            p0 |= (static_cast<uint32_t>(d0) & 0xffu) << (8 * k);
        }
    }
    if (on) {
        StsU32(dq, p2);
        StsU32(dq + dstride, p1);
        StsU32(dq + 2 * dstride, p0);
        StsU32(dq + 3 * dstride, 0u);
    }
    return sc;
}

// RMSNorm of x (n % 32 == 0, shared memory) straight into the digit planes
// and block scales of the normalised vector, which is not stored: a thread
// per four elements, eight threads per 32-block.  Each normalised value is
// x * rsqrt(mean(x^2) + eps) * w in the reference's product order.  Vectors of
// up to 1024 elements stay in registers between the two passes.
__device__ __forceinline__ void RmsNormDigits(const float* x, const float* w, int n, float eps, int8_t* dig,
                                              int dstride, float* sx, float* scratch) {
    const int n4 = n / 4;
    const uint32_t xa = SmemAddr(x), wa = SmemAddr(w), da = SmemAddr(dig);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    float4 v0 = make_float4(0.f, 0.f, 0.f, 0.f);
    if (tid < n4) v0 = LdsF32x4(xa + 16 * tid);
    float ss = 0.0f;
    ss = fmaf(v0.x, v0.x, ss);
    ss = fmaf(v0.y, v0.y, ss);
    ss = fmaf(v0.z, v0.z, ss);
    ss = fmaf(v0.w, v0.w, ss);
    for (int i = tid + 256; i < n4; i += 256) {
        const float4 v = LdsF32x4(xa + 16 * i);
        ss = fmaf(v.x, v.x, ss);
        ss = fmaf(v.y, v.y, ss);
        ss = fmaf(v.z, v.z, ss);
        ss = fmaf(v.w, v.w, ss);
    }
    // one barrier: scratch is not written again before the closing barrier
    ss = WarpSum(ss);
    if (lane == 0) scratch[warp] = ss;
    ConsumerBar();
    const float4 s0 = LdsF32x4(SmemAddr(scratch)), s1 = LdsF32x4(SmemAddr(scratch) + 16);
    const float tot = ((s0.x + s0.y) + (s0.z + s0.w)) + ((s1.x + s1.y) + (s1.z + s1.w));
    const float scale = 1.0f / sqrtf(tot / static_cast<float>(n) + eps);
    // n4 is a multiple of 8, so the eight threads of a block share every trip
    for (int i0 = 0; i0 < n4; i0 += 256) {
        const int i = i0 + tid;
        const bool on = i < n4;
        float y[4] = {0.f, 0.f, 0.f, 0.f};
        if (on) {
            const float4 v = i0 == 0 ? v0 : LdsF32x4(xa + 16 * i);
            const float4 g = LdsF32x4(wa + 16 * i);
            y[0] = v.x * scale * g.x;
            y[1] = v.y * scale * g.y;
            y[2] = v.z * scale * g.z;
            y[3] = v.w * scale * g.w;
        }
        const float sc = QuadDigits(y, on, da + 4 * i, dstride);
        if (on && (tid & 7) == 0) sx[i / 8] = sc;
    }
    ConsumerBar();
}


// ---------------------------------------------------------------- MMA pieces
struct LaneMma {
    uint32_t lrow;  // ldmatrix row offset inside a chunk
    int m;          // integer weight of column 2t against column 2t + 1 (256 or 1)
    float lf;       // the lane's digit factor (256 for t = 0, 1 otherwise)
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
    l.m = l.t == 0 ? 256 : 1;
    l.lf = l.t == 0 ? 256.0f : 1.0f;
    return l;
}

// Up to N chunks (16 rows x 32 inputs each) times their blocks of digits:
// chunk i at ch + i * ch_step, digits at db + i * db_step, block scale
// sx[i * sx_step]; adds the scaled contributions of rows g and g + 8 of chunk i
// to vg[i], vg8[i] (before the lane-pair combine).  The asm statements keep
// program order, so the N ldmatrix loads are issued back to back, then the N
// MMAs, then the scaling: N products in flight instead of one.
// Products of one chunk (16 rows x 32 inputs) with the 4 digit columns of one
// x block (D2, D1, D0, 0) land in lane (g, t) as c0 = col 2t, c1 = col 2t + 1
// of rows g and g + 8.  Lane t = 0 holds D2 and D1, whose weights 65536 and
// 256 are 256 * (256, 1): it forms 256 * c0 + c1 (|.| < 2^28, exact in int32)
// and scales by 256; lane t = 1 holds D0 (weight 1) and the zero column;
// lanes t = 2, 3 hold zero columns.  So every lane computes c0 * m + c1 in
// integer and one conversion per row, with m and the lane factor in LaneMma.
__device__ __forceinline__ float LaneDigits(const LaneMma& L, int c0, int c1) {
    return __int2float_rn(c0 * L.m + c1);
}

__device__ __forceinline__ uint32_t LdsU32(uint32_t a) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
    return v;
}

__device__ __forceinline__ float LdsF32(uint32_t a) {
    float v;
    asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(a));
    return v;
}

__device__ __forceinline__ float LdsHalf(uint32_t a) {
    uint16_t h;
    asm volatile("ld.shared.u16 %0, [%1];" : "=h"(h) : "r"(a));
    return HalfBits(h);
}

// Exactly N chunks (16 rows x 32 inputs) against their digit blocks, summed:
// chunk i at shared address ch + i * ch_step, this lane's B fragment at
// db + i * db_step (db = digit block + g * dstride + 4 t; lanes g >= 4 hold
// the zero columns and load nothing), block scale at sx + 4 * i * sx_step.
// Adds rows g and g + 8 (without the lane factor L.lf, before the lane-pair
// combine) to v, v8.  The asm statements keep program order, so the N ldmatrix
// loads go out back to back, then the N MMAs, then the scaling.
template <int N>
__device__ __forceinline__ void RowChunks(const LaneMma& L, uint32_t ch, int ch_step, uint32_t db, int db_step,
                                          uint32_t sx, int sx_step, float& v, float& v8) {
    uint32_t a[N][4], b[N][2];
#pragma unroll
    for (int i = 0; i < N; ++i) LdMatrixX4(ch + i * ch_step + L.lrow, a[i][0], a[i][1], a[i][2], a[i][3]);
#pragma unroll
    for (int i = 0; i < N; ++i) {
        b[i][0] = b[i][1] = 0;
        if (L.g < 4) {
            b[i][0] = LdsU32(db + i * db_step);
            b[i][1] = LdsU32(db + i * db_step + 16);
        }
    }
    int c[N][4];
#pragma unroll
    for (int i = 0; i < N; ++i)
        MmaS8(c[i][0], c[i][1], c[i][2], c[i][3], a[i][0], a[i][1], a[i][2], a[i][3], b[i][0], b[i][1]);
#pragma unroll
    for (int i = 0; i < N; ++i) {
        const uint32_t sc = ch + i * ch_step + 512 + 2 * L.g;
        const float s = LdsF32(sx + 4 * i * sx_step);
        v = fmaf(LaneDigits(L, c[i][0], c[i][1]), LdsHalf(sc) * s, v);
        v8 = fmaf(LaneDigits(L, c[i][2], c[i][3]), LdsHalf(sc + 16) * s, v8);
    }
}

// Exactly N chunks (ch + i * ch_step) against one digit block (B fragment
// b0, b1 and scale s already loaded): rows g and g + 8 of chunk i into
// vg[i], vg8[i] (without the lane factor).
template <int N>
__device__ __forceinline__ void ColumnChunks(const LaneMma& L, uint32_t ch, int ch_step, uint32_t b0, uint32_t b1,
                                             float s, float* vg, float* vg8) {
    uint32_t a[N][4];
#pragma unroll
    for (int i = 0; i < N; ++i) LdMatrixX4(ch + i * ch_step + L.lrow, a[i][0], a[i][1], a[i][2], a[i][3]);
    int c[N][4];
#pragma unroll
    for (int i = 0; i < N; ++i) MmaS8(c[i][0], c[i][1], c[i][2], c[i][3], a[i][0], a[i][1], a[i][2], a[i][3], b0, b1);
#pragma unroll
    for (int i = 0; i < N; ++i) {
        const uint32_t sc = ch + i * ch_step + 512 + 2 * L.g;
        vg[i] = LaneDigits(L, c[i][0], c[i][1]) * (LdsHalf(sc) * s);
        vg8[i] = LaneDigits(L, c[i][2], c[i][3]) * (LdsHalf(sc + 16) * s);
    }
}

// count (1..8) blocks by RowChunks with an exact compile-time count.
__device__ __forceinline__ void RowChunksN(int count, const LaneMma& L, uint32_t ch, int ch_step, uint32_t db,
                                           int db_step, uint32_t sx, int sx_step, float& v, float& v8) {
    switch (count) {
        case 8: RowChunks<8>(L, ch, ch_step, db, db_step, sx, sx_step, v, v8); break;
        case 7: RowChunks<7>(L, ch, ch_step, db, db_step, sx, sx_step, v, v8); break;
        case 6: RowChunks<6>(L, ch, ch_step, db, db_step, sx, sx_step, v, v8); break;
        case 5: RowChunks<5>(L, ch, ch_step, db, db_step, sx, sx_step, v, v8); break;
        case 4: RowChunks<4>(L, ch, ch_step, db, db_step, sx, sx_step, v, v8); break;
        case 3: RowChunks<3>(L, ch, ch_step, db, db_step, sx, sx_step, v, v8); break;
        case 2: RowChunks<2>(L, ch, ch_step, db, db_step, sx, sx_step, v, v8); break;
        default: RowChunks<1>(L, ch, ch_step, db, db_step, sx, sx_step, v, v8); break;
    }
}

constexpr int kMkMmaBatch = 8;  // chunks a warp has in flight

// Row tiles of a stage (NTILE x nb chunks, row-tile major) against the digits
// of xs; warps split the work by (tile, block); results (one value per row)
// land in red as [warp][tile * 16 + row].  Returns with the partials written
// (no barrier).
template <int NTILE>
__device__ __forceinline__ void RowTilesDotImpl(const int8_t* dig, const float* sxv, float* red, const LaneMma L,
                                                const uint8_t* stage, int nb, int dstride) {
    const int warp = threadIdx.x >> 5;
    constexpr int wpt = kMkConsumerWarps / NTILE;  // warps per tile
    const int tile = warp / wpt, part = warp % wpt;
    const uint32_t tb = SmemAddr(stage) + tile * nb * kR16Chunk;
    const uint32_t dl = SmemAddr(dig) + L.g * dstride + 4 * L.t;
    const uint32_t sl = SmemAddr(sxv);
    float v = 0.0f, v8 = 0.0f;
    int count = part < nb ? (nb - part + wpt - 1) / wpt : 0;  // blocks part, part + wpt, ...
    for (int b = part; count > 0; b += kMkMmaBatch * wpt, count -= kMkMmaBatch)
        RowChunksN(min(count, kMkMmaBatch), L, tb + b * kR16Chunk, wpt * kR16Chunk, dl + b * 32, wpt * 32,
                   sl + 4 * b, wpt, v, v8);
    v *= L.lf;
    v8 *= L.lf;
    v += __shfl_xor_sync(0xffffffffu, v, 1);
    v8 += __shfl_xor_sync(0xffffffffu, v8, 1);
    if (L.t == 0) {
        red[warp * 32 + tile * 16 + L.g] = v;
        red[warp * 32 + tile * 16 + L.g + 8] = v8;
    }
}

__device__ __forceinline__ void RowTilesDot(const MkSmem& s, float* red, const LaneMma& L, const uint8_t* stage,
                                            int ntile, int nb, int dstride) {
    if (ntile == 2) RowTilesDotImpl<2>(s.dig, s.sx, red, L, stage, nb, dstride);
    else RowTilesDotImpl<1>(s.dig, s.sx, red, L, stage, nb, dstride);
}

// Sum of the partials of row r of tile `tile` (after a barrier).
__device__ __forceinline__ float RowTotal(const float* red, int ntile, int tile, int r) {
    const int wpt = kMkConsumerWarps / ntile;
    float v = 0.0f;
    for (int w = tile * wpt; w < (tile + 1) * wpt; ++w) v += red[w * 32 + tile * 16 + r];
    return v;
}

// The partial-sum buffer of chunk n: two alternate, so the chunk after next
// is the first to overwrite one, and the release barrier of the chunk in
// between orders the reads of the totals before it.
__device__ __forceinline__ float* RedBuf(const MkSmem& s, const Ring& rg) { return s.red + (rg.n & 1) * 256; }

// A block column (ntiles chunks of 16 rows x 32 inputs) times one block of
// digits (scale *sxb), added into acc[row] in shared memory (each row has one
// owner lane, so no atomics); warp w takes row tiles w, w + 8, ...
__device__ __forceinline__ void ColumnDotSmem(const LaneMma L, const uint8_t* column, int ntiles, int nrows,
                                              const int8_t* dblk, int dstride, const float* sxb, float* acc) {
    const int warp = threadIdx.x >> 5;
    uint32_t b0 = 0, b1 = 0;
    if (L.g < 4) {
        const uint32_t db = SmemAddr(dblk) + L.g * dstride + 4 * L.t;
        b0 = LdsU32(db);
        b1 = LdsU32(db + 16);
    }
    const float s = *sxb;
    const uint32_t col = SmemAddr(column);
    for (int t0 = warp; t0 < ntiles; t0 += kMkMmaBatch * kMkConsumerWarps) {
        const int count = min(kMkMmaBatch, (ntiles - t0 + kMkConsumerWarps - 1) / kMkConsumerWarps);
        float vg[kMkMmaBatch], vg8[kMkMmaBatch];
        const uint32_t ch = col + t0 * kR16Chunk;
        constexpr int st = kMkConsumerWarps * kR16Chunk;
        switch (count) {
            case 8: ColumnChunks<8>(L, ch, st, b0, b1, s, vg, vg8); break;
            case 7: ColumnChunks<7>(L, ch, st, b0, b1, s, vg, vg8); break;
            case 6: ColumnChunks<6>(L, ch, st, b0, b1, s, vg, vg8); break;
            case 5: ColumnChunks<5>(L, ch, st, b0, b1, s, vg, vg8); break;
            case 4: ColumnChunks<4>(L, ch, st, b0, b1, s, vg, vg8); break;
            case 3: ColumnChunks<3>(L, ch, st, b0, b1, s, vg, vg8); break;
            case 2: ColumnChunks<2>(L, ch, st, b0, b1, s, vg, vg8); break;
            default: ColumnChunks<1>(L, ch, st, b0, b1, s, vg, vg8); break;
        }
#pragma unroll
        for (int i = 0; i < kMkMmaBatch; ++i) {
            if (i >= count) break;
            float a = vg[i] * L.lf, a8 = vg8[i] * L.lf;
            a += __shfl_xor_sync(0xffffffffu, a, 1);
            a8 += __shfl_xor_sync(0xffffffffu, a8, 1);
            const int r0 = (t0 + i * kMkConsumerWarps) * 16 + L.g, r1 = r0 + 8;
            if (L.t == 0 && r0 < nrows) acc[r0] += a;
            if (L.t == 0 && r1 < nrows) acc[r1] += a8;
        }
    }
}

// After a barrier: out[i] += acc[i] (+ addend[i]) for i < n by red.add, one
// coalesced pass, and acc back to zero.
__device__ __forceinline__ void FlushRed(float* acc, float* out, int n, const float* addend) {
    // n is a multiple of 32; acc (shared), out and addend are 16-byte aligned
    for (int i = 4 * threadIdx.x; i < n; i += 4 * 256) {
        float4 a = *reinterpret_cast<const float4*>(acc + i);
        if (addend) {
            const float4 b = __ldcg(reinterpret_cast<const float4*>(addend + i));
            a.x += b.x;
            a.y += b.y;
            a.z += b.z;
            a.w += b.w;
        }
        RedAdd4(out + i, a);
        *reinterpret_cast<float4*>(acc + i) = make_float4(0.f, 0.f, 0.f, 0.f);
    }
}

// Digit planes of one 32-block held by a warp (lane = element): block scale
// into *sxp.  Same digits as RmsNormDigits / DigitsMk.
__device__ __forceinline__ void DigitsWarp(float v, int8_t* dblk, int dstride, float* sxp) {
    const int lane = threadIdx.x & 31;
    const float mx = WarpMax(fabsf(v));
    const int e = static_cast<int>((__float_as_uint(mx) >> 23) & 0xff) - 126;
    int xi = 0;
    float sc = 0.0f;
    if (mx > 0.0f && e >= -104) {
        const float up = __uint_as_float(static_cast<uint32_t>(127 + 22 - e) << 23);
        sc = __uint_as_float(static_cast<uint32_t>(127 + e - 22) << 23);
        xi = RoundSmall(v * up);
    }
    const int d0 = (xi << 24) >> 24;
    const int x1 = (xi - d0) >> 8;
    const int d1 = (x1 << 24) >> 24;
    const int d2 = (x1 - d1) >> 8;
    dblk[lane] = static_cast<int8_t>(d2);
    dblk[dstride + lane] = static_cast<int8_t>(d1);
    dblk[2 * dstride + lane] = static_cast<int8_t>(d0);
    dblk[3 * dstride + lane] = 0;
    if (lane == 0) *sxp = sc;
}

// ---------------------------------------------------------------- schedule
// The chunk sequence of one CTA for one step (weights only, so every step
// repeats it); thread 0 issues it into the ring, the consumers consume it, in
// the same order.

// CTAs per attention head: one per wo block column when every head can have
// that many, so each CTA of a head runs the head's attention and projects
// through its own column; else one CTA per head and all its columns.
struct AttnPlan {
    int hsplit;  // CTAs per head over its wo block columns (1 or hd / 32)
    int rsplit;  // and over the rows of each column (1 or 2)
    int items;   // n_heads x hsplit x rsplit
};

__host__ __device__ __forceinline__ AttnPlan AttnSplit(const MegaParams& p, int G) {
    const int bph = p.hd / 32;
    AttnPlan a;
    a.hsplit = p.n_heads * bph <= G ? bph : 1;
    a.rsplit = (a.hsplit == bph && 2 * p.n_heads * bph <= G && (p.dim + 15) / 16 >= 2) ? 2 : 1;
    a.items = p.n_heads * a.hsplit * a.rsplit;
    return a;
}

// Row tiles [t0, t1) of the wo block column that part rh of rsplit projects.
__host__ __device__ __forceinline__ void AttnRows(int ntiles, int rsplit, int rh, int& t0, int& t1) {
    const int per = (ntiles + rsplit - 1) / rsplit;
    t0 = rh * per < ntiles ? rh * per : ntiles;
    t1 = t0 + per < ntiles ? t0 + per : ntiles;
}


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
    const AttnPlan ap = AttnSplit(p, G);
    for (int l = 0; l < p.n_layers; ++l) {
        const MegaLayer& L = p.layers[l];
        for (int t = c; t < t_qkv; t += G) {
            const int seg = t < tq ? 0 : (t < tq + tk ? 1 : 2);
            const int ti = seg == 0 ? t : (seg == 1 ? t - tq : t - tq - tk);
            f(Chunk{L.wqkv[seg] + size_t(ti) * tile_b, nullptr, tile_b, 0});
        }
        // attention items (head, its wo columns, a row range of them)
        for (int it = G - 1 - c; it < ap.items; it += G) {
            const int per_head = ap.hsplit * ap.rsplit, rem = it % per_head, h = it / per_head;
            const int ci = rem / ap.rsplit, rh = rem % ap.rsplit;
            int t0, t1;
            AttnRows(ntiles_dim, ap.rsplit, rh, t0, t1);
            for (int j = ci * (bph / ap.hsplit); j < (ci + 1) * (bph / ap.hsplit); ++j)
                f(Chunk{L.wo + size_t(h * bph + j) * col_b + size_t(t0) * kR16Chunk, nullptr,
                        static_cast<uint32_t>(t1 - t0) * kR16Chunk, 0});
        }
        // FFN: per 32-unit hidden block j, its gate rows, its up rows, its
        // w_down block column (R16C)
        for (int j = c; j < nj; j += G) {
            f(Chunk{L.gate + size_t(2 * j) * tile_b, nullptr, 2 * tile_b, 0});
            f(Chunk{L.up + size_t(2 * j) * tile_b, nullptr, 2 * tile_b, 0});
            f(Chunk{L.down + size_t(j) * col_b, nullptr, col_b, 0});
        }
    }
    // lm_head: two row tiles per stage
    for (int t2 = c; 2 * t2 < t_lm; t2 += G)
        f(Chunk{p.lm_head + size_t(2 * t2) * tile_b, nullptr, (2 * t2 + 1 < t_lm ? 2u : 1u) * tile_b, 0});
}

// ---------------------------------------------------------------- consumers
// Returns how many chunks it consumed (all of them unless it aborted).
__device__ unsigned Consumers(const MegaParams& p, const MkSmem& s) {
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
    const AttnPlan ap = AttnSplit(p, G);
    const unsigned w_att = ap.items, w_ffn = WorkerCount(G, nj), w_lm = G;
    const int ctr_lm_ticket = kMkPhases * p.n_layers, ctr_token = kMkPhases * p.n_layers + 1;
    Ring rg;  // the chunk sequence thread 0 issued in the prologue, continued here
    rg.n = 0;
    rg.len = static_cast<unsigned>(s.flags[2]);
    rg.total = rg.len * static_cast<unsigned>(p.n_steps);
    rg.li = rg.len ? kMkStages % rg.len : 0;
    rg.pol = L2EvictFirstPolicy();

    for (int step = 0; step < p.n_steps; ++step) {
        const int pos = p.start_pos + step;
        const unsigned k1 = static_cast<unsigned>(step + 1);
        for (int l = 0; l < p.n_layers; ++l) {
            const MegaLayer& Lw = p.layers[l];
            const unsigned tag = p.tag_base + static_cast<unsigned>(step * p.n_layers + l);
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
                    if (step > 0 && !WaitCounter(p, s, ctr_token, k1 - 1)) return rg.n;
                } else if (!WaitCounter(p, s, kMkPhases * (l - 1) + 2, k1 * w_ffn)) {
                    return rg.n;
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
                if (c == 0) {  // x_mid starts as x, the next x at zero; then the attention CTAs may add
                    for (int i = tid; i < p.dim; i += 256) {
                        p.xmid[i] = s.xs[i];
                        xout[i] = 0.0f;
                    }
                    Signal(p, kMkPhases * l + 0);
                }
                RmsNormDigits(s.xs, s.nw, p.dim, p.eps, s.dig, dstride, s.sx, s.scratch);
                Trace(p, step, l, 11);
                for (int t = c, i = 0; t < t_qkv; t += G, ++i) {
                    const int seg = t < tq ? 0 : (t < tq + tk ? 1 : 2);
                    const int ti = seg == 0 ? t : (seg == 1 ? t - tq : t - tq - tk);
                    const int rows = seg == 0 ? p.qd : p.kd;
                    const int off = seg == 0 ? 0 : (seg == 1 ? p.qd : p.qd + p.kd);
                    float* red = RedBuf(s, rg);
                    WaitChunk(p, s, rg);
                    RowTilesDot(s, red, L, StagePtr(p, s, rg), 1, nb_dim, dstride);
                    ReleaseChunk(p, s, rg);  // its barrier publishes red
                    if (tid < 16) {
                        const int r = ti * 16 + tid;
                        if (r < rows) {
                            float v = RowTotal(red, 1, 0, tid);
                            if (Lw.bias[seg]) v += i < 32 ? s.vec[16 * i + tid] : Lw.bias[seg][r];
                            StTagged(p.qkvt + off + r, tag, v);  // read by the attention CTAs directly
                        }
                    }
                }
                Trace(p, step, l, 10);
                ConsumerBar();
                Trace(p, step, l, 1);
            }
            // ---------------- attention + O projection, one query head
            for (int it = G - 1 - c; it < ap.items; it += G) {
                const int per_head = ap.hsplit * ap.rsplit, rem = it % per_head, h = it / per_head;
                const int ci = rem / ap.rsplit, rh = rem % ap.rsplit;
                const int j0 = ci * (bph / ap.hsplit), j1 = j0 + bph / ap.hsplit;
                int rt0, rt1;  // this item's row tiles of its wo columns
                AttnRows(ntiles_dim, ap.rsplit, rh, rt0, rt1);
                const int r0 = rt0 * 16, nrows = (rt1 * 16 < p.dim ? rt1 * 16 : p.dim) - r0;
                const int hd = p.hd, half = hd / 2, kvh = h / p.group;
                const size_t pstride = size_t(p.n_kv) * hd;
                const size_t lbase = size_t(l) * p.max_seq * pstride + size_t(kvh) * hd;
                const int lpr = hd / 4, rpi = 32 / lpr;  // float4 lanes per K/V row, rows per warp pass
                const int rsub = lane / lpr, col = lane % lpr;
                // While QKV runs (none of it depends on the step): the K rows
                // of cached positions 0..nst-1 into shared memory (cp.async;
                // 16-byte piece c of row r at slot c ^ (r % 8), so the score
                // pass reads a row per thread without bank conflicts), this
                // warp's V row pieces of the first pass into registers (the
                // asm loads keep their place before the q, k, v polls), the
                // other cached rows into L2.
                const int nst = pos < p.kst_rows ? pos : p.kst_rows;
                for (int i = tid; i < nst * lpr; i += 256) {
                    const int r = i / lpr, c4 = i - r * lpr;
                    CpAsync16(s.kst + r * hd + 4 * (c4 ^ (r & 7)), p.kc + lbase + size_t(r) * pstride + 4 * c4);
                }
                float4 vpre[16];
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const int r = warp * 32 + i * rpi + rsub;
                    vpre[i] = make_float4(0.f, 0.f, 0.f, 0.f);
                    if (i < lpr && r < pos) vpre[i] = LdCgF4(p.vc + lbase + size_t(r) * pstride + 4 * col);
                }
                for (int pp = tid; pp < pos; pp += 256) {
                    BulkPrefetchL2(p.vc + lbase + size_t(pp) * pstride, static_cast<uint32_t>(hd) * 4);
                    if (pp >= nst)
                        BulkPrefetchL2(p.kc + lbase + size_t(pp) * pstride, static_cast<uint32_t>(hd) * 4);
                }
                // RoPE rows of this position (s.att is free until the values pass)
                float* ct = s.att;
                float* st = s.att + half;
                LoadVecCg(ct, p.rope_cos + size_t(pos) * half, half);
                LoadVecCg(st, p.rope_sin + size_t(pos) * half, half);
                float* q = s.vec;
                float* kn = s.vec + 128;
                float* vn = s.vec + 256;
                float* o = s.vec + 384;
                // q of the head, k and v of its kv head: each thread polls
                // its tagged words until this step's layer-l tag (bounded)
                for (int i = tid; i < 3 * hd; i += 256) {
                    const int part = i / hd, d = i - part * hd;
                    const size_t src = part == 0 ? size_t(h) * hd + d
                                                 : size_t(p.qd) + (part - 1) * p.kd + size_t(kvh) * hd + d;
                    unsigned long long wv = 0;
                    bool got = false;
                    uint64_t t0 = 0;
                    for (int it2 = 0; it2 < kMkSpin; ++it2) {
                        wv = LdTagged(p.qkvt + src);
                        if (static_cast<unsigned>(wv >> 32) == tag) {
                            got = true;
                            break;
                        }
                        if ((it2 & 255) == 255) {
                            if (LdRelaxedInt(p.status) != 0) break;
                            const uint64_t now = GlobalTimerNs();
                            if (t0 == 0) t0 = now;
                            else if (now - t0 > p.wait_ns) break;
                        }
                    }
                    if (!got) {
                        atomicCAS(p.status, 0, MLB_ERR_DEVICE_TIMEOUT);
                        s.flags[0] = 1;
                    }
                    (part == 0 ? q : (part == 1 ? kn : vn))[d] = __uint_as_float(static_cast<unsigned>(wv));
                }
                for (int i = tid; i < hd; i += 256) o[i] = 0.0f;
                CpAsyncWaitAll();  // this thread's RoPE-table and K-row copies; the barrier publishes them
                ConsumerBar();
                if (tid == 0) s.flags[4] = s.flags[0] == 0;
                ConsumerBar();
                if (!s.flags[4]) return rg.n;
                Trace(p, step, l, 2);
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
                if (h % p.group == 0 && j0 == 0 && rh == 0)  // one CTA of the group's first head stores k, v
                    for (int i = tid; i < hd; i += 256) {
                        p.kc[lbase + size_t(pos) * pstride + i] = kn[i];
                        p.vc[lbase + size_t(pos) * pstride + i] = vn[i];
                    }
                // Positions 0..pos in chunks of 256 with a running max and sum.
                // Scores: a thread per position (its K row as float4 loads, all
                // in flight together).  Values: a warp per 32 positions, lanes
                // over (row, float4 column), every row load in flight together.
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
                        } else if (pp < nst) {  // a staged row (first pass), four chains
                            const float4* ks = reinterpret_cast<const float4*>(s.kst + size_t(pp) * hd);
                            float d4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                            for (int i = 0; i < 32; ++i)
                                if (i < lpr) {
                                    const float4 qv = q4[i], kv = ks[i ^ (pp & 7)];
                                    d4[i & 3] = fmaf(qv.x, kv.x, d4[i & 3]);
                                    d4[i & 3] = fmaf(qv.y, kv.y, d4[i & 3]);
                                    d4[i & 3] = fmaf(qv.z, kv.z, d4[i & 3]);
                                    d4[i & 3] = fmaf(qv.w, kv.w, d4[i & 3]);
                                }
                            dot = (d4[0] + d4[1]) + (d4[2] + d4[3]);
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
                    // this warp's first 16 V row pieces (the first pass's
                    // were loaded before the wait; later passes load them
                    // before the softmax reductions so their latency overlaps
                    // them); the current position's row comes from shared memory
                    const int r0 = base + warp * 32;
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        const int r = r0 + i * rpi + rsub;
                        if (base > 0) {
                            vpre[i] = make_float4(0.f, 0.f, 0.f, 0.f);
                            if (i < lpr && r < pos)
                                vpre[i] =
                                    __ldcg(reinterpret_cast<const float4*>(p.vc + lbase + size_t(r) * pstride) + col);
                        }
                        if (i < lpr && r == pos) vpre[i] = reinterpret_cast<const float4*>(vn)[col];
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
                // the normalised output's digit planes, straight from the
                // warps that hold it (warp w: block w; hd is a multiple of 32)
                for (int d = tid; d < hd; d += 256)
                    DigitsWarp(o[d] / l_run, s.vdig + (d >> 5) * 32, vstride, s.vsx + (d >> 5));
                ConsumerBar();
                Trace(p, step, l, 8);
                // this item's wo block columns into acc, then one red.add pass
                for (int j = j0; j < j1; ++j) {
                    WaitChunk(p, s, rg);
                    ColumnDotSmem(L, StagePtr(p, s, rg), rt1 - rt0, nrows, s.vdig + j * 32, vstride, s.vsx + j,
                                  s.acc + r0);
                    ReleaseChunk(p, s, rg);
                }
                if (!WaitCounter(p, s, kMkPhases * l + 0, k1)) return rg.n;  // x_mid holds x
                FlushRed(s.acc + r0, p.xmid + r0, nrows, nullptr);
                Trace(p, step, l, 9);
                Signal(p, kMkPhases * l + 1);
                Trace(p, step, l, 3);
            }
            // ---------------- FFN: per hidden block, gate and up rows, SwiGLU,
            // then the block's w_down column into acc; one red.add pass
            if (c < nj) {
                LoadVecCg(s.nw, Lw.ffn_norm, p.dim);  // independent of the wait
                if (!WaitCounter(p, s, kMkPhases * l + 1, k1 * w_att)) return rg.n;
                Trace(p, step, l, 4);
                LoadVecCg(s.xs, p.xmid, p.dim);
                CpAsyncWaitAll();
                ConsumerBar();
                RmsNormDigits(s.xs, s.nw, p.dim, p.eps, s.dig, dstride, s.sx, s.scratch);
                Trace(p, step, l, 7);
                for (int j = c; j < nj; j += G) {
                    float gu[2];  // warp 0, lane r: gate and up of hidden unit 32 j + r
#pragma unroll
                    for (int part = 0; part < 2; ++part) {
                        float* red = RedBuf(s, rg);
                        WaitChunk(p, s, rg);
                        RowTilesDot(s, red, L, StagePtr(p, s, rg), 2, nb_dim, dstride);
                        ReleaseChunk(p, s, rg);  // its barrier publishes red
                        if (tid < 32) gu[part] = RowTotal(red, 2, tid >> 4, tid & 15);
                    }
                    if (tid < 32) {  // SwiGLU, then the block's digit planes
                        const float sig = 1.0f / (1.0f + expf(-gu[0]));
                        DigitsWarp(gu[0] * sig * gu[1], s.vdig, vstride, s.vsx);
                    }
                    ConsumerBar();
                    WaitChunk(p, s, rg);
                    ColumnDotSmem(L, StagePtr(p, s, rg), ntiles_dim, p.dim, s.vdig, vstride, s.vsx, s.acc);
                    ReleaseChunk(p, s, rg);
                }
                // the residual x_mid joins through CTA 0
                FlushRed(s.acc, xout, p.dim, c == 0 ? p.xmid : nullptr);
                Trace(p, step, l, 6);
                Signal(p, kMkPhases * l + 2);
                Trace(p, step, l, 5);
            }
        }
        // ---------------- lm_head + arg-max
        LoadVecCg(s.nw, p.final_norm, p.dim);  // independent of the wait
        if (!WaitCounter(p, s, kMkPhases * (p.n_layers - 1) + 2, k1 * w_ffn)) return rg.n;
        Trace(p, step, p.n_layers, 0);
        float* xfin = p.xbuf[p.n_layers & 1];
        LoadVecCg(s.xs, xfin, p.dim);
        CpAsyncWaitAll();
        ConsumerBar();
        RmsNormDigits(s.xs, s.nw, p.dim, p.eps, s.dig, dstride, s.sx, s.scratch);
        float best = -INFINITY;
        int besti = 0x7fffffff;
        for (int t2 = c; 2 * t2 < t_lm; t2 += G) {
            // a lone last tile leaves stale bytes in the stage's second half;
            // its rows are past the vocabulary and skipped
            float* red = RedBuf(s, rg);
            WaitChunk(p, s, rg);
            RowTilesDot(s, red, L, StagePtr(p, s, rg), 2, nb_dim, dstride);
            ReleaseChunk(p, s, rg);  // its barrier publishes red
            if (tid < 32) {
                const int r = (2 * t2 + (tid >> 4)) * 16 + (tid & 15);
                if (r < p.vocab) {
                    const float v = RowTotal(red, 2, tid >> 4, tid & 15);
                    p.logits[r] = v;
                    if (v > best || (v == best && r < besti)) {
                        best = v;
                        besti = r;
                    }
                }
            }
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
                RedRelease(p.counters + ctr_token);
            }
        }
        ConsumerBar();
    }
    return rg.n;
}

__global__ void __launch_bounds__(kMkThreads, 1) MegaDecodeKernel(const MegaParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int nb_dim = p.dim / 32;
    // fixed-size buffers first, at compile-time offsets (their addresses
    // need no registers), then the dim-sized ones and the ring
    MkSmem s;
    s.full = reinterpret_cast<uint64_t*>(smem + kOffFull);
    s.flags = reinterpret_cast<int*>(smem + kOffFlags);
    s.scratch = reinterpret_cast<float*>(smem + kOffScratch);
    s.vsx = reinterpret_cast<float*>(smem + kOffVsx);
    s.vdig = reinterpret_cast<int8_t*>(smem + kOffVdig);
    s.red = reinterpret_cast<float*>(smem + kOffRed);
    s.vec = reinterpret_cast<float*>(smem + kOffVec);
    s.att = reinterpret_cast<float*>(smem + kOffAtt);
    s.sc = reinterpret_cast<float*>(smem + kOffSc);
    const size_t vbytes = Round128(4 * size_t(p.dim));
    s.xs = reinterpret_cast<float*>(smem + kOffFixedEnd);
    s.nw = reinterpret_cast<float*>(smem + kOffFixedEnd + vbytes);
    s.dig = reinterpret_cast<int8_t*>(smem + kOffFixedEnd + 2 * vbytes);
    s.sx = reinterpret_cast<float*>(smem + kOffFixedEnd + 2 * vbytes + Round128(4 * size_t(DigitStride(nb_dim))));
    s.acc = reinterpret_cast<float*>(smem + kOffFixedEnd + 2 * vbytes + Round128(4 * size_t(DigitStride(nb_dim))) +
                                     Round128(4 * size_t(nb_dim)));
    const size_t list_off =
        kOffFixedEnd + 3 * vbytes + Round128(4 * size_t(DigitStride(nb_dim))) + Round128(4 * size_t(nb_dim));
    for (int i = threadIdx.x; i < p.dim; i += kMkThreads) s.acc[i] = 0.0f;
    s.list = reinterpret_cast<Chunk*>(smem + list_off);
    s.ring = smem + list_off + Round128(sizeof(Chunk) * size_t(p.list_cap));
    s.kst = reinterpret_cast<float*>(s.ring + Round128(size_t(kMkStages) * p.stage_bytes));
    if (threadIdx.x == 0) {
        for (int i = 0; i < kMkStages; ++i) MbarInit(&s.full[i], 1);
        FenceMbarInit();
        for (int i = 0; i < 8; ++i) s.flags[i] = 0;
        int len = 0;
        ForEachChunk(p, blockIdx.x, gridDim.x, [&](const Chunk& ch) {
            if (len < p.list_cap) s.list[len] = ch;
            ++len;
        });
        s.flags[2] = len;
        if (len > p.list_cap) {  // sized on the host (MegaListCap); an empty list is fine
            atomicCAS(p.status, 0, MLB_ERR_UNSUPPORTED);
            s.flags[0] = 1;
        } else {
            const unsigned total = static_cast<unsigned>(len) * p.n_steps;
            const uint64_t pol = L2EvictFirstPolicy();
            for (unsigned k = 0; k < kMkStages && k < total; ++k) IssueChunk(p, s, k, k % len, pol);
        }
    }
    __syncthreads();
    if (s.flags[0]) return;
    Consumers(p, s);
    // Wait (bounded) for any copy still in flight into this CTA's shared
    // memory.  A slot never holds two copies at once (nothing is issued once
    // the CTA aborts), so the last kMkStages issued chunks cover them all; the
    // ones already consumed return at once.
    ConsumerBar();
    if (threadIdx.x == 0) {
        const unsigned issued = static_cast<unsigned>(s.flags[5]);
        for (unsigned k = issued > kMkStages ? issued - kMkStages : 0; k < issued; ++k)
            MbarWaitFor(&s.full[k % kMkStages], (k / kMkStages) & 1, p.wait_ns, nullptr);
    }
}

}  // namespace

int MegaListCap(const MegaParams& p, int G) {
    auto per = [G](int items) { return (items + G - 1) / G; };  // items of one CTA at most
    const int t_qkv = (p.qd + 15) / 16 + 2 * ((p.kd + 15) / 16);
    const int t_lm = (p.vocab + 15) / 16;
    const AttnPlan ap = AttnSplit(p, G);
    return p.n_layers * (per(t_qkv) + per(ap.items) * (p.hd / 32 / ap.hsplit) + 3 * per(p.hidden / 32)) +
           per((t_lm + 1) / 2);
}

size_t MegaSmemBytes(const MegaParams& p) {
    const int nb_dim = p.dim / 32;
    return kOffFixedEnd + 3 * Round128(4 * size_t(p.dim)) + Round128(4 * size_t(DigitStride(nb_dim))) +
           Round128(4 * size_t(nb_dim)) + Round128(sizeof(Chunk) * size_t(p.list_cap)) +
           Round128(size_t(kMkStages) * p.stage_bytes) + 4 * size_t(p.hd) * p.kst_rows;
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
