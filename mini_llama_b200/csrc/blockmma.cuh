// GEMV for up to 8 rows of x straight from GGUF Q8_0 / Q4_0 / Q4_1 blocks, on
// the integer tensor-core MMA (mma.m16n8k32, s8 or u8 quants x s8 digits ->
// s32), for the quantized linear entry points at row counts 1..8.
//
// Work: a row tile is 16 consecutive weight rows; a unit is one row tile over
// kc consecutive blocks (kc = all blocks of the row when 16 rows fit a slot,
// else a multiple of 8, so every piece of a row starts 16-byte aligned).  A
// group of warps (a pair) owns whole row tiles (all their units in turn) and its
// own ring of shared-memory slots; the leader moves a whole-row unit with one
// bulk copy (16 GGUF rows are contiguous), a split unit with one bulk copy per
// row (lanes 0..15), completing on the slot's mbarrier; weights are read once,
// so the copies mark their lines first to leave the L2.  The group's warps
// split each unit's blocks and meet at one named barrier per unit (after which
// the slot is refilled), adding the followers' partial sums at the end of a
// tile.  Each group starts on two fixed tiles and then takes the next free tile
// from a device counter (fetched one tile ahead, so its latency hides behind a
// tile of work), so groups that run faster take more tiles and all finish
// within about one tile of each other.  After the prologue no group waits on
// another.
//
// MMA operands: A = the quants of one block column of the tile, read from the
// raw blocks (lane (g, t) takes elements 4t..4t+3 and 16+4t..19+4t of rows g
// and g+8; Q8_0/Q4_0 blocks start 2 bytes off a word in every other block, so
// blocks go in pairs: the even block's words are funnel-shifted, the odd
// block's are aligned).  B = x as signed 8-bit digit planes in fragment order,
// built once per CTA: with max|x_b| < 2^E over 32-element block b of x row m,
// X = rint(x * 2^(22-E)) = D2*2^16 + D1*2^8 + D0, and B column 3m + p holds
// plane p, so ceil(3M/8) MMAs per block cover M rows of x.  The int32 sums
// are exact; the accumulator starts at the bit pattern of 1.5*2^23, so the
// result read as a float is 1.5*2^23 + S.  Each column accumulates
// S * w * d_r over the blocks, w = plane weight * 2^(E-22): one FMA of the
// raw result with w and -(1.5*2^23 + c) w gives (S - c) w exactly, a second
// adds it times d_r; the three columns of an x row are added at the end of
// the tile.  Per (row r, x row m) a block adds
//   Q8_0: d_r * 2^(E-22) * (65536 S2 + 256 S1 + S0)           (c = 0)
//   Q4_0: the same with unsigned nibbles n as A and c = 8 sum_k D_p[k],
//         which applies the 8 of (n - 8)
//   Q4_1: d_r * (nibble sums, c = 0) + min_r * sum_k x_b[k].
// The only roundings are the rint of x (2^-23 of the block maximum) and the
// fp32 combine, as in an fp32 dot product.
//
// Replaces the reference kernels Q80LinearKernel / Q40LinearKernel /
// Q41LinearKernel (mini_llama src/cuda_quant.cu:40-135) for 1..8 rows.
#pragma once

#include "qgemv.cuh"

namespace mlb {

constexpr int kBmMaxWarps = 16;
// Warps per group.  A compile-time constant: with the size read from the
// parameters (divisions and loops at run time per unit) a call took 1.6 us
// longer at one row of x on the [151936, 896] shape.  Groups of four
// measured slower at every row count.
constexpr int kBmGroupWarps = 2;
constexpr uint32_t kBmMagic = 0x4B400000u;  // 1.5 * 2^23
constexpr float kBmMagicF = 12582912.0f;

// MMAs per block for M rows of x (three digit columns per row, 8 per MMA).
__host__ __device__ constexpr int BmMmas(int M) { return (3 * M + 7) / 8; }

// Tile scheduler of the launches (one at a time on the library's stream):
// [0] tiles handed out past the fixed ones, [1] CTAs finished.  The last CTA
// to finish puts both back to zero for the next launch.
static __device__ unsigned int g_bm_sched[2];

struct BmParams {
    const float* x;     // [M, K]
    const uint8_t* w;   // GGUF blocks [N, nb], 16-byte aligned
    const float* bias;  // [N] or null
    float* y;           // [M, N]
    int K, N, nb, rowbytes;
    int kc;         // blocks per unit
    int units_k;    // units per row tile (1: whole rows)
    int tiles;      // row tiles
    int slots;      // ring slots per warp group
    int gsize;      // warps per group (kBmGroupWarps): they split each unit's blocks
    int stage_bytes;
    int pitch;      // bytes from one row of a unit to the next in shared memory
    int rowmap;     // 1: MMA rows g, g + 8 are tile rows 2g, 2g + 1; 0: g, g + 8
    int* status;    // MLB_ERR_DEVICE_TIMEOUT when a bounded wait expires
};

template <int QT>
struct BmTraits;
template <>
struct BmTraits<MLB_Q8_0> {
    static constexpr int kBytes = 34;
    static constexpr bool kUnsigned = false;
};
template <>
struct BmTraits<MLB_Q4_0> {
    static constexpr int kBytes = 18;
    static constexpr bool kUnsigned = true;
};
template <>
struct BmTraits<MLB_Q4_1> {
    static constexpr int kBytes = 20;
    static constexpr bool kUnsigned = true;
};

// Shared memory: slots [groups][slots][stage_bytes] | mbarriers
// [groups][slots] | slot tile numbers [groups][slots] int | per group the
// followers' partial sums [2][gsize - 1][NJ][2][32] float2 (the parity buffer
// just read then holds the tile's column sums [16][8 NJ] floats) | B
// fragments [nb][NJ][32] uint2 |
// column records [nb][NJ][4] float4 | Q4_1: x block sums [nb][NJ][4] float2.
struct BmSmem {
    static __host__ __device__ size_t Ring(int groups, int slots, int stage_bytes) {
        return size_t(groups) * slots * stage_bytes;
    }
    static __host__ __device__ size_t Bars(int groups, int slots) {
        return (size_t(groups) * slots * 12 + 15) & ~size_t(15);
    }
    // two buffers (tile parity) of [gsize - 1][NJ][2][32] float2; the leader
    // turns the one it has read into the tile's column sums [16][8 NJ] floats
    static __host__ __device__ size_t GroupScratch(int M, int gsize) {
        return size_t(BmMmas(M)) * 2 * (gsize - 1) * 2 * 32 * 8;
    }
    static __host__ __device__ size_t Scratch(int M, int groups, int gsize) {
        return size_t(groups) * GroupScratch(M, gsize);
    }
    static __host__ __device__ size_t Frag(int M, int nb) { return size_t(nb) * BmMmas(M) * 256; }
    // records (float4), then for Q4_1 the x block sums (float2)
    static __host__ __device__ size_t Rec(int M, int nb, bool sums) {
        return size_t(nb) * BmMmas(M) * (sums ? 64 + 32 : 64);
    }
    static __host__ __device__ size_t Bytes(int M, int nb, int groups, int slots, int stage_bytes, bool sums,
                                            int gsize) {
        return Ring(groups, slots, stage_bytes) + Bars(groups, slots) + Scratch(M, groups, gsize) + Frag(M, nb) +
               Rec(M, nb, sums);
    }
};

__device__ __forceinline__ float2 Half2Bits(uint32_t u) {
    __half2_raw r;
    r.x = static_cast<unsigned short>(u & 0xffffu);
    r.y = static_cast<unsigned short>(u >> 16);
    return __half22float2(__half2(r));
}

template <bool kUnsignedA>
__device__ __forceinline__ void MmaI8(int (&d)[4], const uint32_t (&a)[4], uint2 b, int c0, int c1) {
    if constexpr (kUnsignedA) {
        asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
            "{%8, %9}, {%10, %11, %12, %13};"
            : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b.x), "r"(b.y), "r"(c0), "r"(c1),
              "r"(c0), "r"(c1));
    } else {
        asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
            "{%8, %9}, {%10, %11, %12, %13};"
            : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b.x), "r"(b.y), "r"(c0), "r"(c1),
              "r"(c0), "r"(c1));
    }
}

// One block column of the tile against every x row: NJ MMAs.  acc[j][0] and
// acc[j][1] hold rows g and g + 8 of B columns 8j + 2t and 8j + 2t + 1.  A
// column's record holds w = plane weight * x scale (a power of two, or 0) and
// -(1.5*2^23 + c) * w, c = 8 sum_k D_p[k] for Q4_0 (the 8 of n - 8), else 0;
// one FMA of the raw result gives (S - c) * w exactly, a second adds it times
// d.  dg = (d_g, d_g), d8 = (d_g8, d_g8); for Q4_1, mg and m8 are the rows'
// minimums and xsum[j * 4 + t] the x block sums of the lane's columns (on
// plane-2^16 columns, else 0).
template <int QT, int NJ>
__device__ __forceinline__ void BmBlock(const uint32_t (&a)[4], float2 dg, float2 d8, float mg,
                                        float m8, const uint2* frag, const float4* rec,
                                        const float2* xsum, int lane, int t, float2 (&acc)[NJ][2]) {
#pragma unroll
    for (int j = 0; j < NJ; ++j) {
        const uint2 bf = frag[j * 32 + lane];
        const float4 rc = rec[j * 4 + t];
        int c[4];
        MmaI8<BmTraits<QT>::kUnsigned>(c, a, bf, static_cast<int>(kBmMagic), static_cast<int>(kBmMagic));
        const float2 w = make_float2(rc.x, rc.y), nw = make_float2(rc.z, rc.w);
        const float2 sg = __ffma2_rn(make_float2(__int_as_float(c[0]), __int_as_float(c[1])), w, nw);
        const float2 s8 = __ffma2_rn(make_float2(__int_as_float(c[2]), __int_as_float(c[3])), w, nw);
        acc[j][0] = __ffma2_rn(sg, dg, acc[j][0]);
        acc[j][1] = __ffma2_rn(s8, d8, acc[j][1]);
        if constexpr (QT == MLB_Q4_1) {
            const float2 xs = xsum[j * 4 + t];
            acc[j][0] = __ffma2_rn(make_float2(mg, mg), xs, acc[j][0]);
            acc[j][1] = __ffma2_rn(make_float2(m8, m8), xs, acc[j][1]);
        }
    }
}

// Blocks [i0, i1) of one unit in shared memory (rows of ustride bytes); block
// i is global column b0 + i of the fragment tables.  For Q8_0 / Q4_0, i0 and
// i1 are even.  rowmap picks the tile rows of MMA rows g and g + 8 so that the
// eight rows one load instruction touches start in distinct bank groups: with
// a row pitch of 2 mod 4 words, rows 2g (and 2g + 1) do; with 4 mod 8 words,
// rows g (and g + 8) do.
template <int QT, int NJ>
__device__ __forceinline__ void BmUnit(const uint8_t* unit, int ustride, int rowmap, int i0, int i1, int b0,
                                       const uint2* frags, const float4* recs, const float2* xsums,
                                       int lane, float2 (&acc)[NJ][2]) {
    const int g = lane >> 2, t = lane & 3;
    const uint8_t* rg = unit + (rowmap ? 2 * g : g) * ustride;
    const uint8_t* r8 = rg + (rowmap ? 1 : 8) * ustride;
    if constexpr (QT == MLB_Q4_1) {
        // 20-byte blocks: every block starts on a word
#pragma unroll 2
        for (int i = i0; i < i1; ++i) {
            const uint32_t* pg = reinterpret_cast<const uint32_t*>(rg + i * 20);
            const uint32_t* p8 = reinterpret_cast<const uint32_t*>(r8 + i * 20);
            const uint32_t hg = pg[0], h8 = p8[0];
            const uint32_t qg = pg[1 + t], q8 = p8[1 + t];
            uint32_t a[4];
            a[0] = qg & 0x0F0F0F0Fu;
            a[1] = q8 & 0x0F0F0F0Fu;
            a[2] = (qg >> 4) & 0x0F0F0F0Fu;
            a[3] = (q8 >> 4) & 0x0F0F0F0Fu;
            const float2 dg = Half2Bits(__byte_perm(hg, 0, 0x1010));
            const float2 d8 = Half2Bits(__byte_perm(h8, 0, 0x1010));
            const float2 mn = Half2Bits(__byte_perm(hg, h8, 0x7632));
            const size_t bi = size_t(b0 + i) * NJ;
            BmBlock<QT, NJ>(a, dg, d8, mn.x, mn.y, frags + bi * 32, recs + bi * 4, xsums + bi * 4, lane, t,
                            acc);
        }
    } else {
        // block pairs (2i, 2i+1) start on a word; the even block's quants are
        // 2 bytes past it, the odd block's on a word
        constexpr int kBB = BmTraits<QT>::kBytes;
#pragma unroll 2
        for (int i = i0; i < i1; i += 2) {
            const uint32_t* pg = reinterpret_cast<const uint32_t*>(rg + i * kBB);
            const uint32_t* p8 = reinterpret_cast<const uint32_t*>(r8 + i * kBB);
            uint32_t ae[4], ao[4];
            uint32_t hg, h8, og, o8;  // words holding the even / odd scales
            if constexpr (QT == MLB_Q8_0) {
                // words 0..16 of the 68-byte pair: even d = bytes 0-1, even
                // quants 2..33, odd d = bytes 34-35, odd quants 36..67
                ae[0] = __funnelshift_r(pg[t], pg[t + 1], 16);
                ae[1] = __funnelshift_r(p8[t], p8[t + 1], 16);
                ae[2] = __funnelshift_r(pg[t + 4], pg[t + 5], 16);
                ae[3] = __funnelshift_r(p8[t + 4], p8[t + 5], 16);
                ao[0] = pg[9 + t];
                ao[1] = p8[9 + t];
                ao[2] = pg[13 + t];
                ao[3] = p8[13 + t];
                hg = pg[0];
                h8 = p8[0];
                og = pg[8];
                o8 = p8[8];
            } else {
                // Q4_0, words 0..8 of the 36-byte pair: even d = bytes 0-1,
                // even nibbles 2..17, odd d = bytes 18-19, odd nibbles 20..35
                const uint32_t qg = __funnelshift_r(pg[t], pg[t + 1], 16);
                const uint32_t q8 = __funnelshift_r(p8[t], p8[t + 1], 16);
                const uint32_t vg = pg[5 + t], v8 = p8[5 + t];
                ae[0] = qg & 0x0F0F0F0Fu;
                ae[1] = q8 & 0x0F0F0F0Fu;
                ae[2] = (qg >> 4) & 0x0F0F0F0Fu;
                ae[3] = (q8 >> 4) & 0x0F0F0F0Fu;
                ao[0] = vg & 0x0F0F0F0Fu;
                ao[1] = v8 & 0x0F0F0F0Fu;
                ao[2] = (vg >> 4) & 0x0F0F0F0Fu;
                ao[3] = (v8 >> 4) & 0x0F0F0F0Fu;
                hg = pg[0];
                h8 = p8[0];
                og = pg[4];
                o8 = p8[4];
            }
            const size_t bi = size_t(b0 + i) * NJ;
            BmBlock<QT, NJ>(ae, Half2Bits(__byte_perm(hg, 0, 0x1010)), Half2Bits(__byte_perm(h8, 0, 0x1010)),
                            0.0f, 0.0f, frags + bi * 32, recs + bi * 4, nullptr, lane, t, acc);
            BmBlock<QT, NJ>(ao, Half2Bits(__byte_perm(og, 0, 0x3232)), Half2Bits(__byte_perm(o8, 0, 0x3232)),
                            0.0f, 0.0f, frags + (bi + NJ) * 32, recs + (bi + NJ) * 4, nullptr, lane, t,
                            acc);
        }
    }
}

// Barrier of the warps of a group (named barrier id, `threads` threads) that
// also ORs a flag over them, so all take the same branch after it.
__device__ __forceinline__ bool GroupBarrierOr(int id, int threads, bool flag) {
    uint32_t r;
    asm volatile(
        "{\n .reg .pred p, q;\n setp.ne.u32 q, %1, 0;\n bar.red.or.pred p, %2, %3, q;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(r)
        : "r"(static_cast<uint32_t>(flag)), "r"(id), "r"(threads)
        : "memory");
    return r != 0;
}

// x rows -> digit-plane B fragments and column records (all threads; ends
// with a CTA barrier).  Eight threads per (x row m, block b), one 4-element
// group each, for m < kRows: a row past M fills the spare columns with zero
// digits and weights.  x is read from global memory (rows of K floats).
template <int QT, int M>
__device__ __forceinline__ void BmBuildTables(const float* x, int K, int nb, uint2* frags, float4* recs,
                                              float2* xsums) {
    constexpr int NJ = BmMmas(M);
    constexpr int kCols = 8 * NJ;
    constexpr int kRows = (kCols + 2) / 3;  // x rows whose columns fill the MMAs
    const int sub = threadIdx.x & 7;        // group: elements 4 sub .. 4 sub + 3
    const int total = kRows * nb;
    const int per_round = blockDim.x >> 3;
    // the same number of rounds for every thread, so the group shuffles
    // always see the whole warp
    for (int base = 0; base < total; base += per_round) {
        const int item = base + (threadIdx.x >> 3);
        const bool live = item < total;
        const int m = live ? item / nb : 0, b = live ? item - m * nb : 0;
        float v[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        if (live && m < M) {
            const int k0 = b * 32 + 4 * sub;
            const float* src = x + size_t(m) * K + k0;
            if (k0 + 4 <= K && (reinterpret_cast<uintptr_t>(src) & 15) == 0) {
                const float4 f = __ldg(reinterpret_cast<const float4*>(src));
                v[0] = f.x;
                v[1] = f.y;
                v[2] = f.z;
                v[3] = f.w;
            } else {
#pragma unroll
                for (int i = 0; i < 4; ++i) v[i] = k0 + i < K ? __ldg(src + i) : 0.0f;
            }
        }
        float mx = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
#pragma unroll
        for (int o = 1; o < 8; o <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        const int e = static_cast<int>((__float_as_uint(mx) >> 23) & 0xff) - 126;  // mx < 2^e
        float up = 0.0f, s = 0.0f;
        if (mx > 0.0f && e >= -104) {
            up = __uint_as_float(static_cast<uint32_t>(127 + 22 - e) << 23);
            s = __uint_as_float(static_cast<uint32_t>(127 + e - 22) << 23);
        }
        uint32_t wd[3] = {0u, 0u, 0u};  // planes 2^16, 2^8, 1
        int dsum[3] = {0, 0, 0};
        float xsum = (v[0] + v[1]) + (v[2] + v[3]);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int xi = __float2int_rn(v[i] * up);
            const int d0 = (xi << 24) >> 24;
            const int x1 = (xi - d0) >> 8;
            const int d1 = (x1 << 24) >> 24;
            const int d2 = (x1 - d1) >> 8;
            wd[0] |= (static_cast<uint32_t>(d2) & 0xffu) << (8 * i);
            wd[1] |= (static_cast<uint32_t>(d1) & 0xffu) << (8 * i);
            wd[2] |= (static_cast<uint32_t>(d0) & 0xffu) << (8 * i);
            dsum[0] += d2;
            dsum[1] += d1;
            dsum[2] += d0;
        }
        if constexpr (QT == MLB_Q4_0) {
#pragma unroll
            for (int o = 1; o < 8; o <<= 1)
#pragma unroll
                for (int pl = 0; pl < 3; ++pl) dsum[pl] += __shfl_xor_sync(0xffffffffu, dsum[pl], o);
        }
        if constexpr (QT == MLB_Q4_1) {
#pragma unroll
            for (int o = 1; o < 8; o <<= 1) xsum += __shfl_xor_sync(0xffffffffu, xsum, o);
        }
        if (!live) continue;
        // column c of MMA c / 8 is fragment lane 4 (c % 8) + (k & 15) / 4,
        // word k / 16; this thread's elements k = 4 sub + i
#pragma unroll
        for (int pl = 0; pl < 3; ++pl) {
            const int c = 3 * m + pl;
            if (c < kCols) {
                uint32_t* fw = reinterpret_cast<uint32_t*>(frags + (size_t(b) * NJ + (c >> 3)) * 32);
                fw[(4 * (c & 7) + (sub & 3)) * 2 + (sub >> 2)] = wd[pl];
            }
        }
        // records: lane t of MMA j reads record (b, j, t) = w of columns
        // 8j + 2t (x) and 8j + 2t + 1 (y), then -(1.5*2^23 + c) w of the same
        // two columns (all exact: w is a power of two or 0)
        if (sub == 0) {
            const float pw[3] = {65536.0f, 256.0f, 1.0f};
#pragma unroll
            for (int pl = 0; pl < 3; ++pl) {
                const int c = 3 * m + pl;
                if (c >= kCols) continue;
                const size_t ri = (size_t(b) * NJ + (c >> 3)) * 4 + ((c & 7) >> 1);
                float* rf = reinterpret_cast<float*>(recs + ri);
                const int u = c & 1;
                const float w = pw[pl] * s;
                const float off = (QT == MLB_Q4_0) ? kBmMagicF + static_cast<float>(8 * dsum[pl]) : kBmMagicF;
                rf[u] = w;
                rf[2 + u] = -off * w;
                if constexpr (QT == MLB_Q4_1) reinterpret_cast<float*>(xsums + ri)[u] = pl == 0 ? xsum : 0.0f;
            }
        }
    }
    __syncthreads();
}

template <int QT, int M>
__global__ void __launch_bounds__(kBmMaxWarps * 32, 1) BlockMmaGemvKernel(const BmParams p) {
    constexpr int NJ = BmMmas(M);
    constexpr int kCols = 8 * NJ;
    constexpr int kBB = BmTraits<QT>::kBytes;
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr int gs = kBmGroupWarps;
    const int nw = blockDim.x >> 5, ngroups = nw / gs;  // warp groups
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const int grp = warp / gs, member = warp - grp * gs;
    const bool leader = member == 0;
    const int ns = p.slots;
    uint8_t* ring = smem;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + BmSmem::Ring(ngroups, ns, p.stage_bytes));
    volatile int* slot_tiles = reinterpret_cast<volatile int*>(bars + ngroups * ns);
    uint8_t* scratch_all = reinterpret_cast<uint8_t*>(bars) + BmSmem::Bars(ngroups, ns);
    uint2* frags = reinterpret_cast<uint2*>(scratch_all + BmSmem::Scratch(M, ngroups, gs));
    float4* recs = reinterpret_cast<float4*>(reinterpret_cast<uint8_t*>(frags) + BmSmem::Frag(M, p.nb));
    float2* xsums = reinterpret_cast<float2*>(recs + size_t(p.nb) * NJ * 4);
    uint8_t* myring = ring + size_t(grp) * ns * p.stage_bytes;
    uint64_t* mybars = bars + grp * ns;
    volatile int* mytiles = slot_tiles + grp * ns;
    // per group: the followers' partial sums (two buffers by tile parity) and
    // the tile's column sums
    uint8_t* scratch = scratch_all + size_t(grp) * BmSmem::GroupScratch(M, gs);
    float2* xbuf = reinterpret_cast<float2*>(scratch);
    const int xpar = (gs - 1) * NJ * 2 * 32;  // float2 per parity buffer

    const int gp = blockIdx.x * ngroups + grp, GP = gridDim.x * ngroups;
    const int ustride = p.pitch;

    if (leader && lane == 0) {
        for (int s = 0; s < ns; ++s) MbarInit(&mybars[s], 1);
        FenceMbarInit();
    }
    __syncwarp();

    // Issue cursor (leader warp): the tile and unit to copy next (i_tile < 0:
    // take the next tile when the next unit is issued).  Tiles: gp, gp + GP,
    // then 2 GP + (the device counter), fetched a tile before it is needed.
    int i_tile = gp, i_u = 0, i_slot = 0, inflight = 0, n_fixed = 1;
    bool i_done = false;
    unsigned int pending = 0u;
    auto next_tile = [&]() -> int {
        int tl;
        if (n_fixed < 2) {
            tl = gp + GP;
            n_fixed = 2;
        } else {
            tl = 2 * GP + static_cast<int>(__shfl_sync(0xffffffffu, pending, 0));
        }
        if (tl < p.tiles && lane == 0) pending = atomicAdd(&g_bm_sched[0], 1u);
        return tl;
    };
    auto issue = [&]() {  // leader warp only
        if (i_done) return;
        if (i_tile < 0) i_tile = next_tile();
        uint8_t* dst = myring + size_t(i_slot) * p.stage_bytes;
        uint64_t* bar = &mybars[i_slot];
        ++inflight;
        if (i_tile >= p.tiles) {
            // no more tiles: a phase without data tells the group to stop
            if (lane == 0) {
                mytiles[i_slot] = -1;
                asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(SmemAddr(bar)) : "memory");
            }
            i_done = true;
        } else {
            const int row0 = i_tile * 16;
            const int rows = min(16, p.N - row0);
            if (lane == 0) mytiles[i_slot] = i_tile;  // published by the arrive below
            if (p.units_k == 1) {
                const uint32_t body = static_cast<uint32_t>(rows * p.rowbytes) & ~15u;
                if (lane == 0) {
                    MbarExpectTx(bar, body);
                    BulkLoadHint(dst, p.w + size_t(row0) * p.rowbytes, body, bar, L2EvictFirstPolicy());
                }
            } else {
                const int k0 = i_u * p.kc;
                const uint32_t seg = static_cast<uint32_t>(min(p.kc, p.nb - k0) * kBB);
                if (lane == 0) MbarExpectTx(bar, seg * rows);
                __syncwarp();
                if (lane < rows)
                    BulkLoadHint(dst + size_t(lane) * ustride,
                                 p.w + size_t(row0 + lane) * p.rowbytes + size_t(k0) * kBB, seg, bar,
                                 L2EvictFirstPolicy());
            }
            if (++i_u == p.units_k) {
                i_u = 0;
                i_tile = -1;
            }
        }
        if (++i_slot == ns) i_slot = 0;
    };

    GridDepWait();
    // x's lines into L2 ahead of the weight stream, then one unit per group
    // (x's reads queue behind only half the ring), x's tables, the rest of
    // the ring
    for (int i = threadIdx.x; i < (M * p.K + 31) / 32; i += blockDim.x)
        asm volatile("prefetch.global.L2 [%0];" ::"l"(p.x + size_t(i) * 32));
    if (leader) issue();
    BmBuildTables<QT, M>(p.x, p.K, p.nb, frags, recs, xsums);  // ends with a CTA barrier
    if (leader)
        for (int s = 1; s < ns; ++s) issue();
    GridDepLaunch();

    float2 acc[NJ][2];
#pragma unroll
    for (int j = 0; j < NJ; ++j) acc[j][0] = acc[j][1] = make_float2(0.0f, 0.0f);
    int c_u = 0, c_slot = 0, parity = 0;
    uint32_t phase = 0;
    for (;;) {
        uint8_t* unit = myring + size_t(c_slot) * p.stage_bytes;
        const bool ok = MbarWait(&mybars[c_slot], phase);
        const int tile = ok ? mytiles[c_slot] : -1;  // read before the slot is refilled
        const bool run = tile >= 0;                  // false: stop mark or expired wait
        const int row0 = tile * 16;
        const bool tile_end = c_u + 1 == p.units_k;
        if (run) {
            if (p.units_k == 1) {
                // the last tile may end a few bytes past a 16-byte boundary
                // (both warps write the same bytes)
                const int total = min(16, p.N - row0) * p.rowbytes;
                const int tail = total & 15;
                if (tail) {
                    if (lane < tail) unit[total - tail + lane] = p.w[size_t(row0) * p.rowbytes + total - tail + lane];
                    __syncwarp();
                }
            }
            // member r of the group takes blocks [b_r, b_{r+1}) of the unit
            // (whole block pairs for Q8_0 / Q4_0)
            const int k0 = c_u * p.kc, kcc = min(p.kc, p.nb - k0);
            int i0, i1;
            if (QT == MLB_Q4_1) {
                i0 = kcc * member / gs;
                i1 = kcc * (member + 1) / gs;
            } else {
                i0 = (kcc / 2) * member / gs * 2;
                i1 = (kcc / 2) * (member + 1) / gs * 2;
            }
            BmUnit<QT, NJ>(unit, ustride, p.rowmap, i0, i1, k0, frags, recs, xsums, lane, acc);
            if (tile_end && !leader) {
                float2* xb = xbuf + parity * xpar + (member - 1) * NJ * 2 * 32;
#pragma unroll
                for (int j = 0; j < NJ; ++j) {
                    xb[(j * 2) * 32 + lane] = acc[j][0];
                    xb[(j * 2 + 1) * 32 + lane] = acc[j][1];
                }
            }
        }
        // the group has read the slot; either all go on or all stop (at the
        // stop mark, or when any warp's wait expired)
        if (GroupBarrierOr(1 + grp, 32 * gs, !run)) {
            if (!ok && lane == 0 && p.status) atomicExch(p.status, MLB_ERR_DEVICE_TIMEOUT);
            // leave no copy in flight into shared memory: wait (bounded) for
            // the other issued units (none after the stop mark), then stop
            if (leader) {
                int sl = c_slot;
                uint32_t ph = phase;
                for (int k = 1; k < inflight; ++k) {
                    if (++sl == ns) {
                        sl = 0;
                        ph ^= 1u;
                    }
                    MbarWait(&mybars[sl], ph);
                }
            }
            break;
        }
        if (leader) {
            --inflight;
            issue();  // into the slot just read
        }
        if (++c_slot == ns) {
            c_slot = 0;
            phase ^= 1u;
        }
        if (tile_end) {
            if (leader) {
                // column sums of the tile: leader + follower partials (in
                // member order), written over the partials once all lanes
                // have read them
                float2* xb = xbuf + parity * xpar;
                float* colsum = reinterpret_cast<float*>(xb);
                for (int f = 0; f < gs - 1; ++f) {
#pragma unroll
                    for (int j = 0; j < NJ; ++j) {
                        acc[j][0] = __fadd2_rn(acc[j][0], xb[(f * NJ + j) * 2 * 32 + lane]);
                        acc[j][1] = __fadd2_rn(acc[j][1], xb[((f * NJ + j) * 2 + 1) * 32 + lane]);
                    }
                }
                __syncwarp();
#pragma unroll
                for (int j = 0; j < NJ; ++j) {
#pragma unroll
                    for (int r = 0; r < 2; ++r) {
                        const int trow = p.rowmap ? 2 * g + r : g + 8 * r;
                        float* cs = colsum + trow * kCols + 8 * j + 2 * t;
                        cs[0] = acc[j][r].x;
                        cs[1] = acc[j][r].y;
                    }
                }
                __syncwarp();
                // y[m, n] = sum of the three digit columns of x row m
                for (int e = lane; e < 16 * M; e += 32) {
                    const int r = e & 15, m = e >> 4;
                    const int n = row0 + r;
                    if (n < p.N) {
                        const float* cs = colsum + r * kCols + 3 * m;
                        p.y[size_t(m) * p.N + n] = (cs[0] + cs[1]) + cs[2] + (p.bias ? p.bias[n] : 0.0f);
                    }
                }
                __syncwarp();
            }
#pragma unroll
            for (int j = 0; j < NJ; ++j) acc[j][0] = acc[j][1] = make_float2(0.0f, 0.0f);
            parity ^= 1;
            c_u = 0;
        } else {
            ++c_u;
        }
    }
    // every counter fetch has returned before the CTA reports; the last CTA
    // resets the scheduler for the next launch
    if (leader && lane == 0) asm volatile("" ::"r"(pending));
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        if (atomicAdd(&g_bm_sched[1], 1u) == gridDim.x - 1) {
            atomicExch(&g_bm_sched[0], 0u);
            atomicExch(&g_bm_sched[1], 0u);
        }
    }
}

struct BmPlan {
    bool ok = false;
    int grid = 0;
    int warps = 0;
    size_t smem = 0;
};

// Tiling, ring and grid of one launch; ok = false when the shape needs the
// other GEMV (odd block count of Q8_0/Q4_0, misaligned weights, or no room).
BmPlan PlanBlockMma(BmParams& p, int qtype, int M, int sm_count, int max_smem);
void LaunchBlockMma(int qtype, int M, const BmParams& p, const BmPlan& plan, cudaStream_t stream);

}  // namespace mlb
