// Quantized linear for 9..64 rows of x on the integer MMA (mma.m16n8k32,
// x digits s8 x GGUF quants s8 / u8 -> exact s32 block sums), for the row
// counts where one weight pass must serve many rows but the tcgen05 tile
// pipeline is still dominated by its fixed costs.
//
// Operands of one MMA: A = 16 digit rows of x over one 32-element block (x row
// m split per block as X = rint(x 2^(22-E)) = D2 2^16 + D1 2^8 + D0, digit row
// (plane p, row m)); B = 8 weight rows of the same block, read straight from
// the raw GGUF bytes in shared memory (Q8_0: s8 quants; Q4_0 / Q4_1: the
// nibbles as u8, low nibbles = elements 0..15, high = 16..31, so one 32-bit
// word gives both halves of a fragment).  The accumulator starts at the bit
// pattern of 1.5 * 2^23, so each result read as a float is 1.5 * 2^23 + S;
// one FMA with a per-digit-row record (w, -(1.5 * 2^23 + c) w), w = plane
// weight * 2^(E-22), gives (S - c) w exactly (c = 8 sum D for Q4_0: the 8 of
// n - 8), and a second adds it times the weight row's scale d.  The three
// planes of an x row accumulate into the same fp32 sums; Q4_1 adds
// min * (sum of x over the block) once per block.
//
// x's digit fragments and records are built once per call by WidePrepX into a
// table in global memory (per block, contiguous, so a range of blocks is one
// bulk copy).  The main kernel's CTA owns 128 weight rows and a range of
// blocks: a producer warp streams the rows' raw bytes (2-D tensor-map boxes,
// or one bulk copy per row when the rows do not fit such a view) and the
// table range into a ring of stages; eight warps consume them, two groups of
// four splitting each stage's blocks, each warp 32 weight rows x all x rows
// (one A fragment feeds four MMAs).  With the blocks split over CTAs, partial
// sums go to the workspace and WideReduce adds them in split order with the
// bias (deterministic).
//
// Replaces, for 9..64 rows, the reference kernels Q80LinearKernel /
// Q40LinearKernel / Q41LinearKernel (mini_llama src/cuda_quant.cu:40-135).
#include <algorithm>
#include <cstring>

#include "qgemv.cuh"

namespace mlb {
namespace {

constexpr uint32_t kWMagic = 0x4B400000u;  // 1.5 * 2^23
constexpr float kWMagicF = 12582912.0f;
constexpr int kWRows = 128;                 // weight rows per CTA
constexpr int kWBlocks = 4;                 // blocks per stage
constexpr int kWMaxStages = 4;
constexpr int kWJ = 4;                      // 8-row B fragments per consuming warp
constexpr int kWRowGroups = kWRows / (8 * kWJ);
constexpr int kWWarps = 2 * kWRowGroups;    // consuming warps: two block groups
constexpr int kWThreads = (kWWarps + 1) * 32;
constexpr int kWHeader = 256;
constexpr uint64_t kWWaitNs = 2000000000ull;

template <int QT>
struct WTraits;
template <>
struct WTraits<MLB_Q8_0> {
    static constexpr int kBytes = 34;
};
template <>
struct WTraits<MLB_Q4_0> {
    static constexpr int kBytes = 18;
};
template <>
struct WTraits<MLB_Q4_1> {
    static constexpr int kBytes = 20;
};

// Table bytes of one block for MQ groups of 16 x rows: 3 MQ A fragments
// (32 lanes x 16 bytes), 3 MQ x 8 records (float4: w and -(magic + c) w of
// digit rows g and g + 8), MQ x 8 x sums (float2, Q4_1).
__host__ __device__ constexpr int WTabBlock(int MQ) { return 3 * MQ * 512 + 3 * MQ * 128 + MQ * 64; }
__host__ __device__ constexpr int WTabSums(int MQ) { return 3 * MQ * 640; }

// One launch covers up to kWMaxSegs weight matrices that read the same x
// (same K and block type): their row groups follow one another in the grid.
constexpr int kWMaxSegs = 3;

struct WideParams {
    const uint8_t* w[kWMaxSegs];  // GGUF blocks [N_s, nb], 16-byte aligned
    const float* bias[kWMaxSegs];  // [N_s] or null (applied here when splits == 1)
    float* y[kWMaxSegs];           // [M, N_s]
    float* part[kWMaxSegs];        // partial sums [splits][M][N_s] (splits > 1)
    int N[kWMaxSegs];
    int tma_rows[kWMaxSegs];       // P > 0: rows arrive as P tensor-map boxes per stage; 0: one bulk copy per row
    int rg_end[kWMaxSegs];         // row groups of segments 0..s together
    int nseg;
    const uint8_t* tab;  // x tables [nb][WTabBlock(MQ)]
    int M, nb, rowbytes;
    int kper;            // blocks per split (a multiple of kWBlocks)
    int splits;
    int pitch;           // bytes per weight row in a stage
    int stage_bytes;     // kWRows * pitch + kWBlocks * WTabBlock(MQ)
    int stages;          // ring stages (2..kWMaxStages)
    int* status;
};

__device__ __forceinline__ float2 HalfPair(uint32_t lo16, uint32_t hi16) {
    __half2_raw r;
    r.x = static_cast<unsigned short>(lo16 & 0xffffu);
    r.y = static_cast<unsigned short>(hi16 & 0xffffu);
    return __half22float2(__half2(r));
}

__device__ __forceinline__ void WTmaLoad2D(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        ::"r"(SmemAddr(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(SmemAddr(bar))
        : "memory");
}

__device__ __forceinline__ void WArrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(SmemAddr(bar)) : "memory");
}

template <bool kUnsignedB>
__device__ __forceinline__ void WMma(int (&d)[4], const uint4& a, uint32_t b0, uint32_t b1) {
    const int c = static_cast<int>(kWMagic);
    if constexpr (kUnsignedB) {
        asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.u8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
            "{%8, %9}, {%10, %10, %10, %10};"
            : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
            : "r"(a.x), "r"(a.y), "r"(a.z), "r"(a.w), "r"(b0), "r"(b1), "r"(c));
    } else {
        asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
            "{%8, %9}, {%10, %10, %10, %10};"
            : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
            : "r"(a.x), "r"(a.y), "r"(a.z), "r"(a.w), "r"(b0), "r"(b1), "r"(c));
    }
}

// ---------------------------------------------------------------- x tables
// Eight threads per (x row m < 16 MQ, block b), four elements each; rows
// past M get zero digits, records and sums.  Fragment lane of digit row r of
// a 16-row fragment, element k: lane 4 (r % 8) + (k % 16) / 4, word
// 2 (k / 16) + r / 8 (the m16n8k32 A layout).
template <int QT, int MQ>
__global__ void __launch_bounds__(256) WidePrepX(const float* x, int M, int K, int nb, uint8_t* tab) {
    GridDepWait();    // x belongs to the previous kernel until it finishes
    GridDepLaunch();  // the main kernel's prologue (barriers, weight copies) may start
    constexpr int NF = 3 * MQ;
    const int sub = threadIdx.x & 7;
    const int item = blockIdx.x * 32 + (threadIdx.x >> 3);
    const bool live = item < 16 * MQ * nb;
    const int m = live ? item / nb : 0, b = live ? item - m * nb : 0;
    float v[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    const int k0 = b * 32 + 4 * sub;
    if (live && m < M) {
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
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) {
#pragma unroll
        for (int pl = 0; pl < 3; ++pl) dsum[pl] += __shfl_xor_sync(0xffffffffu, dsum[pl], o);
        xsum += __shfl_xor_sync(0xffffffffu, xsum, o);
    }
    if (!live) return;
    uint8_t* tb = tab + size_t(b) * WTabBlock(MQ);
    const int q = m >> 4, r = m & 15, g = r & 7, hi = r >> 3;
    const int lane = 4 * g + (sub & 3), word = 2 * (sub >> 2) + hi;
#pragma unroll
    for (int pl = 0; pl < 3; ++pl) {
        const int f = pl * MQ + q;
        reinterpret_cast<uint32_t*>(tb)[(f * 32 + lane) * 4 + word] = wd[pl];
    }
    if (sub == 0) {
        const float pw[3] = {65536.0f, 256.0f, 1.0f};
        float* rec = reinterpret_cast<float*>(tb + NF * 512);
#pragma unroll
        for (int pl = 0; pl < 3; ++pl) {
            const int f = pl * MQ + q;
            const float wv = pw[pl] * s;
            const float off = (QT == MLB_Q4_0) ? kWMagicF + static_cast<float>(8 * dsum[pl]) : kWMagicF;
            rec[(f * 8 + g) * 4 + 2 * hi] = wv;
            rec[(f * 8 + g) * 4 + 2 * hi + 1] = -off * wv;
        }
        float* xs = reinterpret_cast<float*>(tb + WTabSums(MQ));
        xs[(q * 8 + g) * 2 + hi] = (QT == MLB_Q4_1 && m < M) ? xsum : 0.0f;
    }
}

// Sum of the split partials [splits][M][N] in split order, plus bias.
__global__ void __launch_bounds__(256) WideReduce(const float* part, int splits, int M, int N, const float* bias,
                                                  float* y) {
    GridDepWait();
    const size_t mn = size_t(M) * N;
    for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < mn; i += size_t(gridDim.x) * blockDim.x) {
        float acc = bias ? bias[i % N] : 0.0f;
        for (int s = 0; s < splits; ++s) acc += __ldg(part + s * mn + i);
        y[i] = acc;
    }
}


// One CTA: weight rows [n0, n0 + 128) over blocks [kb0, kb1) of its split.
// The last warp produces the stages; the others consume them (warp w: block
// group w / kWRowGroups, weight rows 8 kWJ (w % kWRowGroups) onwards).  Every
// wait is bounded: an expired wait sets the status word and the abort flag,
// the consumers skip the epilogue, and the producer waits (bounded) for its
// copies in flight.
template <int QT, int MQ>
__global__ void __launch_bounds__(kWThreads, 1) WideGemvKernel(const WideParams p,
                                                                const __grid_constant__ CUtensorMap wmap0,
                                                                const __grid_constant__ CUtensorMap wmap1,
                                                                const __grid_constant__ CUtensorMap wmap2) {
    constexpr int NF = 3 * MQ;
    constexpr int kBB = WTraits<QT>::kBytes;
    constexpr int kTab = WTabBlock(MQ);
    constexpr bool kU = QT != MLB_Q8_0;
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);
    uint64_t* empty = full + kWMaxStages;
    volatile int* abort = reinterpret_cast<volatile int*>(empty + kWMaxStages);
    uint8_t* stages = smem + kWHeader;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    // this CTA's weight matrix (fields picked with constant indices, so the
    // parameters stay where they are)
    int seg = 0;
    if (p.nseg > 1 && static_cast<int>(blockIdx.x) >= p.rg_end[0]) seg = 1;
    if (p.nseg > 2 && static_cast<int>(blockIdx.x) >= p.rg_end[1]) seg = 2;
    auto pick = [&](auto a0, auto a1, auto a2) { return seg == 0 ? a0 : (seg == 1 ? a1 : a2); };
    const uint8_t* const W = pick(p.w[0], p.w[1], p.w[2]);
    const int N = pick(p.N[0], p.N[1], p.N[2]);
    const int tma = pick(p.tma_rows[0], p.tma_rows[1], p.tma_rows[2]);
    const CUtensorMap* const wmap = pick(&wmap0, &wmap1, &wmap2);
    const int rg_first = seg == 0 ? 0 : pick(0, p.rg_end[0], p.rg_end[1]);
    const int n0 = (static_cast<int>(blockIdx.x) - rg_first) * kWRows, sp = blockIdx.y;
    const int kb0 = sp * p.kper, kb1 = min(p.nb, kb0 + p.kper);
    const int nst = (kb1 - kb0 + kWBlocks - 1) / kWBlocks;
    const size_t rowbytes = static_cast<size_t>(p.rowbytes);
    const int ns = p.stages;
    if (threadIdx.x == 0) {
        for (int i = 0; i < ns; ++i) {
            MbarInit(&full[i], 2);  // the producer's expect_tx, then its arrival after any tail bytes
            MbarInit(&empty[i], kWWarps);
        }
        *abort = 0;
        FenceMbarInit();
    }
    __syncthreads();

    if (warp == kWWarps) {
        // ---------------------------------------------------------- producer
        const uintptr_t wend = reinterpret_cast<uintptr_t>(W) + size_t(N) * rowbytes;
        auto fail = [&]() {
            if (lane == 0) {
                *abort = 1;
                if (p.status) atomicExch(p.status, MLB_ERR_DEVICE_TIMEOUT);
            }
        };
        // stage s's weight rows (first arrival, with the whole stage's bytes)
        auto issue_rows = [&](int s) {
            const int slot = s % ns;
            const int b0 = kb0 + s * kWBlocks, nblk = min(kWBlocks, kb1 - b0);
            uint8_t* st = stages + size_t(slot) * p.stage_bytes;
            if (tma) {
                // P boxes of (pitch bytes x 128 / P rows): weight row P i + j
                // lands in box j, row i (rows past N and bytes past a row read
                // as zeros)
                if (lane == 0) {
                    const int P = tma, rows = kWRows / P;
                    MbarExpectTx(&full[slot], static_cast<uint32_t>(kWRows * p.pitch + nblk * kTab));
                    const long long k0 = static_cast<long long>(b0) * kBB;
                    for (int j = 0; j < P; ++j)
                        WTmaLoad2D(st + size_t(j) * rows * p.pitch, wmap,
                                   static_cast<int>((j * static_cast<long long>(rowbytes) + k0) & ~15LL), n0 / P,
                                   &full[slot]);
                }
                __syncwarp();
                return;
            }
            // one bulk copy per row (rows lane + 32 i), 16-byte aligned
            // around the range; the buffer's last bytes by plain loads
            uint32_t bytes = 0;
            uintptr_t src[4], s16[4];
            uint32_t len[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int n = min(n0 + lane + 32 * i, N - 1);
                src[i] = reinterpret_cast<uintptr_t>(W) + size_t(n) * rowbytes + size_t(b0) * kBB;
                const uintptr_t end = src[i] + size_t(nblk) * kBB;
                s16[i] = src[i] & ~uintptr_t(15);
                uintptr_t l = (end - s16[i] + 15) & ~uintptr_t(15);
                if (s16[i] + l > wend) l = (wend - s16[i]) & ~uintptr_t(15);
                len[i] = static_cast<uint32_t>(l);
                bytes += len[i];
            }
            bytes = __reduce_add_sync(0xffffffffu, bytes);
            if (lane == 0) MbarExpectTx(&full[slot], bytes + static_cast<uint32_t>(nblk * kTab));
            __syncwarp();
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                uint8_t* dst = st + size_t(lane + 32 * i) * p.pitch;
                if (len[i])
                    BulkLoadHint(dst, reinterpret_cast<const void*>(s16[i]), len[i], &full[slot], L2EvictFirstPolicy());
                const uintptr_t end = src[i] + size_t(nblk) * kBB;
                for (uintptr_t q = s16[i] + len[i]; q < end; ++q)
                    dst[q - s16[i]] = __ldg(reinterpret_cast<const unsigned char*>(q));
            }
        };
        // stage s's table range (second arrival, after the warp's tail bytes)
        auto issue_tab = [&](int s) {
            const int slot = s % ns;
            const int b0 = kb0 + s * kWBlocks, nblk = min(kWBlocks, kb1 - b0);
            uint8_t* st = stages + size_t(slot) * p.stage_bytes;
            if (lane == 0)
                BulkLoad(st + size_t(kWRows) * p.pitch, p.tab + size_t(b0) * kTab, static_cast<uint32_t>(nblk * kTab),
                         &full[slot]);
            __syncwarp();
            if (lane == 0) WArrive(&full[slot]);
        };
        // the first stages' weight rows do not depend on the previous kernels
        const int first = min(nst, ns);
        for (int s = 0; s < first; ++s) issue_rows(s);
        GridDepWait();  // x's tables are the pre-pass's output
        for (int s = 0; s < first; ++s) issue_tab(s);
        int issued = first;
        for (int s = ns; s < nst; ++s) {
            const int slot = s % ns, use = s / ns;
            if (!MbarWaitFor(&empty[slot], (use - 1) & 1, kWWaitNs, abort)) {
                if (!*abort) fail();
                break;
            }
            issue_rows(s);
            issue_tab(s);
            issued = s + 1;
        }
        // copies still in flight land before the CTA can leave
        if (lane == 0)
            for (int s = max(0, issued - ns); s < issued; ++s)
                if (!MbarWaitFor(&full[s % ns], (s / ns) & 1, kWWaitNs, nullptr)) fail();
        return;
    }

    // -------------------------------------------------------------- consumers
    const int kg = warp / kWRowGroups, rg = warp % kWRowGroups;
    constexpr int kRW = 8 * kWJ;  // weight rows per warp
    // per B fragment j: stage row of the lane's quants (weight row
    // kRW rg + 8 j + g) and of the scales of its two columns (rows
    // kRW rg + 8 j + 2 t, + 1), each with its row's byte offset mod 16 in the
    // weight buffer; with P boxes per stage, weight row r sits at stage row
    // (r % P) 128 / P + r / P
    auto srow = [&](int r) { return tma > 1 ? (r % tma) * (kWRows / tma) + r / tma : r; };
    int rq[kWJ], rd0[kWJ], rd1[kWJ];
    uint32_t mq[kWJ], md0[kWJ], md1[kWJ];
#pragma unroll
    for (int j = 0; j < kWJ; ++j) {
        const int a = kRW * rg + 8 * j + g, b = kRW * rg + 8 * j + 2 * t;
        mq[j] = static_cast<uint32_t>((size_t(min(n0 + a, N - 1)) * rowbytes) & 15);
        md0[j] = static_cast<uint32_t>((size_t(min(n0 + b, N - 1)) * rowbytes) & 15);
        md1[j] = static_cast<uint32_t>((size_t(min(n0 + b + 1, N - 1)) * rowbytes) & 15);
        rq[j] = srow(a);
        rd0[j] = srow(b);
        rd1[j] = srow(b + 1);
    }
    float2 acc[MQ][kWJ][2];
#pragma unroll
    for (int q = 0; q < MQ; ++q)
#pragma unroll
        for (int j = 0; j < kWJ; ++j) acc[q][j][0] = acc[q][j][1] = make_float2(0.0f, 0.0f);

    // one block (tb: its table; bq / dd: the fragment words and the two
    // columns' scales per j) against every x fragment; per group of 16 x
    // rows the three planes' MMAs are issued before their results are
    // combined
    auto block = [&](const uint8_t* tb, const uint32_t (&bq)[kWJ][2], const float2 (&dd)[kWJ]) {
        const uint4* af = reinterpret_cast<const uint4*>(tb);
        const float4* rc = reinterpret_cast<const float4*>(tb + NF * 512);
#pragma unroll
        for (int q = 0; q < MQ; ++q) {
            uint4 a[3];
            float4 r[3];
#pragma unroll
            for (int pl = 0; pl < 3; ++pl) {
                a[pl] = af[(pl * MQ + q) * 32 + lane];
                r[pl] = rc[(pl * MQ + q) * 8 + g];
            }
            int c[3][kWJ][4];
#pragma unroll
            for (int pl = 0; pl < 3; ++pl)
#pragma unroll
                for (int j = 0; j < kWJ; ++j) WMma<kU>(c[pl][j], a[pl], bq[j][0], bq[j][1]);
#pragma unroll
            for (int pl = 0; pl < 3; ++pl)
#pragma unroll
                for (int j = 0; j < kWJ; ++j) {
                    const float2 sg = __ffma2_rn(make_float2(__int_as_float(c[pl][j][0]), __int_as_float(c[pl][j][1])),
                                                 make_float2(r[pl].x, r[pl].x), make_float2(r[pl].y, r[pl].y));
                    const float2 s8 = __ffma2_rn(make_float2(__int_as_float(c[pl][j][2]), __int_as_float(c[pl][j][3])),
                                                 make_float2(r[pl].z, r[pl].z), make_float2(r[pl].w, r[pl].w));
                    acc[q][j][0] = __ffma2_rn(sg, dd[j], acc[q][j][0]);
                    acc[q][j][1] = __ffma2_rn(s8, dd[j], acc[q][j][1]);
                }
        }
    };

    for (int s = 0; s < nst; ++s) {
        const int slot = s % ns, use = s / ns;
        if (!MbarWaitFor(&full[slot], use & 1, kWWaitNs, abort)) {
            if (!*abort && lane == 0) {
                *abort = 1;
                if (p.status) atomicExch(p.status, MLB_ERR_DEVICE_TIMEOUT);
            }
            break;
        }
        const uint8_t* st = stages + size_t(slot) * p.stage_bytes;
        const uint8_t* tabs = st + size_t(kWRows) * p.pitch;
        const int b0 = kb0 + s * kWBlocks, nblk = min(kWBlocks, kb1 - b0);
        const uint32_t sadd = static_cast<uint32_t>((size_t(b0) * kBB) & 15);
        const int i0 = 2 * kg;  // this group's first block of the stage
        const uint8_t* pq[kWJ];
        const uint8_t* pd0[kWJ];
        const uint8_t* pd1[kWJ];
#pragma unroll
        for (int j = 0; j < kWJ; ++j) {
            pq[j] = st + rq[j] * p.pitch + ((mq[j] + sadd) & 15) + i0 * kBB;
            pd0[j] = st + rd0[j] * p.pitch + ((md0[j] + sadd) & 15) + i0 * kBB;
            pd1[j] = st + rd1[j] * p.pitch + ((md1[j] + sadd) & 15) + i0 * kBB;
        }
        if constexpr (QT == MLB_Q4_1) {
            // 20-byte blocks, every one word-aligned: d, m, then the nibbles
            for (int i = i0; i < min(i0 + 2, nblk); ++i) {
                const int e = i - i0;
                uint32_t bq[kWJ][2];
                float2 dd[kWJ], mn[kWJ];
#pragma unroll
                for (int j = 0; j < kWJ; ++j) {
                    const uint32_t* pg = reinterpret_cast<const uint32_t*>(pq[j] + e * kBB);
                    const uint32_t v = pg[1 + t];
                    bq[j][0] = v & 0x0F0F0F0Fu;
                    bq[j][1] = (v >> 4) & 0x0F0F0F0Fu;
                    const uint32_t h0 = *reinterpret_cast<const uint32_t*>(pd0[j] + e * kBB);
                    const uint32_t h1 = *reinterpret_cast<const uint32_t*>(pd1[j] + e * kBB);
                    dd[j] = HalfPair(h0, h1);
                    mn[j] = HalfPair(h0 >> 16, h1 >> 16);
                }
                const uint8_t* tb = tabs + size_t(i) * kTab;
                block(tb, bq, dd);
                const float2* xs = reinterpret_cast<const float2*>(tb + WTabSums(MQ));
#pragma unroll
                for (int q = 0; q < MQ; ++q) {
                    const float2 v = xs[q * 8 + g];
#pragma unroll
                    for (int j = 0; j < kWJ; ++j) {
                        acc[q][j][0] = __ffma2_rn(make_float2(v.x, v.x), mn[j], acc[q][j][0]);
                        acc[q][j][1] = __ffma2_rn(make_float2(v.y, v.y), mn[j], acc[q][j][1]);
                    }
                }
            }
        } else if (i0 < nblk) {
            // a block pair (i0, i0 + 1) starts on a word: the even block's
            // quants 2 bytes past it, the odd block's on a word
            uint32_t be[kWJ][2], bo[kWJ][2];
            float2 de[kWJ], dod[kWJ];
#pragma unroll
            for (int j = 0; j < kWJ; ++j) {
                const uint32_t* pg = reinterpret_cast<const uint32_t*>(pq[j]);
                const uint32_t* h0 = reinterpret_cast<const uint32_t*>(pd0[j]);
                const uint32_t* h1 = reinterpret_cast<const uint32_t*>(pd1[j]);
                if constexpr (QT == MLB_Q8_0) {
                    // words 0..16 of the 68-byte pair: even d, even quants
                    // 2..33, odd d at 34, odd quants 36..67
                    be[j][0] = __funnelshift_r(pg[t], pg[t + 1], 16);
                    be[j][1] = __funnelshift_r(pg[t + 4], pg[t + 5], 16);
                    bo[j][0] = pg[9 + t];
                    bo[j][1] = pg[13 + t];
                    de[j] = HalfPair(h0[0], h1[0]);
                    dod[j] = HalfPair(h0[8] >> 16, h1[8] >> 16);
                } else {
                    // Q4_0, words 0..8 of the 36-byte pair: even d, even
                    // nibbles 2..17, odd d at 18, odd nibbles 20..35
                    const uint32_t qe = __funnelshift_r(pg[t], pg[t + 1], 16);
                    const uint32_t qo = pg[5 + t];
                    be[j][0] = qe & 0x0F0F0F0Fu;
                    be[j][1] = (qe >> 4) & 0x0F0F0F0Fu;
                    bo[j][0] = qo & 0x0F0F0F0Fu;
                    bo[j][1] = (qo >> 4) & 0x0F0F0F0Fu;
                    de[j] = HalfPair(h0[0], h1[0]);
                    dod[j] = HalfPair(h0[4] >> 16, h1[4] >> 16);
                }
            }
            block(tabs + size_t(i0) * kTab, be, de);
            block(tabs + size_t(i0 + 1) * kTab, bo, dod);
        }
        __syncwarp();
        if (lane == 0) WArrive(&empty[slot]);
    }

    // ------------------------------------------------------------ epilogue
    // group 1 hands its sums to group 0 through the (now idle) stage memory;
    // the barrier also ORs the abort flag over the consumers, so all of them
    // take the same branch
    uint32_t aborted;
    asm volatile(
        "{\n .reg .pred p, q;\n setp.ne.u32 q, %1, 0;\n bar.red.or.pred p, 1, %2, q;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(aborted)
        : "r"(static_cast<uint32_t>(*abort)), "r"(kWWarps * 32)
        : "memory");
    if (aborted) return;
    float2* xch = reinterpret_cast<float2*>(stages) + size_t(rg) * (MQ * kWJ * 2) * 32;
    if (kg == 1) {
#pragma unroll
        for (int q = 0; q < MQ; ++q)
#pragma unroll
            for (int j = 0; j < kWJ; ++j) {
                xch[((q * kWJ + j) * 2) * 32 + lane] = acc[q][j][0];
                xch[((q * kWJ + j) * 2 + 1) * 32 + lane] = acc[q][j][1];
            }
    }
    asm volatile("bar.sync 1, %0;" ::"r"(kWWarps * 32) : "memory");
    GridDepLaunch();
    if (kg == 1) return;
    GridDepWait();  // the outputs may still be read by earlier kernels until they finish
    const bool single = p.splits == 1;
    const float* const bias = pick(p.bias[0], p.bias[1], p.bias[2]);
    float* out = single ? pick(p.y[0], p.y[1], p.y[2]) : pick(p.part[0], p.part[1], p.part[2]) + size_t(sp) * p.M * N;
#pragma unroll
    for (int q = 0; q < MQ; ++q)
#pragma unroll
        for (int j = 0; j < kWJ; ++j) {
            const int n = n0 + kRW * rg + 8 * j + 2 * t;
            float b0v = 0.0f, b1v = 0.0f;
            if (single && bias) {
                if (n < N) b0v = bias[n];
                if (n + 1 < N) b1v = bias[n + 1];
            }
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                const int m = 16 * q + g + 8 * r;
                if (m >= p.M) continue;
                const float2 o = xch[((q * kWJ + j) * 2 + r) * 32 + lane];
                const float2 v = make_float2(acc[q][j][r].x + o.x, acc[q][j][r].y + o.y);
                float* yr = out + size_t(m) * N;
                if (n < N) yr[n] = v.x + b0v;
                if (n + 1 < N) yr[n + 1] = v.y + b1v;
            }
        }
}

struct WidePlan {
    bool ok = false;
    int MQ = 0, kper = 0, splits = 0, pitch = 0, stage_bytes = 0, stages = 0, row_groups = 0;
    size_t smem = 0, tab_bytes = 0, part_off = 0, total = 0;
};

// Stage geometry and the block split for `row_groups` CTAs' worth of weight
// rows (n_total rows in all): the split count minimises a cost in SM cycles
// -- waves of CTAs x (blocks per split x the MMA time of a block, 48 MQ MMAs
// at about 2.1 cycles each, plus a fixed cost per CTA) -- plus the
// partial-sum pass (its bytes at about 25 B per cycle per SM).
WidePlan PlanWide(int qtype, int M, int K, int row_groups, long long n_total, int sms, int max_smem) {
    WidePlan pl;
    if (M < 1 || M > kWideMaxRows || K < 1 || row_groups < 1) return pl;
    const int bb = BlockBytes(qtype);
    const int nb = (K + 31) / 32;
    if (qtype != MLB_Q4_1 && (nb & 1)) return pl;  // Q8_0 / Q4_0 blocks are read in pairs
    pl.MQ = (M + 15) / 16;
    // a row's range plus its misalignment, rounded to 16 bytes, at a pitch of
    // 4 mod 8 words: the eight rows one fragment load touches start in
    // distinct bank groups
    int pitch = (kWBlocks * bb + 15 + 15) & ~15;
    while ((pitch / 4) % 8 != 4) pitch += 16;
    pl.pitch = pitch;
    pl.stage_bytes = kWRows * pitch + kWBlocks * WTabBlock(pl.MQ);
    pl.stages = std::min<int>(kWMaxStages,
                              static_cast<int>((static_cast<size_t>(max_smem) - 1024 - kWHeader) / pl.stage_bytes));
    if (pl.stages < 2) return pl;
    pl.smem = kWHeader + size_t(pl.stages) * pl.stage_bytes;
    pl.row_groups = row_groups;
    const double blk = 48.0 * pl.MQ * 2.13, fixed = 5000.0;
    double best = 1e300;
    for (int s = 1; s <= 32; ++s) {
        const int kper = ((nb + s - 1) / s + kWBlocks - 1) / kWBlocks * kWBlocks;
        const int splits = (nb + kper - 1) / kper;
        if (splits != s) continue;
        const long long ctas = static_cast<long long>(row_groups) * splits;
        const long long waves = (ctas + sms - 1) / sms;
        double t = double(waves) * (kper * blk + fixed);
        if (splits > 1) t += 2000.0 + double(M) * n_total * 4.0 * (splits + 1) / (25.0 * sms);
        if (t < best) {
            best = t;
            pl.kper = kper;
            pl.splits = splits;
        }
    }
    pl.tab_bytes = size_t(nb) * WTabBlock(pl.MQ);
    pl.part_off = (pl.tab_bytes + 255) / 256 * 256;
    pl.total = pl.part_off + (pl.splits > 1 ? size_t(pl.splits) * M * size_t(n_total) * 4 : 0);
    pl.ok = true;
    return pl;
}

// The weight blocks as a 2-D tensor map (uint8, no swizzle, no multicast):
// rows viewed P at a time (P the smallest of 1, 2, 4, 8 that makes the row
// stride a multiple of 16 bytes), boxes of pitch bytes x 128 / P rows.
// Returns P, or 0 (per-row bulk copies) when N does not divide into such
// groups, the base is not 16-byte aligned or the driver offers no encoder.
int WideWeightMap(const uint8_t* w, int N, size_t rowbytes, int pitch, CUtensorMap& map) {
    std::memset(&map, 0, sizeof(map));
    int P = 1;
    while (P <= 8 && (P * rowbytes) % 16 != 0) P *= 2;
    if (P > 8 || N % P != 0 || (reinterpret_cast<uintptr_t>(w) & 15) != 0 || pitch > 256) return 0;
    const cuuint64_t gdim[2] = {cuuint64_t(P * rowbytes), cuuint64_t(N / P)};
    const cuuint64_t gstride[1] = {cuuint64_t(P * rowbytes)};
    const cuuint32_t box[2] = {cuuint32_t(pitch), cuuint32_t(kWRows / P)};
    const cuuint32_t estride[2] = {1, 1};
    const PFN_cuTensorMapEncodeTiled_v12000 encode = TensorMapEncoder();
    if (!encode) return 0;
    const CUresult r = encode(&map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(w), gdim, gstride, box,
                              estride, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? P : 0;
}

template <int QT, int MQ>
void LaunchWideT(DeviceContext& c, const WidePlan& pl, const float* x, int M, int K, const WideSeg* segs, int nseg,
                 int* status, uint8_t* ws, bool reuse_x) {
    const int nb = (K + 31) / 32;
    const bool reuse = reuse_x && c.tc_x == x && c.tc_ws == ws && c.tc_m == M && c.tc_k == K && c.tc_mx == 0 &&
                       c.tc_mtiles == MQ;
    if (!reuse)
        Launch("WidePrepX", WidePrepX<QT, MQ>, dim3((16 * MQ * nb + 31) / 32), dim3(256), 0, c.stream, true, x, M,
               K, nb, ws);
    c.tc_x = x;
    c.tc_ws = ws;
    c.tc_m = M;
    c.tc_k = K;
    c.tc_mx = 0;  // marks this path's tables (the tcgen05 path's x images have tc_mx >= 16)
    c.tc_mtiles = MQ;
    WideParams p{};
    p.nseg = nseg;
    p.tab = ws;
    p.M = M;
    p.nb = nb;
    p.rowbytes = nb * BlockBytes(QT);
    p.kper = pl.kper;
    p.splits = pl.splits;
    p.pitch = pl.pitch;
    p.stage_bytes = pl.stage_bytes;
    p.stages = pl.stages;
    p.status = status;
    CUtensorMap maps[kWMaxSegs];
    float* part = reinterpret_cast<float*>(ws + pl.part_off);
    int rg = 0;
    for (int i = 0; i < kWMaxSegs; ++i) {
        const int j = i < nseg ? i : nseg - 1;  // unused slots repeat the last segment
        p.w[i] = segs[j].w;
        p.bias[i] = segs[j].bias;
        p.y[i] = segs[j].y;
        p.N[i] = segs[j].N;
        p.part[i] = part;
        p.tma_rows[i] = WideWeightMap(segs[j].w, segs[j].N, size_t(p.rowbytes), pl.pitch, maps[i]);
        if (i < nseg) {
            rg += (segs[i].N + kWRows - 1) / kWRows;
            part += size_t(pl.splits) * M * segs[i].N;
        }
        p.rg_end[i] = rg;
    }
    static int configured[64] = {};
    if (c.device >= 64 || configured[c.device] < static_cast<int>(pl.smem)) {
        CheckCuda(cudaFuncSetAttribute(WideGemvKernel<QT, MQ>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(pl.smem)),
                  "cudaFuncSetAttribute(WideGemvKernel)");
        if (c.device < 64) configured[c.device] = static_cast<int>(pl.smem);
    }
    Launch("WideGemvKernel", WideGemvKernel<QT, MQ>, dim3(pl.row_groups, pl.splits), dim3(kWThreads), pl.smem,
           c.stream, true, p, maps[0], maps[1], maps[2]);
    if (pl.splits > 1) {
        for (int i = 0; i < nseg; ++i) {
            const size_t mn = size_t(M) * segs[i].N;
            const int g = static_cast<int>(std::max<size_t>(1, std::min<size_t>((mn + 255) / 256, size_t(8) * c.sm_count)));
            Launch("WideReduce", WideReduce, dim3(g), dim3(256), 0, c.stream, true, static_cast<const float*>(p.part[i]),
                   pl.splits, M, segs[i].N, segs[i].bias, segs[i].y);
        }
    }
}

template <int QT>
void LaunchWideQ(DeviceContext& c, const WidePlan& pl, const float* x, int M, int K, const WideSeg* segs, int nseg,
                 int* status, uint8_t* ws, bool reuse_x) {
    switch (pl.MQ) {
        case 1: return LaunchWideT<QT, 1>(c, pl, x, M, K, segs, nseg, status, ws, reuse_x);
        case 2: return LaunchWideT<QT, 2>(c, pl, x, M, K, segs, nseg, status, ws, reuse_x);
        case 3: return LaunchWideT<QT, 3>(c, pl, x, M, K, segs, nseg, status, ws, reuse_x);
        default: return LaunchWideT<QT, 4>(c, pl, x, M, K, segs, nseg, status, ws, reuse_x);
    }
}

}  // namespace

bool WidePreferred(int M, int K, int N) {
    return M <= kWideMaxRows && (M <= 32 || static_cast<long long>(N) * K <= (8LL << 20));
}

size_t WideWorkspaceBytes(int M, int K, int N, int sm_count, int max_smem) {
    size_t total = 0;
    for (int qt : {MLB_Q8_0, MLB_Q4_0, MLB_Q4_1}) {
        const WidePlan pl = PlanWide(qt, M, K, (N + kWRows - 1) / kWRows, N, sm_count, max_smem);
        if (pl.ok) total = std::max(total, pl.total);
    }
    return total;
}

bool LaunchWideLinearSegs(DeviceContext& c, int qtype, const float* x, int M, int K, const WideSeg* segs, int nseg,
                          int* status, void* workspace, bool reuse_x) {
    if (nseg < 1 || nseg > kWMaxSegs) return false;
    int row_groups = 0;
    long long n_total = 0;
    for (int i = 0; i < nseg; ++i) {
        if (segs[i].N < 1 || (reinterpret_cast<uintptr_t>(segs[i].w) & 15)) return false;
        row_groups += (segs[i].N + kWRows - 1) / kWRows;
        n_total += segs[i].N;
    }
    const WidePlan pl = PlanWide(qtype, M, K, row_groups, n_total, c.sm_count, c.max_smem_optin);
    if (!pl.ok) return false;
    uint8_t* ws = static_cast<uint8_t*>(workspace ? workspace : Workspace(c, pl.total));
    switch (qtype) {
        case MLB_Q8_0: LaunchWideQ<MLB_Q8_0>(c, pl, x, M, K, segs, nseg, status, ws, reuse_x); break;
        case MLB_Q4_0: LaunchWideQ<MLB_Q4_0>(c, pl, x, M, K, segs, nseg, status, ws, reuse_x); break;
        default: LaunchWideQ<MLB_Q4_1>(c, pl, x, M, K, segs, nseg, status, ws, reuse_x); break;
    }
    return true;
}

bool LaunchWideLinear(DeviceContext& c, int qtype, const float* x, const uint8_t* w, int M, int K, int N,
                      const float* bias, float* y, int* status, void* workspace, bool reuse_x) {
    const WideSeg seg{w, bias, y, N};
    return LaunchWideLinearSegs(c, qtype, x, M, K, &seg, 1, status, workspace, reuse_x);
}

}  // namespace mlb
