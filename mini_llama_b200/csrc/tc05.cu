// Quantized linear for M >= 9 rows (prefill): y = x W^T (+ bias) on the
// 5th-generation tensor cores (tcgen05.mma, accumulator in tensor memory).
// Replaces the reference's Q8_0 / Q4_0 / Q4_1 linear kernels
// (src/cuda_quant.cu:40-135) for batches of rows.
//
// Exactness: the reference multiplies fp32 x by the fp32 dequantized weight
// w = fp16(d) * q (Q4_0: d * (q - 8); Q4_1: d * q + m, rounded once) and sums
// in fp32.  Every value v is split into fp16 v_hi = rn(v) and
// v_lo = rn(v - v_hi), and the tensor cores accumulate
// x_hi w_hi + x_hi w_lo + x_lo w_hi in fp32 (the x_lo w_lo term is below
// 2^-22 relative).  Each x row is first scaled by a power of two so that its
// largest |x| sits in [2^14, 2^15) (exact; undone in the epilogue).  W needs
// no scale: fp16(d) and m are multiples of 2^-24, so d q and w - w_hi are too,
// and the split is exact for Q8_0 / Q4_0 (d q has at most 19 significant
// bits; computed on half2 pairs as hi = rn(d q), lo = fma(d, q, -hi)) and
// within 2^-22 for Q4_1, subnormal halves included.  Only an fp16 overflow of
// w_hi could break it: a block whose |w| bound reaches 2^15 marks the tile,
// which is then recomputed with each W row scaled by a power of two that
// brings its largest |w| into [2^14, 2^15).  Result: within ~1e-6 relative of
// the fp32 reference.
//
// Operands: A = W (128 W rows per MMA = tensor-memory lanes), B = x (MX x
// rows per MMA = accumulator columns, MX a multiple of 16, <= 256), both
// K-major in the canonical no-swizzle layout of 8-row x 16-byte core matrices:
// an R-row x 16-element image is
//   offset(r, k) = (k / 8) * 16 R + (r / 8) * 128 + (r % 8) * 16 + (k % 8) * 2
// (leading byte offset 16 R between the two 8-element k chunks, stride byte
// offset 128 between 8-row groups).
//
// Batches of up to 128 rows may instead run with the roles swapped: A = the x
// tile padded to 128 rows, B = 256 W rows in one image, so a stage takes three
// 128 x 256 MMAs rather than six narrow ones (tcgen05.mma issue, about 95
// cycles each, bounds the narrow form).  The planner picks by a cycle model.
//
// A CTA owns NW x 128 W rows (NW = 1 or 2) and MX x rows over a range of K
// (split-K when the tile grid alone would leave SMs idle); its NW accumulators
// of 128 x MX fp32 fill up to all 512 tensor-memory columns.  One stage is 16
// elements of K (half a quantization block); four stages are in flight:
//   warps 0-7  stream the raw W blocks of the tile into a shared ring of
//              three windows of 2 (Q8_0) or 3 blocks, one bulk copy per row
//              and window (completion on rawfull), then
//              dequantize: each thread converts one 8-element chunk of one or
//              two rows from the ring into the stage's hi / lo images, and
//              each warp arrives on wfull.  Afterwards they are the epilogue.
//   warp 8     bulk-copies the x hi / lo images of each stage (written by the
//              pre-pass TcPrepX) into their own ring of 64 KB (4 stages at
//              MX = 256, up to 16 for small MX), completing on xfull.
//   warp 9     allocates tensor memory; one lane issues the 3 NW MMAs of a
//              stage (3 products x NW sub-tiles) and commits them to the
//              stage's W and x empty barriers, and after the last stage to
//              accfull.
// The pre-pass, this kernel and the split-K sum are chained with programmatic
// dependent launch: each starts its independent prologue while the previous
// one runs and waits (griddepcontrol.wait) before touching its output.
// Every wait is bounded (an expired wait records MLB_ERR_DEVICE_TIMEOUT and
// raises the CTA's abort flag); in-flight copies and MMAs are waited for and
// tensor memory is freed on every path.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cmath>
#include <cstring>

#include "common.cuh"
#include "qgemv.cuh"

namespace mlb {
namespace {

constexpr int kTcRows = 128;                        // W rows per MMA (M of the instruction)
constexpr int kTcMaxX = 256;                        // x rows per MMA at most (N of the instruction)
constexpr int kTcK = 16;                            // elements of K per stage: half a block
constexpr int kTcStages = 4;                        // W image stages in flight
constexpr int kTcWImg = kTcRows * kTcK * 2;         // one fp16 image of a 128-row W sub-tile
constexpr int kTcWBytes = 2 * kTcWImg;              // its hi + lo images
constexpr int kTcStageBytes = 2 * kTcWBytes;        // room for two W sub-tiles: 16 KB
constexpr int kTcXRing = 64 * 1024;                 // x image stages: 64 MX bytes each
constexpr int kTcXSlotsMax = 16;
constexpr int kTcRawSlots = 3;                      // raw windows in flight
constexpr int kTcHeader = 2048;
constexpr int kTcDqWarps = 8;
constexpr int kTcDqThreads = kTcDqWarps * 32;
constexpr int kTcThreads = kTcDqThreads + 64;       // + x-copy warp + MMA warp
constexpr uint64_t kTcWaitNs = 2000000000ull;

// 2^e as a float for -126 <= e <= 127, from its exponent bits.
__device__ __forceinline__ float Pow2(int e) { return __uint_as_float(static_cast<uint32_t>(127 + e) << 23); }

// Exponent s with (bound * 2^s) in [2^14, 2^15) (0 when bound is 0 or not finite).
__device__ __forceinline__ int ScaleExp(float bound) {
    if (!(bound > 0.0f) || !isfinite(bound)) return 0;
    const int e = static_cast<int>((__float_as_uint(bound) >> 23) & 0xff) - 127;  // 2^e <= bound < 2^(e+1)
    int s = 14 - e;
    return s > 100 ? 100 : (s < -100 ? -100 : s);
}

__device__ __forceinline__ uint32_t PackHalf2(__half a, __half b) {
    return static_cast<uint32_t>(__half_as_ushort(a)) | (static_cast<uint32_t>(__half_as_ushort(b)) << 16);
}

// ---------------------------------------------------------------- x pre-pass
// One CTA per x row of the padded tiles (mtiles * MX rows): its scale
// exponent (largest |x| into [2^14, 2^15)), the undo factor 2^-s, and its
// hi / lo images [m tile][stage][hi, lo] in the B-operand layout.  Rows past M
// and elements past K are zero.
__global__ void __launch_bounds__(128) TcPrepX(const float* x, int M, int K, int MX, int kst, float* xundo,
                                               uint8_t* images) {
    __shared__ float red[4];
    GridDepWait();    // x and the workspace belong to earlier kernels until they finish
    GridDepLaunch();  // the linear kernel's prologue (barriers, tensor memory, W) may start now
    const int row = blockIdx.x, tid = threadIdx.x;
    const int mt = row / MX, r = row % MX;
    const bool live = row < M;
    const float* xr = x + size_t(live ? row : 0) * K;
    const bool vec = (K & 3) == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0;
    // rows of up to 4 x 128 8-element chunks stay in registers (chunk
    // tid + 128 j in va[j], vb[j]): x is read once
    constexpr int kRegChunks = 4;
    const bool inreg = vec && kst * 2 <= kRegChunks * 128;
    float4 va[kRegChunks], vb[kRegChunks];
    float mx = 0.0f;
    if (inreg) {
#pragma unroll
        for (int j = 0; j < kRegChunks; ++j) {
            const int k0 = 8 * (tid + 128 * j);
            const float4 z = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            va[j] = (live && k0 + 4 <= K) ? *reinterpret_cast<const float4*>(xr + k0) : z;
            vb[j] = (live && k0 + 8 <= K) ? *reinterpret_cast<const float4*>(xr + k0 + 4) : z;
            mx = fmaxf(mx, fmaxf(fmaxf(fabsf(va[j].x), fabsf(va[j].y)), fmaxf(fabsf(va[j].z), fabsf(va[j].w))));
            mx = fmaxf(mx, fmaxf(fmaxf(fabsf(vb[j].x), fabsf(vb[j].y)), fmaxf(fabsf(vb[j].z), fabsf(vb[j].w))));
        }
    } else if (live) {
        for (int k = tid; k < K; k += 128) mx = fmaxf(mx, fabsf(xr[k]));
    }
    mx = WarpMax(mx);
    if ((tid & 31) == 0) red[tid >> 5] = mx;
    __syncthreads();
    mx = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
    const int s = ScaleExp(mx);
    const float sc = live ? Pow2(s) : 0.0f;
    if (live && tid == 0) xundo[row] = Pow2(-s);
    const size_t img = size_t(MX) * kTcK * 2;  // bytes of one image
    for (int ch = tid, j = 0; ch < kst * 2; ch += 128, ++j) {
        const int kt = ch >> 1, c = ch & 1, k0 = kt * kTcK + c * 8;
        float v[8];
        if (inreg) {
            float4 a = va[0], b = vb[0];
#pragma unroll
            for (int q = 1; q < kRegChunks; ++q)
                if (j == q) {
                    a = va[q];
                    b = vb[q];
                }
            v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
        } else if (live && vec && k0 + 8 <= K) {
            const float4 a = *reinterpret_cast<const float4*>(xr + k0);
            const float4 b = *reinterpret_cast<const float4*>(xr + k0 + 4);
            v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
        } else {
#pragma unroll
            for (int j = 0; j < 8; ++j) v[j] = (live && k0 + j < K) ? xr[k0 + j] : 0.0f;
        }
        uint32_t hi[4], lo[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float a = v[2 * j] * sc, b = v[2 * j + 1] * sc;
            const __half ah = __float2half_rn(a), bh = __float2half_rn(b);
            hi[j] = PackHalf2(ah, bh);
            lo[j] = PackHalf2(__float2half_rn(a - __half2float(ah)), __float2half_rn(b - __half2float(bh)));
        }
        uint8_t* base = images + (size_t(mt) * kst + kt) * 2 * img + size_t(c) * MX * 16 + (r >> 3) * 128 +
                        (r & 7) * 16;
        *reinterpret_cast<uint4*>(base) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
        *reinterpret_cast<uint4*>(base + img) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
    }
}

// Sum of the split-K partials [splits][M][N] plus bias.
__global__ void __launch_bounds__(256) TcReduce(const float* part, int splits, int M, int N, const float* bias,
                                                float* y) {
    const size_t mn = size_t(M) * N;
    GridDepWait();
    if ((N & 3) == 0 && mn < (size_t(1) << 32) &&
        ((reinterpret_cast<uintptr_t>(part) | reinterpret_cast<uintptr_t>(y) | reinterpret_cast<uintptr_t>(bias)) & 15) == 0) {
        // four columns per thread (the same sum order per element)
        const uint32_t mn4 = static_cast<uint32_t>(mn >> 2), n4 = static_cast<uint32_t>(N >> 2);
        const float4* p4 = reinterpret_cast<const float4*>(part);
        for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < mn4; i += gridDim.x * blockDim.x) {
            float4 acc = bias ? reinterpret_cast<const float4*>(bias)[i % n4] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll 8
            for (int s = 0; s < splits; ++s) {
                const float4 v = __ldg(p4 + size_t(s) * mn4 + i);
                acc.x += v.x;
                acc.y += v.y;
                acc.z += v.z;
                acc.w += v.w;
            }
            reinterpret_cast<float4*>(y)[i] = acc;
        }
        return;
    }
    for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < mn; i += size_t(gridDim.x) * blockDim.x) {
        float acc = bias ? bias[i % N] : 0.0f;
#pragma unroll 8
        for (int s = 0; s < splits; ++s) acc += __ldg(part + s * mn + i);
        y[i] = acc;
    }
}

// ---------------------------------------------------------------- tcgen05
__device__ __forceinline__ uint64_t SmemDesc(uint32_t addr, uint32_t lbo) {
    // K-major, no swizzle: leading byte offset lbo (k chunks), stride byte offset 128 (8-row groups),
    // descriptor version 1
    return static_cast<uint64_t>((addr >> 4) & 0x3FFFu) | (static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16) |
           (static_cast<uint64_t>(128 >> 4) << 32) | (1ull << 46);
}

// kind::f16 instruction descriptor: fp32 accumulate, fp16 A and B, both
// K-major, M = 128, N = n.
__device__ __forceinline__ uint32_t Idesc(int n) {
    return (1u << 4) | (static_cast<uint32_t>(n >> 3) << 17) | (static_cast<uint32_t>(kTcRows >> 4) << 24);
}

__device__ __forceinline__ void TcMma(uint32_t dtmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                      uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n"
        :
        : "r"(dtmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0));
}

__device__ __forceinline__ void TcCommit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(SmemAddr(bar))
                 : "memory");
}

__device__ __forceinline__ void TcFenceBefore() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void TcFenceAfter() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void TcLoad8(uint32_t taddr, float (&v)[8]) {
    uint32_t r[8];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void MbarArrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(SmemAddr(bar)) : "memory");
}

__device__ __forceinline__ uint32_t LdgU16(const uint8_t* p) {
    return __ldg(reinterpret_cast<const unsigned short*>(p));
}

template <int QT>
struct TcBlock {
    static constexpr int kBytes = QT == MLB_Q8_0 ? 34 : (QT == MLB_Q4_0 ? 18 : 20);
    static constexpr int kQOff = QT == MLB_Q4_1 ? 4 : 2;
    // blocks of a row in one raw window, and the bytes that row takes in the
    // ring: its blocks plus up to 14 bytes of leading alignment, rounded to an
    // odd number of 16-byte pieces so that 8 consecutive rows start in 8
    // different bank groups
    static constexpr int kWin = QT == MLB_Q8_0 ? 2 : 3;
    static constexpr int kPieces = (kWin * kBytes + 14 + 15) / 16;
    static constexpr int kRawRow = 16 * (kPieces | 1);
};

template <int QT>
constexpr size_t TcSmemBytes() {
    return kTcHeader + size_t(kTcStages) * kTcStageBytes + kTcXRing +
           size_t(kTcRawSlots) * 2 * kTcRows * TcBlock<QT>::kRawRow;
}

// The raw bytes one lane converts: the block's fp16 d (and Q4_1's m in the
// high half) and the 8 quant bytes of its chunk.
struct TcRaw {
    uint32_t d, q0, q1;
};

__device__ __forceinline__ uint32_t LdsU16(uint32_t addr) {
    unsigned short v;
    asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(addr));
    return v;
}

__device__ __forceinline__ uint32_t LdsU32(uint32_t addr) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr));
    return v;
}

// From a raw block in shared memory (blk: its first byte, 2-byte aligned):
// the quant bytes of elements 16 h + 8 c .. + 7 (Q8_0), or the bytes whose
// nibbles hold them (Q4: bytes 8 c .. 8 c + 7, low nibbles for h = 0).
template <int QT>
__device__ __forceinline__ TcRaw TcLoadRawSmem(uint32_t blk, int c, int h) {
    TcRaw r;
    r.d = LdsU16(blk);
    if constexpr (QT == MLB_Q4_1) r.d |= LdsU16(blk + 2) << 16;
    const uint32_t q = blk + TcBlock<QT>::kQOff + (QT == MLB_Q8_0 ? 16 * h + 8 * c : 8 * c);
    const uint32_t p = q & ~3u, sh = (q & 2) ? 16u : 0u;
    const uint32_t w0 = LdsU32(p), w1 = LdsU32(p + 4);
    const uint32_t w2 = sh ? LdsU32(p + 8) : 0u;
    r.q0 = __funnelshift_r(w0, w1, sh);
    r.q1 = __funnelshift_r(w1, w2, sh);
    return r;
}

// Upper bound of |w| over one block, from its d (and m).
template <int QT>
__device__ __forceinline__ float TcBound(uint32_t dm) {
    const float d = fabsf(HalfBits(static_cast<uint16_t>(dm)));
    if constexpr (QT == MLB_Q8_0) return d * 128.0f;
    else if constexpr (QT == MLB_Q4_0) return d * 8.0f;
    else return d * 15.0f + fabsf(HalfBits(static_cast<uint16_t>(dm >> 16)));
}

template <int QT>
__device__ __forceinline__ float TcBlockBound(const uint8_t* blk) {
    uint32_t dm = LdgU16(blk);
    if constexpr (QT == MLB_Q4_1) dm |= LdgU16(blk + 2) << 16;
    return TcBound<QT>(dm);
}

// Four quant values as two half2 pairs, from four bytes (Q8_0: signed bytes;
// Q4: one nibble per byte, 0..15): 0x64xx is the fp16 value 1024 + xx.
template <int QT>
__device__ __forceinline__ void TcQuads(uint32_t bytes, __half2& q01, __half2& q23) {
    uint32_t u;
    __half2 bias;
    if constexpr (QT == MLB_Q8_0) {
        u = bytes ^ 0x80808080u;
        bias = __half2half2(__ushort_as_half(0x6480));  // 1152
    } else {
        u = bytes;
        bias = __half2half2(__ushort_as_half(QT == MLB_Q4_0 ? 0x6408 : 0x6400));  // 1032 (q - 8) / 1024 (q)
    }
    const uint32_t a = __byte_perm(u, 0x64646464u, 0x4140), b = __byte_perm(u, 0x64646464u, 0x4342);
    q01 = __hsub2(*reinterpret_cast<const __half2*>(&a), bias);
    q23 = __hsub2(*reinterpret_cast<const __half2*>(&b), bias);
}

// Converts one lane's chunk (8 weights of half h, scaled by mul) into hi / lo
// halves.
template <int QT>
__device__ __forceinline__ void TcConvert(const TcRaw& r, int h, float mul, uint4& hi, uint4& lo) {
    uint32_t hv[4], lv[4];
    uint32_t b0 = r.q0, b1 = r.q1;
    if constexpr (QT != MLB_Q8_0) {
        const int shift = 4 * h;  // elements 16..31: the high nibbles
        b0 = (b0 >> shift) & 0x0F0F0F0Fu;
        b1 = (b1 >> shift) & 0x0F0F0F0Fu;
    }
    __half2 q[4];
    TcQuads<QT>(b0, q[0], q[1]);
    TcQuads<QT>(b1, q[2], q[3]);
    if constexpr (QT == MLB_Q4_1) {
        const float d = HalfBits(static_cast<uint16_t>(r.d)), m = HalfBits(static_cast<uint16_t>(r.d >> 16));
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float2 qf = __half22float2(q[j]);
            const float a = __fmaf_rn(d, qf.x, m) * mul, b = __fmaf_rn(d, qf.y, m) * mul;
            const __half ah = __float2half_rn(a), bh = __float2half_rn(b);
            hv[j] = PackHalf2(ah, bh);
            lv[j] = PackHalf2(__float2half_rn(a - __half2float(ah)), __float2half_rn(b - __half2float(bh)));
        }
    } else {
        const __half2 dd = __half2half2(__float2half_rn(HalfBits(static_cast<uint16_t>(r.d)) * mul));
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const __half2 hh = __hmul2(dd, q[j]);
            const __half2 ll = __hfma2(dd, q[j], __hneg2(hh));
            hv[j] = *reinterpret_cast<const uint32_t*>(&hh);
            lv[j] = *reinterpret_cast<const uint32_t*>(&ll);
        }
    }
    hi = make_uint4(hv[0], hv[1], hv[2], hv[3]);
    lo = make_uint4(lv[0], lv[1], lv[2], lv[3]);
}

struct TcShared {
    uint64_t xfull[kTcXSlotsMax];
    uint64_t xempty[kTcXSlotsMax];
    uint64_t wfull[kTcStages];
    uint64_t wempty[kTcStages];
    uint64_t rawfull[kTcRawSlots];
    uint64_t rawempty[kTcRawSlots];
    uint64_t accfull;
    uint32_t tmem;
    int abort;
    int overflow;  // a block's |w| bound reached 2^15: recompute with row scales
    float wundo[2 * kTcRows];
};

struct TcArgs {
    const uint8_t* w;
    int N, K, nb, M;
    int mx, mtiles, kst, kper;
    const uint8_t* ximg;
    const float* xundo;
    const float* bias;
    float* y;     // splits == 1
    float* part;  // splits > 1: [splits][M][N]
    int splits;
    int* status;
    int tma_rows;  // 0: one bulk copy per row; else P: the tensor map views P rows as one
};

// One 2-D tensor-map box (no multicast) into shared memory, completing on bar.
__device__ __forceinline__ void TmaLoad2D(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        ::"r"(SmemAddr(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(SmemAddr(bar))
        : "memory");
}

__device__ __forceinline__ void TcFail(TcShared& sh, int* status) {
    atomicCAS(status, 0, MLB_ERR_DEVICE_TIMEOUT);
    *reinterpret_cast<volatile int*>(&sh.abort) = 1;
}

// SW (swapped roles, small batches): NW == 2, A = the x tile padded to 128
// rows (MX == 128), B = the CTA's 256 W rows as one image, one 128 x 256
// accumulator; three MMAs per stage instead of six.
template <int QT, int NW, bool SW>
__global__ void __launch_bounds__(kTcThreads, 1) TcLinearKernel(const TcArgs a, const __grid_constant__ CUtensorMap wmap) {
    static_assert(!SW || NW == 2, "the swapped form covers 256 W rows");
    extern __shared__ __align__(1024) uint8_t smem[];
    TcShared& sh = *reinterpret_cast<TcShared*>(smem);
    uint8_t* stages = smem + kTcHeader;
    uint8_t* xring = stages + kTcStages * kTcStageBytes;
    uint8_t* raw = xring + kTcXRing;
    constexpr int kItems = NW;                              // W rows per dequant thread
    constexpr int kBB = TcBlock<QT>::kBytes;
    constexpr int kRawRow = TcBlock<QT>::kRawRow;
    constexpr int kRawSlot = NW * kTcRows * kRawRow;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int mt = blockIdx.x % a.mtiles, split = blockIdx.x / a.mtiles;
    const int n0 = blockIdx.y * NW * kTcRows, m0 = mt * a.mx;
    const int kb0 = split * a.kper, kb1 = min(a.nb, kb0 + a.kper), nk = kb1 - kb0, nst = 2 * nk;
    const int mx = a.mx;
    const int xslots = min(kTcXSlotsMax, kTcXRing / (64 * mx));  // x image stages in flight
    const size_t rowbytes = size_t(a.nb) * kBB;
    const uintptr_t wend = reinterpret_cast<uintptr_t>(a.w) + size_t(a.N) * rowbytes;
    const volatile int* abort = &sh.abort;

    if (tid == 0) {
        for (int i = 0; i < kTcStages; ++i) {
            MbarInit(&sh.wfull[i], kTcDqWarps);
            MbarInit(&sh.wempty[i], 1);
        }
        for (int i = 0; i < kTcXSlotsMax; ++i) {
            MbarInit(&sh.xfull[i], 1);
            MbarInit(&sh.xempty[i], 1);
        }
        for (int i = 0; i < kTcRawSlots; ++i) {
            // one arrival per warp with its rows' bulk copies, or one for the tensor-map boxes
            MbarInit(&sh.rawfull[i], a.tma_rows ? 1 : kTcDqWarps);
            MbarInit(&sh.rawempty[i], kTcDqWarps);
        }
        MbarInit(&sh.accfull, 1);
        FenceMbarInit();
        sh.abort = 0;
        sh.overflow = 0;
    }
    if (tid < 2 * kTcRows) sh.wundo[tid] = 1.0f;
    uint32_t ncols = 32;
    while (ncols < static_cast<uint32_t>(SW ? 2 * kTcRows : NW * mx)) ncols <<= 1;
    if (warp == kTcDqWarps + 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(SmemAddr(&sh.tmem)),
                     "r"(ncols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
    }
    TcFenceBefore();
    __syncthreads();
    TcFenceAfter();
    const uint32_t tmem = sh.tmem;

    // dequantizing threads: rows rb + 128 i, chunk c of each half block; each
    // 8-lane group of a warp stores one chunk of 8 consecutive rows (128
    // contiguous bytes of a W image)
    const int c = (lane >> 3) & 1, rb = 16 * warp + (lane & 7) + 8 * (lane >> 4);
    const uint8_t* rowp[kItems];
    float mul[kItems];
#pragma unroll
    for (int i = 0; i < kItems; ++i) {
        const int n = n0 + rb + kTcRows * i;
        rowp[i] = a.w + size_t(n < a.N ? n : a.N - 1) * rowbytes;
        mul[i] = n < a.N ? 1.0f : 0.0f;
    }

    int pass = 0;
    for (;; ++pass) {
        if (warp < kTcDqWarps) {
            // ------------------------------------------------ raw W blocks -> W images
            // Raw window wi of this pass (TcBlock<QT>::kWin blocks of every row; global
            // window count gw) goes to ring slot gw % kTcRawSlots: thread t
            // bulk-copies row t's window with the 16-byte aligned bytes around
            // it (the last bytes of the weight buffer, where rounding up would
            // run past it, by plain loads); lane 0 of each warp arrives on
            // rawfull expecting the warp's bytes.
            const int nwin = (nk + TcBlock<QT>::kWin - 1) / TcBlock<QT>::kWin;
            auto issue = [&](int wi) -> bool {
                if (wi >= nwin) return true;
                const int gw = pass * nwin + wi, rs = gw % kTcRawSlots;
                if (gw >= kTcRawSlots &&
                    !MbarWaitFor(&sh.rawempty[rs], (gw / kTcRawSlots - 1) & 1, kTcWaitNs, abort))
                    return false;
                if (a.tma_rows) {  // P boxes of (NW x 128 / P rows, kRawRow bytes): row P i + j -> box j, row i
                    if (tid == 0) {
                        const int P = a.tma_rows, rows = NW * kTcRows / P;
                        const long long k0 = (long long)(kb0 + wi * TcBlock<QT>::kWin) * kBB;
                        MbarExpectTx(&sh.rawfull[rs], static_cast<uint32_t>(NW * kTcRows * kRawRow));
                        for (int j = 0; j < P; ++j)
                            TmaLoad2D(raw + rs * kRawSlot + j * rows * kRawRow, &wmap,
                                      static_cast<int>((j * (long long)rowbytes + k0) & ~15LL), n0 / P, &sh.rawfull[rs]);
                    }
                    return true;
                }
                uint32_t bytes = 0;
                if (tid < NW * kTcRows) {
                    const int n = n0 + tid, b0 = wi * TcBlock<QT>::kWin;
                    const int nblk = min(TcBlock<QT>::kWin, nk - b0);
                    const uintptr_t src = reinterpret_cast<uintptr_t>(a.w) +
                                          size_t(n < a.N ? n : a.N - 1) * rowbytes + size_t(kb0 + b0) * kBB;
                    const uintptr_t s16 = src & ~uintptr_t(15), end = src + size_t(nblk) * kBB;
                    uint32_t len = static_cast<uint32_t>((end - s16 + 15) & ~uintptr_t(15));
                    uint8_t* dst = raw + rs * kRawSlot + tid * kRawRow;
                    if (s16 + len > wend) {  // the buffer's last block: whole pieces + a plain tail
                        len = static_cast<uint32_t>((wend - s16) & ~uintptr_t(15));
                        for (uintptr_t p = s16 + len; p < end; p += 2)
                            *reinterpret_cast<uint16_t*>(dst + (p - s16)) = LdgU16(reinterpret_cast<const uint8_t*>(p));
                    }
                    if (len) BulkLoad(dst, reinterpret_cast<const void*>(s16), len, &sh.rawfull[rs]);
                    bytes = len;
                }
                bytes = __reduce_add_sync(0xffffffffu, bytes);
                __syncwarp();
                if (lane == 0) MbarExpectTx(&sh.rawfull[rs], bytes);
                return true;
            };
            bool ok = true;
            int issued = 0;  // windows of this pass whose copies were issued
            for (int wi = 0; wi < kTcRawSlots && ok; ++wi) {
                ok = issue(wi);
                if (ok && wi < nwin) issued = wi + 1;
            }
            for (int wi = 0; wi < nwin && ok; ++wi) {
                const int gw = pass * nwin + wi, rs = gw % kTcRawSlots;
                if (!MbarWaitFor(&sh.rawfull[rs], (gw / kTcRawSlots) & 1, kTcWaitNs, abort)) {
                    ok = false;
                    break;
                }
                const uint32_t rbase = SmemAddr(raw + rs * kRawSlot);
                const int b0 = wi * TcBlock<QT>::kWin, nblk = min(TcBlock<QT>::kWin, nk - b0);
                uint32_t rowbase[kItems];
#pragma unroll
                for (int i = 0; i < kItems; ++i) {
                    const uintptr_t src = reinterpret_cast<uintptr_t>(rowp[i]) + size_t(kb0 + b0) * kBB;
                    const int r = rb + kTcRows * i;
                    const int roff = a.tma_rows ? (r % a.tma_rows) * (NW * kTcRows / a.tma_rows) + r / a.tma_rows : r;
                    rowbase[i] = rbase + roff * kRawRow + static_cast<uint32_t>(src & 15);
                }
                bool big = false;
                for (int j = 0; j < nblk && ok; ++j) {
                    const int b = b0 + j;
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const int git = pass * nst + 2 * b + h, slot = git % kTcStages, use = git / kTcStages;
                        if (use > 0 && !MbarWaitFor(&sh.wempty[slot], (use - 1) & 1, kTcWaitNs, abort)) {
                            ok = false;
                            break;
                        }
                        uint8_t* st = stages + size_t(slot) * kTcStageBytes;
#pragma unroll
                        for (int i = 0; i < kItems; ++i) {
                            const TcRaw r = TcLoadRawSmem<QT>(rowbase[i] + j * kBB, c, h);
                            if (h == 0 && mul[i] != 0.0f && TcBound<QT>(r.d) * mul[i] >= 32768.0f) big = true;
                            uint4 hi, lo;
                            TcConvert<QT>(r, h, mul[i], hi, lo);
                            const int row = rb + kTcRows * i, t = row >> 7, rr = row & 127;
                            // SW: one 256-row hi image, then the lo image
                            uint8_t* dst = SW ? st + c * (2 * kTcRows * 16) + (row >> 3) * 128 + (row & 7) * 16
                                              : st + t * kTcWBytes + c * (kTcRows * 16) + (rr >> 3) * 128 + (rr & 7) * 16;
                            *reinterpret_cast<uint4*>(dst) = hi;
                            *reinterpret_cast<uint4*>(dst + (SW ? 2 * kTcWImg : kTcWImg)) = lo;
                        }
                        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                        __syncwarp();
                        if (lane == 0) MbarArrive(&sh.wfull[slot]);
                    }
                }
                if (!ok) break;
                if (big) sh.overflow = 1;
                __syncwarp();
                if (lane == 0) MbarArrive(&sh.rawempty[rs]);
                ok = issue(wi + kTcRawSlots);
                if (ok && wi + kTcRawSlots < nwin) issued = wi + kTcRawSlots + 1;
            }
            if (!ok && !*abort) TcFail(sh, a.status);
            // raw copies still in flight land before the CTA moves on (the
            // latest phase of each ring slot)
            if (lane == 0)
                for (int wi = max(0, issued - kTcRawSlots); wi < issued; ++wi) {
                    const int gw = pass * nwin + wi;
                    if (!MbarWaitFor(&sh.rawfull[gw % kTcRawSlots], (gw / kTcRawSlots) & 1, kTcWaitNs, nullptr))
                        TcFail(sh, a.status);
                }
            __syncwarp();
        } else if (warp == kTcDqWarps) {
            // ------------------------------------------------ x images: bulk copies
            if (lane == 0) {
                GridDepWait();  // the x images are the pre-pass's output
                const uint32_t bytes = static_cast<uint32_t>(mx) * kTcK * 4;
                int issued = 0;
                int slot = (pass * nst) % xslots, use = (pass * nst) / xslots;
                const uint8_t* src = a.ximg + (size_t(mt) * a.kst + 2 * kb0) * bytes;
                for (int it = 0; it < nst; ++it) {
                    if (use > 0 && !MbarTryWait(&sh.xempty[slot], (use - 1) & 1) &&
                        !MbarWaitFor(&sh.xempty[slot], (use - 1) & 1, kTcWaitNs, abort)) {
                        if (!*abort) TcFail(sh, a.status);
                        break;
                    }
                    if (*abort) break;
                    MbarExpectTx(&sh.xfull[slot], bytes);
                    BulkLoad(xring + size_t(slot) * bytes, src + size_t(it) * bytes, bytes, &sh.xfull[slot]);
                    issued = it + 1;
                    if (++slot == xslots) slot = 0, ++use;
                }
                // copies still in flight land before the CTA moves on
                for (int it = max(0, issued - xslots); it < issued; ++it) {
                    const int git = pass * nst + it;
                    if (!MbarWaitFor(&sh.xfull[git % xslots], (git / xslots) & 1, kTcWaitNs, nullptr))
                        TcFail(sh, a.status);
                }
            }
        } else {
            // ------------------------------------------------ MMA issue
            // One thread runs this loop at dependent-instruction latency, so
            // it keeps per-stage work minimal: descriptors are a base plus a
            // slot offset (the 14-bit start-address field never carries),
            // slots and phases advance by increments, and a completed barrier
            // costs one try_wait.
            if (lane == 0) {
                const uint32_t idesc = Idesc(SW ? 2 * kTcRows : mx);
                const uint64_t w0 = SmemDesc(SmemAddr(stages), (SW ? 2 : 1) * kTcRows * 16);
                const uint64_t x0 = SmemDesc(SmemAddr(xring), static_cast<uint32_t>(mx) * 16);
                const uint64_t wstep = kTcStageBytes >> 4, wsub = kTcWBytes >> 4, wlo = kTcWImg >> 4;
                const uint64_t xstep = static_cast<uint64_t>(4 * mx), xlo = static_cast<uint64_t>(2 * mx);
                int slot = (pass * nst) % kTcStages, use = (pass * nst) / kTcStages;
                int xs = (pass * nst) % xslots, xuse = (pass * nst) / xslots;
                int last = -1;  // stage (of this pass) of the last commit
                int lslot = 0, luse = 0;
                for (int it = 0; it < nst; ++it) {
                    if ((!MbarTryWait(&sh.xfull[xs], xuse & 1) &&
                         !MbarWaitFor(&sh.xfull[xs], xuse & 1, kTcWaitNs, abort)) ||
                        (!MbarTryWait(&sh.wfull[slot], use & 1) &&
                         !MbarWaitFor(&sh.wfull[slot], use & 1, kTcWaitNs, abort))) {
                        if (!*abort) TcFail(sh, a.status);
                        break;
                    }
                    TcFenceAfter();
                    const uint64_t xhi = x0 + xs * xstep, xlo2 = xhi + xlo;
                    const uint64_t aw = w0 + slot * wstep;
                    if constexpr (SW) {  // A = x (128 rows), B = W (256 rows)
                        const uint64_t whi = aw, wlo2 = aw + 2 * wlo;
                        TcMma(tmem, xhi, whi, idesc, it != 0);
                        TcMma(tmem, xhi, wlo2, idesc, 1);
                        TcMma(tmem, xlo2, whi, idesc, 1);
                    } else {  // A = W (128 rows per sub-tile), B = x (MX rows)
#pragma unroll
                        for (int t = 0; t < NW; ++t) {
                            const uint64_t ahi = aw + t * wsub, alo = ahi + wlo;
                            const uint32_t d = tmem + t * mx;
                            TcMma(d, ahi, xhi, idesc, it != 0);
                            TcMma(d, alo, xhi, idesc, 1);
                            TcMma(d, ahi, xlo2, idesc, 1);
                        }
                    }
                    TcCommit(&sh.wempty[slot]);
                    TcCommit(&sh.xempty[xs]);
                    last = it;
                    lslot = slot;
                    luse = use;
                    if (++slot == kTcStages) slot = 0, ++use;
                    if (++xs == xslots) xs = 0, ++xuse;
                }
                if (last == nst - 1 && nst > 0) {
                    TcCommit(&sh.accfull);
                } else if (last >= 0) {
                    // aborted: the MMAs issued so far finish before tensor memory is freed
                    if (!MbarWaitFor(&sh.wempty[lslot], luse & 1, kTcWaitNs, nullptr)) TcFail(sh, a.status);
                }
            }
        }
        __syncthreads();
        if (*abort || pass == 1 || !sh.overflow) break;
        // a block could overflow fp16 unscaled: recompute with per-row power-of-two scales
        // (after the first pass's accumulator phase has completed, so the
        // epilogue's wait on the second one is unambiguous)
        if (warp < kTcDqWarps) {
            if (!MbarWaitFor(&sh.accfull, 0, kTcWaitNs, abort) && !*abort) TcFail(sh, a.status);
#pragma unroll
            for (int i = 0; i < kItems; ++i) {
                const int row = rb + kTcRows * i, n = n0 + row;
                float bound = 0.0f;
                for (int b = kb0 + c; b < kb1; b += 2) bound = fmaxf(bound, TcBlockBound<QT>(rowp[i] + size_t(b) * kBB));
                bound = fmaxf(bound, __shfl_xor_sync(0xffffffffu, bound, 8));
                const int s = ScaleExp(bound);
                mul[i] = n < a.N ? Pow2(s) : 0.0f;
                if (c == 0) sh.wundo[row] = Pow2(-s);
            }
        }
        __syncthreads();
    }

    GridDepLaunch();  // the split-K sum may launch; it waits for this grid's partials
    // ------------------------------------------------ epilogue
    if (warp < kTcDqWarps && !*abort) {
        bool ok = MbarWaitFor(&sh.accfull, pass & 1, kTcWaitNs, abort);
        if (!ok && !*abort) TcFail(sh, a.status);
        TcFenceAfter();
        if (ok && !*abort && SW) {
            // lanes = x rows, columns = W rows (half 0: 0..127, half 1: 128..255)
            const int q = warp & 3, half = warp >> 2;
            const int m = m0 + 32 * q + lane;
            const float xu = m < a.M ? __ldg(a.xundo + m) : 0.0f;
            float* dst = (a.splits == 1 ? a.y : a.part + size_t(split) * a.M * a.N) + size_t(m < a.M ? m : 0) * a.N;
            const bool vec = (a.N & 3) == 0;
            for (int col = half * kTcRows; col < (half + 1) * kTcRows; col += 8) {
                float v[8];
                TcLoad8(tmem + (static_cast<uint32_t>(32 * q) << 16) + col, v);
                if (m >= a.M) continue;
                const int nb = n0 + col;
                float out[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const int n = nb + i;
                    out[i] = n < a.N ? v[i] * xu * sh.wundo[col + i] + ((a.splits == 1 && a.bias) ? a.bias[n] : 0.0f)
                                     : 0.0f;
                }
                if (vec && nb + 8 <= a.N) {
                    reinterpret_cast<float4*>(dst + nb)[0] = make_float4(out[0], out[1], out[2], out[3]);
                    reinterpret_cast<float4*>(dst + nb)[1] = make_float4(out[4], out[5], out[6], out[7]);
                } else {
                    for (int i = 0; i < 8; ++i)
                        if (nb + i < a.N) dst[nb + i] = out[i];
                }
            }
        } else if (ok && !*abort) {
            const int q = warp & 3, half = warp >> 2;
            const int t = NW == 2 ? half : 0;
            const int r = 32 * q + lane, n = n0 + t * kTcRows + r;
            const int cbeg = NW == 2 ? 0 : half * (mx >> 1), cend = NW == 2 ? mx : cbeg + (mx >> 1);
            const float wu = sh.wundo[t * kTcRows + r];
            const float bn = (a.splits == 1 && a.bias && n < a.N) ? a.bias[n] : 0.0f;
            float* dst = a.splits == 1 ? a.y : a.part + size_t(split) * a.M * a.N;
            for (int col = cbeg; col < cend; col += 8) {
                float v[8];
                TcLoad8(tmem + (static_cast<uint32_t>(32 * q) << 16) + t * mx + col, v);
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const int m = m0 + col + i;
                    if (m < a.M && n < a.N) dst[size_t(m) * a.N + n] = v[i] * wu * __ldg(a.xundo + m) + bn;
                }
            }
        }
    }
    TcFenceBefore();
    __syncthreads();
    if (warp == kTcDqWarps + 1) {
        TcFenceAfter();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(ncols));
    }
}

// ---------------------------------------------------------------- host plan
struct TcPlan {
    int nw, mx, mtiles, kper, splits;
    bool sw;  // swapped roles: A = x (128 rows), B = 256 W rows
};

// Tile shape and split-K from a cost model in SM cycles: per 32-element block
// the largest of the tensor time (3 NW MX), the shared-memory traffic of the
// MMA operand reads, the W images and the raw ring at 128 B per cycle, and the
// weight stream's share of HBM (~190 NW); plus a fixed cost per CTA and its
// epilogue, times the waves of CTAs over the SMs, plus the partial-sum pass
// when K is split.
TcPlan PlanTc(int M, int N, int nb, int sms) {
    TcPlan best{2, 16, 1, nb, 1, false};
    double best_t = 1e300;
    auto consider = [&](int nw, int mx, int mtiles, bool sw, double block) {
        const long long ntiles = (N + nw * kTcRows - 1) / (nw * kTcRows);
        for (int s = 1; s <= std::min(nb, 32); ++s) {
            const int kper = (nb + s - 1) / s;
            const int splits = (nb + kper - 1) / kper;
            if (splits != s) continue;
            const long long ctas = ntiles * mtiles * splits;
            const long long waves = (ctas + sms - 1) / sms;
            double t = double(waves) * (3000.0 + kper * block + 12.0 * nw * mx);
            if (splits > 1) t += 2000.0 + double(M) * N * 4.0 * (splits + 1) / (23.5 * sms);
            if (t < best_t) {
                best_t = t;
                best = TcPlan{nw, mx, mtiles, kper, splits, sw};
            }
        }
    };
    // per-block cycles: the MMA thread (~160 a tcgen05.mma with its share of
    // the stage's waits and commits, measured), tensor time, shared-memory
    // wavefronts (operand reads, images, raw ring) and the HBM share of W
    constexpr double kMmaCycles = 160.0;
    if (M <= kTcRows) {
        const double smem_bytes = 2.0 * (3.0 * (kTcWImg + 2.0 * kTcWImg) + kTcWBytes * 2.0 + kTcRows * kTcK * 4.0) +
                                  2.0 * 2 * kTcRows * 48.0;
        const double block = std::max({2 * 3 * kMmaCycles, 2 * 3 * 128.0, smem_bytes / 128.0, 380.0}) + 150.0;
        consider(2, kTcRows, 1, true, block);
    }
    const int mt_min = (M + kTcMaxX - 1) / kTcMaxX;
    for (int nw = 1; nw <= 2; ++nw) {
        for (int mtiles = mt_min; mtiles <= mt_min + 3; ++mtiles) {
            const int mx = ((M + mtiles - 1) / mtiles + 15) / 16 * 16;
            if (mx > kTcMaxX || (mtiles > mt_min && mx < 64)) continue;
            const double smem_bytes = 2.0 * nw * (3.0 * (kTcWImg + 2.0 * kTcK * mx) + kTcWBytes) +
                                      2.0 * nw * kTcRows * 48.0;
            const double block =
                std::max({2 * 3 * kMmaCycles * nw, 3.0 * nw * mx, smem_bytes / 128.0, 190.0 * nw}) + 150.0;
            consider(nw, mx, mtiles, false, block);
        }
    }
    return best;
}

// The weight blocks as a 2-D tensor map for the raw-window copies: rows viewed
// P at a time (P the smallest of 1, 2, 4, 8 that makes the row stride a
// multiple of 16 bytes), boxes of kRawRow bytes x (cta_rows / P) rows.
// Returns P, or 0 (per-row bulk copies) when the rows do not divide into
// such groups or the base is not 16-byte aligned.
template <int QT>
int WeightMap(const uint8_t* w, int N, int nb, int cta_rows, CUtensorMap& map) {
    std::memset(&map, 0, sizeof(map));
    const size_t rowbytes = size_t(nb) * TcBlock<QT>::kBytes;
    int P = 1;
    while (P <= 8 && (P * rowbytes) % 16 != 0) P *= 2;
    if (P > 8 || N % P != 0 || (reinterpret_cast<uintptr_t>(w) & 15) != 0 || cta_rows / P > 256) return 0;
    const cuuint64_t gdim[2] = {cuuint64_t(P * rowbytes), cuuint64_t(N / P)};
    const cuuint64_t gstride[1] = {cuuint64_t(P * rowbytes)};
    const cuuint32_t box[2] = {cuuint32_t(TcBlock<QT>::kRawRow), cuuint32_t(cta_rows / P)};
    const cuuint32_t estride[2] = {1, 1};
    const PFN_cuTensorMapEncodeTiled_v12000 encode = TensorMapEncoder();
    if (!encode) return 0;
    const CUresult r = encode(&map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(w), gdim, gstride, box,
                              estride, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? P : 0;
}

template <int QT, int NW, bool SW>
void LaunchTcKernel(DeviceContext& c, dim3 grid, const TcArgs& a, const CUtensorMap& wmap) {
    constexpr size_t smem = TcSmemBytes<QT>();
    static int configured[64] = {};
    if (c.device >= 64 || !configured[c.device]) {
        CheckCuda(cudaFuncSetAttribute(TcLinearKernel<QT, NW, SW>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem)),
                  "cudaFuncSetAttribute(TcLinearKernel)");
        if (c.device < 64) configured[c.device] = 1;
    }
    Launch("TcLinearKernel", TcLinearKernel<QT, NW, SW>, grid, dim3(kTcThreads), smem, c.stream, true, a, wmap);
}

// Workspace layout of one call: x images, x undo factors, split-K partials.
struct TcLayout {
    TcPlan plan;
    int nb, kst;
    size_t undo_off, part_off, total;
};

TcLayout LayoutTc(int M, int K, int N, int sms) {
    TcLayout L;
    L.nb = (K + 31) / 32;
    L.kst = 2 * L.nb;  // stages of 16 elements
    L.plan = PlanTc(M, N, L.nb, sms);
    const size_t img_bytes = size_t(L.plan.mtiles) * L.kst * L.plan.mx * kTcK * 4;
    L.undo_off = (img_bytes + 255) / 256 * 256;
    L.part_off = L.undo_off + (size_t(M) * 4 + 255) / 256 * 256;
    L.total = L.part_off + (L.plan.splits > 1 ? size_t(L.plan.splits) * M * N * 4 : 0);
    return L;
}

template <int QT>
void LaunchTcT(DeviceContext& c, const float* x, const uint8_t* w, int M, int K, int N, const float* bias,
               float* y, int* status, void* workspace, bool reuse_x) {
    const TcLayout L = LayoutTc(M, K, N, c.sm_count);
    const TcPlan& p = L.plan;
    const int nb = L.nb, kst = L.kst;
    const size_t undo_off = L.undo_off, part_off = L.part_off;
    uint8_t* ws = static_cast<uint8_t*>(workspace ? workspace : Workspace(c, L.total));
    float* undo = reinterpret_cast<float*>(ws + undo_off);
    float* part = reinterpret_cast<float*>(ws + part_off);
    const bool reuse = reuse_x && c.tc_x == x && c.tc_ws == ws && c.tc_m == M && c.tc_k == K &&
                       c.tc_mx == p.mx && c.tc_mtiles == p.mtiles;
    if (!reuse)
        Launch("TcPrepX", TcPrepX, dim3(p.mtiles * p.mx), dim3(128), 0, c.stream, true, x, M, K, p.mx, kst, undo,
               ws);
    c.tc_x = x;
    c.tc_ws = ws;
    c.tc_m = M;
    c.tc_k = K;
    c.tc_mx = p.mx;
    c.tc_mtiles = p.mtiles;
    TcArgs a{w, N, K, nb, M, p.mx, p.mtiles, kst, p.kper, ws, undo, bias, y, part, p.splits, status, 0};
    const dim3 grid(p.mtiles * p.splits, (N + p.nw * kTcRows - 1) / (p.nw * kTcRows));
    CUtensorMap wmap;
    a.tma_rows = WeightMap<QT>(w, N, nb, p.nw * kTcRows, wmap);
    if (p.sw) LaunchTcKernel<QT, 2, true>(c, grid, a, wmap);
    else if (p.nw == 2) LaunchTcKernel<QT, 2, false>(c, grid, a, wmap);
    else LaunchTcKernel<QT, 1, false>(c, grid, a, wmap);
    if (p.splits > 1) {
        const size_t mn = size_t(M) * N;
        // four columns per thread when N % 4 == 0 (TcReduce's vector path)
        const size_t items = (N & 3) == 0 ? mn / 4 : mn;
        const int g = static_cast<int>(std::max<size_t>(1, std::min<size_t>((items + 255) / 256, size_t(8) * c.sm_count)));
        Launch("TcReduce", TcReduce, dim3(g), dim3(256), 0, c.stream, true, static_cast<const float*>(part), p.splits,
               M, N, bias, y);
    }
}

}  // namespace

size_t TcWorkspaceBytes(int M, int K, int N, int sm_count) {
    size_t total = LayoutTc(M, K, N, sm_count).total;
    if (WidePreferred(M, K, N)) total = std::max(total, WideWorkspaceBytes(M, K, N, sm_count, 227 * 1024));
    return total;
}

void LaunchTcLinear(DeviceContext& c, int qtype, const float* x, const uint8_t* w, int M, int K, int N,
                    const float* bias, float* y, int* status, void* workspace, bool reuse_x) {
    static_assert(sizeof(TcShared) <= kTcHeader, "shared header");
    Require((reinterpret_cast<uintptr_t>(w) & 1) == 0, "mlb_quant_linear", "weight blocks must be 2-byte aligned");
    if (WidePreferred(M, K, N) && LaunchWideLinear(c, qtype, x, w, M, K, N, bias, y, status, workspace, reuse_x))
        return;
    switch (qtype) {
        case MLB_Q8_0: LaunchTcT<MLB_Q8_0>(c, x, w, M, K, N, bias, y, status, workspace, reuse_x); break;
        case MLB_Q4_0: LaunchTcT<MLB_Q4_0>(c, x, w, M, K, N, bias, y, status, workspace, reuse_x); break;
        default: LaunchTcT<MLB_Q4_1>(c, x, w, M, K, N, bias, y, status, workspace, reuse_x); break;
    }
}

}  // namespace mlb
