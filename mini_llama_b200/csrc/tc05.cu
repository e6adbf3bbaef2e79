// Quantized linear for M >= 64 rows (prefill): y = x W^T (+ bias) on the
// 5th-generation tensor cores (tcgen05.mma, accumulator in tensor memory).
// Replaces the reference's Q8_0 / Q4_0 / Q4_1 linear kernels
// (src/cuda_quant.cu:40-135) for batches of rows.
//
// Exactness: the reference multiplies fp32 x by the fp32 dequantized weight
// w = fp16(d) * q (Q4_0: d * (q - 8); Q4_1: d * q + m, rounded once) and sums
// in fp32.  Here each row of W is scaled by a power of two 2^s_n and each row
// of x by 2^s_m (exact) so that their largest magnitudes sit in [2^14, 2^15),
// then every value v is split into fp16 v_hi = rn(v) and v_lo = rn(v - v_hi)
// (v_hi + v_lo carries 22 significant bits; a Q8_0 / Q4_0 weight has at most
// 19 and is split exactly).  The tensor cores accumulate
//   x_hi w_hi + x_hi w_lo + x_lo w_hi
// in fp32 (the x_lo w_lo term is below 2^-22 relative), and the epilogue
// undoes the scales.  Result: within ~1e-6 relative of the fp32 reference.
//
// Layout: both operands K-major in the canonical no-swizzle tcgen05 layout,
// 8-row x 16-byte core matrices; a 128-row x 64-element stage image is
//   offset(r, k) = ((k / 8) * 16 + r / 8) * 128 + (r % 8) * 16 + (k % 8) * 2
// (leading byte offset 2048 between 8-element k chunks, stride byte offset 128
// between 8-row groups), hi image then lo image.  The x images are written by
// a pre-pass (TcSplitX) so a stage of x is one 32 KB bulk copy; the W images
// are dequantized in shared memory by the CTA itself (thread t: W row t).
//
// Per CTA one 128 x 128 output tile, two stages in flight: while the tensor
// cores run stage k, the threads dequantize stage k + 1.  Thread 0 issues the
// MMAs (4 k-steps x 3 products a stage) and commits them to the stage's
// mbarrier.  The epilogue reads the accumulator with tcgen05.ld (warp w reads
// tensor-memory lanes 32w .. 32w + 31 = output rows).  Every wait is bounded
// (an expired wait records MLB_ERR_DEVICE_TIMEOUT); tensor memory is freed
// on every path.
#include <algorithm>
#include <cmath>

#include "common.cuh"
#include "qgemv.cuh"

namespace mlb {
namespace {

constexpr int kTcM = 128;          // output rows (x rows) per tile
constexpr int kTcN = 128;          // output columns (W rows) per tile
constexpr int kTcK = 64;           // elements of K per stage
constexpr int kTcImage = 16384;    // bytes of one fp16 128 x 64 image
constexpr int kTcStageBytes = 4 * kTcImage;  // x hi, x lo, w hi, w lo
constexpr int kTcThreads = 128;
constexpr uint64_t kTcWaitNs = 2000000000ull;

__host__ __device__ constexpr size_t TcImageOffset(int r, int k) {
    return (size_t((k / 8) * 16 + r / 8) * 128) + (r % 8) * 16 + (k % 8) * 2;
}

// 2^e as a float for -126 <= e <= 127, from its exponent bits.
__device__ __forceinline__ float Pow2(int e) { return __uint_as_float(static_cast<uint32_t>(127 + e) << 23); }

// Exponent s with (bound * 2^s) in [2^14, 2^15) (0 when bound is 0 or not finite).
__device__ __forceinline__ int ScaleExp(float bound) {
    if (!(bound > 0.0f) || !isfinite(bound)) return 0;
    const int e = static_cast<int>((__float_as_uint(bound) >> 23) & 0xff) - 127;  // 2^e <= bound < 2^(e+1)
    int s = 14 - e;
    return s > 100 ? 100 : (s < -100 ? -100 : s);
}

__device__ __forceinline__ void SplitHalf(float v, __half& hi, __half& lo) {
    hi = __float2half_rn(v);
    lo = __float2half_rn(v - __half2float(hi));
}

// ---------------------------------------------------------------- x pre-pass
// One warp per x row: its scale exponent (largest |x| into [2^14, 2^15)),
// written as the undo factor 2^-s (and kept for the split).
__global__ void __launch_bounds__(256) TcRowScale(const float* x, int M, int K, float* undo, int* sexp) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= M) return;
    const float* row = x + size_t(warp) * K;
    float mx = 0.0f;
    for (int k = lane; k < K; k += 32) mx = fmaxf(mx, fabsf(row[k]));
    mx = WarpMax(mx);
    if (lane == 0) {
        const int s = ScaleExp(mx);
        sexp[warp] = s;
        undo[warp] = Pow2(-s);
    }
}

// x -> hi / lo stage images [m_tile][k_stage][hi, lo], rows past M and
// columns past K zero.  One thread per (row, 8-element chunk).
__global__ void __launch_bounds__(256) TcSplitX(const float* x, int M, int K, int ktiles, const int* sexp,
                                                uint8_t* images) {
    const int mtiles = (M + kTcM - 1) / kTcM;
    const long long total = 1LL * mtiles * kTcM * ktiles * (kTcK / 8);
    for (long long i = blockIdx.x * 1LL * blockDim.x + threadIdx.x; i < total; i += 1LL * gridDim.x * blockDim.x) {
        const int chunk = static_cast<int>(i % (kTcK / 8));
        long long rest = i / (kTcK / 8);
        const int kt = static_cast<int>(rest % ktiles);
        rest /= ktiles;
        const int r = static_cast<int>(rest % kTcM);
        const int mt = static_cast<int>(rest / kTcM);
        const int m = mt * kTcM + r;
        const int k0 = kt * kTcK + chunk * 8;
        __align__(16) __half hi[8], lo[8];
        const float sc = m < M ? Pow2(sexp[m]) : 0.0f;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float v = (m < M && k0 + j < K) ? x[size_t(m) * K + k0 + j] * sc : 0.0f;
            SplitHalf(v, hi[j], lo[j]);
        }
        uint8_t* img = images + (size_t(mt) * ktiles + kt) * (2 * kTcImage);
        const size_t off = TcImageOffset(r, chunk * 8);
        *reinterpret_cast<uint4*>(img + off) = *reinterpret_cast<const uint4*>(hi);
        *reinterpret_cast<uint4*>(img + kTcImage + off) = *reinterpret_cast<const uint4*>(lo);
    }
}

// ---------------------------------------------------------------- tcgen05
__device__ __forceinline__ uint64_t SmemDesc(uint32_t addr) {
    // K-major, no swizzle: LBO 2048 B (k chunks), SBO 128 B (8-row groups), version 1
    return static_cast<uint64_t>((addr >> 4) & 0x3FFFu) | (static_cast<uint64_t>(2048 >> 4) << 16) |
           (static_cast<uint64_t>(128 >> 4) << 32) | (1ull << 46);
}

// kind::f16, fp32 accumulate, fp16 A and B, both K-major, N = 128, M = 128.
constexpr uint32_t kTcIdesc = (1u << 4) | (0u << 7) | (0u << 10) | (static_cast<uint32_t>(kTcN >> 3) << 17) |
                              (static_cast<uint32_t>(kTcM >> 4) << 24);

__device__ __forceinline__ void TcMma(uint32_t dtmem, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n"
        :
        : "r"(dtmem), "l"(adesc), "l"(bdesc), "r"(kTcIdesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0));
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

// Dequantized weight j (0..31) of a block, before the row scale.
template <int QT>
__device__ __forceinline__ float BlockWeight(const uint8_t* blk, int j) {
    const float d = HalfBits(static_cast<uint16_t>(blk[0] | (blk[1] << 8)));
    if constexpr (QT == MLB_Q8_0) {
        return __fmul_rn(d, static_cast<float>(static_cast<int8_t>(blk[2 + j])));
    } else if constexpr (QT == MLB_Q4_0) {
        const int q = j < 16 ? (blk[2 + j] & 15) : (blk[2 + j - 16] >> 4);
        return __fmul_rn(d, static_cast<float>(q - 8));
    } else {
        const float mn = HalfBits(static_cast<uint16_t>(blk[2] | (blk[3] << 8)));
        const int q = j < 16 ? (blk[4 + j] & 15) : (blk[4 + j - 16] >> 4);
        return __fadd_rn(__fmul_rn(d, static_cast<float>(q)), mn);
    }
}

// Upper bound of |w| over one block.
template <int QT>
__device__ __forceinline__ float BlockBound(const uint8_t* blk) {
    const float d = fabsf(HalfBits(static_cast<uint16_t>(blk[0] | (blk[1] << 8))));
    if constexpr (QT == MLB_Q8_0) return d * 128.0f;
    else if constexpr (QT == MLB_Q4_0) return d * 8.0f;
    else return d * 15.0f + fabsf(HalfBits(static_cast<uint16_t>(blk[2] | (blk[3] << 8))));
}

struct TcShared {
    uint64_t xfull[2];
    uint64_t mmadone[2];
    uint32_t tmem;
    int abort;
    int last;  // stage of the last commit (-1: none)
    float wundo[kTcN];
};

template <int QT>
__global__ void __launch_bounds__(kTcThreads, 1)
    TcLinearKernel(const uint8_t* w, int N, int K, int nb, int M, int ktiles, const uint8_t* ximages,
                   const float* xundo, const float* bias, float* y, int* status) {
    extern __shared__ __align__(1024) uint8_t smem[];
    TcShared& sh = *reinterpret_cast<TcShared*>(smem);
    uint8_t* stages = smem + 1024;  // 2 x kTcStageBytes, 1024-aligned
    const int tid = threadIdx.x, warp = tid >> 5;
    const int n0 = blockIdx.x * kTcN, mt = blockIdx.y, m0 = mt * kTcM;
    constexpr int kBB = QT == MLB_Q8_0 ? 34 : (QT == MLB_Q4_0 ? 18 : 20);

    if (tid == 0) {
        for (int i = 0; i < 2; ++i) {
            MbarInit(&sh.xfull[i], 1);
            MbarInit(&sh.mmadone[i], 1);
        }
        FenceMbarInit();
        sh.abort = 0;
        sh.last = -1;
    }
    if (warp == 0) {  // 128 tensor-memory columns: the 128 x 128 fp32 accumulator
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(SmemAddr(&sh.tmem)),
                     "r"(kTcN));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
    }
    // this thread's W row: its scale from the largest block bound
    const int n = n0 + tid;
    const uint8_t* wrow = w + size_t(n < N ? n : 0) * nb * kBB;
    float bound = 0.0f;
    if (n < N)
        for (int b = 0; b < nb; ++b) bound = fmaxf(bound, BlockBound<QT>(wrow + size_t(b) * kBB));
    const int sw = ScaleExp(bound);
    const float wsc = Pow2(sw);
    sh.wundo[tid] = Pow2(-sw);
    TcFenceBefore();
    __syncthreads();
    TcFenceAfter();
    const uint32_t tmem = sh.tmem;

    for (int kt = 0; kt < ktiles; ++kt) {
        const int slot = kt & 1;
        uint8_t* st = stages + size_t(slot) * kTcStageBytes;
        if (kt >= 2 && !MbarWaitFor(&sh.mmadone[slot], ((kt - 2) >> 1) & 1, kTcWaitNs, &sh.abort)) {
            atomicCAS(status, 0, MLB_ERR_DEVICE_TIMEOUT);
            sh.abort = 1;
        }
        __syncthreads();
        if (sh.abort) break;
        if (tid == 0) {  // the x hi / lo images of this stage, one bulk copy
            MbarExpectTx(&sh.xfull[slot], 2 * kTcImage);
            BulkLoad(st, ximages + (size_t(mt) * ktiles + kt) * (2 * kTcImage), 2 * kTcImage, &sh.xfull[slot]);
        }
        // W row tid, elements kt*64 .. +63 (two blocks), into the w images
        uint8_t* wimg = st + 2 * kTcImage;
#pragma unroll
        for (int half = 0; half < 2; ++half) {
            const int b = kt * 2 + half;
            const bool on = n < N && b < nb;
            const uint8_t* blk = wrow + size_t(on ? b : 0) * kBB;
#pragma unroll
            for (int c = 0; c < 4; ++c) {  // 8-element chunks
                __align__(16) __half hi[8], lo[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const int e = c * 8 + j;
                    // (elements past K in the last block meet zero x)
                    SplitHalf(on ? BlockWeight<QT>(blk, e) * wsc : 0.0f, hi[j], lo[j]);
                }
                const size_t off = TcImageOffset(tid, half * 32 + c * 8);
                *reinterpret_cast<uint4*>(wimg + off) = *reinterpret_cast<const uint4*>(hi);
                *reinterpret_cast<uint4*>(wimg + kTcImage + off) = *reinterpret_cast<const uint4*>(lo);
            }
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncthreads();
        if (tid == 0) {
            if (!MbarWaitFor(&sh.xfull[slot], (kt >> 1) & 1, kTcWaitNs, nullptr)) {
                atomicCAS(status, 0, MLB_ERR_DEVICE_TIMEOUT);
                sh.abort = 1;
            } else {
                TcFenceAfter();
                const uint32_t a = SmemAddr(st), b = a + 2 * kTcImage;
#pragma unroll
                for (int j = 0; j < kTcK / 16; ++j) {  // k-steps of 16: two 8-element chunks
                    const uint32_t ko = j * 2 * 2048;
                    const uint64_t ahi = SmemDesc(a + ko), alo = SmemDesc(a + kTcImage + ko);
                    const uint64_t bhi = SmemDesc(b + ko), blo = SmemDesc(b + kTcImage + ko);
                    TcMma(tmem, ahi, bhi, (kt | j) != 0);
                    TcMma(tmem, ahi, blo, 1);
                    TcMma(tmem, alo, bhi, 1);
                }
                TcCommit(&sh.mmadone[slot]);
                sh.last = kt;
            }
        }
    }
    // the last commit covers every MMA issued before it: wait for it (also
    // after an abort, before the memory is freed)
    __syncthreads();
    const int last = sh.last;
    if (last >= 0 && !MbarWaitFor(&sh.mmadone[last & 1], (last >> 1) & 1, kTcWaitNs, nullptr)) {
        atomicCAS(status, 0, MLB_ERR_DEVICE_TIMEOUT);
        sh.abort = 1;
    }
    if (last != ktiles - 1) sh.abort = 1;
    __syncthreads();
    TcFenceAfter();
    if (!sh.abort) {
        // epilogue: warp w holds output rows 32 w .. 32 w + 31 (tensor-memory lanes)
        const int r = warp * 32 + (tid & 31);
        const int m = m0 + r;
        const float xu = m < M ? xundo[m] : 0.0f;
        for (int c0 = 0; c0 < kTcN; c0 += 8) {
            float v[8];
            TcLoad8(tmem + (static_cast<uint32_t>(warp * 32) << 16) + c0, v);
            if (m >= M) continue;
            float out[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int nn = n0 + c0 + i;
                out[i] = nn < N ? v[i] * xu * sh.wundo[c0 + i] + (bias ? bias[nn] : 0.0f) : 0.0f;
            }
            float* yr = y + size_t(m) * N + n0 + c0;
            if (n0 + c0 + 8 <= N && (N & 3) == 0) {
                reinterpret_cast<float4*>(yr)[0] = make_float4(out[0], out[1], out[2], out[3]);
                reinterpret_cast<float4*>(yr)[1] = make_float4(out[4], out[5], out[6], out[7]);
            } else {
                for (int i = 0; i < 8; ++i)
                    if (n0 + c0 + i < N) yr[i] = out[i];
            }
        }
    }
    TcFenceBefore();
    __syncthreads();
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTcN));
}

template <int QT>
void LaunchTcT(DeviceContext& c, const float* x, const uint8_t* w, int M, int K, int N, const float* bias,
               float* y, int* status) {
    const int nb = (K + 31) / 32;
    const int ktiles = (K + kTcK - 1) / kTcK;
    const int mtiles = (M + kTcM - 1) / kTcM;
    const size_t img_bytes = size_t(mtiles) * ktiles * 2 * kTcImage;
    uint8_t* ws = static_cast<uint8_t*>(Workspace(c, img_bytes + size_t(M) * 8 + 256));
    uint8_t* images = ws;
    float* undo = reinterpret_cast<float*>(ws + img_bytes);
    int* sexp = reinterpret_cast<int*>(ws + img_bytes + size_t(M) * 4);
    TcRowScale<<<(M * 32 + 255) / 256, 256, 0, c.stream>>>(x, M, K, undo, sexp);
    CheckCuda(cudaGetLastError(), "TcRowScale");
    const long long chunks = 1LL * mtiles * kTcM * ktiles * (kTcK / 8);
    const int grid = static_cast<int>(std::min<long long>((chunks + 255) / 256, 16LL * c.sm_count));
    TcSplitX<<<grid, 256, 0, c.stream>>>(x, M, K, ktiles, sexp, images);
    CheckCuda(cudaGetLastError(), "TcSplitX");
    const size_t smem = 1024 + 2 * size_t(kTcStageBytes);
    static int configured[64] = {};
    if (c.device >= 64 || configured[c.device] < static_cast<int>(smem)) {
        CheckCuda(cudaFuncSetAttribute(TcLinearKernel<QT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem)),
                  "cudaFuncSetAttribute(TcLinearKernel)");
        if (c.device < 64) configured[c.device] = static_cast<int>(smem);
    }
    dim3 g((N + kTcN - 1) / kTcN, mtiles);
    TcLinearKernel<QT><<<g, kTcThreads, smem, c.stream>>>(w, N, K, nb, M, ktiles, images, undo, bias, y, status);
    CheckCuda(cudaGetLastError(), "TcLinearKernel");
}

}  // namespace

void LaunchTcLinear(DeviceContext& c, int qtype, const float* x, const uint8_t* w, int M, int K, int N,
                    const float* bias, float* y, int* status) {
    static_assert(sizeof(TcShared) <= 1024, "shared header");
    switch (qtype) {
        case MLB_Q8_0: LaunchTcT<MLB_Q8_0>(c, x, w, M, K, N, bias, y, status); break;
        case MLB_Q4_0: LaunchTcT<MLB_Q4_0>(c, x, w, M, K, N, bias, y, status); break;
        default: LaunchTcT<MLB_Q4_1>(c, x, w, M, K, N, bias, y, status); break;
    }
}

}  // namespace mlb
