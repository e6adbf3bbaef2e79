// F32 linear and matmul (replace the cuBLAS path of mini_llama
// src/cuda_matmul.cpp:118-229, which creates a cuBLAS handle per call).
//
// F32 linear (y = x . W^T + bias, rows <= 8 per pass) is bandwidth-bound: a
// warp owns an output row, streams the weight row with 16-byte loads
// (four rows in flight per warp) and dots it with x held in shared memory.
// The general matmul (C = A . B, B row-major [K, N]) is a 64x64 shared-memory
// tiled FMA kernel; it serves the reference's CudaMatmul, a test utility.
#include <algorithm>

#include "common.cuh"

namespace mlb {
namespace {

constexpr int kF32Rows = 8;   // x rows per pass
constexpr int kRowsPerWarp = 4;

template <int M>
__global__ void __launch_bounds__(256) F32LinearKernel(const float* x, const float* w,
                                                       const float* bias, float* y, int K, int N) {
    extern __shared__ __align__(16) float xs[];  // [M][K]
    StageFloats(xs, x, M * K);
    CpAsyncWaitAll();
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nwarps = gridDim.x * (blockDim.x >> 5);
    const bool vec = (K % 4 == 0) && ((reinterpret_cast<uintptr_t>(w) & 15) == 0);
    for (int r0 = (blockIdx.x * (blockDim.x >> 5) + warp) * kRowsPerWarp; r0 < N;
         r0 += nwarps * kRowsPerWarp) {
        float acc[kRowsPerWarp][M];
#pragma unroll
        for (int i = 0; i < kRowsPerWarp; ++i)
#pragma unroll
            for (int m = 0; m < M; ++m) acc[i][m] = 0.0f;
        if (vec) {
            const int k4 = K / 4;
            for (int c = lane; c < k4; c += 32) {
                float4 wv[kRowsPerWarp];
#pragma unroll
                for (int i = 0; i < kRowsPerWarp; ++i)
                    wv[i] = r0 + i < N ? __ldcs(reinterpret_cast<const float4*>(w + size_t(r0 + i) * K) + c)
                                       : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
                for (int m = 0; m < M; ++m) {
                    const float4 xv = reinterpret_cast<const float4*>(xs + m * K)[c];
#pragma unroll
                    for (int i = 0; i < kRowsPerWarp; ++i) {
                        acc[i][m] = fmaf(wv[i].x, xv.x, acc[i][m]);
                        acc[i][m] = fmaf(wv[i].y, xv.y, acc[i][m]);
                        acc[i][m] = fmaf(wv[i].z, xv.z, acc[i][m]);
                        acc[i][m] = fmaf(wv[i].w, xv.w, acc[i][m]);
                    }
                }
            }
        } else {
            for (int k = lane; k < K; k += 32) {
#pragma unroll
                for (int i = 0; i < kRowsPerWarp; ++i) {
                    const float wv = r0 + i < N ? w[size_t(r0 + i) * K + k] : 0.0f;
#pragma unroll
                    for (int m = 0; m < M; ++m) acc[i][m] = fmaf(wv, xs[m * K + k], acc[i][m]);
                }
            }
        }
#pragma unroll
        for (int i = 0; i < kRowsPerWarp; ++i)
#pragma unroll
            for (int m = 0; m < M; ++m) {
                const float v = WarpSum(acc[i][m]);
                if (lane == 0 && r0 + i < N)
                    y[size_t(m) * N + r0 + i] = v + (bias ? bias[r0 + i] : 0.0f);
            }
    }
}

__global__ void F32MatmulKernel(const float* a, const float* b, float* c, int M, int K, int N) {
    __shared__ float as[64][17];
    __shared__ float bs[16][65];
    const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;  // 16 x 16 threads, 4x4 outputs each
    const int row0 = blockIdx.y * 64, col0 = blockIdx.x * 64;
    float acc[4][4] = {};
    for (int k0 = 0; k0 < K; k0 += 16) {
        for (int i = threadIdx.x; i < 64 * 16; i += 256) {
            const int r = i / 16, kk = i % 16;
            as[r][kk] = (row0 + r < M && k0 + kk < K) ? a[size_t(row0 + r) * K + k0 + kk] : 0.0f;
            const int kr = i / 64, cc = i % 64;
            bs[kr][cc] = (k0 + kr < K && col0 + cc < N) ? b[size_t(k0 + kr) * N + col0 + cc] : 0.0f;
        }
        __syncthreads();
        for (int kk = 0; kk < 16; ++kk)
            for (int i = 0; i < 4; ++i)
                for (int j = 0; j < 4; ++j)
                    acc[i][j] = fmaf(as[ty * 4 + i][kk], bs[kk][tx * 4 + j], acc[i][j]);
        __syncthreads();
    }
    for (int i = 0; i < 4; ++i)
        for (int j = 0; j < 4; ++j) {
            const int r = row0 + ty * 4 + i, cc = col0 + tx * 4 + j;
            if (r < M && cc < N) c[size_t(r) * N + cc] = acc[i][j];
        }
}

template <int M>
void LaunchF32(DeviceContext& c, const float* x, const float* w, const float* bias, float* y, int K,
               int N) {
    const size_t smem = size_t(M) * K * 4;
    Require(smem + 1024 <= static_cast<size_t>(c.max_smem_optin), "CudaLinear",
            "in_features too large for the F32 GEMV", MLB_ERR_UNSUPPORTED);
    static int configured[64] = {};
    if (c.device >= 64 || configured[c.device] < static_cast<int>(smem)) {
        CheckCuda(cudaFuncSetAttribute(F32LinearKernel<M>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem)),
                  "cudaFuncSetAttribute(F32LinearKernel)");
        if (c.device < 64) configured[c.device] = static_cast<int>(smem);
    }
    const int warps_needed = (N + kRowsPerWarp - 1) / kRowsPerWarp;
    const int grid = std::max(1, std::min((warps_needed + 7) / 8, c.sm_count * 4));
    F32LinearKernel<M><<<grid, 256, smem, c.stream>>>(x, w, bias, y, K, N);
    CheckCuda(cudaGetLastError(), "F32LinearKernel");
}

}  // namespace
}  // namespace mlb

using namespace mlb;

extern "C" {

int mlb_f32_linear(int device, const float* x, const float* w, int rows, int in_features,
                   int out_features, const float* bias, float* y) {
    return Guard([&] {
        const char* c = "CudaLinear";
        Require(x && w && y, c, "device weight is null");
        Require(rows > 0 && in_features > 0 && out_features > 0, c, "empty tensors are not supported");
        DeviceContext& ctx = Ctx(device);
        for (int m0 = 0; m0 < rows; m0 += kF32Rows) {
            const int M = std::min(kF32Rows, rows - m0);
            const float* xm = x + size_t(m0) * in_features;
            float* ym = y + size_t(m0) * out_features;
            switch (M) {
                case 1: LaunchF32<1>(ctx, xm, w, bias, ym, in_features, out_features); break;
                case 2: LaunchF32<2>(ctx, xm, w, bias, ym, in_features, out_features); break;
                case 3: LaunchF32<3>(ctx, xm, w, bias, ym, in_features, out_features); break;
                case 4: LaunchF32<4>(ctx, xm, w, bias, ym, in_features, out_features); break;
                case 5: LaunchF32<5>(ctx, xm, w, bias, ym, in_features, out_features); break;
                case 6: LaunchF32<6>(ctx, xm, w, bias, ym, in_features, out_features); break;
                case 7: LaunchF32<7>(ctx, xm, w, bias, ym, in_features, out_features); break;
                default: LaunchF32<8>(ctx, xm, w, bias, ym, in_features, out_features); break;
            }
        }
    });
}

int mlb_f32_matmul(int device, const float* a, const float* b, int m, int k, int n, float* c) {
    return Guard([&] {
        Require(a && b && c, "CudaMatmul", "tensor is null");
        Require(m > 0 && k > 0 && n > 0, "CudaMatmul", "tensor must be 2D and non-empty");
        DeviceContext& ctx = Ctx(device);
        dim3 grid((n + 63) / 64, (m + 63) / 64);
        F32MatmulKernel<<<grid, 256, 0, ctx.stream>>>(a, b, c, m, k, n);
        CheckCuda(cudaGetLastError(), "F32MatmulKernel");
    });
}

}  // extern "C"
