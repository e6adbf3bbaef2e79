// Row-wise element kernels shared by the batched decode driver (batch.cu)
// and the session's prompt pass (decode.cu): each works on `rows` vectors at
// once with the arithmetic of the reference CPU path (src/ops.cpp).  All are
// launched with programmatic dependent launch and wait for the previous grid
// before reading.
#pragma once

#include "common.cuh"

namespace mlb {
namespace {

__device__ __forceinline__ float RowsBlockSum(float v, float* scratch) {
    v = WarpSum(v);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) scratch[warp] = v;
    __syncthreads();
    float t = 0.0f;
    for (int w = 0; w < (blockDim.x >> 5); ++w) t += scratch[w];
    __syncthreads();
    return t;
}

// y[b] = x[b] * rsqrt(mean(x[b]^2) + eps) * w, one CTA per row (the order of
// the final products of src/ops.cpp:49-69).
// Rows of up to 8 float4 per thread (aligned, n % 4 == 0) stay in registers:
// one read of x, one write of y; other rows read x twice.
__global__ void RowsRmsNormKernel(const float* x, const float* w, float* y, int n, float eps) {
    __shared__ float scratch[32];
    GridDepWait();
    GridDepLaunch();
    const float* xr = x + size_t(blockIdx.x) * n;
    float* yr = y + size_t(blockIdx.x) * n;
    constexpr int kPer = 8;
    const int n4 = n >> 2;
    if ((n & 3) == 0 && n4 <= kPer * static_cast<int>(blockDim.x) &&
        ((reinterpret_cast<uintptr_t>(xr) | reinterpret_cast<uintptr_t>(yr) | reinterpret_cast<uintptr_t>(w)) & 15) == 0) {
        const float4* x4 = reinterpret_cast<const float4*>(xr);
        const float4* w4 = reinterpret_cast<const float4*>(w);
        float4* y4 = reinterpret_cast<float4*>(yr);
        float4 v[kPer];
        float ss = 0.0f;
#pragma unroll
        for (int k = 0; k < kPer; ++k) {
            const int i = threadIdx.x + k * blockDim.x;
            v[k] = i < n4 ? x4[i] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        }
#pragma unroll
        for (int k = 0; k < kPer; ++k) {
            ss = fmaf(v[k].x, v[k].x, ss);
            ss = fmaf(v[k].y, v[k].y, ss);
            ss = fmaf(v[k].z, v[k].z, ss);
            ss = fmaf(v[k].w, v[k].w, ss);
        }
        ss = RowsBlockSum(ss, scratch);
        const float scale = 1.0f / sqrtf(ss / static_cast<float>(n) + eps);
#pragma unroll
        for (int k = 0; k < kPer; ++k) {
            const int i = threadIdx.x + k * blockDim.x;
            if (i < n4) {
                const float4 wv = w4[i];
                y4[i] = make_float4(v[k].x * scale * wv.x, v[k].y * scale * wv.y, v[k].z * scale * wv.z,
                                    v[k].w * scale * wv.w);
            }
        }
        return;
    }
    float ss = 0.0f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) ss = fmaf(xr[i], xr[i], ss);
    ss = RowsBlockSum(ss, scratch);
    const float scale = 1.0f / sqrtf(ss / static_cast<float>(n) + eps);
    for (int i = threadIdx.x; i < n; i += blockDim.x) yr[i] = xr[i] * scale * w[i];
}

// y = silu(g) * u (SiLU of src/ops.cpp: x / (1 + e^-x)).
__global__ void RowsSwigluKernel(const float* g, const float* u, size_t n, float* y) {
    GridDepWait();
    GridDepLaunch();
    for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < n; i += size_t(gridDim.x) * blockDim.x) {
        const float a = g[i];
        y[i] = a / (1.0f + expf(-a)) * u[i];
    }
}

// y = a + b.
__global__ void RowsAddKernel(const float* a, const float* b, size_t n, float* y) {
    GridDepWait();
    GridDepLaunch();
    for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < n; i += size_t(gridDim.x) * blockDim.x)
        y[i] = a[i] + b[i];
}

// x[i] = table[tokens[i]] for i < rows; an out-of-range token records the
// status and leaves zeros.
__global__ void RowsEmbedKernel(const float* table, int vocab, int dim, const int* tokens, float* x, int* status) {
    GridDepWait();
    GridDepLaunch();
    const int tok = tokens[blockIdx.x];
    const bool ok = tok >= 0 && tok < vocab;
    if (!ok && threadIdx.x == 0) atomicExch(status, MLB_ERR_OUT_OF_RANGE);
    const float* row = table + size_t(ok ? tok : 0) * dim;
    for (int i = threadIdx.x; i < dim; i += blockDim.x) x[size_t(blockIdx.x) * dim + i] = ok ? row[i] : 0.0f;
}

// Token i of a prompt at position start + i: RoPE of its q heads in place and
// of its k heads (reference CPU tables, src/context.cpp:16-25, pair layouts of
// src/ops.cpp:123-168), and k, v into the cache at (layer, position); one CTA
// per token.  positions[i] = start + i for the attention pass.
__global__ void RowsRopeKvKernel(float* q, const float* k, const float* v, int n_heads, int n_kv, int hd, int start,
                                 const float* rope_cos, const float* rope_sin, int neox, float* kc, float* vc,
                                 int layer, int max_seq_len, int* positions) {
    GridDepWait();
    GridDepLaunch();
    const int i = blockIdx.x, pos = start + i, half = hd / 2;
    const float* ct = rope_cos + size_t(pos) * half;
    const float* st = rope_sin + size_t(pos) * half;
    float* qr = q + size_t(i) * n_heads * hd;
    const float* kr = k + size_t(i) * n_kv * hd;
    const float* vr = v + size_t(i) * n_kv * hd;
    const size_t row = (size_t(layer) * max_seq_len + pos) * n_kv * hd;
    for (int t = threadIdx.x; t < (n_heads + n_kv) * half; t += blockDim.x) {
        const int head = t / half, j = t - head * half;
        const int a = neox ? j : 2 * j, b = neox ? j + half : 2 * j + 1;
        const float cs = ct[j], sn = st[j];
        if (head < n_heads) {
            float* base = qr + size_t(head) * hd;
            const float x0 = base[a], x1 = base[b];
            base[a] = __fsub_rn(__fmul_rn(x0, cs), __fmul_rn(x1, sn));
            base[b] = __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, cs));
        } else {
            const int kh = head - n_heads;
            const float* base = kr + size_t(kh) * hd;
            const float x0 = base[a], x1 = base[b];
            kc[row + size_t(kh) * hd + a] = __fsub_rn(__fmul_rn(x0, cs), __fmul_rn(x1, sn));
            kc[row + size_t(kh) * hd + b] = __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, cs));
        }
    }
    for (int t = threadIdx.x; t < n_kv * hd; t += blockDim.x) vc[row + t] = vr[t];
    if (threadIdx.x == 0) positions[i] = pos;
}

inline int RowsGrid(size_t n, int threads, int sms) {
    const size_t g = (n + threads - 1) / threads;
    return static_cast<int>(g < 1 ? 1 : (g > size_t(4) * sms ? size_t(4) * sms : g));
}

}  // namespace
}  // namespace mlb
