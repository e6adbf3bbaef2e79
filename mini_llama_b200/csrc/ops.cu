// Element-wise / normalisation / RoPE / embedding / arg-max / KV-write /
// quantizer / synthetic-input kernels and their C-ABI entry points.
// Replace mini_llama include/cuda_ops.h:11-46 (kernels src/cuda_ops.cu:22-172),
// CudaKVCache::WriteDevice (src/cuda_kv_cache.cpp:157-182) and the host
// quantizers of src/quant.cpp:104-317.
#include <cmath>
#include <vector>

#include "common.cuh"

namespace mlb {

namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ float BlockSum(float v, float* scratch) {
    v = WarpSum(v);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) scratch[warp] = v;
    __syncthreads();
    float t = 0.0f;
    const int nw = blockDim.x >> 5;
    for (int w = 0; w < nw; ++w) t += scratch[w];
    __syncthreads();
    return t;
}

__device__ __forceinline__ float BlockMax(float v, float* scratch) {
    v = WarpMax(v);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) scratch[warp] = v;
    __syncthreads();
    float t = -INFINITY;
    const int nw = blockDim.x >> 5;
    for (int w = 0; w < nw; ++w) t = fmaxf(t, scratch[w]);
    __syncthreads();
    return t;
}

// y = x * rsqrt(mean(x^2) + eps) * w, one CTA (src/ops.cpp:49-69 order of the
// final products).
__global__ void RmsNormKernel(const float* x, const float* w, float* y, int n, float eps) {
    __shared__ float scratch[32];
    float ss = 0.0f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) ss = fmaf(x[i], x[i], ss);
    ss = BlockSum(ss, scratch);
    const float scale = 1.0f / sqrtf(ss / static_cast<float>(n) + eps);
    for (int i = threadIdx.x; i < n; i += blockDim.x) y[i] = x[i] * scale * w[i];
}

struct RopeAngles {
    float c[256];
    float s[256];
};

// In-place rotation of q [n_heads, hd] and k [n_kv_heads, hd]; angles are the
// host-computed table row of the position.
__global__ void RopeKernel(float* q, float* k, int n_heads, int n_kv_heads, int hd, int neox,
                           const RopeAngles ang) {
    const int half = hd / 2;
    const int total = (n_heads + n_kv_heads) * half;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
        int head = i / half, j = i - head * half;
        float* base = head < n_heads ? q + size_t(head) * hd : k + size_t(head - n_heads) * hd;
        int a = neox ? j : 2 * j, b = neox ? j + half : 2 * j + 1;
        float c = ang.c[j], s = ang.s[j];
        float x0 = base[a], x1 = base[b];
        base[a] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
        base[b] = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
    }
}

__global__ void SiluKernel(const float* x, float* y, size_t n) {
    for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < n;
         i += size_t(gridDim.x) * blockDim.x)
        y[i] = x[i] / (1.0f + expf(-x[i]));
}

__global__ void MulKernel(const float* a, const float* b, float* y, size_t n) {
    for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < n;
         i += size_t(gridDim.x) * blockDim.x)
        y[i] = a[i] * b[i];
}

__global__ void AddKernel(const float* a, const float* b, float* y, size_t n) {
    for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < n;
         i += size_t(gridDim.x) * blockDim.x)
        y[i] = a[i] + b[i];
}

__global__ void SoftmaxKernel(const float* x, float* y, int n) {
    __shared__ float scratch[32];
    float mx = -INFINITY;
    for (int i = threadIdx.x; i < n; i += blockDim.x) mx = fmaxf(mx, x[i]);
    mx = BlockMax(mx, scratch);
    float sum = 0.0f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        float e = expf(x[i] - mx);
        y[i] = e;
        sum += e;
    }
    sum = BlockSum(sum, scratch);
    for (int i = threadIdx.x; i < n; i += blockDim.x) y[i] = y[i] / sum;
}

__global__ void EmbeddingKernel(const float* table, int dim, const int* token_dev, int token,
                                float* y) {
    const int t = token_dev ? *token_dev : token;
    const float* row = table + size_t(t) * dim;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < dim; i += gridDim.x * blockDim.x)
        y[i] = row[i];
}

// First maximum (lowest index among equal maxima), one CTA.
__global__ void ArgmaxKernel(const float* x, int n, int* out) {
    __shared__ float sv[1024];
    __shared__ int si[1024];
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        float v = x[i];
        if (v > bv) {
            bv = v;
            bi = i;
        }
    }
    sv[threadIdx.x] = bv;
    si[threadIdx.x] = bi;
    __syncthreads();
    for (int o = blockDim.x / 2; o > 0; o >>= 1) {
        if (threadIdx.x < o) {
            float ov = sv[threadIdx.x + o];
            int oi = si[threadIdx.x + o];
            if (ov > sv[threadIdx.x] || (ov == sv[threadIdx.x] && oi < si[threadIdx.x])) {
                sv[threadIdx.x] = ov;
                si[threadIdx.x] = oi;
            }
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) *out = si[0] == 0x7fffffff ? 0 : si[0];
}

__global__ void KvWriteKernel(float* kc, float* vc, size_t slot, const float* k, const float* v,
                              int n) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        kc[slot + i] = k[i];
        vc[slot + i] = v[i];
    }
}

// ---------------------------------------------------------------- quantizer
// fp16 conversion with the reference's rounding (round half up on bit 12,
// src/quant.cpp:17-52), not the IEEE ties-to-even of __float2half.
__device__ uint16_t F32ToF16Ref(float value) {
    uint32_t bits = __float_as_uint(value);
    uint32_t sign = (bits >> 16) & 0x8000u;
    int exponent = static_cast<int>((bits >> 23) & 0xffu) - 127 + 15;
    uint32_t mantissa = bits & 0x7fffffu;
    if (exponent <= 0) {
        if (exponent < -10) return static_cast<uint16_t>(sign);
        mantissa |= 0x800000u;
        uint32_t shifted = mantissa >> (1 - exponent);
        if (shifted & 0x1000u) shifted += 0x2000u;
        return static_cast<uint16_t>(sign | (shifted >> 13));
    }
    if (exponent >= 31) return static_cast<uint16_t>(sign | 0x7c00u);
    if (mantissa & 0x1000u) {
        mantissa += 0x2000u;
        if (mantissa & 0x800000u) {
            mantissa = 0;
            if (++exponent >= 31) return static_cast<uint16_t>(sign | 0x7c00u);
        }
    }
    return static_cast<uint16_t>(sign | (static_cast<uint32_t>(exponent) << 10) | (mantissa >> 13));
}

// One thread per 32-element block; every fp32 operation is an explicitly
// rounded intrinsic so no FMA contraction changes the reference's rounding.
__global__ void QuantizeKernel(int qtype, const float* x, int rows, int cols, uint8_t* out) {
    const int nb = (cols + 31) / 32;
    const long long total = 1LL * rows * nb;
    for (long long idx = blockIdx.x * 1LL * blockDim.x + threadIdx.x; idx < total;
         idx += 1LL * gridDim.x * blockDim.x) {
        const int r = static_cast<int>(idx / nb), b = static_cast<int>(idx % nb);
        const int begin = b * 32;
        const int len = min(32, cols - begin);
        const float* src = x + size_t(r) * cols + begin;
        if (qtype == MLB_Q8_0) {
            uint8_t* o = out + idx * 34;
            float mx = 0.0f;
            for (int i = 0; i < len; ++i) mx = fmaxf(mx, fabsf(src[i]));
            uint16_t d = 0;
            int8_t q[32] = {};
            if (mx > 0.0f) {
                d = F32ToF16Ref(__fdiv_rn(mx, 127.0f));
                float stored = HalfBits(d);
                float inv = stored == 0.0f ? 0.0f : __fdiv_rn(1.0f, stored);
                for (int i = 0; i < len; ++i) {
                    int v = static_cast<int>(roundf(__fmul_rn(src[i], inv)));
                    q[i] = static_cast<int8_t>(v > 127 ? 127 : (v < -127 ? -127 : v));
                }
            }
            o[0] = d & 0xff;
            o[1] = d >> 8;
            for (int i = 0; i < 32; ++i) o[2 + i] = static_cast<uint8_t>(q[i]);
        } else if (qtype == MLB_Q4_0) {
            uint8_t* o = out + idx * 18;
            float mx = 0.0f;
            for (int i = 0; i < len; ++i) mx = fmaxf(mx, fabsf(src[i]));
            uint16_t d = 0;
            uint8_t qs[16] = {};
            if (mx > 0.0f) {
                d = F32ToF16Ref(__fdiv_rn(mx, 7.0f));
                float stored = HalfBits(d);
                float inv = stored == 0.0f ? 0.0f : __fdiv_rn(1.0f, stored);
                for (int i = 0; i < 16; ++i) {
                    float x0 = i < len ? __fmul_rn(src[i], inv) : 0.0f;
                    float x1 = i + 16 < len ? __fmul_rn(src[i + 16], inv) : 0.0f;
                    int q0 = static_cast<int>(roundf(__fadd_rn(x0, 8.0f)));
                    int q1 = static_cast<int>(roundf(__fadd_rn(x1, 8.0f)));
                    q0 = q0 < 0 ? 0 : (q0 > 15 ? 15 : q0);
                    q1 = q1 < 0 ? 0 : (q1 > 15 ? 15 : q1);
                    qs[i] = static_cast<uint8_t>((q1 << 4) | q0);
                }
            }
            o[0] = d & 0xff;
            o[1] = d >> 8;
            for (int i = 0; i < 16; ++i) o[2 + i] = qs[i];
        } else {  // MLB_Q4_1, rule of test/gpu_core_test.cpp:156-198
            uint8_t* o = out + idx * 20;
            float mn = INFINITY, mx = -INFINITY;
            for (int i = 0; i < len; ++i) {
                mn = fminf(mn, src[i]);
                mx = fmaxf(mx, src[i]);
            }
            float range = __fsub_rn(mx, mn);
            uint16_t d = F32ToF16Ref(range > 0.0f ? __fdiv_rn(range, 15.0f) : 0.0f);
            uint16_t m = F32ToF16Ref(isfinite(mn) ? mn : 0.0f);
            float df = HalfBits(d), mf = HalfBits(m);
            o[0] = d & 0xff;
            o[1] = d >> 8;
            o[2] = m & 0xff;
            o[3] = m >> 8;
            for (int i = 0; i < 16; ++i) {
                int q0 = (i < len && df != 0.0f)
                             ? static_cast<int>(roundf(__fdiv_rn(__fsub_rn(src[i], mf), df)))
                             : 0;
                int q1 = (i + 16 < len && df != 0.0f)
                             ? static_cast<int>(roundf(__fdiv_rn(__fsub_rn(src[i + 16], mf), df)))
                             : 0;
                q0 = q0 < 0 ? 0 : (q0 > 15 ? 15 : q0);
                q1 = q1 < 0 ? 0 : (q1 > 15 ? 15 : q1);
                o[4 + i] = static_cast<uint8_t>(q0 | (q1 << 4));
            }
        }
    }
}

// Exact dequantization (src/quant.cpp:153-317): w = d*q, Q4_1 w = d*q + m.
__global__ void DequantizeKernel(int qtype, const uint8_t* blocks, int rows, int cols, float* y) {
    const int nb = (cols + 31) / 32;
    const int bb = qtype == MLB_Q8_0 ? 34 : (qtype == MLB_Q4_0 ? 18 : 20);
    const long long total = 1LL * rows * cols;
    for (long long i = blockIdx.x * 1LL * blockDim.x + threadIdx.x; i < total;
         i += 1LL * gridDim.x * blockDim.x) {
        const int r = static_cast<int>(i / cols), k = static_cast<int>(i % cols);
        const uint8_t* blk = blocks + (size_t(r) * nb + k / 32) * bb;
        const int e = k & 31;
        float d = HalfBits(static_cast<uint16_t>(blk[0] | (blk[1] << 8)));
        float v;
        if (qtype == MLB_Q8_0) {
            v = __fmul_rn(d, static_cast<float>(static_cast<int8_t>(blk[2 + e])));
        } else {
            const int off = qtype == MLB_Q4_0 ? 2 : 4;
            int q = e < 16 ? (blk[off + e] & 15) : (blk[off + e - 16] >> 4);
            if (qtype == MLB_Q4_0) {
                v = __fmul_rn(d, static_cast<float>(q - 8));
            } else {
                float m = HalfBits(static_cast<uint16_t>(blk[2] | (blk[3] << 8)));
                v = __fadd_rn(__fmul_rn(d, static_cast<float>(q)), m);
            }
        }
        y[i] = v;
    }
}

// ---------------------------------------------------------------- synthetic inputs
__device__ __forceinline__ uint64_t Mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    return z ^ (z >> 31);
}

__global__ void SynthNormalKernel(float* out, size_t n, uint64_t key, double sigma) {
    constexpr uint64_t kGamma = 0x9E3779B97F4A7C15ULL;
    for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < n;
         i += size_t(gridDim.x) * blockDim.x) {
        uint64_t s = 0;
#pragma unroll
        for (uint64_t j = 0; j < 6; ++j) {
            uint64_t r = Mix64(key + (i * 6ULL + j + 1ULL) * kGamma);
            s += (r & 0xFFFFFFFFULL) + (r >> 32);
        }
        double z = __dadd_rn(__dmul_rn(static_cast<double>(s), 1.0 / 4294967296.0), -6.0);
        out[i] = __double2float_rn(__dmul_rn(z, sigma));
    }
}

int GridFor(size_t n, int threads, int sm_count) {
    size_t blocks = (n + threads - 1) / threads;
    size_t cap = size_t(sm_count) * 8;
    return static_cast<int>(blocks < 1 ? 1 : (blocks > cap ? cap : blocks));
}

}  // namespace

uint64_t SynthKey(uint64_t seed, uint64_t stream) {
    // same derivation as the host generator
    uint64_t z = seed * 0x9E3779B97F4A7C15ULL + stream * 0xD1B54A32D192ED03ULL + 1ULL;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    return z ^ (z >> 31);
}

void LaunchSynthNormal(DeviceContext& c, float* out, size_t n, uint64_t seed, uint64_t stream,
                       double sigma) {
    SynthNormalKernel<<<GridFor(n, kThreads, c.sm_count), kThreads, 0, c.stream>>>(
        out, n, SynthKey(seed, stream), sigma);
    CheckCuda(cudaGetLastError(), "SynthNormalKernel");
}

void LaunchQuantize(DeviceContext& c, int qtype, const float* x, int rows, int cols, void* out) {
    const size_t blocks = size_t(rows) * ((cols + 31) / 32);
    QuantizeKernel<<<GridFor(blocks, kThreads, c.sm_count), kThreads, 0, c.stream>>>(
        qtype, x, rows, cols, static_cast<uint8_t*>(out));
    CheckCuda(cudaGetLastError(), "QuantizeKernel");
}

// Host rotation angles of one position, with the reference CPU table formula
// (src/context.cpp:16-25); glibc powf/cosf/sinf as the reference uses.
void RopeAnglesHost(int pos, int head_dim, float theta, float* c, float* s) {
    const int half = head_dim / 2;
    for (int i = 0; i < half; ++i) {
        float freq = 1.0f / std::pow(theta, static_cast<float>(2 * i) / static_cast<float>(head_dim));
        c[i] = std::cos(static_cast<float>(pos) * freq);
        s[i] = std::sin(static_cast<float>(pos) * freq);
    }
}

}  // namespace mlb

using namespace mlb;

extern "C" {

int mlb_rmsnorm(int device, const float* x, const float* weight, int n, float eps, float* y) {
    return Guard([&] {
        const char* c = "CudaRmsNormDeviceWeight";
        Require(x && weight && y, c, "weight is empty");
        Require(n > 0, c, "tensor is empty");
        Require(std::isfinite(eps) && eps > 0.0f, c, "eps must be positive and finite");
        DeviceContext& ctx = Ctx(device);
        RmsNormKernel<<<1, 1024, 0, ctx.stream>>>(x, weight, y, n, eps);
        CheckCuda(cudaGetLastError(), "RmsNormKernel");
    });
}

int mlb_rope(int device, float* q, float* k, int n_heads, int n_kv_heads, int head_dim, int pos,
             float theta, int rope_type) {
    return Guard([&] {
        const char* c = "CudaRopeDeviceInput";
        Require(q && k, c, "input tensor is null");
        Require(n_heads > 0 && n_kv_heads > 0 && head_dim > 0 && head_dim % 2 == 0, c,
                "head shape is invalid");
        Require(head_dim <= 512, c, "head_dim above 512 is not supported", MLB_ERR_UNSUPPORTED);
        Require(pos >= 0, c, "pos must be positive", MLB_ERR_OUT_OF_RANGE);
        Require(std::isfinite(theta) && theta > 0.0f, c, "theta must be positive");
        DeviceContext& ctx = Ctx(device);
        RopeAngles ang;
        RopeAnglesHost(pos, head_dim, theta, ang.c, ang.s);
        const int total = (n_heads + n_kv_heads) * (head_dim / 2);
        RopeKernel<<<GridFor(total, kThreads, ctx.sm_count), kThreads, 0, ctx.stream>>>(
            q, k, n_heads, n_kv_heads, head_dim, rope_type == MLB_ROPE_NEOX ? 1 : 0, ang);
        CheckCuda(cudaGetLastError(), "RopeKernel");
    });
}

int mlb_silu(int device, const float* x, size_t n, float* y) {
    return Guard([&] {
        Require(x && y, "CudaSiluDeviceInput", "tensor is null");
        if (n == 0) return;
        DeviceContext& ctx = Ctx(device);
        SiluKernel<<<GridFor(n, kThreads, ctx.sm_count), kThreads, 0, ctx.stream>>>(x, y, n);
        CheckCuda(cudaGetLastError(), "SiluKernel");
    });
}

int mlb_mul(int device, const float* a, const float* b, size_t n, float* y) {
    return Guard([&] {
        Require(a && b && y, "CudaElementMutmulDeviceInput", "tensor is null");
        if (n == 0) return;
        DeviceContext& ctx = Ctx(device);
        MulKernel<<<GridFor(n, kThreads, ctx.sm_count), kThreads, 0, ctx.stream>>>(a, b, y, n);
        CheckCuda(cudaGetLastError(), "MulKernel");
    });
}

int mlb_add(int device, const float* a, const float* b, size_t n, float* y) {
    return Guard([&] {
        Require(a && b && y, "CudaElementAddDeviceInput", "tensor is null");
        if (n == 0) return;
        DeviceContext& ctx = Ctx(device);
        AddKernel<<<GridFor(n, kThreads, ctx.sm_count), kThreads, 0, ctx.stream>>>(a, b, y, n);
        CheckCuda(cudaGetLastError(), "AddKernel");
    });
}

int mlb_softmax(int device, const float* x, int n, float* y) {
    return Guard([&] {
        Require(x && y, "CudaSoftmax", "tensor is null");
        Require(n > 0, "CudaSoftmax", "tensor is empty");
        DeviceContext& ctx = Ctx(device);
        SoftmaxKernel<<<1, 1024, 0, ctx.stream>>>(x, y, n);
        CheckCuda(cudaGetLastError(), "SoftmaxKernel");
    });
}

int mlb_embedding(int device, const float* table, int vocab_size, int dim, int token, float* y) {
    return Guard([&] {
        const char* c = "CudaEmbeddingDevcieWeightInput";
        Require(table != nullptr && y != nullptr, c, "embedding is empty");
        Require(vocab_size > 0 && dim > 0, c, "embedding shape must be positive");
        Require(token >= 0 && token < vocab_size, c, "token is out of range");
        DeviceContext& ctx = Ctx(device);
        EmbeddingKernel<<<GridFor(dim, kThreads, ctx.sm_count), kThreads, 0, ctx.stream>>>(
            table, dim, nullptr, token, y);
        CheckCuda(cudaGetLastError(), "EmbeddingKernel");
    });
}

int mlb_argmax(int device, const float* x, int n, int* out_index) {
    return Guard([&] {
        Require(x && out_index, "GetArgMax", "tensor is null");
        Require(n > 0, "GetArgMax", "tensor is empty");
        DeviceContext& ctx = Ctx(device);
        ArgmaxKernel<<<1, 1024, 0, ctx.stream>>>(x, n, out_index);
        CheckCuda(cudaGetLastError(), "ArgmaxKernel");
    });
}

int mlb_kv_write(int device, float* key_cache, float* value_cache, int n_layers, int max_seq_len,
                 int n_kv_heads, int head_dim, int layer, int pos, const float* k, const float* v) {
    return Guard([&] {
        const char* c = "CudaKvCache";
        Require(key_cache && value_cache && k && v, c, "cache is empty");
        Require(n_layers > 0 && max_seq_len > 0 && n_kv_heads > 0 && head_dim > 0, c,
                "cache shape must be positive");
        Require(layer >= 0 && layer < n_layers, c, "layer out of range", MLB_ERR_OUT_OF_RANGE);
        Require(pos >= 0 && pos < max_seq_len, c, "position out of range", MLB_ERR_OUT_OF_RANGE);
        DeviceContext& ctx = Ctx(device);
        const int n = n_kv_heads * head_dim;
        const size_t slot = (size_t(layer) * max_seq_len + pos) * n;
        KvWriteKernel<<<GridFor(n, kThreads, ctx.sm_count), kThreads, 0, ctx.stream>>>(
            key_cache, value_cache, slot, k, v, n);
        CheckCuda(cudaGetLastError(), "KvWriteKernel");
    });
}

int mlb_quantize(int device, int qtype, const float* x, int rows, int cols, void* blocks) {
    return Guard([&] {
        Require(qtype == MLB_Q8_0 || qtype == MLB_Q4_0 || qtype == MLB_Q4_1, "mlb_quantize",
                "unsupported block type");
        Require(x && blocks, "mlb_quantize", "tensor is null");
        Require(rows > 0 && cols > 0, "mlb_quantize", "dimension must be positive");
        LaunchQuantize(Ctx(device), qtype, x, rows, cols, blocks);
    });
}

int mlb_dequantize(int device, int qtype, const void* blocks, int rows, int cols, float* y) {
    return Guard([&] {
        Require(qtype == MLB_Q8_0 || qtype == MLB_Q4_0 || qtype == MLB_Q4_1, "mlb_dequantize",
                "unsupported block type");
        Require(blocks && y, "mlb_dequantize", "tensor is null");
        Require(rows > 0 && cols > 0, "mlb_dequantize", "dimension must be positive");
        DeviceContext& ctx = Ctx(device);
        const size_t n = size_t(rows) * cols;
        DequantizeKernel<<<GridFor(n, kThreads, ctx.sm_count), kThreads, 0, ctx.stream>>>(
            qtype, static_cast<const uint8_t*>(blocks), rows, cols, y);
        CheckCuda(cudaGetLastError(), "DequantizeKernel");
    });
}

int mlb_synth_normal(int device, float* out, size_t n, uint64_t seed, uint64_t stream,
                     double sigma) {
    return Guard([&] {
        Require(out != nullptr, "mlb_synth_normal", "output is null");
        if (n == 0) return;
        LaunchSynthNormal(Ctx(device), out, n, seed, stream, sigma);
    });
}

}  // extern "C"
