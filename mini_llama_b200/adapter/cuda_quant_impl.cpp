// include/cuda_quant.h over the C ABI (replaces src/cuda_quant.cu and
// src/cuda_quant.cpp).  Validation and messages follow the reference
// (src/cuda_quant.cu:148-210); the kernels are mlb_q80/q40/q41_linear.
#include "include/cuda_quant.h"

#include "adapter_common.h"

namespace mini_llama {
using adapter::Check;

namespace {

struct LinearShape {
    int rows, in, out;
    bool one_d;
};

LinearShape Validate(const std::vector<int>& x_shape, const std::string& x_str,
                     const std::vector<int>& w_shape, size_t blocks, const char* caller) {
    if (w_shape.size() != 2)
        throw std::runtime_error(std::string(caller) + ": expected weight shape [out_features, in_features]");
    LinearShape s{1, 0, 0, x_shape.size() == 1};
    if (x_shape.size() == 1) s.in = x_shape[0];
    else if (x_shape.size() == 2) {
        s.rows = x_shape[0];
        s.in = x_shape[1];
    } else {
        throw std::runtime_error(std::string(caller) +
                                 ": expected x shape [in_features] or [batch, in_features], got " + x_str);
    }
    if (s.in <= 0 || w_shape[0] <= 0 || w_shape[1] <= 0)
        throw std::runtime_error(std::string(caller) + ": empty tensors are not supported");
    if (w_shape[1] != s.in)
        throw std::runtime_error(std::string(caller) + ": dimension mismatch x=" + x_str + " weight=[" +
                                 std::to_string(w_shape[0]) + ", " + std::to_string(w_shape[1]) + "]");
    s.out = w_shape[0];
    const size_t expected = static_cast<size_t>(s.out) * ((s.in + 31) / 32);
    if (blocks != expected)
        throw std::runtime_error(std::string(caller) + ": block count mismatch: expected " +
                                 std::to_string(expected) + ", got " + std::to_string(blocks));
    return s;
}

void AddBias(Tensor& y, const Tensor& bias, int rows, int cols, const char* caller) {
    if (bias.DimNum() != 1 || bias.shape[0] != cols)
        throw std::runtime_error(std::string(caller) + ": expected bias shape [out_features]");
    for (int r = 0; r < rows; ++r)
        for (int c = 0; c < cols; ++c) y.data[static_cast<size_t>(r) * cols + c] += bias.data[c];
}

// host x, device weights
Tensor LinearHostX(int qtype, const Tensor& x, const void* w, size_t blocks,
                   const std::vector<int>& w_shape, const Tensor* bias, int dev, const char* caller) {
    if (w == nullptr) throw std::runtime_error(std::string(caller) + ": device weight pointer is null");
    LinearShape s = Validate(x.shape, x.ShapeString(), w_shape, blocks, caller);
    Tensor y(s.one_d ? std::vector<int>{s.out} : std::vector<int>{s.rows, s.out}, 0.0f);
    CudaDeviceBuffer x_dev(x.Size() * sizeof(float), dev);
    CudaDeviceBuffer y_dev(y.Size() * sizeof(float), dev);
    x_dev.Upload(x.data.data(), x.Size() * sizeof(float));
    Check(mlb_quant_linear(dev, qtype, static_cast<const float*>(x_dev.GetData()), w, blocks, s.rows,
                           s.in, s.out, nullptr, static_cast<float*>(y_dev.GetData())));
    y_dev.Download(y.data.data(), y.Size() * sizeof(float));
    if (bias != nullptr) AddBias(y, *bias, s.rows, s.out, caller);
    return y;
}

// device x, device weights
CudaTensor LinearDeviceX(int qtype, const CudaTensor& x, const void* w, size_t blocks,
                         const std::vector<int>& w_shape, int dev, const char* caller) {
    if (w == nullptr) throw std::runtime_error(std::string(caller) + ": device weight pointer is null");
    if (x.GetDeviceId() != dev)
        throw std::runtime_error(std::string(caller) + ": input tensor is on a different CUDA device");
    LinearShape s = Validate(x.Shape(), x.ShapeString(), w_shape, blocks, caller);
    CudaTensor y(s.one_d ? std::vector<int>{s.out} : std::vector<int>{s.rows, s.out}, dev);
    Check(mlb_quant_linear(dev, qtype, static_cast<const float*>(x.GetData()), w, blocks, s.rows, s.in,
                           s.out, nullptr, static_cast<float*>(y.GetData())));
    return y;
}

template <typename Block>
Tensor LinearHostW(int qtype, const Tensor& x, const std::vector<Block>& w,
                   const std::vector<int>& w_shape, const Tensor* bias, int dev, const char* caller) {
    Validate(x.shape, x.ShapeString(), w_shape, w.size(), caller);
    CudaDeviceBuffer w_dev(w.size() * sizeof(Block), dev);
    w_dev.Upload(w.data(), w.size() * sizeof(Block));
    return LinearHostX(qtype, x, w_dev.GetData(), w.size(), w_shape, bias, dev, caller);
}

}  // namespace

bool CheckCudaQuantBuilt() { return true; }

Tensor CudaQ80Linear(const Tensor& x, const std::vector<BlockQ80>& w, const std::vector<int>& shape,
                     const Tensor* bias, int dev) {
    return LinearHostW(MLB_Q8_0, x, w, shape, bias, dev, "CudaQ80Linear");
}
Tensor CudaQ80LinearDeviceWeight(const Tensor& x, const void* w, size_t blocks,
                                 const std::vector<int>& shape, const Tensor* bias, int dev) {
    return LinearHostX(MLB_Q8_0, x, w, blocks, shape, bias, dev, "CudaQ80LinearDevicePointer");
}
CudaTensor CudaQ80LinearDeviceInput(const CudaTensor& x, const void* w, size_t blocks,
                                    const std::vector<int>& shape, int dev) {
    return LinearDeviceX(MLB_Q8_0, x, w, blocks, shape, dev, "CudaQ80LinearDevicePointer");
}

Tensor CudaQ40Linear(const Tensor& x, const std::vector<BlockQ40>& w, const std::vector<int>& shape,
                     const Tensor* bias, int dev) {
    return LinearHostW(MLB_Q4_0, x, w, shape, bias, dev, "CudaQ40Linear");
}
Tensor CudaQ40LinearDeviceWeight(const Tensor& x, const void* w, size_t blocks,
                                 const std::vector<int>& shape, const Tensor* bias, int dev) {
    return LinearHostX(MLB_Q4_0, x, w, blocks, shape, bias, dev, "CudaQ40Linear");
}
CudaTensor CudaQ40LinearDeviceInput(const CudaTensor& x, const void* w, size_t blocks,
                                    const std::vector<int>& shape, int dev) {
    return LinearDeviceX(MLB_Q4_0, x, w, blocks, shape, dev, "CudaQ40Linear");
}

Tensor CudaQ41Linear(const Tensor& x, const std::vector<BlockQ41>& w, const std::vector<int>& shape,
                     const Tensor* bias, int dev) {
    return LinearHostW(MLB_Q4_1, x, w, shape, bias, dev, "CudaQ41Linear");
}
Tensor CudaQ41LinearDeviceWeight(const Tensor& x, const void* w, size_t blocks,
                                 const std::vector<int>& shape, const Tensor* bias, int dev) {
    return LinearHostX(MLB_Q4_1, x, w, blocks, shape, bias, dev, "CudaQ41Linear");
}
CudaTensor CudaQ41LinearDeviceInput(const CudaTensor& x, const void* w, size_t blocks,
                                    const std::vector<int>& shape, int dev) {
    return LinearDeviceX(MLB_Q4_1, x, w, blocks, shape, dev, "CudaQ41Linear");
}

}  // namespace mini_llama
