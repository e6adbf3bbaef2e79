// include/cuda_matmul.h over the C ABI (replaces the cuBLAS path of
// src/cuda_matmul.cpp: no library handle, the library's own F32 kernels).
#include "include/cuda_matmul.h"

#include "adapter_common.h"

namespace mini_llama {
using adapter::Check;

namespace {
void ValidateLinear(const std::vector<int>& x_shape, const std::vector<int>& w_shape, const char* c,
                    int& rows, int& in) {
    if (w_shape.size() != 2)
        throw std::runtime_error(std::string(c) + ": expect w shape is [out_feature, in_feature]");
    if (x_shape.size() == 1) {
        rows = 1;
        in = x_shape[0];
    } else if (x_shape.size() == 2) {
        rows = x_shape[0];
        in = x_shape[1];
    } else {
        throw std::runtime_error(std::string(c) + "expect x shape [in_feature] or [batch, in_feature]");
    }
    if (w_shape[1] != in)
        throw std::runtime_error(std::string(c) + "x is not match w, x in_feature is " +
                                 std::to_string(in) + "w infeature is " + std::to_string(w_shape[1]));
}
}  // namespace

bool CheckCudaMatmulBuilt() { return true; }

Tensor CudaMatmul(const Tensor& a, const Tensor& b, int dev) {
    if (a.DimNum() != 2 || b.DimNum() != 2) throw std::runtime_error("CudaMatmul: tensor must be 2D");
    if (a.shape[1] != b.shape[0]) throw std::runtime_error("CudaMatmul: tensor must be match");
    CudaTensor ad = CudaTensorFromHost(a, dev), bd = CudaTensorFromHost(b, dev);
    CudaTensor cd({a.shape[0], b.shape[1]}, dev);
    Check(mlb_f32_matmul(dev, static_cast<const float*>(ad.GetData()),
                         static_cast<const float*>(bd.GetData()), a.shape[0], a.shape[1], b.shape[1],
                         static_cast<float*>(cd.GetData())));
    return cd.Download();
}

Tensor CudaLinearDeviceWeight(const Tensor& x, const void* w, const std::vector<int>& w_shape,
                              const Tensor* bias, int dev) {
    const char* c = "CudaLinearWithDeviceWeight";
    if (w == nullptr) throw std::runtime_error(std::string(c) + ": device weight is null");
    int rows = 0, in = 0;
    ValidateLinear(x.shape, w_shape, c, rows, in);
    const int out = w_shape[0];
    if (bias != nullptr && (bias->DimNum() != 1 || bias->shape[0] != out))
        throw std::runtime_error("CudaLinear: expect bias shape [out_feature]");
    CudaTensor xd = CudaTensorFromHost(x, dev);
    CudaTensor bd;
    if (bias != nullptr) bd = CudaTensorFromHost(*bias, dev);
    CudaTensor yd(x.DimNum() == 1 ? std::vector<int>{out} : std::vector<int>{rows, out}, dev);
    Check(mlb_f32_linear(dev, static_cast<const float*>(xd.GetData()), static_cast<const float*>(w),
                         rows, in, out, bias ? static_cast<const float*>(bd.GetData()) : nullptr,
                         static_cast<float*>(yd.GetData())));
    return yd.Download();
}

Tensor CudaLinear(const Tensor& x, const Tensor& weight, const Tensor* bias, int dev) {
    if (weight.DimNum() != 2)
        throw std::runtime_error("CudaLinear: weight expect shape [out_feature, in_feature]");
    CudaTensor wd = CudaTensorFromHost(weight, dev);
    return CudaLinearDeviceWeight(x, wd.GetData(), weight.shape, bias, dev);
}

CudaTensor CudaLinearDeviceInput(const CudaTensor& x, const void* w, const std::vector<int>& w_shape,
                                 int dev) {
    const char* c = "CudaLinearDeviceInput";
    if (w == nullptr) throw std::runtime_error(std::string(c) + ": device weight is null");
    if (x.GetDeviceId() != dev) throw std::runtime_error(std::string(c) + ": input is on another device");
    int rows = 0, in = 0;
    ValidateLinear(x.Shape(), w_shape, c, rows, in);
    const int out = w_shape[0];
    CudaTensor y(x.GetDimNum() == 1 ? std::vector<int>{out} : std::vector<int>{rows, out}, dev);
    Check(mlb_f32_linear(dev, static_cast<const float*>(x.GetData()), static_cast<const float*>(w), rows,
                         in, out, nullptr, static_cast<float*>(y.GetData())));
    return y;
}

}  // namespace mini_llama
