// include/cuda_ops.h over the C ABI (replaces src/cuda_ops.cu:310-554).
#include "include/cuda_ops.h"

#include <cmath>

#include "adapter_common.h"

namespace mini_llama {
using adapter::Check;

namespace {
const float* F(const CudaTensor& t) { return static_cast<const float*>(t.GetData()); }
float* F(CudaTensor& t) { return static_cast<float*>(t.GetData()); }

void SameShape(const CudaTensor& a, const CudaTensor& b, const char* c) {
    if (a.Shape() != b.Shape())
        throw std::runtime_error(std::string(c) + ": shape is not match form " + a.ShapeString() +
                                 " to " + b.ShapeString());
    if (a.GetDeviceId() != b.GetDeviceId())
        throw std::runtime_error(std::string(c) + "tensor is on differen cuda devices");
}

void Check1D(const std::vector<int>& shape, size_t n, const char* c) {
    if (shape.size() != 1) throw std::runtime_error(std::string(c) + ": tensor shape is not 1D");
    if (n == 0) throw std::runtime_error(std::string(c) + ": tensor is empty");
}

void CheckEps(float eps, const char* c) {
    if (!std::isfinite(eps) || eps <= 0.0f)
        throw std::runtime_error(std::string(c) + ": eps must be positive and finite");
}

// Host helper: y = op(a, b) with both uploaded, downloaded after.
template <typename Op>
Tensor Host2(const Tensor& a, const Tensor& b, int dev, Op op) {
    CudaTensor ad = CudaTensorFromHost(a, dev), bd = CudaTensorFromHost(b, dev);
    CudaTensor yd(a.shape, dev);
    op(ad, bd, yd);
    return yd.Download();
}
}  // namespace

bool CheckCudaOpsBuild() { return true; }

Tensor CudaElementMutmul(const Tensor& a, const Tensor& b, int dev) {
    if (a.shape != b.shape) throw std::runtime_error("CudaElementMutmul: shape is not match");
    return Host2(a, b, dev, [&](CudaTensor& x, CudaTensor& y, CudaTensor& o) {
        Check(mlb_mul(dev, F(x), F(y), x.GetSize(), F(o)));
    });
}

CudaTensor CudaElementMutmulDeviceInput(const CudaTensor& a, const CudaTensor& b, int dev) {
    SameShape(a, b, "CudaElementMutmulDeviceInput");
    if (a.GetDeviceId() != dev)
        throw std::runtime_error("CudaElementMutmulDeviceInput: two tensor is not on this device");
    CudaTensor y(a.Shape(), dev);
    Check(mlb_mul(dev, F(a), F(b), a.GetSize(), F(y)));
    return y;
}

Tensor CudaElementAdd(const Tensor& a, const Tensor& b, int dev) {
    if (a.shape != b.shape) throw std::runtime_error("CudaElementAdd: shape is not match");
    return Host2(a, b, dev, [&](CudaTensor& x, CudaTensor& y, CudaTensor& o) {
        Check(mlb_add(dev, F(x), F(y), x.GetSize(), F(o)));
    });
}

CudaTensor CudaElementAddDeviceInput(const CudaTensor& a, const CudaTensor& b, int dev) {
    SameShape(a, b, "CudaElementAddDeviceInput");
    if (a.GetDeviceId() != dev)
        throw std::runtime_error("CudaElementAddDeviceInput: two tensor is not on this device");
    CudaTensor y(a.Shape(), dev);
    Check(mlb_add(dev, F(a), F(b), a.GetSize(), F(y)));
    return y;
}

CudaTensor CudaElementAddDeviceWeight(const CudaTensor& a, const void* b_data,
                                      const std::vector<int>& b_shape, int dev) {
    if (a.GetDeviceId() != dev)
        throw std::runtime_error("CudaAddDeviceWeightInput: current tensor is not on this device");
    if (b_data == nullptr) throw std::runtime_error("CudaAddDeviceWeightInput: data is empty");
    if (a.Shape() != b_shape)
        throw std::runtime_error("CudaAddDeviceWeightInput: input and weight is not match");
    CudaTensor y(a.Shape(), dev);
    Check(mlb_add(dev, F(a), static_cast<const float*>(b_data), a.GetSize(), F(y)));
    return y;
}

Tensor CudaSilu(const Tensor& x, int dev) {
    CudaTensor xd = CudaTensorFromHost(x, dev);
    CudaTensor yd(x.shape, dev);
    Check(mlb_silu(dev, F(xd), xd.GetSize(), F(yd)));
    return yd.Download();
}

CudaTensor CudaSiluDeviceInput(const CudaTensor& x, int dev) {
    if (x.GetDeviceId() != dev)
        throw std::runtime_error("CudaSiluDeviceInput: this tensor device is not this device");
    CudaTensor y(x.Shape(), dev);
    Check(mlb_silu(dev, F(x), x.GetSize(), F(y)));
    return y;
}

Tensor CudaSoftmax(const Tensor& x, int dev) {
    Check1D(x.shape, x.Size(), "CudaSoftmax");
    CudaTensor xd = CudaTensorFromHost(x, dev);
    CudaTensor yd(x.shape, dev);
    Check(mlb_softmax(dev, F(xd), static_cast<int>(x.Size()), F(yd)));
    return yd.Download();
}

Tensor CudaRmsNorm(const Tensor& x, const Tensor& weight, float eps, int dev) {
    Check1D(x.shape, x.Size(), "CudaRmsNorm");
    Check1D(weight.shape, weight.Size(), "CudaRmsNorm");
    if (x.shape != weight.shape) throw std::runtime_error("CudaRmsNorm: x and weight shape is not match");
    CheckEps(eps, "CudaRmsNorm");
    CudaTensor xd = CudaTensorFromHost(x, dev), wd = CudaTensorFromHost(weight, dev);
    CudaTensor yd(x.shape, dev);
    Check(mlb_rmsnorm(dev, F(xd), F(wd), static_cast<int>(x.Size()), eps, F(yd)));
    return yd.Download();
}

CudaTensor CudaRmsNormDeviceInput(const CudaTensor& x, const Tensor& weight, float eps, int dev) {
    CudaTensor wd = CudaTensorFromHost(weight, dev);
    return CudaRmsNormDeviceWeight(x, wd.GetData(), weight.shape, eps, dev);
}

CudaTensor CudaRmsNormDeviceWeight(const CudaTensor& x, const void* weight,
                                   const std::vector<int>& weight_shape, float eps, int dev) {
    const char* c = "CudaRmsNormDeviceWeightInput";
    Check1D(x.Shape(), x.GetSize(), c);
    if (weight == nullptr) throw std::runtime_error(std::string(c) + ": weight is empty");
    if (x.Shape() != weight_shape) throw std::runtime_error(std::string(c) + ": shape is not match");
    if (x.GetDeviceId() != dev)
        throw std::runtime_error(std::string(c) + ": current tensor is not on this device");
    CheckEps(eps, c);
    CudaTensor y(x.Shape(), dev);
    Check(mlb_rmsnorm(dev, F(x), static_cast<const float*>(weight), static_cast<int>(x.GetSize()), eps,
                      F(y)));
    return y;
}

void CudaRope(Tensor& q, Tensor& k, int pos, float theta, RopeType type, int dev) {
    if (q.DimNum() != 2 || k.DimNum() != 2) throw std::runtime_error("CudaRope: tensor is not 2D");
    if (pos < 0) throw std::out_of_range("CudaRope: pos must be positive");
    if (!std::isfinite(theta) || theta <= 0.0f)
        throw std::runtime_error("CudaRope: theta must be finite and positive");
    if (q.shape[1] != k.shape[1]) throw std::runtime_error("CudaRope: q and k head_dim is not match");
    if (q.shape[1] <= 0 || q.shape[1] % 2 != 0)
        throw std::runtime_error("CudaRope: head_dim must be even and positive");
    CudaTensor qd = CudaTensorFromHost(q, dev), kd = CudaTensorFromHost(k, dev);
    Check(mlb_rope(dev, F(qd), F(kd), q.shape[0], k.shape[0], q.shape[1], pos, theta,
                   type == RopeType::kNeoX ? MLB_ROPE_NEOX : MLB_ROPE_NORMAL));
    qd.DownloadTo(q);
    kd.DownloadTo(k);
}

void CudaRopeDeviceInput(CudaTensor& q, CudaTensor& k, int n_heads, int n_kv_heads, int head_dim,
                         int pos, float theta, RopeType type, int dev) {
    const char* c = "CudaRopeDeviceInput";
    if (q.GetDeviceId() != dev || k.GetDeviceId() != dev)
        throw std::runtime_error(std::string(c) + ": input tensor is not on this CUDA device");
    if (n_heads <= 0 || n_kv_heads <= 0 || head_dim <= 0 || head_dim % 2 != 0)
        throw std::runtime_error(std::string(c) + ": head shape is invalid");
    if (q.GetSize() != static_cast<size_t>(n_heads) * head_dim)
        throw std::runtime_error(std::string(c) + ": q shape is not match");
    if (k.GetSize() != static_cast<size_t>(n_kv_heads) * head_dim)
        throw std::runtime_error(std::string(c) + ": k shape is not match");
    if (pos < 0) throw std::out_of_range(std::string(c) + ": pos must be positive");
    if (!std::isfinite(theta) || theta <= 0.0f)
        throw std::runtime_error(std::string(c) + ": theta must be positive");
    Check(mlb_rope(dev, F(q), F(k), n_heads, n_kv_heads, head_dim, pos, theta,
                   type == RopeType::kNeoX ? MLB_ROPE_NEOX : MLB_ROPE_NORMAL));
}

CudaTensor CudaEmbedding(const void* table, const std::vector<int>& shape, int token, int dev) {
    const char* c = "CudaEmbeddingDevcieWeightInput";
    if (table == nullptr) throw std::runtime_error(std::string(c) + ": embedding is empty");
    if (shape.size() != 2) throw std::runtime_error(std::string(c) + ": shape must be 2D");
    if (shape[0] <= 0 || shape[1] <= 0)
        throw std::runtime_error(std::string(c) + ": embedding shape must be positive");
    if (token < 0 || token >= shape[0]) throw std::runtime_error(std::string(c) + ": token is out of range");
    CudaTensor y({shape[1]}, dev);
    Check(mlb_embedding(dev, static_cast<const float*>(table), shape[0], shape[1], token, F(y)));
    return y;
}

}  // namespace mini_llama
