// include/cuda_tensor.h over the C ABI (replaces src/cuda_tensor.cpp).
//
// A CudaTensor is an fp32 shape plus one CudaDeviceBuffer from the library
// pool.  The class layout is fixed by the reference header; the error texts
// are part of its interface (callers match on them), so they are kept.
#include "include/cuda_tensor.h"

#include <sstream>

#include "adapter_common.h"

namespace mini_llama {
namespace {

// Elements of a shape (0 for the empty shape); every extent must be positive
// and the product must fit in size_t.
size_t ShapeElements(const std::vector<int>& shape) {
    size_t n = shape.empty() ? 0 : 1;
    for (const int extent : shape) {
        if (extent <= 0) throw std::runtime_error("CudaTensor Reset: shape is must positive");
        if (__builtin_mul_overflow(n, static_cast<size_t>(extent), &n))
            throw std::runtime_error("CudaTensor Reset: shape size is over limit");
    }
    return n;
}

}  // namespace

std::string CudaTensor::ShapeString() const {
    std::ostringstream os;
    os << '[';
    const char* sep = "";
    for (const int extent : shape_) {
        os << sep << extent;
        sep = ",";
    }
    os << ']';
    return os.str();
}

CudaTensor::CudaTensor(const std::vector<int>& shape, int device_id) : element_num_(0), device_id_(device_id) {
    Reset(shape, device_id);
}

void CudaTensor::Reset(const std::vector<int>& shape, int device_id) {
    // validate and allocate before touching the members, so a failure leaves
    // the tensor as it was
    const size_t n = ShapeElements(shape);
    buffer_.Reset(n * sizeof(float), device_id);
    shape_ = shape;
    element_num_ = n;
    device_id_ = device_id;
}

void CudaTensor::Reset() {
    buffer_.Reset();
    shape_ = {};
    element_num_ = 0;
    device_id_ = 0;
}

void CudaTensor::Upload(const Tensor& src) {
    if (shape_ != src.shape) throw std::runtime_error("CudaTensor Upload: shape is not match.");
    buffer_.Upload(src.data.data(), element_num_ * sizeof(float));
}

void CudaTensor::DownloadTo(Tensor& dst) const {
    if (dst.shape != shape_)
        throw std::runtime_error("CUDA DownloadTo: CudaTensor shape is not match dst shape");
    buffer_.Download(dst.data.data(), element_num_ * sizeof(float));
}

Tensor CudaTensor::Download() const {
    Tensor host;
    if (!shape_.empty()) {
        host = Tensor(shape_, 0.0f);
        DownloadTo(host);
    }
    return host;
}

CudaTensor CudaTensorFromHost(const Tensor& src, int device_id) {
    CudaTensor t(src.shape, device_id);
    t.Upload(src);
    return t;
}

}  // namespace mini_llama
