// include/cuda_tensor.h over the C ABI (replaces src/cuda_tensor.cpp).
#include "include/cuda_tensor.h"

#include <limits>

#include "adapter_common.h"

namespace mini_llama {
namespace {
size_t ElementCount(const std::vector<int>& shape, const char* caller) {
    if (shape.empty()) return 0;
    size_t total = 1;
    for (int dim : shape) {
        if (dim <= 0) throw std::runtime_error(std::string(caller) + ": shape is must positive");
        if (total > std::numeric_limits<size_t>::max() / static_cast<size_t>(dim))
            throw std::runtime_error(std::string(caller) + ": shape size is over limit");
        total *= static_cast<size_t>(dim);
    }
    return total;
}
}  // namespace

std::string CudaTensor::ShapeString() const {
    std::string out = "[";
    for (size_t i = 0; i < shape_.size(); ++i) {
        if (i) out += ',';
        out += std::to_string(shape_[i]);
    }
    return out + ']';
}

CudaTensor::CudaTensor(const std::vector<int>& shape, int device_id)
    : shape_(shape), element_num_(0), device_id_(device_id) {
    Reset(shape, device_id);
}

void CudaTensor::Reset(const std::vector<int>& shape, int device_id) {
    element_num_ = ElementCount(shape, "CudaTensor Reset");
    shape_ = shape;
    device_id_ = device_id;
    buffer_.Reset(element_num_ * sizeof(float), device_id_);
}

void CudaTensor::Reset() {
    shape_.clear();
    device_id_ = 0;
    element_num_ = 0;
    buffer_.Reset();
}

void CudaTensor::Upload(const Tensor& src) {
    if (src.shape != shape_) throw std::runtime_error("CudaTensor Upload: shape is not match.");
    buffer_.Upload(src.data.data(), src.Size() * sizeof(float));
}

void CudaTensor::DownloadTo(Tensor& dst) const {
    if (shape_ != dst.shape)
        throw std::runtime_error("CUDA DownloadTo: CudaTensor shape is not match dst shape");
    buffer_.Download(dst.data.data(), dst.Size() * sizeof(float));
}

Tensor CudaTensor::Download() const {
    if (shape_.empty()) return Tensor();
    Tensor dst(shape_, 0.0f);
    DownloadTo(dst);
    return dst;
}

CudaTensor CudaTensorFromHost(const Tensor& src, int device_id) {
    CudaTensor dst(src.shape, device_id);
    dst.Upload(src);
    return dst;
}

}  // namespace mini_llama
