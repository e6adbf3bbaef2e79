// include/cuda_data.h over the C ABI: device queries, the pooled
// stream-ordered allocator and copies.  Replaces src/cuda_data.cpp (a
// cudaMalloc/cudaFree per buffer and synchronous cudaMemcpy).
#include "include/cuda_data.h"

#include <sstream>

#include "adapter_common.h"

namespace mini_llama {
namespace adapter {
int& CurrentDevice() {
    thread_local int device = 0;
    return device;
}
}  // namespace adapter

using adapter::Check;

bool CheckCudaRuntimeBuilt() { return true; }

int GetCudaDeviceCount() {
    int n = 0;
    Check(mlb_device_count(&n));
    return n;
}

void CudaSetDevice(int device_id) {
    Check(mlb_set_device(device_id));
    adapter::CurrentDevice() = device_id;
}

CudaDeviceInfo GetCudaDeviceInfo(int device_id) {
    int count = GetCudaDeviceCount();
    if (device_id < 0 || device_id >= count) {
        throw std::runtime_error("CUDA device: " + std::to_string(device_id) + "is not available");
    }
    mlb_device_info d;
    Check(mlb_get_device_info(device_id, &d));
    CudaDeviceInfo info;
    info.id = device_id;
    info.name = d.name;
    info.compute_major = d.compute_major;
    info.compute_minor = d.compute_minor;
    info.total_memory_bytes = d.total_memory_bytes;
    info.driver_version = d.driver_version;
    info.runtime_version = d.runtime_version;
    return info;
}

std::string CudaFormatDeviceInfo(const CudaDeviceInfo& info) {
    std::ostringstream oss;
    oss << "device " << info.id << ": " << info.name << ", compute capability "
        << info.compute_major << '.' << info.compute_minor << ", total memory "
        << static_cast<double>(info.total_memory_bytes) / (1024.0 * 1024.0 * 1024.0) << "GB"
        << ", cuda runtime toolkit version" << info.runtime_version
        << ", cuda driver version" << info.driver_version;
    return oss.str();
}

void* CudaMallocBytes(size_t bytes) {
    if (bytes == 0) return nullptr;
    void* p = nullptr;
    Check(mlb_malloc(adapter::CurrentDevice(), bytes, &p));
    return p;
}

void CudaFreeBytes(void* ptr) {
    if (ptr == nullptr) return;
    Check(mlb_free(adapter::CurrentDevice(), ptr));
}

void CudaMemcpyBytes(void* dst, const void* src, size_t bytes, MemcpyKind kind) {
    if (bytes == 0) return;
    if (dst == nullptr || src == nullptr) throw std::runtime_error("cuda memcpy dst or src is nullptr");
    const int dev = adapter::CurrentDevice();
    switch (kind) {
        case MemcpyKind::kHostToDevice: Check(mlb_memcpy_h2d(dev, dst, src, bytes)); return;
        case MemcpyKind::kDeviceToHost: Check(mlb_memcpy_d2h(dev, dst, src, bytes)); return;
        case MemcpyKind::kDeviceToDevice: Check(mlb_memcpy_d2d(dev, dst, src, bytes)); return;
    }
    throw std::runtime_error("unknow CUDA memcpy kind");
}

CudaDeviceBuffer::CudaDeviceBuffer(size_t bytes, int device_id) { Reset(bytes, device_id); }

CudaDeviceBuffer::~CudaDeviceBuffer() { ReleaseNoexcept(); }

CudaDeviceBuffer::CudaDeviceBuffer(CudaDeviceBuffer&& other) noexcept
    : data_(other.data_), bytes_(other.bytes_), device_id_(other.device_id_) {
    other.data_ = nullptr;
    other.bytes_ = 0;
    other.device_id_ = 0;
}

CudaDeviceBuffer& CudaDeviceBuffer::operator=(CudaDeviceBuffer&& other) noexcept {
    if (this == &other) return *this;
    ReleaseNoexcept();
    data_ = other.data_;
    bytes_ = other.bytes_;
    device_id_ = other.device_id_;
    other.data_ = nullptr;
    other.bytes_ = 0;
    other.device_id_ = 0;
    return *this;
}

void CudaDeviceBuffer::Reset() {
    if (data_ == nullptr) return;
    Check(mlb_free(device_id_, data_));  // stream-ordered: pending kernels finish first
    data_ = nullptr;
    bytes_ = 0;
    device_id_ = 0;
}

void CudaDeviceBuffer::Reset(size_t bytes, int device_id) {
    Reset();
    device_id_ = device_id;
    if (bytes == 0) return;
    Check(mlb_malloc(device_id, bytes, &data_));
    bytes_ = bytes;
}

void CudaDeviceBuffer::Upload(const void* src, size_t bytes) {
    if (bytes > bytes_) throw std::runtime_error("CUDA upload: CUDA must more size");
    if (bytes == 0) return;
    if (src == nullptr || data_ == nullptr) throw std::runtime_error("cuda memcpy dst or src is nullptr");
    Check(mlb_memcpy_h2d(device_id_, data_, src, bytes));
}

void CudaDeviceBuffer::Download(void* dst, size_t bytes) const {
    if (bytes > bytes_) throw std::runtime_error("CUDA download: need size is too more");
    if (bytes == 0) return;
    if (dst == nullptr || data_ == nullptr) throw std::runtime_error("cuda memcpy dst or src is nullptr");
    Check(mlb_memcpy_d2h(device_id_, dst, data_, bytes));
}

void CudaDeviceBuffer::ReleaseNoexcept() noexcept {
    try {
        Reset();
    } catch (...) {
    }
}

}  // namespace mini_llama
