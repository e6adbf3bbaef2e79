// include/cuda_kv_cache.h over the C ABI (replaces src/cuda_kv_cache.cpp):
// WriteDevice is one kernel instead of two synchronous D2D copies, Clear a
// memset instead of uploading a host tensor of zeros.
#include "include/cuda_kv_cache.h"

#include <limits>

#include "adapter_common.h"

namespace mini_llama {
using adapter::Check;

namespace {
void CheckPositive(int value, const char* what) {
    if (value <= 0) throw std::runtime_error("Cuda kv_cache: " + std::string(what) + "must be positive");
}
}  // namespace

bool CheckCudaKVCacheBuilt() { return true; }

CudaKVCache::CudaKVCache(int n_layers, int max_seq_len, int n_kv_heads, int head_dim, int device_id) {
    Reset(n_layers, max_seq_len, n_kv_heads, head_dim, device_id);
}

void CudaKVCache::Clear() {
    if (Empty()) return;
    Check(mlb_memset(device_id_, keys_.GetData(), 0, keys_.GetBytes()));
    Check(mlb_memset(device_id_, values_.GetData(), 0, values_.GetBytes()));
}

void CudaKVCache::Reset() {
    keys_.Reset();
    values_.Reset();
    n_layers_ = max_seq_len_ = n_kv_heads_ = head_dim_ = device_id_ = 0;
}

void CudaKVCache::Reset(int n_layers, int max_seq_len, int n_kv_heads, int head_dim, int device_id) {
    CheckPositive(n_layers, "n_layers");
    CheckPositive(max_seq_len, "max_seq_len");
    CheckPositive(n_kv_heads, "n_kv_heads");
    CheckPositive(head_dim, "head_dim");
    n_layers_ = n_layers;
    max_seq_len_ = max_seq_len;
    n_kv_heads_ = n_kv_heads;
    head_dim_ = head_dim;
    device_id_ = device_id;
    keys_.Reset({n_layers, max_seq_len, n_kv_heads, head_dim}, device_id);
    values_.Reset({n_layers, max_seq_len, n_kv_heads, head_dim}, device_id);
    Clear();
}

void CudaKVCache::ValidateIndices(int layer, int pos) const {
    if (Empty()) throw std::runtime_error("CudaKvCache: cache is empty");
    if (layer < 0 || layer >= n_layers_) throw std::out_of_range("CudaKvCache layer out of range");
    if (pos < 0 || pos >= max_seq_len_) throw std::out_of_range("CudaKvCache position out of range");
}

void CudaKVCache::ValidateHeadIndex(int kv_head) const {
    if (kv_head < 0 || kv_head >= n_kv_heads_) throw std::out_of_range("CudaKvCache head out of range");
}

void CudaKVCache::ValidateWriteTensors(const Tensor& k, const Tensor& v) const {
    if (k.DimNum() != 2 || v.DimNum() != 2 || k.shape != v.shape)
        throw std::out_of_range("CudaKvCache::Write expected matching [n_kv_heads, head_dim] tensors");
    if (k.shape[0] != n_kv_heads_ || k.shape[1] != head_dim_)
        throw std::out_of_range("CudaKvCache::Write tensor shape does not match cache shape");
}

size_t CudaKVCache::SlotOffsetBytes(int layer, int pos) const {
    return ((static_cast<size_t>(layer) * max_seq_len_ + pos) * n_kv_heads_ * head_dim_) * sizeof(float);
}

size_t CudaKVCache::HeadOffsetBytes(int layer, int pos, int kv_head) const {
    return SlotOffsetBytes(layer, pos) + static_cast<size_t>(kv_head) * head_dim_ * sizeof(float);
}

void CudaKVCache::Write(int layer, int pos, const Tensor& k, const Tensor& v) {
    ValidateIndices(layer, pos);
    ValidateWriteTensors(k, v);
    const size_t off = SlotOffsetBytes(layer, pos);
    const size_t bytes = k.Size() * sizeof(float);
    Check(mlb_memcpy_h2d(device_id_, static_cast<char*>(keys_.GetData()) + off, k.data.data(), bytes));
    Check(mlb_memcpy_h2d(device_id_, static_cast<char*>(values_.GetData()) + off, v.data.data(), bytes));
}

void CudaKVCache::WriteDevice(int layer, int pos, const CudaTensor& k, const CudaTensor& v) {
    ValidateIndices(layer, pos);
    if (k.GetDeviceId() != device_id_ || v.GetDeviceId() != device_id_)
        throw std::runtime_error("Cuda kv_cache: tensor is not on same device");
    const size_t expected = static_cast<size_t>(n_kv_heads_) * head_dim_;
    if (k.GetSize() != expected || v.GetSize() != expected)
        throw std::out_of_range("Cuda kv_cache: tensor shape is not match");
    Check(mlb_kv_write(device_id_, static_cast<float*>(keys_.GetData()),
                       static_cast<float*>(values_.GetData()), n_layers_, max_seq_len_, n_kv_heads_,
                       head_dim_, layer, pos, static_cast<const float*>(k.GetData()),
                       static_cast<const float*>(v.GetData())));
}

namespace {
Tensor ReadSlot(const CudaTensor& t, int device, size_t off, std::vector<int> shape) {
    Tensor dst(shape, 0.0f);
    Check(mlb_memcpy_d2h(device, dst.data.data(), static_cast<const char*>(t.GetData()) + off,
                         dst.Size() * sizeof(float)));
    return dst;
}
}  // namespace

Tensor CudaKVCache::ReadKey(int layer, int pos) const {
    ValidateIndices(layer, pos);
    return ReadSlot(keys_, device_id_, SlotOffsetBytes(layer, pos), {n_kv_heads_, head_dim_});
}

Tensor CudaKVCache::ReadValue(int layer, int pos) const {
    ValidateIndices(layer, pos);
    return ReadSlot(values_, device_id_, SlotOffsetBytes(layer, pos), {n_kv_heads_, head_dim_});
}

Tensor CudaKVCache::ReadKeyHead(int layer, int pos, int kv_head) const {
    ValidateIndices(layer, pos);
    ValidateHeadIndex(kv_head);
    return ReadSlot(keys_, device_id_, HeadOffsetBytes(layer, pos, kv_head), {head_dim_});
}

Tensor CudaKVCache::ReadValueHead(int layer, int pos, int kv_head) const {
    ValidateIndices(layer, pos);
    ValidateHeadIndex(kv_head);
    return ReadSlot(values_, device_id_, HeadOffsetBytes(layer, pos, kv_head), {head_dim_});
}

}  // namespace mini_llama
