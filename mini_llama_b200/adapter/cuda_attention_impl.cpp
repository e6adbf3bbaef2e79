// include/cuda_attention.h over the C ABI (replaces src/cuda_attention.cu:184-251).
#include "include/cuda_attention.h"

#include "adapter_common.h"

namespace mini_llama {
using adapter::Check;

namespace {
void ValidateCommon(const CudaKVCache& kv, int layer, int pos, int n_heads, int n_kv_heads,
                    int head_dim, const char* caller) {
    if (kv.Empty()) throw std::runtime_error(std::string(caller) + ": CUDA KV cache is empty");
    if (layer < 0 || layer >= kv.GetNLayers())
        throw std::out_of_range(std::string(caller) + ": layer out of range");
    if (pos < 0 || pos >= kv.GetMaxSeqLen())
        throw std::out_of_range(std::string(caller) + ": position out of range");
    if (n_heads <= 0 || n_kv_heads <= 0 || head_dim <= 0)
        throw std::runtime_error(std::string(caller) + ": head counts and head_dim must be positive");
    if (n_heads % n_kv_heads != 0)
        throw std::runtime_error(std::string(caller) + ": n_heads must be divisible by n_kv_heads");
}
}  // namespace

bool CheckCudaAttentionBuilt() { return true; }

Tensor CudaAttentionDecode(const Tensor& q, const CudaKVCache& kv, int layer, int pos, int max_seq_len,
                           int n_heads, int n_kv_heads, int head_dim, int dev) {
    const char* c = "CudaAttentionDecode";
    if (q.shape != std::vector<int>{n_heads, head_dim})
        throw std::runtime_error(std::string(c) + ": expected q shape [" + std::to_string(n_heads) +
                                 ", " + std::to_string(head_dim) + "], got " + q.ShapeString());
    ValidateCommon(kv, layer, pos, n_heads, n_kv_heads, head_dim, c);
    if (kv.GetNKVHeads() != n_kv_heads || kv.GetHeadDim() != head_dim)
        throw std::runtime_error(std::string(c) + ": KV cache shape does not match attention shape");
    CudaTensor q_dev = CudaTensorFromHost(q, dev);
    CudaTensor out({n_heads, head_dim}, dev);
    Check(mlb_attention_decode(dev, static_cast<const float*>(q_dev.GetData()),
                               static_cast<const float*>(kv.GetKeyData()),
                               static_cast<const float*>(kv.GetValueData()), kv.GetNLayers(),
                               max_seq_len, layer, pos, n_heads, n_kv_heads, head_dim,
                               static_cast<float*>(out.GetData())));
    return out.Download();
}

CudaTensor CudaAttentionDecodeDeviceInputs(const CudaTensor& q, const CudaKVCache& kv, int layer,
                                           int pos, int max_seq_len, int n_heads, int n_kv_heads,
                                           int head_dim, int dev) {
    const char* c = "CudaAttentionDecodeDeviceInput";
    if (q.GetDeviceId() != dev)
        throw std::runtime_error(std::string(c) + ": q tensor is on a different CUDA device");
    if (q.GetSize() != static_cast<size_t>(n_heads) * head_dim)
        throw std::runtime_error(std::string(c) + ": q shape mismatch");
    ValidateCommon(kv, layer, pos, n_heads, n_kv_heads, head_dim, c);
    if (kv.GetNKVHeads() != n_kv_heads || kv.GetHeadDim() != head_dim || kv.GetDeviceId() != dev)
        throw std::runtime_error(std::string(c) +
                                 ": KV cache shape or device does not match attention shape");
    CudaTensor out({n_heads * head_dim}, dev);
    Check(mlb_attention_decode(dev, static_cast<const float*>(q.GetData()),
                               static_cast<const float*>(kv.GetKeyData()),
                               static_cast<const float*>(kv.GetValueData()), kv.GetNLayers(),
                               max_seq_len, layer, pos, n_heads, n_kv_heads, head_dim,
                               static_cast<float*>(out.GetData())));
    return out;
}

}  // namespace mini_llama
