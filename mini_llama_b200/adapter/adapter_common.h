// Shared helpers of the adapter: the C++17 implementation of mini_llama's CUDA
// headers (include/cuda_data.h, cuda_tensor.h, cuda_kv_cache.h, cuda_quant.h,
// cuda_attention.h, cuda_ops.h, cuda_matmul.h) over the mini_llama_b200 C ABI
// (include/mlb.h).  Compiled against the reference's own headers, so
// mini_llama's forward.cpp, model.cpp, loaders and sampler link unchanged.
#pragma once

#include <stdexcept>
#include <string>
#include <vector>

#include "mlb.h"

namespace mini_llama {
namespace adapter {

// Maps a C-ABI status to the exception type the reference throws.
inline void Check(int status) {
    if (status == MLB_OK) return;
    const std::string msg = mlb_last_error();
    if (status == MLB_ERR_OUT_OF_RANGE) throw std::out_of_range(msg);
    throw std::runtime_error(msg);
}

// Device selected by the last CudaSetDevice of this thread.
int& CurrentDevice();

inline size_t Product(const std::vector<int>& shape) {
    size_t n = 1;
    for (int s : shape) n *= static_cast<size_t>(s);
    return n;
}

}  // namespace adapter
}  // namespace mini_llama
