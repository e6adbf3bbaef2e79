// Exposes two helpers of the reference GPU unit test (test/gpu_core_test.cpp)
// to the harness: the Q4_1 quantizer (gpu_core_test.cpp:156-198, the only Q4_1
// quantizer the reference has) and the CPU attention reference
// (gpu_core_test.cpp:221-247).  The test source is compiled from where it lies
// in the reference tree; its main() is renamed so the harness keeps its own.
// TEST INFRASTRUCTURE ONLY.
#define main mini_llama_gpu_core_test_main
#include "test/gpu_core_test.cpp"
#undef main

namespace mini_llama {

std::vector<BlockQ41> HarnessQuantizeQ41(const Tensor& t) { return QuantizeQ41ForTest(t); }

Tensor HarnessAttentionReference(const Tensor& q, const KVCache& cache, int layer, int pos,
                                 int n_heads, int n_kv_heads, int head_dim) {
    return AttentionReference(q, cache, layer, pos, n_heads, n_kv_heads, head_dim);
}

}  // namespace mini_llama
