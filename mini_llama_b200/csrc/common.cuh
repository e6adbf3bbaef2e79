// Shared device/host helpers of the mini_llama_b200 CUDA library (sm_100a).
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdio>
#include <stdexcept>
#include <string>

#include "../../include/mlb.h"

namespace mlb {

// ---------------------------------------------------------------- errors
// Every C-ABI entry point runs its body inside Guard(): a thrown Error (or any
// std::exception) becomes a status code plus a thread-local message that
// mlb_last_error() returns, so no C++ exception crosses the C boundary.
struct Error : std::runtime_error {
    int status;
    Error(int s, const std::string& m) : std::runtime_error(m), status(s) {}
};

void SetLastError(const std::string& msg);
void ClearLastError();

[[noreturn]] inline void Fail(int status, const std::string& msg) { throw Error(status, msg); }

inline void Require(bool ok, const char* caller, const std::string& msg,
                    int status = MLB_ERR_INVALID_ARGUMENT) {
    if (!ok) Fail(status, std::string(caller) + ": " + msg);
}

inline void CheckCuda(cudaError_t err, const char* caller) {
    if (err != cudaSuccess) {
        Fail(MLB_ERR_CUDA, std::string("CUDA error in ") + caller + ": " + cudaGetErrorString(err));
    }
}

template <typename F>
int Guard(F&& body) {
    try {
        body();
        ClearLastError();
        return MLB_OK;
    } catch (const Error& e) {
        SetLastError(e.what());
        return e.status;
    } catch (const std::exception& e) {
        SetLastError(e.what());
        return MLB_ERR_INVALID_ARGUMENT;
    }
}

// ---------------------------------------------------------------- device context
// One context per device: the library stream (non-blocking, all work of the
// library is ordered on it), a stream-ordered memory pool that keeps freed
// memory for reuse (no cudaFree in steady state), and a grow-only workspace
// for kernel scratch.
struct DeviceContext {
    int device = -1;
    int sm_count = 0;
    int max_smem_optin = 0;
    cudaStream_t stream = nullptr;
    cudaMemPool_t pool = nullptr;
    void* workspace = nullptr;
    size_t workspace_bytes = 0;
    void* pinned = nullptr;  // small pinned staging buffer for host<->device scalars
    size_t pinned_bytes = 0;
    int* status = nullptr;   // device status word of the op kernels with bounded waits
    // the x images the tensor-core linear's pre-pass last wrote (on this
    // context's stream): input, workspace and their shape
    const void* tc_x = nullptr;
    const void* tc_ws = nullptr;
    int tc_m = 0, tc_k = 0, tc_mx = 0, tc_mtiles = 0;
};

DeviceContext& Ctx(int device);                     // creates on first use, makes device current
void* Workspace(DeviceContext& ctx, size_t bytes);  // stream-ordered, grow-only
void* PinnedStaging(DeviceContext& ctx, size_t bytes);

inline size_t CeilDiv(size_t a, size_t b) { return (a + b - 1) / b; }

// The driver's tensor-map encoder, reached through the runtime (the library
// does not link the driver library); null when the driver does not offer it.
PFN_cuTensorMapEncodeTiled_v12000 TensorMapEncoder();

// Kernel launch with programmatic dependent launch enabled, so a kernel
// captured behind another may start its independent prologue (weight
// prefetch) before the previous grid finishes; it calls GridDepWait() before
// touching data the previous grid produced.
template <typename Kernel, typename... Args>
void Launch(const char* name, Kernel kernel, dim3 grid, dim3 block, size_t smem,
            cudaStream_t stream, bool pdl, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    CheckCuda(cudaLaunchKernelEx(&cfg, kernel, args...), name);
}

// ---------------------------------------------------------------- device helpers
__device__ __forceinline__ void GridDepWait() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void GridDepLaunch() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ float HalfBits(uint16_t bits) {
    __half_raw r;
    r.x = bits;
    return __half2float(__half(r));
}

__device__ __forceinline__ float WarpSum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float WarpMax(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// mbarrier + bulk-copy (TMA, non-tensor, no multicast) wrappers.
__device__ __forceinline__ uint32_t SmemAddr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void MbarInit(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(SmemAddr(bar)), "r"(count)
                 : "memory");
}

__device__ __forceinline__ void FenceMbarInit() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void MbarExpectTx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(SmemAddr(bar)),
                 "r"(bytes)
                 : "memory");
}

// Bounded wait on an mbarrier phase.  Returns false when the bound expired
// (the caller records an error status and skips the data).
__device__ __forceinline__ bool MbarWait(uint64_t* bar, uint32_t parity) {
    uint32_t addr = SmemAddr(bar);
    for (uint32_t spin = 0; spin < (1u << 26); ++spin) {
        uint32_t done;
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
            " selp.u32 %0, 1, 0, p;\n}\n"
            : "=r"(done)
            : "r"(addr), "r"(parity)
            : "memory");
        if (done) return true;
    }
    return false;
}

__device__ __forceinline__ uint64_t GlobalTimerNs() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// One test of an mbarrier phase (no wait): true when it has completed.
__device__ __forceinline__ bool MbarTryWait(uint64_t* bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(SmemAddr(bar)), "r"(parity)
        : "memory");
    return done != 0;
}

// Time-bounded wait on an mbarrier phase; also gives up when *abort becomes
// nonzero (a shared flag another warp sets).  Returns false when it gave up.
__device__ __forceinline__ bool MbarWaitFor(uint64_t* bar, uint32_t parity, uint64_t timeout_ns,
                                            const volatile int* abort) {
    const uint32_t addr = SmemAddr(bar);
    // a phase that has already completed costs one test, no timer read
    if (MbarTryWait(bar, parity)) return true;
    const uint64_t t0 = GlobalTimerNs();
    for (uint32_t spin = 0;; ++spin) {
        uint32_t done;
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
            " selp.u32 %0, 1, 0, p;\n}\n"
            : "=r"(done)
            : "r"(addr), "r"(parity)
            : "memory");
        if (done) return true;
        if ((spin & 63) == 63) {
            if (abort && *abort) return false;
            if (GlobalTimerNs() - t0 > timeout_ns) return false;
        }
    }
}

// Global -> shared bulk copy of `bytes` (multiple of 16, both addresses
// 16-byte aligned), completing on `bar`.
__device__ __forceinline__ void BulkLoad(void* smem_dst, const void* gmem_src, uint32_t bytes,
                                         uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
        ::"r"(SmemAddr(smem_dst)), "l"(gmem_src), "r"(bytes), "r"(SmemAddr(bar))
        : "memory");
}

// L2 policy for data read once per pass (streamed weights): evicted first, so
// it does not push out what is reused (KV cache, activations, counters).
__device__ __forceinline__ uint64_t L2EvictFirstPolicy() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}

// BulkLoad with an L2 cache policy (L2EvictFirstPolicy).
__device__ __forceinline__ void BulkLoadHint(void* smem_dst, const void* gmem_src, uint32_t bytes,
                                             uint64_t* bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;"
        ::"r"(SmemAddr(smem_dst)), "l"(gmem_src), "r"(bytes), "r"(SmemAddr(bar)), "l"(policy)
        : "memory");
}

// Asynchronous global -> shared copies (cp.async): every copy of a batch is in
// flight at once, so staging a vector costs one memory round trip.
__device__ __forceinline__ void CpAsync4(void* smem_dst, const void* gmem_src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(SmemAddr(smem_dst)),
                 "l"(gmem_src)
                 : "memory");
}
__device__ __forceinline__ void CpAsync16(void* smem_dst, const void* gmem_src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(SmemAddr(smem_dst)),
                 "l"(gmem_src)
                 : "memory");
}
__device__ __forceinline__ void CpAsyncWaitAll() {
    asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;" ::: "memory");
}

// Block-cooperative staging of n floats into shared memory (no wait).
__device__ __forceinline__ void StageFloats(float* dst, const float* src, int n) {
    const bool vec = ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 15) == 0;
    int done = 0;
    if (vec) {
        const int n4 = n >> 2;
        for (int i = threadIdx.x; i < n4; i += blockDim.x) CpAsync16(dst + 4 * i, src + 4 * i);
        done = n4 << 2;
    }
    for (int i = done + threadIdx.x; i < n; i += blockDim.x) CpAsync4(dst + i, src + i);
}

// L2 prefetch of a global range (bulk, no shared memory involved).
__device__ __forceinline__ void BulkPrefetchL2(const void* gmem_src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(gmem_src), "r"(bytes)
                 : "memory");
}

}  // namespace mlb
