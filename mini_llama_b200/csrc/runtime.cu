// Device runtime: per-device contexts (library stream, stream-ordered memory
// pool, kernel workspace), error reporting and the memory entry points of the
// C ABI.  Replaces the synchronous cudaMalloc/cudaMemcpy/cudaFree runtime of
// mini_llama src/cuda_data.cpp:50-151.
#include <cstring>
#include <mutex>
#include <vector>

#include "common.cuh"

namespace mlb {

namespace {
thread_local std::string g_last_error;
std::mutex g_ctx_mutex;
std::vector<DeviceContext*> g_ctx;
// The op kernels' device status words: part of the library image (every
// device that loads the library holds its own copy, zero at load), so setting
// up a device allocates no device memory.  Word 0 is the status the op
// kernels set and mlb_synchronize reads.
__device__ __align__(256) int g_status_words[64];
}  // namespace

void SetLastError(const std::string& msg) { g_last_error = msg; }
void ClearLastError() { g_last_error.clear(); }

DeviceContext& Ctx(int device) {
    std::lock_guard<std::mutex> lock(g_ctx_mutex);
    int count = 0;
    CheckCuda(cudaGetDeviceCount(&count), "cudaGetDeviceCount");
    if (device < 0 || device >= count) {
        Fail(MLB_ERR_INVALID_ARGUMENT, "CUDA device " + std::to_string(device) +
                                           " is not available (" + std::to_string(count) +
                                           " visible)");
    }
    if (g_ctx.size() < static_cast<size_t>(count)) g_ctx.resize(count, nullptr);
    CheckCuda(cudaSetDevice(device), "cudaSetDevice");
    if (g_ctx[device] == nullptr) {
        auto* c = new DeviceContext();
        c->device = device;
        CheckCuda(cudaDeviceGetAttribute(&c->sm_count, cudaDevAttrMultiProcessorCount, device),
                  "cudaDeviceGetAttribute(SM count)");
        CheckCuda(cudaDeviceGetAttribute(&c->max_smem_optin,
                                         cudaDevAttrMaxSharedMemoryPerBlockOptin, device),
                  "cudaDeviceGetAttribute(smem)");
        CheckCuda(cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking),
                  "cudaStreamCreate");
        cudaMemPoolProps props = {};
        props.allocType = cudaMemAllocationTypePinned;
        props.location.type = cudaMemLocationTypeDevice;
        props.location.id = device;
        CheckCuda(cudaMemPoolCreate(&c->pool, &props), "cudaMemPoolCreate");
        uint64_t keep = UINT64_MAX;  // never hand freed blocks back to the driver
        CheckCuda(cudaMemPoolSetAttribute(c->pool, cudaMemPoolAttrReleaseThreshold, &keep),
                  "cudaMemPoolSetAttribute");
        void* st = nullptr;  // this device's copy of g_status_words (the device is current)
        CheckCuda(cudaGetSymbolAddress(&st, g_status_words), "cudaGetSymbolAddress(status)");
        c->status = static_cast<int*>(st);
        g_ctx[device] = c;
    }
    return *g_ctx[device];
}

PFN_cuTensorMapEncodeTiled_v12000 TensorMapEncoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 encode = [] {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault, &q) !=
                cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            fn = nullptr;
        return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }();
    return encode;
}

void* Workspace(DeviceContext& ctx, size_t bytes) {
    if (bytes <= ctx.workspace_bytes) return ctx.workspace;
    if (ctx.workspace) CheckCuda(cudaFreeAsync(ctx.workspace, ctx.stream), "cudaFreeAsync");
    size_t want = bytes < (1u << 20) ? (1u << 20) : bytes;
    CheckCuda(cudaMallocFromPoolAsync(&ctx.workspace, want, ctx.pool, ctx.stream),
              "cudaMallocFromPoolAsync(workspace)");
    ctx.workspace_bytes = want;
    return ctx.workspace;
}

void* PinnedStaging(DeviceContext& ctx, size_t bytes) {
    if (bytes <= ctx.pinned_bytes) return ctx.pinned;
    if (ctx.pinned) {
        CheckCuda(cudaStreamSynchronize(ctx.stream), "cudaStreamSynchronize");
        CheckCuda(cudaFreeHost(ctx.pinned), "cudaFreeHost");
    }
    size_t want = bytes < 4096 ? 4096 : bytes;
    CheckCuda(cudaMallocHost(&ctx.pinned, want), "cudaMallocHost");
    ctx.pinned_bytes = want;
    return ctx.pinned;
}

}  // namespace mlb

using namespace mlb;

extern "C" {

const char* mlb_last_error(void) { return g_last_error.c_str(); }

int mlb_abi_version(void) { return MLB_ABI_VERSION; }

int mlb_device_count(int* count) {
    return Guard([&] {
        Require(count != nullptr, "mlb_device_count", "count is null");
        int n = 0;
        cudaError_t err = cudaGetDeviceCount(&n);
        if (err == cudaErrorNoDevice || err == cudaErrorInsufficientDriver) {
            cudaGetLastError();
            n = 0;
        } else {
            CheckCuda(err, "cudaGetDeviceCount");
        }
        *count = n;
    });
}

int mlb_set_device(int device) { return Guard([&] { Ctx(device); }); }

int mlb_get_device_info(int device, mlb_device_info* info) {
    return Guard([&] {
        Require(info != nullptr, "mlb_get_device_info", "info is null");
        DeviceContext& c = Ctx(device);
        cudaDeviceProp prop = {};
        CheckCuda(cudaGetDeviceProperties(&prop, device), "cudaGetDeviceProperties");
        std::memset(info, 0, sizeof(*info));
        std::strncpy(info->name, prop.name, sizeof(info->name) - 1);
        info->compute_major = prop.major;
        info->compute_minor = prop.minor;
        info->total_memory_bytes = prop.totalGlobalMem;
        info->sm_count = c.sm_count;
        CheckCuda(cudaDriverGetVersion(&info->driver_version), "cudaDriverGetVersion");
        CheckCuda(cudaRuntimeGetVersion(&info->runtime_version), "cudaRuntimeGetVersion");
    });
}

int mlb_get_stream(int device, void** cuda_stream) {
    return Guard([&] {
        Require(cuda_stream != nullptr, "mlb_get_stream", "out pointer is null");
        *cuda_stream = Ctx(device).stream;
    });
}

int mlb_malloc(int device, size_t bytes, void** ptr) {
    return Guard([&] {
        Require(ptr != nullptr, "mlb_malloc", "out pointer is null");
        *ptr = nullptr;
        if (bytes == 0) return;
        DeviceContext& c = Ctx(device);
        CheckCuda(cudaMallocFromPoolAsync(ptr, bytes, c.pool, c.stream), "cudaMallocFromPoolAsync");
    });
}

int mlb_free(int device, void* ptr) {
    return Guard([&] {
        if (ptr == nullptr) return;
        DeviceContext& c = Ctx(device);
        CheckCuda(cudaFreeAsync(ptr, c.stream), "cudaFreeAsync");
    });
}

int mlb_memcpy_h2d(int device, void* dst, const void* src, size_t bytes) {
    return Guard([&] {
        if (bytes == 0) return;
        Require(dst && src, "mlb_memcpy_h2d", "cuda memcpy dst or src is nullptr");
        DeviceContext& c = Ctx(device);
        // Pageable sources are staged by the driver before the copy call
        // returns, so the caller may reuse them at once; pinned (or
        // registered) sources are read asynchronously, so those copies are
        // waited for.
        cudaPointerAttributes attr{};
        const cudaError_t ar = cudaPointerGetAttributes(&attr, src);
        if (ar != cudaSuccess) cudaGetLastError();  // not a pointer CUDA knows: treat it as pinned, and wait
        const bool pageable = ar == cudaSuccess && attr.type == cudaMemoryTypeUnregistered;
        CheckCuda(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, c.stream),
                  "cudaMemcpyAsync(H2D)");
        if (!pageable) CheckCuda(cudaStreamSynchronize(c.stream), "cudaStreamSynchronize(H2D)");
    });
}

int mlb_memcpy_d2h(int device, void* dst, const void* src, size_t bytes) {
    return Guard([&] {
        if (bytes == 0) return;
        Require(dst && src, "mlb_memcpy_d2h", "cuda memcpy dst or src is nullptr");
        DeviceContext& c = Ctx(device);
        CheckCuda(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, c.stream),
                  "cudaMemcpyAsync(D2H)");
        CheckCuda(cudaStreamSynchronize(c.stream), "cudaStreamSynchronize(D2H)");
    });
}

int mlb_memcpy_d2d(int device, void* dst, const void* src, size_t bytes) {
    return Guard([&] {
        if (bytes == 0) return;
        Require(dst && src, "mlb_memcpy_d2d", "cuda memcpy dst or src is nullptr");
        DeviceContext& c = Ctx(device);
        CheckCuda(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, c.stream),
                  "cudaMemcpyAsync(D2D)");
    });
}

int mlb_memset(int device, void* dst, int value, size_t bytes) {
    return Guard([&] {
        if (bytes == 0) return;
        Require(dst != nullptr, "mlb_memset", "dst is null");
        DeviceContext& c = Ctx(device);
        CheckCuda(cudaMemsetAsync(dst, value, bytes, c.stream), "cudaMemsetAsync");
    });
}

int mlb_synchronize(int device) {
    return Guard([&] {
        DeviceContext& c = Ctx(device);
        CheckCuda(cudaStreamSynchronize(c.stream), "cudaStreamSynchronize");
        int st = 0;
        CheckCuda(cudaMemcpy(&st, c.status, sizeof(int), cudaMemcpyDeviceToHost), "cudaMemcpy(status)");
        if (st != 0) {
            CheckCuda(cudaMemset(c.status, 0, sizeof(int)), "cudaMemset(status)");
            Fail(st, "a bounded device wait of an op kernel expired");
        }
    });
}

}  // extern "C"
