// Library-level C entry points (version and status-code text) and the per-device host
// caches the launchers share.
#include <atomic>
#include <map>
#include <mutex>
#include <utility>

#include "asu_common.cuh"

namespace {

constexpr int kMaxDevices = 64;
std::atomic<int> g_sm_count[kMaxDevices];  // 0: not queried yet
std::mutex g_smem_mu;
std::map<std::pair<int, const void*>, int> g_smem_limit;  // (device, kernel) -> max dynamic smem

int current_device(int* dev) {
    const cudaError_t e = cudaGetDevice(dev);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return ASU_ERR_CUDA_BASE + static_cast<int>(e);
    }
    return (*dev >= 0 && *dev < kMaxDevices) ? ASU_OK : ASU_ERR_ARG;
}

}  // namespace

int asu_sm_count() {
    int dev = 0;
    if (current_device(&dev) != ASU_OK) return 1;
    int n = g_sm_count[dev].load(std::memory_order_relaxed);
    if (n > 0) return n;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) {
        cudaGetLastError();
        return 1;
    }
    g_sm_count[dev].store(n, std::memory_order_relaxed);
    return n;
}

int asu_max_dynamic_smem(const void* kernel, int* max_dynamic) {
    int dev = 0;
    int rc = current_device(&dev);
    if (rc != ASU_OK) return rc;
    std::lock_guard<std::mutex> lock(g_smem_mu);
    const auto key = std::make_pair(dev, kernel);
    const auto it = g_smem_limit.find(key);
    if (it != g_smem_limit.end()) {
        *max_dynamic = it->second;
        return ASU_OK;
    }
    int optin = 0;
    cudaFuncAttributes fa;
    cudaError_t e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&fa, kernel);
    int limit = 0;
    if (e == cudaSuccess) {
        limit = optin - static_cast<int>(fa.sharedSizeBytes);
        e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, limit);
    }
    if (e != cudaSuccess) {
        cudaGetLastError();  // leave no error behind for the caller's runtime checks
        return ASU_ERR_CUDA_BASE + static_cast<int>(e);
    }
    g_smem_limit.emplace(key, limit);
    *max_dynamic = limit;
    return ASU_OK;
}

extern "C" int asu_version(void) { return 10000; /* 1.0.0 */ }

extern "C" const char* asu_status_string(int code) {
    switch (code) {
        case ASU_OK: return "ok";
        case ASU_ERR_ARG: return "invalid argument (null pointer or size out of range)";
        case ASU_ERR_ALIGN: return "pointer or row size not 16-byte aligned";
        case ASU_ERR_NOALLOC_CAPACITY:
            return "topk_numel exceeds the fixed scratch of asu_kv_resolver_noalloc (ASU_RESOLVER_NOALLOC_MAX_TOPK)";
        default: break;
    }
    if (code >= ASU_ERR_CUDA_BASE) return cudaGetErrorString(static_cast<cudaError_t>(code - ASU_ERR_CUDA_BASE));
    return "unknown status";
}
