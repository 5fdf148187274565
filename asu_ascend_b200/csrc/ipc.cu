// Cross-process plumbing of the multi-GPU swap-in balancing (host code only).
//
// A rank whose host link is the slower one hands part of its swap-in to a rank on a faster link.
// The helper reads the owner's host rows through its own link and stores them into the owner's
// HBM slot pool over NVLink, so it needs two mappings in its own CUDA context:
//  * the owner's pinned host pool: a shared-memory mapping (memfd) registered here with
//    cudaHostRegister(mapped), see asu_host_register;
//  * the owner's slot pool: a CUDA IPC mapping of the owner's device allocation, see
//    asu_ipc_export / asu_ipc_open.
// The reference has no counterpart: its swap-in is a per-request MicroKV socket fetch on one NPU
// (docs/v0.1/kv-cache-offload-v0.1-real-ops-design.md:293-312).
#include <cuda.h>

#include <cstring>

#include "asu_common.cuh"

namespace {

int cuda_rc(cudaError_t e) {
    if (e == cudaSuccess) return ASU_OK;
    cudaGetLastError();  // leave no sticky error behind for the caller
    return ASU_ERR_CUDA_BASE + static_cast<int>(e);
}

// cuMemGetAddressRange (v2) through the runtime's driver entry point, so the library does not link
// libcuda itself (it must load on hosts without a driver for its CPU tests).
using AddressRangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);

AddressRangeFn address_range_fn() {
    static AddressRangeFn fn = [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
        if (cudaGetDriverEntryPointByVersion("cuMemGetAddressRange", &p, 12000, cudaEnableDefault, &q) !=
                cudaSuccess ||
            q != cudaDriverEntryPointSuccess) {
            cudaGetLastError();
            p = nullptr;
        }
        return reinterpret_cast<AddressRangeFn>(p);
    }();
    return fn;
}

}  // namespace

extern "C" int asu_host_register(void* host_ptr, uint64_t bytes, void** device_ptr) {
    if (!host_ptr || bytes == 0 || !device_ptr) return ASU_ERR_ARG;
    int rc = cuda_rc(cudaHostRegister(host_ptr, bytes, cudaHostRegisterPortable | cudaHostRegisterMapped));
    if (rc != ASU_OK) return rc;
    void* d = nullptr;
    rc = cuda_rc(cudaHostGetDevicePointer(&d, host_ptr, 0));
    if (rc != ASU_OK) {
        cudaHostUnregister(host_ptr);
        cudaGetLastError();
        return rc;
    }
    *device_ptr = d;
    return ASU_OK;
}

extern "C" int asu_host_unregister(void* host_ptr) {
    if (!host_ptr) return ASU_OK;
    return cuda_rc(cudaHostUnregister(host_ptr));
}

extern "C" int asu_ipc_export(const void* device_ptr, uint8_t* handle, uint64_t* offset) {
    if (!device_ptr || !handle || !offset) return ASU_ERR_ARG;
    const AddressRangeFn range = address_range_fn();
    if (range == nullptr) return ASU_ERR_CUDA_BASE + static_cast<int>(cudaErrorNotSupported);
    CUdeviceptr base = 0;
    size_t size = 0;
    if (range(&base, &size, reinterpret_cast<CUdeviceptr>(device_ptr)) != CUDA_SUCCESS)
        return ASU_ERR_CUDA_BASE + static_cast<int>(cudaErrorInvalidValue);
    cudaIpcMemHandle_t h;
    const int rc = cuda_rc(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)));
    if (rc != ASU_OK) return rc;
    std::memcpy(handle, &h, sizeof(h));
    *offset = reinterpret_cast<uint64_t>(device_ptr) - static_cast<uint64_t>(base);
    return ASU_OK;
}

extern "C" int asu_ipc_open(const uint8_t* handle, void** base_ptr) {
    if (!handle || !base_ptr) return ASU_ERR_ARG;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    void* p = nullptr;
    const int rc = cuda_rc(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
    if (rc != ASU_OK) return rc;
    *base_ptr = p;
    return ASU_OK;
}

extern "C" int asu_ipc_close(void* base_ptr) {
    if (!base_ptr) return ASU_OK;
    return cuda_rc(cudaIpcCloseMemHandle(base_ptr));
}
