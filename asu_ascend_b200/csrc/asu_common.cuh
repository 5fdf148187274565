// Shared device helpers for the ASU resolver kernels (sm_100a).
//
// Conventions used by every kernel in this library:
//  * One request row per CTA for the stateful ops: every read-modify-write of a
//    request's maps happens inside one CTA, ordered by __syncthreads().  Mutable
//    state is read with ld.global.cg (L2, never a stale L1 line) and written
//    with st.global.cg.
//  * Kernels never trap.  Problems are OR-ed into a per-request int32 status
//    word (ASU_ST_* bits) when the caller passes one, and the offending
//    element is skipped.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#include "../../include/asu_b200.h"

namespace asu {

constexpr int32_t kNotFound = -1;
constexpr int32_t kClaimBase = INT32_MIN;  // claim value of query position p: kClaimBase + p

__host__ __device__ __forceinline__ uint32_t hash32(uint32_t x) {
    // Integer mixer of ops/asu_hbm_index_maintain_aicpu_kernel.aicpu:25-33 (same constants, same steps).
    x ^= x >> 16;
    x *= 0x7feb352dU;
    x ^= x >> 15;
    x *= 0x846ca68bU;
    x ^= x >> 16;
    return x;
}

__device__ __forceinline__ int32_t ld_cg(const int32_t* p) { return __ldcg(p); }
__device__ __forceinline__ void st_cg(int32_t* p, int32_t v) { __stcg(p, v); }

// Programmatic dependent launch (PDL).  A kernel launched with launch_pdl() may have its CTAs
// scheduled while the previous grid on the stream is still draining; it calls pdl_wait() before
// its first global-memory access, which returns once that grid has completed and its writes are
// visible, so stream order holds.  pdl_trigger() lets the next PDL grid be scheduled early.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename... KArgs, typename... Args>
inline int launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                      Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return ASU_ERR_CUDA_BASE + static_cast<int>(e);
    }
    return ASU_OK;
}

__device__ __forceinline__ void flag_status(int32_t* status, int row, int32_t bits) {
    if (status != nullptr) atomicOr(status + row, bits);
}

// Block-wide exclusive scan of one int per thread (blockDim.x a multiple of 32, <= 1024).
// `warp_sums` must hold 33 ints of shared memory.  Returns the exclusive prefix and
// writes the block total to *total.  Contains three __syncthreads() (the last one lets
// back-to-back scans reuse `warp_sums`); every thread of the block must call it.
__device__ __forceinline__ int block_exclusive_scan(int v, int* warp_sums, int* total) {
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int nwarps = blockDim.x >> 5;
    int x = v;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
        int y = __shfl_up_sync(0xffffffffu, x, d);
        if (lane >= d) x += y;
    }
    if (lane == 31) warp_sums[warp] = x;
    __syncthreads();
    if (warp == 0) {
        int w = lane < nwarps ? warp_sums[lane] : 0;
        int s = w;
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
            int y = __shfl_up_sync(0xffffffffu, s, d);
            if (lane >= d) s += y;
        }
        if (lane < nwarps) warp_sums[lane] = s - w;  // exclusive warp offsets
        if (lane == 31) warp_sums[32] = s;
    }
    __syncthreads();
    int res = warp_sums[warp] + x - v;
    *total = warp_sums[32];
    __syncthreads();
    return res;
}

// Block-wide exclusive scan with a single __syncthreads(): every warp scans the per-warp
// totals itself instead of waiting for one warp to do it.  `warp_sums` (32 ints of shared
// memory) is read after the barrier, so the caller must not write it again before another
// barrier -- alternate two buffers between back-to-back scans.  Returns the exclusive prefix
// and writes the block total to *total; every thread of the block must call it.
__device__ __forceinline__ int block_exclusive_scan_1b(int v, int* warp_sums, int* total) {
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int nwarps = blockDim.x >> 5;
    int x = v;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, d);
        if (lane >= d) x += y;
    }
    if (lane == 31) warp_sums[warp] = x;
    __syncthreads();
    const int w = lane < nwarps ? warp_sums[lane] : 0;
    int s = w;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, s, d);
        if (lane >= d) s += y;
    }
    const int before = __shfl_sync(0xffffffffu, s - w, warp);  // sum of the warps before this one
    *total = __shfl_sync(0xffffffffu, s, 31);
    return before + x - v;
}

}  // namespace asu

// Host-side helpers shared by the entry points (defined in capi_misc.cu; thread-safe).
// SM count of the current device, queried once per device; 1 if the query fails (the launch
// that follows then reports the device's error itself).
int asu_sm_count();
// Opt-in dynamic shared-memory limit of `kernel` on the current device (the device's opt-in
// maximum minus the kernel's static shared memory), set as the kernel's attribute once per
// (device, kernel).  Returns ASU_OK or ASU_ERR_CUDA_BASE + cudaError_t.
int asu_max_dynamic_smem(const void* kernel, int* max_dynamic);

// Host-side launch-error helper shared by the entry points.
static inline int asu_launch_status() {
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? ASU_OK : ASU_ERR_CUDA_BASE + static_cast<int>(e);
}
