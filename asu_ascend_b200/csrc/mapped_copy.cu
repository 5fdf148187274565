// Transfers between HBM and page-locked, mapped host memory done by SMs (zero-copy) instead of a
// copy engine: the end-to-end path's top-k upload before a resolve and its result read-back.
//
// Why: on a box where several GPUs share the host memory system, the copy engines' share of it
// falls first.  On the 8-GPU B200 boxes measured here, pinned H2D copies reach ~29 GB/s per GPU on
// GPUs 0-3 with those four copying, while the swap-in kernel's own reads of mapped host memory
// reach ~45 GB/s there; a 1 MB top-k upload queued behind seven other GPUs' swap-ins then costs
// far more than its size.  Reading (or writing) the host buffer from the SMs puts these small
// transfers on the same path as the swap-in.
//
// The reference has no counterpart: its top-k comes from the indexer on the NPU and the resolved
// slots stay there (patch/0003, patch lines 561-575); the host copies exist only where a caller
// hands the resolver host buffers.
#include "asu_common.cuh"

namespace asu {
namespace {

constexpr int kThreads = 256;
constexpr int kInFlight = 4;  // loads in flight per thread before their stores

template <typename V>
__global__ void __launch_bounds__(kThreads) mapped_copy_kernel(V* __restrict__ dst, const V* __restrict__ src,
                                                               uint64_t n) {
    pdl_wait();  // launched with launch_pdl: the source written by the grid before is visible
    pdl_trigger();
    const uint64_t stride = static_cast<uint64_t>(gridDim.x) * kThreads;
    uint64_t i = static_cast<uint64_t>(blockIdx.x) * kThreads + threadIdx.x;
    for (; i + (kInFlight - 1) * stride < n; i += kInFlight * stride) {
        V v[kInFlight];
#pragma unroll
        for (int u = 0; u < kInFlight; ++u) v[u] = src[i + u * stride];
#pragma unroll
        for (int u = 0; u < kInFlight; ++u) dst[i + u * stride] = v[u];
    }
    for (; i < n; i += stride) dst[i] = src[i];
}

template <typename V>
int launch_copy(cudaStream_t s, void* dst, const void* src, uint64_t bytes) {
    const uint64_t n = bytes / sizeof(V);
    uint64_t grid = (n + static_cast<uint64_t>(kThreads) * kInFlight - 1) / (static_cast<uint64_t>(kThreads) * kInFlight);
    const uint64_t cap = static_cast<uint64_t>(asu_sm_count()) * 8;
    if (grid > cap) grid = cap;
    if (grid < 1) grid = 1;
    return launch_pdl(mapped_copy_kernel<V>, dim3(static_cast<uint32_t>(grid)), dim3(kThreads), 0, s,
                      static_cast<V*>(dst), static_cast<const V*>(src), n);
}

}  // namespace
}  // namespace asu

using namespace asu;

extern "C" int asu_mapped_copy(void* stream, void* dst, const void* src, uint64_t bytes) {
    if (bytes == 0) return ASU_OK;
    if (dst == nullptr || src == nullptr) return ASU_ERR_ARG;
    const uintptr_t d = reinterpret_cast<uintptr_t>(dst), s = reinterpret_cast<uintptr_t>(src);
    // the copied ranges must not overlap (the units are copied in no particular order)
    if (d < s + bytes && s < d + bytes) return ASU_ERR_ARG;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if ((d | s | bytes) % 16 == 0) return launch_copy<int4>(st, dst, src, bytes);
    if ((d | s | bytes) % 4 == 0) return launch_copy<int32_t>(st, dst, src, bytes);
    return launch_copy<uint8_t>(st, dst, src, bytes);
}
