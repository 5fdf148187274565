// Write-back of KV rows from HBM into the pinned, GPU-mapped host row pool (the producer side
// of the swap-in).
//
// Reference behaviour: the v0/v0.1 offload designs store every prefilled (request, layer,
// token) record in MicroKV with batch_put over a Unix socket, one serialized record per key
// (docs/v0.1/kv-cache-offload-v0.1-real-ops-design.md:243-292; MicroKV/src/server.cpp
// CMD_BATCH_PUT).  The bytes stored for a key are the record's bytes, unchanged.
//
// B200 design: zero-copy stores.  The host pool is mapped into the GPU's address space, so the
// GPU writes the rows itself over the host link with 16-byte stores (posted PCIe writes, no
// host thread, no staging copy).  Work unit: the flattened (item, 16-byte chunk) space, so a
// warp's stores to one row are contiguous and coalesce into full-line writes; each thread keeps
// kUnroll HBM loads in flight before its stores.  Item i copies source row src_index[i] (or i)
// to host row dst_row[i] (or i); a negative dst_row skips the item.
#include "asu_common.cuh"

namespace asu {
namespace {

constexpr int kThreads = 256;
constexpr int kUnroll = 8;

__global__ void __launch_bounds__(kThreads)
writeback_kernel(int4* host, int64_t pool_rows, uint32_t cpr, uint32_t wpr, uint32_t pitch16,
                 const int4* __restrict__ src, int64_t src_rows, uint64_t src_pitch16,
                 const int32_t* __restrict__ src_index, const int32_t* __restrict__ dst_row, uint32_t n,
                 int32_t* status) {
    // wpr >= cpr units are written per row: the row's cpr chunks, then zeros over the row's
    // padding up to the host pitch, so a padded row goes out as whole lines
    const uint32_t total = n * wpr;  // < 2^31, checked by the launcher
    const uint32_t stride = gridDim.x * kThreads;
    int32_t bits = 0;
    for (uint32_t u0 = blockIdx.x * kThreads + threadIdx.x; u0 < total; u0 += stride * kUnroll) {
        int4 buf[kUnroll];
        int4* dst[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            dst[u] = nullptr;
            const uint32_t uu = u0 + u * stride;
            if (uu >= total) continue;
            const uint32_t i = uu / wpr;
            const uint32_t ch = uu - i * wpr;
            const int64_t d = dst_row ? static_cast<int64_t>(__ldg(dst_row + i)) : static_cast<int64_t>(i);
            const int64_t s = src_index ? static_cast<int64_t>(__ldg(src_index + i)) : static_cast<int64_t>(i);
            if (d < 0) continue;
            if (d >= pool_rows) {
                bits |= ASU_ST_BAD_STATE;
                continue;
            }
            if (s < 0 || s >= src_rows) {
                bits |= ASU_ST_BAD_SOURCE;
                continue;
            }
            buf[u] = ch < cpr ? __ldg(src + s * src_pitch16 + ch) : make_int4(0, 0, 0, 0);
            dst[u] = host + d * pitch16 + ch;
        }
#pragma unroll
        for (int u = 0; u < kUnroll; ++u)
            if (dst[u]) *dst[u] = buf[u];
    }
    if (bits) flag_status(status, 0, bits);
}

}  // namespace
}  // namespace asu

using namespace asu;

extern "C" int asu_host_pool_writeback(void* stream, void* host_pool, int64_t pool_rows, uint32_t row_bytes,
                                       uint32_t host_pitch, const void* src, int64_t src_rows, uint64_t src_pitch,
                                       const int32_t* src_index, const int32_t* dst_row, int64_t n,
                                       int32_t* status) {
    if (n == 0) return ASU_OK;
    if (n < 0 || !host_pool || !src || pool_rows <= 0 || row_bytes == 0 || src_rows <= 0)
        return ASU_ERR_ARG;
    if (host_pitch == 0) host_pitch = row_bytes;
    if (src_pitch == 0) src_pitch = row_bytes;
    if (host_pitch < row_bytes || src_pitch < row_bytes) return ASU_ERR_ARG;
    if (row_bytes % 16 != 0 || host_pitch % 16 != 0 || src_pitch % 16 != 0 ||
        reinterpret_cast<uintptr_t>(host_pool) % 16 != 0 || reinterpret_cast<uintptr_t>(src) % 16 != 0)
        return ASU_ERR_ALIGN;
    const uint32_t cpr = row_bytes / 16;
    // pad a row up to its pitch when the padding is under one 128-byte line: partial-line PCIe
    // writes cost more than the padding bytes (656-byte rows at a 768-byte pitch: 70% -> ~85%
    // of the link)
    const uint32_t wpr = (host_pitch - row_bytes) < 128 ? host_pitch / 16 : cpr;
    const uint64_t total = static_cast<uint64_t>(n) * wpr;
    if (total >= (1ull << 31)) return ASU_ERR_ARG;  // split larger write-backs
    uint64_t grid = (total + kThreads * kUnroll - 1) / (kThreads * kUnroll);
    const uint64_t cap = static_cast<uint64_t>(asu_sm_count()) * 8ull;
    if (grid > cap) grid = cap;
    writeback_kernel<<<static_cast<uint32_t>(grid), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<int4*>(host_pool), pool_rows, cpr, wpr, host_pitch / 16, static_cast<const int4*>(src), src_rows,
        src_pitch / 16, src_index, dst_row, static_cast<uint32_t>(n), status);
    return asu_launch_status();
}
