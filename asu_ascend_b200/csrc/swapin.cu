// Swap-in gather: copy the KV rows of newly installed keys from a pinned, GPU-mapped host
// row pool into the HBM slot pool.
//
// Reference behaviour: the v0/v0.1 designs fetch each missed (request, layer, token) record
// from MicroKV over a Unix socket, deserialize it on the CPU and copy it to the device
// (docs/v0.1/kv-cache-offload-v0.1-real-ops-design.md:293-312; MicroKV/src/server.cpp:220-251).
// The bytes that land in slot `s` are the record's bytes, unchanged.
//
// B200 design: zero-copy.  The host pool is page-locked and mapped (rows host_pitch bytes
// apart), so the GPU reads it
// directly over the host link with 16-byte loads and writes 16-byte stores into HBM; no
// host thread, no staging copy, no synchronisation with the CPU.  Work unit: one warp per
// 32 query positions of one request.  The warp ballots the install flags, compacts the
// (source row, destination row) pairs of its installs into shared memory, and then copies
// the flattened (row, 16-byte chunk) space lane-strided with 8 loads in flight per lane
// before their stores, so a 656-byte DSA row (41 chunks) and a 41,984-byte block row both
// keep the link busy.  Grid: enough warps for every group, capped at 8 CTAs per SM.
#include "asu_common.cuh"

namespace asu {
namespace {

constexpr int kWarps = 8;
constexpr int kUnroll = 8;

template <bool kPeer>
__global__ void __launch_bounds__(kWarps * 32)
swapin_kernel(const int4* host, int64_t pool_rows, uint32_t cpr, uint32_t pitch16,
              const int32_t* __restrict__ rec, uint32_t K, const int32_t* __restrict__ query,
              const int32_t* __restrict__ slot,
              const uint8_t* __restrict__ inst, uint32_t Q, int4* __restrict__ pool, uint32_t S, uint32_t R,
              int32_t* status) {
    pdl_wait();     // launched with launch_pdl: the masks and slots of the step before are visible
    pdl_trigger();
    __shared__ int64_t src_row[kWarps][32];
    __shared__ int64_t dst_row[kWarps][32];
    const int lane = threadIdx.x & 31;
    const int w = threadIdx.x >> 5;
    const uint32_t groups_per_row = (Q + 31) / 32;
    const uint64_t total_groups = static_cast<uint64_t>(R) * groups_per_row;
    for (uint64_t g = static_cast<uint64_t>(blockIdx.x) * kWarps + w; g < total_groups;
         g += static_cast<uint64_t>(gridDim.x) * kWarps) {
        const uint32_t r = static_cast<uint32_t>(g / groups_per_row);
        const uint32_t pos = static_cast<uint32_t>(g - static_cast<uint64_t>(r) * groups_per_row) * 32 + lane;
        const uint64_t qi = static_cast<uint64_t>(r) * Q + pos;
        const bool flag = pos < Q && __ldg(inst + qi) != 0;
        if (__ballot_sync(0xffffffffu, flag) == 0u) continue;
        bool ok = false;
        int64_t src = 0, dst = 0;
        if (flag) {
            const int32_t key = __ldg(query + qi);
            const int32_t s = __ldg(slot + qi);
            int32_t bits = 0;
            if (static_cast<uint32_t>(key) >= K) {
                bits |= ASU_ST_BAD_QUERY;
            } else if (static_cast<uint32_t>(s) >= S) {
                bits |= ASU_ST_BAD_STATE;
            } else {
                const int32_t row = __ldg(rec + static_cast<uint64_t>(r) * K + key);
                if (row < 0 || row >= pool_rows) {
                    bits |= ASU_ST_BAD_SOURCE;
                } else {
                    ok = true;
                    src = row;
                    dst = static_cast<int64_t>(r) * S + s;
                }
            }
            if (bits) flag_status(status, r, bits);
        }
        const unsigned okmask = __ballot_sync(0xffffffffu, ok);
        if (ok) {
            const int rank = __popc(okmask & ((1u << lane) - 1u));
            src_row[w][rank] = src;
            dst_row[w][rank] = dst;
        }
        __syncwarp();
        const uint32_t n = __popc(okmask);
        const uint32_t total = n * cpr;
        for (uint32_t base = 0; base < total; base += 32 * kUnroll) {
            int4 buf[kUnroll];
#pragma unroll
            for (int u = 0; u < kUnroll; ++u) {
                const uint32_t c = base + u * 32 + lane;
                if (c < total) {
                    const uint32_t ri = c / cpr;
                    const uint32_t ch = c - ri * cpr;
                    buf[u] = host[src_row[w][ri] * pitch16 + ch];
                }
            }
#pragma unroll
            for (int u = 0; u < kUnroll; ++u) {
                const uint32_t c = base + u * 32 + lane;
                if (c < total) {
                    const uint32_t ri = c / cpr;
                    const uint32_t ch = c - ri * cpr;
                    pool[dst_row[w][ri] * cpr + ch] = buf[u];
                }
            }
        }
        __syncwarp();
    }
    // rows stored into another GPU's memory: performed at system scope before the grid
    // completes, so whatever the host orders after this launch sees them
    if constexpr (kPeer) __threadfence_system();
}

// ---------------------------------------------------------------------------------------
// Rows up to kBulkMaxRow bytes: one TMA bulk copy per row.  Each lane owns a shared-memory slot
// and an mbarrier; for an installing position it issues cp.async.bulk host row -> slot
// (completion counted in bytes on the mbarrier), waits for it with a bounded try_wait loop,
// then issues cp.async.bulk slot -> HBM row.  A lane's next load into its slot waits until the
// previous store has read it (cp.async.bulk.wait_group.read).  Measured on B200 with 656-byte
// rows, 128-byte-aligned host rows read this way reach ~48 GB/s against ~44 GB/s for the
// 16-byte-load kernel above; the copy engine (cudaMemcpyAsync of 256 MiB) reaches ~56 GB/s.
// A wait that runs out sets ASU_ST_TIMEOUT, waits once more (bounded) for the copy still in
// flight into the slot, and the lane stops.  A bulk copy cannot be cancelled: if that second
// wait runs out too, the copy may still land in this CTA's shared memory after the CTA has
// exited, i.e. in whichever CTA the SM runs next.  ASU_ST_TIMEOUT therefore reports a failed
// host link, not a skipped row: the results of this stream's later launches are not to be
// trusted (the caller treats it like a CUDA error of the context).
constexpr int kBulkWarps = 4;
constexpr uint32_t kBulkMaxRow = 1024;
constexpr int kBulkSpinLimit = 1 << 18;  // ~1 s of try_wait on B200 (each try suspends ~4 us)

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
    uint32_t done = 0;
    for (int it = 0; it < kBulkSpinLimit && !done; ++it) {
        asm volatile(
            "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
            : "=r"(done)
            : "r"(bar), "r"(parity)
            : "memory");
    }
    return done != 0;
}

// kPeer: the slot pool is another GPU's memory (a CUDA IPC mapping reached over NVLink).  The row
// is then written from shared memory with plain 16-byte stores instead of a bulk store, and every
// thread fences at system scope before it exits.
template <bool kPeer>
__global__ void __launch_bounds__(kBulkWarps * 32)
swapin_bulk_kernel(const uint8_t* host, int64_t pool_rows, uint32_t row_bytes, uint32_t pitch,
                   const int32_t* __restrict__ rec, uint32_t K, const int32_t* __restrict__ query,
                   const int32_t* __restrict__ slot, const uint8_t* __restrict__ inst, uint32_t Q,
                   uint8_t* __restrict__ pool, uint32_t S, uint32_t R, int32_t* status, uint32_t slot_stride) {
    pdl_wait();     // launched with launch_pdl: the masks and slots of the step before are visible
    pdl_trigger();
    extern __shared__ __align__(128) uint8_t slots[];
    __shared__ __align__(8) uint64_t bars[kBulkWarps * 32];
    const int lane = threadIdx.x & 31;
    const int w = threadIdx.x >> 5;
    const uint32_t my_slot = smem_addr(slots + (w * 32 + lane) * slot_stride);
    const uint32_t my_bar = smem_addr(&bars[w * 32 + lane]);
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(my_bar) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    uint32_t parity = 0;
    const uint32_t groups_per_row = (Q + 31) / 32;
    const uint64_t total_groups = static_cast<uint64_t>(R) * groups_per_row;
    for (uint64_t g = static_cast<uint64_t>(blockIdx.x) * kBulkWarps + w; g < total_groups;
         g += static_cast<uint64_t>(gridDim.x) * kBulkWarps) {
        const uint32_t r = static_cast<uint32_t>(g / groups_per_row);
        const uint32_t pos = static_cast<uint32_t>(g - static_cast<uint64_t>(r) * groups_per_row) * 32 + lane;
        const uint64_t qi = static_cast<uint64_t>(r) * Q + pos;
        if (pos >= Q || __ldg(inst + qi) == 0) continue;
        const int32_t key = __ldg(query + qi);
        const int32_t s = __ldg(slot + qi);
        if (static_cast<uint32_t>(key) >= K) {
            flag_status(status, r, ASU_ST_BAD_QUERY);
            continue;
        }
        if (static_cast<uint32_t>(s) >= S) {
            flag_status(status, r, ASU_ST_BAD_STATE);
            continue;
        }
        const int32_t row = __ldg(rec + static_cast<uint64_t>(r) * K + key);
        if (row < 0 || row >= pool_rows) {
            flag_status(status, r, ASU_ST_BAD_SOURCE);
            continue;
        }
        const uint8_t* src = host + static_cast<uint64_t>(row) * pitch;
        uint8_t* dst = pool + (static_cast<uint64_t>(r) * S + s) * row_bytes;
        if constexpr (!kPeer)
            asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");  // the slot's last store has read it
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(my_bar), "r"(row_bytes)
                     : "memory");
        asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                         my_slot),
                     "l"(src), "r"(row_bytes), "r"(my_bar)
                     : "memory");
        if (!mbar_wait(my_bar, parity)) {
            flag_status(status, r, ASU_ST_TIMEOUT);
            mbar_wait(my_bar, parity);  // the copy into the slot may still land: wait once more, then stop
            break;
        }
        parity ^= 1u;
        if constexpr (kPeer) {
            // the bulk copy completed on the mbarrier: its bytes are visible to this thread
            const int4* s16 = reinterpret_cast<const int4*>(slots + (w * 32 + lane) * slot_stride);
            int4* d16 = reinterpret_cast<int4*>(dst);
            for (uint32_t c = 0; c < row_bytes / 16; ++c) d16[c] = s16[c];
        } else {
            asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst), "r"(my_slot),
                         "r"(row_bytes)
                         : "memory");
            asm volatile("cp.async.bulk.commit_group;" ::: "memory");
        }
    }
    if constexpr (kPeer) {
        __threadfence_system();  // peer stores performed before the grid completes
    } else {
        asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");  // every store done before the CTA exits
    }
}

// Self-test of the swap-in's bounded wait (mbar_wait): one thread waits on an mbarrier with an
// arrival count of one.  With `arrive` 0 nothing arrives -- the flag that nothing sets --, the
// wait gives up after kBulkSpinLimit tries and the kernel reports ASU_ST_TIMEOUT in status[0],
// the path a bulk copy that never completes would take; with `arrive` 1 the thread arrives first
// and the wait succeeds.  No copy is in flight either way, so the kernel returns normally.
__global__ void __launch_bounds__(32) wait_selftest_kernel(int32_t arrive, int32_t* status) {
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x != 0) return;
    const uint32_t b = smem_addr(&bar);
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(b) : "memory");
    if (arrive) asm volatile("{ .reg .b64 st; mbarrier.arrive.shared::cta.b64 st, [%0]; }" ::"r"(b) : "memory");
    if (!mbar_wait(b, 0)) flag_status(status, 0, ASU_ST_TIMEOUT);
}

}  // namespace
}  // namespace asu

using namespace asu;

namespace {

// Dynamic shared memory limit of swapin_bulk_kernel<kPeer>, configured once per device.
template <bool kPeer>
int bulk_configure(uint32_t smem) {
    int max_dynamic = 0;
    const int rc = asu_max_dynamic_smem(reinterpret_cast<const void*>(swapin_bulk_kernel<kPeer>), &max_dynamic);
    if (rc != ASU_OK) return rc;
    return smem <= static_cast<uint32_t>(max_dynamic) ? ASU_OK : ASU_ERR_ARG;
}

template <bool kPeer>
int swapin_launch(void* stream, const void* host_pool, int64_t pool_rows, uint32_t row_bytes, uint32_t host_pitch,
                  const int32_t* record_addr, uint32_t key_space, const int32_t* query, const int32_t* slot,
                  const uint8_t* install_mask, uint32_t query_count, void* slot_pool, uint32_t slot_count,
                  uint32_t req_num, int32_t* status) {
    if (req_num == 0 || query_count == 0) return ASU_OK;
    if (!host_pool || !record_addr || !query || !slot || !install_mask || !slot_pool || pool_rows <= 0 ||
        row_bytes == 0 || key_space == 0 || slot_count == 0)
        return ASU_ERR_ARG;
    if (host_pitch == 0) host_pitch = row_bytes;
    if (host_pitch < row_bytes) return ASU_ERR_ARG;
    if (row_bytes % 16 != 0 || host_pitch % 16 != 0 || reinterpret_cast<uintptr_t>(host_pool) % 16 != 0 ||
        reinterpret_cast<uintptr_t>(slot_pool) % 16 != 0)
        return ASU_ERR_ALIGN;
    const uint64_t groups = static_cast<uint64_t>(req_num) * ((query_count + 31) / 32);
    if (row_bytes <= kBulkMaxRow) {
        const uint32_t stride = (row_bytes + 127) / 128 * 128;
        const uint32_t smem = kBulkWarps * 32 * stride;
        const int rc = bulk_configure<kPeer>(smem);
        if (rc != ASU_OK) return rc;
        uint64_t grid = (groups + kBulkWarps - 1) / kBulkWarps;
        const uint64_t per_sm = stride <= 768 ? 2 : 1;  // two CTAs per SM while their slots fit
        const uint64_t cap = static_cast<uint64_t>(asu_sm_count()) * per_sm;
        if (grid > cap) grid = cap;
        return launch_pdl(swapin_bulk_kernel<kPeer>, dim3(static_cast<uint32_t>(grid)), dim3(kBulkWarps * 32), smem,
                          static_cast<cudaStream_t>(stream), static_cast<const uint8_t*>(host_pool), pool_rows,
                          row_bytes, host_pitch, record_addr, key_space, query, slot, install_mask, query_count,
                          static_cast<uint8_t*>(slot_pool), slot_count, req_num, status, stride);
    }
    uint64_t grid = (groups + kWarps - 1) / kWarps;
    const uint64_t cap = static_cast<uint64_t>(asu_sm_count()) * 8ull;
    if (grid > cap) grid = cap;
    return launch_pdl(swapin_kernel<kPeer>, dim3(static_cast<uint32_t>(grid)), dim3(kWarps * 32), 0,
                      static_cast<cudaStream_t>(stream), static_cast<const int4*>(host_pool), pool_rows,
                      row_bytes / 16, host_pitch / 16, record_addr, key_space, query, slot, install_mask, query_count,
                      static_cast<int4*>(slot_pool), slot_count, req_num, status);
}

}  // namespace

extern "C" int asu_swapin_gather(void* stream, const void* host_pool, int64_t pool_rows, uint32_t row_bytes,
                                 uint32_t host_pitch, const int32_t* record_addr, uint32_t key_space,
                                 const int32_t* query, const int32_t* slot, const uint8_t* install_mask,
                                 uint32_t query_count,
                                 void* slot_pool, uint32_t slot_count, uint32_t req_num, int32_t* status) {
    return swapin_launch<false>(stream, host_pool, pool_rows, row_bytes, host_pitch, record_addr, key_space, query,
                                slot, install_mask, query_count, slot_pool, slot_count, req_num, status);
}

extern "C" int asu_swapin_gather_to_peer(void* stream, const void* host_pool, int64_t pool_rows, uint32_t row_bytes,
                                         uint32_t host_pitch, const int32_t* record_addr, uint32_t key_space,
                                         const int32_t* query, const int32_t* slot, const uint8_t* install_mask,
                                         uint32_t query_count, void* peer_slot_pool, uint32_t slot_count,
                                         uint32_t req_num, int32_t* status) {
    return swapin_launch<true>(stream, host_pool, pool_rows, row_bytes, host_pitch, record_addr, key_space, query,
                               slot, install_mask, query_count, peer_slot_pool, slot_count, req_num, status);
}

extern "C" int asu_host_pool_alloc(uint64_t bytes, void** host_ptr, void** device_ptr) {
    if (!host_ptr || bytes == 0) return ASU_ERR_ARG;
    void* h = nullptr;
    cudaError_t e = cudaHostAlloc(&h, bytes, cudaHostAllocPortable | cudaHostAllocMapped);
    if (e != cudaSuccess) return ASU_ERR_CUDA_BASE + static_cast<int>(e);
    void* d = nullptr;
    e = cudaHostGetDevicePointer(&d, h, 0);
    if (e != cudaSuccess) {
        cudaFreeHost(h);
        return ASU_ERR_CUDA_BASE + static_cast<int>(e);
    }
    *host_ptr = h;
    if (device_ptr) *device_ptr = d;
    return ASU_OK;
}

extern "C" int asu_host_pool_free(void* host_ptr) {
    if (!host_ptr) return ASU_OK;
    cudaError_t e = cudaFreeHost(host_ptr);
    return e == cudaSuccess ? ASU_OK : ASU_ERR_CUDA_BASE + static_cast<int>(e);
}

extern "C" int asu_host_device_pointer(const void* host_ptr, void** device_ptr) {
    if (!host_ptr || !device_ptr) return ASU_ERR_ARG;
    void* d = nullptr;
    const cudaError_t e = cudaHostGetDevicePointer(&d, const_cast<void*>(host_ptr), 0);
    if (e != cudaSuccess) {
        cudaGetLastError();  // not page-locked and mapped: leave no error behind
        return ASU_ERR_CUDA_BASE + static_cast<int>(e);
    }
    *device_ptr = d;
    return ASU_OK;
}

extern "C" int asu_selftest_bounded_wait(void* stream, int32_t arrive, int32_t* status) {
    if (!status) return ASU_ERR_ARG;
    wait_selftest_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(arrive != 0, status);
    return asu_launch_status();
}
