// Single-request KV resolver: map top-k token ids to managed slots, installing the missing
// tokens' KV row pairs into the managed cache.
//
// Reference behaviour: patch/0001 vllm_ascend/ops/asu_kv_resolver.py::asu_resolve_kv_slots_single_req
// (patch lines 954-1039) and its AscendC kernel op_kernel/asu_kv_resolver.cpp (patch lines
// 394-452), which runs on ONE core and copies the KV pair element by element:
//   HBM_RESIDENT -> slot = hbm_slot_of_token[tok]
//   ASU_ONLY     -> source = asu_record_addr[tok]
//   TAIL_HBM     -> source = block_table[tok / block_size] * block_size + tok % block_size
//   miss         -> slot = free_slot_stack[--free_slot_count]; copy kv0/kv1 rows source -> slot;
//                   token_state = HBM_RESIDENT; hbm_slot_of_token[tok] = slot; owner[slot] = tok
//
// B200 design: two launches on the caller's stream.
//  1. resolve: one CTA of 1024 threads walks topk in chunks of 2048 (chunks in order, so
//     later chunks see earlier installs exactly as the serial loop does).  First
//     occurrences of non-resident tokens are found with an atomicMin claim on token_state
//     (the states were read before any claim), ranked in topk order with a block scan,
//     and rank k pops free_slot_stack[count - 1 - k] -- the serial --count order.  The
//     (source row, managed slot) pairs go to a compact install list in `workspace`.
//  2. copy: one warp per install list entry copies the kv0 and kv1 rows with 16-byte
//     vectors (4-byte / 1-byte fallbacks for odd row sizes), spread over the whole GPU
//     instead of one core.
#include "asu_common.cuh"

namespace asu {
namespace {

constexpr int kThreads = 1024;
constexpr int kItems = 2;
constexpr int kChunk = kThreads * kItems;
constexpr int kCopyWarps = 8;

__global__ void __launch_bounds__(kThreads)
resolve_kernel(const int32_t* __restrict__ topk, int64_t n, int32_t* __restrict__ token_state,
               const int32_t* __restrict__ record, int32_t* __restrict__ hbm_slot, int32_t* __restrict__ owner,
               const int32_t* __restrict__ stack, int32_t* __restrict__ count_ptr, int64_t stack_len,
               const int32_t* __restrict__ block_table, int64_t bt_len, int64_t src_rows, int64_t slot_count,
               int64_t max_seq, int64_t actual, int64_t bs, int32_t* __restrict__ resolved,
               int32_t* __restrict__ ws, int32_t* status) {
    __shared__ int scan_buf[33];
    const int tid = threadIdx.x;
    int32_t count = ld_cg(count_ptr);
    int32_t bits = 0;
    int64_t n_inst = 0;
    const int64_t limit = actual < max_seq ? actual : max_seq;
    for (int64_t base = 0; base < n; base += kChunk) {
        int32_t tok[kItems], slot[kItems], st[kItems];
        bool miss[kItems];
#pragma unroll
        for (int j = 0; j < kItems; ++j) {
            const int64_t pos = base + tid * kItems + j;
            tok[j] = -1;
            slot[j] = kNotFound;
            st[j] = ASU_TOKEN_INVALID;
            miss[j] = false;
            if (pos < n) {
                tok[j] = __ldg(topk + pos);
                if (tok[j] < 0 || tok[j] >= limit) {
                    bits |= ASU_ST_BAD_QUERY;
                    tok[j] = -1;
                } else {
                    st[j] = ld_cg(token_state + tok[j]);
                    if (st[j] == ASU_TOKEN_HBM_RESIDENT) {
                        slot[j] = ld_cg(hbm_slot + tok[j]);
                    } else if (st[j] == ASU_TOKEN_ASU_ONLY || st[j] == ASU_TOKEN_TAIL_HBM) {
                        miss[j] = true;
                    } else {
                        bits |= ASU_ST_BAD_TOKEN_STATE;
                    }
                }
            }
        }
        __syncthreads();
#pragma unroll
        for (int j = 0; j < kItems; ++j)
            if (miss[j]) atomicMin(token_state + tok[j], kClaimBase + static_cast<int32_t>(tid * kItems + j));
        __syncthreads();
        int canon[kItems];
        int local = 0;
#pragma unroll
        for (int j = 0; j < kItems; ++j) {
            canon[j] = miss[j] && ld_cg(token_state + tok[j]) == kClaimBase + static_cast<int32_t>(tid * kItems + j);
            local += canon[j];
        }
        int M = 0;
        int rank = block_exclusive_scan(local, scan_buf, &M);
#pragma unroll
        for (int j = 0; j < kItems; ++j) {
            if (!canon[j]) continue;
            const int32_t k = rank++;
            const int32_t c = count - 1 - k;
            int32_t s = kNotFound;
            int64_t src = -1;
            bool ok = false;
            if (c >= 0 && c >= stack_len) {
                bits |= ASU_ST_BAD_STATE;  // free_slot_count exceeds the stack
            } else if (c >= 0) {
                s = ld_cg(stack + c);
                if (st[j] == ASU_TOKEN_ASU_ONLY) {
                    src = ld_cg(record + tok[j]);
                } else {
                    const int64_t lb = tok[j] / bs;
                    if (lb < bt_len) src = static_cast<int64_t>(__ldg(block_table + lb)) * bs + tok[j] % bs;
                }
                if (src < 0 || src >= src_rows) bits |= ASU_ST_BAD_SOURCE;
                else if (s < 0 || s >= slot_count) bits |= ASU_ST_BAD_STATE;
                else ok = true;
            } else {
                bits |= ASU_ST_FREE_EXHAUSTED;
            }
            if (ok) {
                st_cg(token_state + tok[j], ASU_TOKEN_HBM_RESIDENT);
                st_cg(hbm_slot + tok[j], s);
                st_cg(owner + s, tok[j]);
                slot[j] = s;
            } else {
                st_cg(token_state + tok[j], st[j]);  // undo the claim
                slot[j] = kNotFound;
            }
            if (c >= 0) {  // a popped entry, usable or not, keeps its place in the install list
                int32_t* e = ws + 1 + 2 * (n_inst + k);
                e[0] = ok ? static_cast<int32_t>(src) : -1;
                e[1] = s;
            }
            miss[j] = false;
        }
        const int32_t popped = M < count ? M : (count > 0 ? count : 0);
        __syncthreads();
#pragma unroll
        for (int j = 0; j < kItems; ++j) {
            const int64_t pos = base + tid * kItems + j;
            if (miss[j]) {  // later duplicate of a token installed in this chunk
                slot[j] = ld_cg(token_state + tok[j]) == ASU_TOKEN_HBM_RESIDENT ? ld_cg(hbm_slot + tok[j]) : kNotFound;
            }
            if (pos < n) resolved[pos] = slot[j];
        }
        count -= popped;
        n_inst += popped;
        __syncthreads();
    }
    if (tid == 0) {
        st_cg(count_ptr, count);
        ws[0] = static_cast<int32_t>(n_inst);
    }
    if (bits) flag_status(status, 0, bits);
}

__device__ __forceinline__ void copy_row(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst, int64_t bytes,
                                         int lane) {
    const uintptr_t m = reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst) |
                        static_cast<uintptr_t>(bytes);
    if ((m & 15) == 0) {
        const int4* s = reinterpret_cast<const int4*>(src);
        int4* d = reinterpret_cast<int4*>(dst);
        for (int64_t i = lane; i < bytes / 16; i += 32) d[i] = __ldg(s + i);
    } else if ((m & 3) == 0) {
        const int32_t* s = reinterpret_cast<const int32_t*>(src);
        int32_t* d = reinterpret_cast<int32_t*>(dst);
        for (int64_t i = lane; i < bytes / 4; i += 32) d[i] = __ldg(s + i);
    } else {
        for (int64_t i = lane; i < bytes; i += 32) dst[i] = __ldg(src + i);
    }
}

__global__ void __launch_bounds__(kCopyWarps * 32)
resolver_copy_kernel(const int32_t* __restrict__ ws, int64_t max_entries, const uint8_t* __restrict__ kv0_src,
                     const uint8_t* __restrict__ kv1_src, uint8_t* __restrict__ kv0_dst, uint8_t* __restrict__ kv1_dst,
                     int64_t rb0, int64_t rb1) {
    const int lane = threadIdx.x & 31;
    const int64_t n = ws[0];
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * kCopyWarps + (threadIdx.x >> 5); i < n && i < max_entries;
         i += static_cast<int64_t>(gridDim.x) * kCopyWarps) {
        const int32_t src = ws[1 + 2 * i];
        const int32_t dst = ws[2 + 2 * i];
        if (src < 0 || dst < 0) continue;
        if (rb0 > 0) copy_row(kv0_src + src * rb0, kv0_dst + dst * rb0, rb0, lane);
        if (rb1 > 0) copy_row(kv1_src + src * rb1, kv1_dst + dst * rb1, rb1, lane);
    }
}

}  // namespace
}  // namespace asu

using namespace asu;

extern "C" int64_t asu_kv_resolver_workspace_bytes(int64_t topk_numel) {
    if (topk_numel < 0) return -1;
    return ((1 + 2 * topk_numel) * 4 + 15) / 16 * 16;
}

extern "C" int asu_kv_resolver_do(void* stream, const int32_t* topk, int64_t topk_numel, int32_t* token_state,
                                  const int32_t* asu_record_addr, int32_t* hbm_slot_of_token,
                                  int32_t* slot_owner_token, const int32_t* free_slot_stack,
                                  int32_t* free_slot_count, int64_t free_slot_stack_len, const int32_t* block_table,
                                  int64_t block_table_len, const void* kv0_src, const void* kv1_src, void* kv0_dst,
                                  void* kv1_dst, int64_t kv0_row_bytes, int64_t kv1_row_bytes, int64_t src_rows,
                                  int64_t slot_count, int64_t max_seq_len, int64_t actual_seq_len, int64_t block_size,
                                  int32_t* resolved, void* workspace, int32_t* status) {
    if (topk_numel == 0) return ASU_OK;
    if (topk_numel < 0 || topk_numel > 0x3fffffff || !topk || !token_state || !asu_record_addr ||
        !hbm_slot_of_token || !slot_owner_token || !free_slot_stack || !free_slot_count || !resolved || !workspace)
        return ASU_ERR_ARG;
    if (block_size <= 0 || actual_seq_len < 0 || max_seq_len <= 0 || slot_count < 0 || src_rows < 0 ||
        src_rows > 0x7fffffff || free_slot_stack_len < 0 || kv0_row_bytes < 0 || kv1_row_bytes < 0 ||
        (block_table_len > 0 && !block_table))
        return ASU_ERR_ARG;
    if ((kv0_row_bytes > 0 && (!kv0_src || !kv0_dst)) || (kv1_row_bytes > 0 && (!kv1_src || !kv1_dst)))
        return ASU_ERR_ARG;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    int32_t* ws = static_cast<int32_t*>(workspace);
    resolve_kernel<<<1, kThreads, 0, s>>>(topk, topk_numel, token_state, asu_record_addr, hbm_slot_of_token,
                                          slot_owner_token, free_slot_stack, free_slot_count, free_slot_stack_len,
                                          block_table, block_table_len, src_rows, slot_count, max_seq_len,
                                          actual_seq_len, block_size, resolved, ws, status);
    int rc = asu_launch_status();
    if (rc != ASU_OK) return rc;
    if (kv0_row_bytes == 0 && kv1_row_bytes == 0) return ASU_OK;
    int64_t grid = (topk_numel + kCopyWarps - 1) / kCopyWarps;
    if (grid > 148 * 8) grid = 148 * 8;
    resolver_copy_kernel<<<static_cast<uint32_t>(grid), kCopyWarps * 32, 0, s>>>(
        ws, topk_numel, static_cast<const uint8_t*>(kv0_src), static_cast<const uint8_t*>(kv1_src),
        static_cast<uint8_t*>(kv0_dst), static_cast<uint8_t*>(kv1_dst), kv0_row_bytes, kv1_row_bytes);
    return asu_launch_status();
}

// ---------------------------------------------------------------------------
// Resolver entry point that allocates nothing.
//
// Some callers cannot allocate device memory when they resolve a layer.  Examples: a serving
// engine that hands nearly all HBM to its KV-block pool at start-up and forbids cudaMalloc in
// the decode loop (it could fail there, and it synchronises the device); or a C / FFI host
// with no caching allocator, which would otherwise pay a cudaMalloc + cudaFree per layer per
// step.  For them the install list lives in a fixed file-scope device array instead of a
// caller-provided workspace.
//
// * Capacity: ASU_RESOLVER_NOALLOC_MAX_TOPK top-k entries per call (128 KiB of device memory
//   that every GPU loading this library holds until the process exits).  Larger calls are
//   rejected with ASU_ERR_NOALLOC_CAPACITY before anything is launched.
// * Set-up: the first call on a device looks up the array's device address with
//   cudaGetSymbolAddress (with that device current) and caches it.  Make that first call
//   before any stream capture on the device.
// * Sharing: every call on a device uses the same array.  The resolve kernel rewrites the
//   install count and every entry it later reads, so nothing has to start at zero, but two
//   calls whose launches overlap on the GPU (different streams, no ordering between them)
//   race on the array.  Order such calls on one stream.
// ---------------------------------------------------------------------------
#include <mutex>

namespace {

constexpr int64_t kNoAllocScratchInts = 1 + 2 * static_cast<int64_t>(ASU_RESOLVER_NOALLOC_MAX_TOPK);
static __device__ __align__(256) int32_t g_noalloc_scratch[kNoAllocScratchInts];

std::mutex g_noalloc_mu;
int32_t* g_noalloc_addr[64] = {};  // device address of g_noalloc_scratch per device ordinal

int noalloc_scratch(int32_t** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return ASU_ERR_CUDA_BASE + static_cast<int>(e);
    }
    if (dev < 0 || dev >= 64) return ASU_ERR_ARG;
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (g_noalloc_addr[dev] == nullptr) {
        void* p = nullptr;
        // The host-side name g_noalloc_scratch is only a stand-in; the kernel needs this address.
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || p == nullptr) {
            cudaGetLastError();
            return e != cudaSuccess ? ASU_ERR_CUDA_BASE + static_cast<int>(e) : ASU_ERR_ARG;
        }
        g_noalloc_addr[dev] = static_cast<int32_t*>(p);
    }
    *out = g_noalloc_addr[dev];
    return ASU_OK;
}

}  // namespace

extern "C" int asu_kv_resolver_noalloc(void* stream, const int32_t* topk, int64_t topk_numel, int32_t* token_state,
                                       const int32_t* asu_record_addr, int32_t* hbm_slot_of_token,
                                       int32_t* slot_owner_token, const int32_t* free_slot_stack,
                                       int32_t* free_slot_count, int64_t free_slot_stack_len,
                                       const int32_t* block_table, int64_t block_table_len, const void* kv0_src,
                                       const void* kv1_src, void* kv0_dst, void* kv1_dst, int64_t kv0_row_bytes,
                                       int64_t kv1_row_bytes, int64_t src_rows, int64_t slot_count,
                                       int64_t max_seq_len, int64_t actual_seq_len, int64_t block_size,
                                       int32_t* resolved, int32_t* status) {
    if (topk_numel > ASU_RESOLVER_NOALLOC_MAX_TOPK) return ASU_ERR_NOALLOC_CAPACITY;
    if (topk_numel == 0) return ASU_OK;
    int32_t* scratch = nullptr;
    const int rc = noalloc_scratch(&scratch);
    if (rc != ASU_OK) return rc;
    return asu_kv_resolver_do(stream, topk, topk_numel, token_state, asu_record_addr, hbm_slot_of_token,
                              slot_owner_token, free_slot_stack, free_slot_count, free_slot_stack_len, block_table,
                              block_table_len, kv0_src, kv1_src, kv0_dst, kv1_dst, kv0_row_bytes, kv1_row_bytes,
                              src_rows, slot_count, max_seq_len, actual_seq_len, block_size, resolved, scratch,
                              status);
}
