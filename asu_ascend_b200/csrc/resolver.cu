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
// B200 design: two launches on the caller's stream, the second a programmatic dependent launch.
//  1. resolve: one thread-block cluster (kCluster CTAs on kCluster SMs) walks topk in chunks
//     of kChunk entries, one entry per thread, chunks in order so later chunks see earlier
//     installs exactly as the serial loop does.  A single CTA is bound by how many random
//     4-byte loads one SM keeps in flight (token_state, hbm_slot_of_token, asu_record_addr and
//     the block table per entry); the cluster spreads them over its SMs.  Per chunk:
//       - every CTA clears its part of a distributed hash table and prefetches its share of
//         the free-stack window free_slot_stack[count - 1 - k];
//       - each thread loads its top-k entry and then the four state words at once;
//       - a non-resident token claims its first position in the table of its home CTA
//         (hash-selected) through distributed shared memory (atomicCAS + atomicMin);
//       - first occurrences are ranked in topk order (block scan + per-CTA totals exchanged
//         through distributed shared memory); rank k takes stack entry k -- the serial
//         --count order --, installs the token, publishes its slot in the home table (where
//         later duplicates read it) and writes (source row, slot) to the install list in
//         `workspace` (count, then pairs in install order).
//     Cluster barriers (barrier.cluster, hardware) separate the phases.
//  2. copy: the flattened (install, unit) space of the kv0 + kv1 rows (16-, 4- or 1-byte
//     units), spread over the GPU with several independent loads in flight per thread.  It is
//     launched with programmatic stream serialization: its CTAs are scheduled while the
//     resolve cluster runs and wait in griddepcontrol.wait until the resolve grid has
//     completed and its writes are visible.
//     Row pairs of up to kInClusterMaxRowBytes whose starts are 16-byte aligned (DSA / MLA
//     token rows) skip this launch: after each chunk every CTA of the cluster copies the rows
//     of its own installs, listed in shared memory in rank order.
// Measured on B200 (16 layers x top-k 2048 per step, L2 flushed per step): ~14.5 us per call
// for this design and for a single 1024-thread CTA alike, against ~3.5 us for two empty
// launches; a call is bound by the latency of its dependent steps, not by bandwidth.
#include <cooperative_groups.h>

#include "asu_common.cuh"

namespace cg = cooperative_groups;

namespace asu {
namespace {

constexpr int kCluster = 8;                   // CTAs (SMs) of the resolve cluster
constexpr int kThreads = 256;                 // threads per CTA, one top-k entry each
constexpr int kChunk = kCluster * kThreads;   // 2048 entries per chunk
constexpr int kHash = 2 * kChunk;             // per-CTA table: even if every key of a chunk hashes
                                              // to one CTA its load factor stays <= 1/2
constexpr int kCopyThreads = 256;
constexpr int kCopyUnroll = 4;
constexpr int64_t kInClusterMaxRowBytes = 1280;  // kv0 + kv1 bytes per token copied by the resolve cluster itself
constexpr int kInClusterUnroll = 12;             // 16-byte loads in flight per thread in that copy
constexpr int64_t kMaxRowBytes = 1 << 20;     // kv0 + kv1 bytes per token
constexpr int64_t kMaxCopyEntries = 2048;     // per copy launch: kMaxCopyEntries * kMaxRowBytes <= 2^31

__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Claim `tok` in a (possibly remote) table: the smallest position `li` wins.  Returns the
// table index; -1 cannot happen (fewer distinct keys than slots) but ends the probe loop.
__device__ __forceinline__ int hash_claim(int32_t* keys, int32_t* first, uint32_t hv, int32_t tok, int32_t li) {
    uint32_t h = hv & (kHash - 1);
    for (int probe = 0; probe < kHash; ++probe) {
        const int32_t prev = atomicCAS(keys + h, -1, tok);
        if (prev == -1 || prev == tok) {
            atomicMin(first + h, li);
            return static_cast<int>(h);
        }
        h = (h + 1) & (kHash - 1);
    }
    return -1;
}

// Copy kernel: unit u of the flattened (install, unit) space, V-sized units, kCopyUnroll
// independent loads in flight per thread.  The install count and the entries are read
// together (entries past the count lie inside the list and are ignored), so one L2 round
// trip precedes the row loads.
template <typename V>
__global__ void __launch_bounds__(kCopyThreads)
resolver_copy_kernel(const int32_t* __restrict__ ws, int64_t first, uint32_t max_entries,
                     const uint8_t* __restrict__ kv0_src, const uint8_t* __restrict__ kv1_src,
                     uint8_t* __restrict__ kv0_dst, uint8_t* __restrict__ kv1_dst, uint32_t c0, uint32_t c1) {
    asm volatile("griddepcontrol.wait;" ::: "memory");  // the previous grid completed, its writes visible
    const uint32_t cpr = c0 + c1;
    const uint32_t bound = max_entries * cpr;  // < 2^31: max_entries <= kMaxCopyEntries, cpr <= kMaxRowBytes
    const uint32_t stride = gridDim.x * kCopyThreads;
    const V* s0 = reinterpret_cast<const V*>(kv0_src);
    const V* s1 = reinterpret_cast<const V*>(kv1_src);
    V* d0 = reinterpret_cast<V*>(kv0_dst);
    V* d1 = reinterpret_cast<V*>(kv1_dst);
    const int64_t n = static_cast<int64_t>(ld_cg(ws)) - first;  // installs of this launch's range
    ws += 2 * first;
    for (uint32_t u0 = blockIdx.x * kCopyThreads + threadIdx.x; u0 < bound; u0 += stride * kCopyUnroll) {
        V buf[kCopyUnroll];
        V* dst[kCopyUnroll];
#pragma unroll
        for (int u = 0; u < kCopyUnroll; ++u) {
            dst[u] = nullptr;
            const uint32_t uu = u0 + static_cast<uint32_t>(u) * stride;
            if (uu >= bound) continue;
            const uint32_t e = uu / cpr;
            const uint32_t ch = uu - e * cpr;
            const int64_t src = ld_cg(ws + 1 + 2 * e);  // inside the list even past its count
            const int64_t d = ld_cg(ws + 2 + 2 * e);
            if (static_cast<int64_t>(e) >= n || src < 0 || d < 0) continue;
            if (ch < c0) {
                buf[u] = __ldg(s0 + src * c0 + ch);
                dst[u] = d0 + d * c0 + ch;
            } else {
                buf[u] = __ldg(s1 + src * c1 + (ch - c0));
                dst[u] = d1 + d * c1 + (ch - c0);
            }
        }
#pragma unroll
        for (int u = 0; u < kCopyUnroll; ++u)
            if (dst[u]) *dst[u] = buf[u];
        if (static_cast<int64_t>((u0 + stride * kCopyUnroll) / cpr) >= n) break;  // past the last install
    }
}

// Logical block and in-block offset of token `tok` (>= 0) for block size `bs` (> 0), in
// 32-bit arithmetic where bs fits.
__device__ __forceinline__ void block_of(int32_t tok, int64_t bs, int64_t* lb, int64_t* off) {
    if (bs <= 0x7fffffff) {
        const uint32_t b = static_cast<uint32_t>(bs);
        const uint32_t q = static_cast<uint32_t>(tok) / b;
        *lb = q;
        *off = static_cast<uint32_t>(tok) - q * b;
    } else {
        *lb = 0;
        *off = tok;
    }
}

// In-cluster copy of one chunk's installs by one CTA: its `m` installs are listed in shared
// memory in rank order (source row, or -1 for an unusable pop; managed slot), and the CTA's
// threads walk the flattened (install, 16-byte unit) space of the kv0 + kv1 rows with
// kInClusterUnroll independent loads in flight per thread.
__device__ __forceinline__ void copy_installs(const int32_t* s_isrc, const int32_t* s_islot, int m,
                                              const int4* __restrict__ s0, const int4* __restrict__ s1,
                                              int4* __restrict__ d0, int4* __restrict__ d1, uint32_t u0, uint32_t u1) {
    const uint32_t upr = u0 + u1;
    const uint32_t total = static_cast<uint32_t>(m) * upr;  // <= kThreads * kInClusterMaxRowBytes / 16
    for (uint32_t base = threadIdx.x; base < total; base += kThreads * kInClusterUnroll) {
        int4 buf[kInClusterUnroll];
        int4* dst[kInClusterUnroll];
#pragma unroll
        for (int k = 0; k < kInClusterUnroll; ++k) {
            dst[k] = nullptr;
            const uint32_t u = base + static_cast<uint32_t>(k) * kThreads;
            if (u >= total) continue;
            const uint32_t e = u / upr;
            const uint32_t ch = u - e * upr;
            const int64_t src = s_isrc[e];
            if (src < 0) continue;
            const int64_t slot = s_islot[e];
            if (ch < u0) {
                buf[k] = __ldg(s0 + src * u0 + ch);
                dst[k] = d0 + slot * u0 + ch;
            } else {
                buf[k] = __ldg(s1 + src * u1 + (ch - u0));
                dst[k] = d1 + slot * u1 + (ch - u0);
            }
        }
#pragma unroll
        for (int k = 0; k < kInClusterUnroll; ++k)
            if (dst[k]) *dst[k] = buf[k];
    }
}

// The global writes of one install: the token's state and slot, the slot's owner (when the
// popped slot was usable) and its (source row, slot) entry of the install list.
__device__ __forceinline__ void install_writes(int32_t* token_state, int32_t* hbm_slot, int32_t* owner, int32_t* ws,
                                               int32_t tok, bool ok, int32_t slot, int32_t src, int64_t entry) {
    if (ok) {
        st_cg(token_state + tok, ASU_TOKEN_HBM_RESIDENT);
        st_cg(hbm_slot + tok, slot);
        st_cg(owner + slot, tok);
    }
    if (entry >= 0) {
        int32_t* e = ws + 1 + 2 * entry;
        e[0] = src;
        e[1] = slot;
    }
}

__global__ void __cluster_dims__(kCluster, 1, 1) __launch_bounds__(kThreads)
resolve_kernel(const int32_t* __restrict__ topk, int64_t n, int32_t* __restrict__ token_state,
               const int32_t* __restrict__ record, int32_t* __restrict__ hbm_slot, int32_t* __restrict__ owner,
               const int32_t* __restrict__ stack, int32_t* __restrict__ count_ptr, int64_t stack_len,
               const int32_t* __restrict__ block_table, int64_t bt_len, int64_t src_rows, int64_t slot_count,
               int64_t max_seq, int64_t actual, int64_t bs, int32_t* __restrict__ resolved,
               int32_t* __restrict__ ws, int32_t* status, const int4* __restrict__ kv0_src,
               const int4* __restrict__ kv1_src, int4* __restrict__ kv0_dst, int4* __restrict__ kv1_dst, uint32_t u0,
               uint32_t u1) {
    // u0 + u1 > 0: this kernel copies the installed rows itself (u0 / u1 16-byte units per
    // kv0 / kv1 row); 0: the copy kernel launched after it does
    // Launched as a programmatic dependent: the CTAs may be resident before the previous grid on
    // the stream has finished; nothing is read before it has completed and its writes are visible.
    asm volatile("griddepcontrol.wait;" ::: "memory");
    // the next grid (the copy kernel, or the next resolve) may be scheduled from now on; it
    // waits for this grid's completion itself
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    __shared__ int scan_buf[33];
    __shared__ int32_t h_key[kHash];        // token id; reused for the installed slot after ranking
    __shared__ int32_t h_first[kHash];      // first chunk position of the token
    __shared__ int32_t s_stack[kThreads];   // free_slot_stack[count - 1 - (rank * kThreads + t)]
    __shared__ int32_t s_counts[kCluster];  // first occurrences per CTA of the cluster
    __shared__ int32_t s_isrc[kThreads];    // this CTA's installs of the chunk in rank order: source row
    __shared__ int32_t s_islot[kThreads];   // ... and managed slot
    cg::cluster_group cluster = cg::this_cluster();
    const int rank = static_cast<int>(cluster.block_rank());
    const int tid = threadIdx.x;
    const int32_t li = rank * kThreads + tid;  // position inside the chunk
    int32_t count = ld_cg(count_ptr);
    int32_t bits = 0;
    int64_t n_inst = 0;
    const int64_t limit = actual < max_seq ? actual : max_seq;
    for (int64_t base = 0; base < n; base += kChunk) {
        for (int i = tid; i < kHash; i += kThreads) {
            h_key[i] = -1;
            h_first[i] = INT32_MAX;
        }
        {
            const int64_t c = static_cast<int64_t>(count) - 1 - li;
            s_stack[tid] = (c >= 0 && c < stack_len) ? __ldg(stack + c) : kNotFound;
        }
        const int64_t pos = base + li;
        int32_t tok = pos < n ? __ldg(topk + pos) : -1;
        int32_t st = ASU_TOKEN_INVALID, hs = kNotFound, rec = -1, btv = -1;
        if (pos < n && (tok < 0 || tok >= limit)) {
            bits |= ASU_ST_BAD_QUERY;
            tok = -1;
        }
        int64_t lb = 0, boff = 0;
        if (tok >= 0) {
            block_of(tok, bs, &lb, &boff);
            st = ld_cg(token_state + tok);
            hs = ld_cg(hbm_slot + tok);
            rec = __ldg(record + tok);
            if (lb < bt_len) btv = __ldg(block_table + lb);
        }
        cluster_sync_all();  // every table of the cluster cleared
        int32_t slot = kNotFound, w_slot = kNotFound, w_src = -1;
        int64_t w_entry = -1;
        bool w_ok = false;
        int h = -1;
        int32_t* home_key = nullptr;
        int32_t* home_first = nullptr;
        bool miss = false;
        if (tok >= 0) {
            if (st == ASU_TOKEN_HBM_RESIDENT) {
                slot = hs;
            } else if (st == ASU_TOKEN_ASU_ONLY || st == ASU_TOKEN_TAIL_HBM) {
                const uint32_t hv = hash32(static_cast<uint32_t>(tok));
                const unsigned home = hv & (kCluster - 1);
                home_key = cluster.map_shared_rank(h_key, home);
                home_first = cluster.map_shared_rank(h_first, home);
                h = hash_claim(home_key, home_first, hv >> 3, tok, li);
                miss = h >= 0;
                if (h < 0) bits |= ASU_ST_BAD_STATE;
            } else {
                bits |= ASU_ST_BAD_TOKEN_STATE;
            }
        }
        cluster_sync_all();  // every claim made
        const int canon = miss && home_first[h] == li;
        int m = 0;
        const int local_rank = block_exclusive_scan(canon, scan_buf, &m);
        if (tid < kCluster) cluster.map_shared_rank(s_counts, tid)[rank] = m;
        cluster_sync_all();  // per-CTA totals everywhere; every table read done (h_key is free)
        int offset = 0, M = 0;
#pragma unroll
        for (int q = 0; q < kCluster; ++q) {
            const int v = s_counts[q];
            offset += q < rank ? v : 0;
            M += v;
        }
        if (canon) {
            const int32_t k = offset + local_rank;
            const int64_t c = static_cast<int64_t>(count) - 1 - k;
            int32_t s = kNotFound;
            int64_t src = -1;
            bool ok = false;
            if (c >= 0 && c >= stack_len) {
                bits |= ASU_ST_BAD_STATE;  // free_slot_count exceeds the stack
            } else if (c >= 0) {
                s = cluster.map_shared_rank(s_stack, static_cast<unsigned>(k / kThreads))[k % kThreads];
                if (st == ASU_TOKEN_ASU_ONLY) src = rec;
                else if (lb < bt_len) src = static_cast<int64_t>(btv) * bs + boff;
                if (src < 0 || src >= src_rows) bits |= ASU_ST_BAD_SOURCE;
                else if (s < 0 || s >= slot_count) bits |= ASU_ST_BAD_STATE;
                else ok = true;
            } else {
                bits |= ASU_ST_FREE_EXHAUSTED;
            }
            slot = ok ? s : kNotFound;
            home_key[h] = slot;
            w_ok = ok;
            w_slot = s;
            w_src = ok ? static_cast<int32_t>(src) : -1;
            w_entry = c >= 0 ? n_inst + k : -1;  // a popped entry, usable or not, keeps its place
            s_isrc[local_rank] = w_src;
            s_islot[local_rank] = s;
        }
        // The global writes of the last chunk wait until after its final cluster barrier: a
        // barrier's release would otherwise wait for them to reach L2.  An earlier chunk writes
        // before its final barrier, whose release/acquire makes the installs visible to the
        // next chunk's state loads in every CTA.
        const bool last = base + kChunk >= n;
        if (!last && canon) install_writes(token_state, hbm_slot, owner, ws, tok, w_ok, w_slot, w_src, w_entry);
        cluster_sync_all();  // first-occurrence slots published
        if (miss && !canon) slot = home_key[h];  // later duplicate of a token installed in this chunk
        if (!last && pos < n) resolved[pos] = slot;
        const int32_t popped = M < count ? M : (count > 0 ? count : 0);
        count -= popped;
        n_inst += popped;
        cluster_sync_all();  // no CTA reads another's tables any more: next chunk / exit
        if (last) {
            if (canon) install_writes(token_state, hbm_slot, owner, ws, tok, w_ok, w_slot, w_src, w_entry);
            if (pos < n) resolved[pos] = slot;
        }
        // the chunk's rows; the next chunk rewrites the lists only after its third barrier
        if (u0 + u1 > 0) copy_installs(s_isrc, s_islot, m, kv0_src, kv1_src, kv0_dst, kv1_dst, u0, u1);
    }
    if (rank == 0 && tid == 0) {
        st_cg(count_ptr, count);
        ws[0] = static_cast<int32_t>(n_inst);
    }
    if (bits) flag_status(status, 0, bits);
}

template <typename V>
int launch_copy(cudaStream_t s, int64_t grid, const int32_t* ws, int64_t first, int64_t entries, const void* kv0_src,
                const void* kv1_src, void* kv0_dst, void* kv1_dst, uint32_t c0, uint32_t c1) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<uint32_t>(grid));
    cfg.blockDim = dim3(kCopyThreads);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, resolver_copy_kernel<V>, ws, first, static_cast<uint32_t>(entries),
                                             static_cast<const uint8_t*>(kv0_src), static_cast<const uint8_t*>(kv1_src),
                                             static_cast<uint8_t*>(kv0_dst), static_cast<uint8_t*>(kv1_dst), c0, c1);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return ASU_ERR_CUDA_BASE + static_cast<int>(e);
    }
    return ASU_OK;
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
    if (kv0_row_bytes + kv1_row_bytes > kMaxRowBytes) return ASU_ERR_ARG;
    // widest copy unit that every row start divides (0: nothing to copy)
    const uintptr_t align = (kv0_row_bytes > 0 ? reinterpret_cast<uintptr_t>(kv0_src) |
                                                     reinterpret_cast<uintptr_t>(kv0_dst) |
                                                     static_cast<uintptr_t>(kv0_row_bytes)
                                               : 0) |
                            (kv1_row_bytes > 0 ? reinterpret_cast<uintptr_t>(kv1_src) |
                                                     reinterpret_cast<uintptr_t>(kv1_dst) |
                                                     static_cast<uintptr_t>(kv1_row_bytes)
                                               : 0);
    const int vec = (kv0_row_bytes == 0 && kv1_row_bytes == 0) ? 0 : (align & 15) == 0 ? 16 : (align & 3) == 0 ? 4 : 1;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    int32_t* ws = static_cast<int32_t*>(workspace);
    // Small 16-byte-aligned row pairs (DSA / MLA token rows) are copied by the resolve cluster
    // as it installs them, which saves the copy launch; larger rows go to the copy kernel,
    // which spreads them over the whole GPU.
    const bool in_cluster = vec == 16 && kv0_row_bytes + kv1_row_bytes <= kInClusterMaxRowBytes;
    const uint32_t u0 = in_cluster ? static_cast<uint32_t>(kv0_row_bytes / 16) : 0;
    const uint32_t u1 = in_cluster ? static_cast<uint32_t>(kv1_row_bytes / 16) : 0;
    {
        // programmatic stream serialization: the cluster is scheduled while the previous grid
        // drains (the kernel's griddepcontrol.wait keeps stream order for its memory accesses)
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(kCluster);
        cfg.blockDim = dim3(kThreads);
        cfg.dynamicSmemBytes = 0;
        cfg.stream = s;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        const cudaError_t e = cudaLaunchKernelEx(
            &cfg, resolve_kernel, topk, topk_numel, token_state, asu_record_addr, hbm_slot_of_token, slot_owner_token,
            free_slot_stack, free_slot_count, free_slot_stack_len, block_table, block_table_len, src_rows, slot_count,
            max_seq_len, actual_seq_len, block_size, resolved, ws, status, static_cast<const int4*>(kv0_src),
            static_cast<const int4*>(kv1_src), static_cast<int4*>(kv0_dst), static_cast<int4*>(kv1_dst), u0, u1);
        if (e != cudaSuccess) {
            cudaGetLastError();
            return ASU_ERR_CUDA_BASE + static_cast<int>(e);
        }
    }
    int rc = asu_launch_status();
    if (rc != ASU_OK || vec == 0 || in_cluster) return rc;
    // one copy launch per kMaxCopyEntries install-list entries (one for any top-k up to that size)
    for (int64_t first = 0; first < topk_numel && rc == ASU_OK; first += kMaxCopyEntries) {
        const int64_t entries = topk_numel - first < kMaxCopyEntries ? topk_numel - first : kMaxCopyEntries;
        const uint32_t c0 = static_cast<uint32_t>(kv0_row_bytes / vec), c1 = static_cast<uint32_t>(kv1_row_bytes / vec);
        int64_t grid = (entries * (c0 + c1) + kCopyThreads * kCopyUnroll - 1) / (kCopyThreads * kCopyUnroll);
        const int64_t cap = static_cast<int64_t>(asu_sm_count()) * 4;
        if (grid > cap) grid = cap;
        if (grid < 1) grid = 1;
        rc = vec == 16 ? launch_copy<int4>(s, grid, ws, first, entries, kv0_src, kv1_src, kv0_dst, kv1_dst, c0, c1)
           : vec == 4  ? launch_copy<int32_t>(s, grid, ws, first, entries, kv0_src, kv1_src, kv0_dst, kv1_dst, c0, c1)
                       : launch_copy<uint8_t>(s, grid, ws, first, entries, kv0_src, kv1_src, kv0_dst, kv1_dst, c0, c1);
    }
    return rc;
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
