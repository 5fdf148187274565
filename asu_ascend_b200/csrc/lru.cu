// Exact LRU slot pool, one pool per request row: step-boundary maintain + resolve in one kernel.
//
// Reference behaviour: LRUManagedCache in simu/kv_cache_eviction_sim.py
//   prepare_free_slots :124-131  popitem(last=False) until free >= target; each victim slot is
//                                appended to the free list (the list's end is the top)
//   resolve_query      :133-150  hit -> move_to_end; miss -> free.pop() (top); empty -> shortage
//   free list init     :109      [S-1, ..., 0], so the first pops return 0, 1, 2, ...
//
// State layout (int32, row-major by request):
//   token_to_slot [R, K]  slot_to_token [R, S]
//   lru_order     [R, S]  first S - free_count entries: resident slots, LRU first
//   free_stack    [R, S]  first free_count entries, top last
//   free_count    [R]
//
// B200 design: one CTA of 1024 threads per request row, everything in one launch.
//  1. Eviction needs no sort: the victims are the head of lru_order.  Each is unmapped and
//     pushed on the free stack in order (evicted keys are written in eviction order).
//  2. Lookup: queries are thread-contiguous; the first occurrence of each missing key is
//     found with an atomicMin claim (INT32_MIN + position) on its token_to_slot entry; a
//     block scan ranks first occurrences in query order and rank k pops
//     free_stack[free - 1 - k].  Later duplicates read the installed slot (serially they
//     are hits).  Every touch records its position with a shared-memory atomicMax on
//     last_pos[slot], so the last occurrence of a slot is known.
//  3. The new LRU order is [untouched residents in old order] ++ [touched slots ordered by
//     their last touching position] -- exactly the OrderedDict order after the serial
//     loop.  Both parts are stable compactions done with two block scans; the remaining
//     old order was held in registers, so the order row is rewritten in place.
// Per step and request the kernel reads/writes the order row once (8*S bytes) plus 14
// bytes per query; no global scratch.
#include "asu_common.cuh"

namespace asu {
namespace {

constexpr int kThreads = 1024;

enum : uint8_t { kInvalid = 0, kHit = 1, kMiss = 2 };

template <int IPT_Q, int IPT_S>
__global__ void __launch_bounds__(kThreads)
lru_step_kernel(int32_t* __restrict__ t2s, int32_t* __restrict__ s2t, int32_t* __restrict__ order,
                int32_t* __restrict__ stack, int32_t* __restrict__ count, const int32_t* __restrict__ query,
                int32_t* __restrict__ slot_out, uint8_t* __restrict__ hit_mask, uint8_t* __restrict__ install_mask,
                int32_t* __restrict__ evicted, uint32_t ev_stride, int32_t* __restrict__ ev_count,
                int64_t* __restrict__ stats, int32_t* status, uint32_t req_num, uint32_t K, uint32_t S, uint32_t Q,
                uint32_t target) {
    extern __shared__ int32_t last_pos[];  // [S]
    __shared__ int scan_buf[33];
    __shared__ int n_hits, n_valid;
    const int tid = threadIdx.x;
    for (uint32_t r = blockIdx.x; r < req_num; r += gridDim.x) {
        int32_t* trow = t2s + static_cast<uint64_t>(r) * K;
        int32_t* srow = s2t + static_cast<uint64_t>(r) * S;
        int32_t* orow = order + static_cast<uint64_t>(r) * S;
        int32_t* krow = stack + static_cast<uint64_t>(r) * S;
        const int32_t* qrow = query + static_cast<uint64_t>(r) * Q;
        int32_t bits = 0;

        const int32_t free0 = ld_cg(count + r);
        if (free0 < 0 || free0 > static_cast<int32_t>(S)) {  // uniform across the block
            if (tid == 0) flag_status(status, r, ASU_ST_BAD_STATE);
            continue;
        }
        const int32_t resident0 = static_cast<int32_t>(S) - free0;
        const int32_t tgt = static_cast<int32_t>(target < S ? target : S);
        int32_t E = 0;
        if (free0 < tgt) E = (tgt - free0) < resident0 ? (tgt - free0) : resident0;

        if (tid == 0) {
            n_hits = 0;
            n_valid = 0;
        }
        for (uint32_t s = tid; s < S; s += kThreads) last_pos[s] = -1;

        // ---- 1. eviction: victims are lru_order[0, E) ----
        for (int32_t k = tid; k < E; k += kThreads) {
            const int32_t v = ld_cg(orow + k);
            int32_t key = kNotFound;
            if (static_cast<uint32_t>(v) < S) {
                key = ld_cg(srow + v);
                if (static_cast<uint32_t>(key) < K) st_cg(trow + key, kNotFound);
                else bits |= ASU_ST_BAD_STATE;
                st_cg(srow + v, kNotFound);
                st_cg(krow + free0 + k, v);
            } else {
                bits |= ASU_ST_BAD_STATE;
            }
            if (static_cast<uint32_t>(k) < ev_stride) evicted[static_cast<uint64_t>(r) * ev_stride + k] = key;
        }
        if (tid == 0) ev_count[r] = E;
        const int32_t n_rem = resident0 - E;
        int32_t oldv[IPT_S];
#pragma unroll
        for (int j = 0; j < IPT_S; ++j) {
            const int32_t idx = tid * IPT_S + j;
            oldv[j] = idx < n_rem ? ld_cg(orow + E + idx) : -1;
        }
        const int32_t free1 = free0 + E;
        __syncthreads();

        // ---- 2. lookup ----
        int32_t key[IPT_Q], slot[IPT_Q];
        uint8_t st[IPT_Q];
        int valid_local = 0;
#pragma unroll
        for (int j = 0; j < IPT_Q; ++j) {
            const uint32_t pos = tid * IPT_Q + j;
            key[j] = -1;
            slot[j] = kNotFound;
            st[j] = kInvalid;
            if (pos < Q) {
                key[j] = __ldg(qrow + pos);
                if (static_cast<uint32_t>(key[j]) < K) {
                    ++valid_local;
                    const int32_t v = ld_cg(trow + key[j]);
                    if (v >= 0 && static_cast<uint32_t>(v) < S) {
                        st[j] = kHit;
                        slot[j] = v;
                    } else if (v == kNotFound) {
                        st[j] = kMiss;
                    } else {
                        bits |= ASU_ST_BAD_STATE;
                    }
                } else {
                    bits |= ASU_ST_BAD_QUERY;
                }
            }
        }
        __syncthreads();  // all pre-step values read before any claim lands
#pragma unroll
        for (int j = 0; j < IPT_Q; ++j) {
            const int32_t pos = tid * IPT_Q + j;
            if (st[j] == kMiss) atomicMin(trow + key[j], kClaimBase + pos);
            else if (st[j] == kHit) atomicMax(&last_pos[slot[j]], pos);
        }
        __syncthreads();
        int canon[IPT_Q];
        int local = 0;
#pragma unroll
        for (int j = 0; j < IPT_Q; ++j) {
            const int32_t pos = tid * IPT_Q + j;
            canon[j] = st[j] == kMiss && ld_cg(trow + key[j]) == kClaimBase + pos;
            local += canon[j];
        }
        int n_canon = 0;
        int rank = block_exclusive_scan(local, scan_buf, &n_canon);
        uint8_t inst[IPT_Q];
#pragma unroll
        for (int j = 0; j < IPT_Q; ++j) {
            inst[j] = 0;
            if (!canon[j]) continue;
            const int32_t pos = tid * IPT_Q + j;
            const int32_t k = rank++;
            int32_t s = kNotFound;
            if (k < free1) {
                s = ld_cg(krow + (free1 - 1 - k));
                if (static_cast<uint32_t>(s) >= S) {
                    bits |= ASU_ST_BAD_STATE;
                    s = kNotFound;
                }
            }
            st_cg(trow + key[j], s);
            if (s >= 0) {
                st_cg(srow + s, key[j]);
                atomicMax(&last_pos[s], pos);
                inst[j] = 1;
            } else {
                bits |= ASU_ST_SHORTAGE;
            }
            slot[j] = s;
        }
        const int32_t n_inst = n_canon < free1 ? n_canon : free1;
        const int32_t free2 = free1 - n_inst;
        __syncthreads();
        int hits_local = 0;
#pragma unroll
        for (int j = 0; j < IPT_Q; ++j) {
            const int32_t pos = tid * IPT_Q + j;
            bool hit = st[j] == kHit;
            if (st[j] == kMiss && !canon[j]) {  // later duplicate of a missing key
                const int32_t v = ld_cg(trow + key[j]);
                if (v >= 0) {
                    slot[j] = v;
                    hit = true;
                    atomicMax(&last_pos[v], pos);
                }
            }
            hits_local += hit;
            if (static_cast<uint32_t>(pos) < Q) {
                const uint64_t o = static_cast<uint64_t>(r) * Q + pos;
                slot_out[o] = slot[j];
                hit_mask[o] = hit;
                install_mask[o] = inst[j];
            }
        }
        if (hits_local) atomicAdd(&n_hits, hits_local);
        if (valid_local) atomicAdd(&n_valid, valid_local);
        __syncthreads();

        // ---- 3. new LRU order ----
        int keep_local = 0;
        bool keep[IPT_S];
#pragma unroll
        for (int j = 0; j < IPT_S; ++j) {
            keep[j] = static_cast<uint32_t>(oldv[j]) < S && last_pos[oldv[j]] == -1;
            if (tid * IPT_S + j < n_rem && static_cast<uint32_t>(oldv[j]) >= S) bits |= ASU_ST_BAD_STATE;
            keep_local += keep[j];
        }
        int n_keep = 0;
        int a = block_exclusive_scan(keep_local, scan_buf, &n_keep);
        int touched_local = 0;
        bool touched[IPT_Q];
#pragma unroll
        for (int j = 0; j < IPT_Q; ++j) {
            const int32_t pos = tid * IPT_Q + j;
            touched[j] = slot[j] >= 0 && last_pos[slot[j]] == pos;
            touched_local += touched[j];
        }
        int n_touched = 0;
        int b = block_exclusive_scan(touched_local, scan_buf, &n_touched);
        // A consistent state has n_keep + n_touched == S - free2 <= S; the bounds guard only
        // matters for corrupt input (duplicate slots across the maps), which is flagged below.
#pragma unroll
        for (int j = 0; j < IPT_S; ++j) {
            if (keep[j]) {
                if (a < static_cast<int>(S)) st_cg(orow + a, oldv[j]);
                ++a;
            }
        }
#pragma unroll
        for (int j = 0; j < IPT_Q; ++j) {
            if (touched[j]) {
                const int o = n_keep + b++;
                if (o < static_cast<int>(S)) st_cg(orow + o, slot[j]);
            }
        }
        if (tid == 0) {
            st_cg(count + r, free2);
            if (n_keep + n_touched != static_cast<int>(S) - free2) bits |= ASU_ST_BAD_STATE;
            if (stats != nullptr) {
                int64_t* row = stats + static_cast<uint64_t>(r) * ASU_LRU_STAT_COLS;
                row[ASU_LRU_STAT_HITS] += n_hits;
                row[ASU_LRU_STAT_MISSES] += n_valid - n_hits;
                row[ASU_LRU_STAT_INSTALLS] += n_inst;
                row[ASU_LRU_STAT_SHORTAGES] += n_valid - n_hits - n_inst;
                row[ASU_LRU_STAT_EVICTIONS] += E;
            }
        }
        if (bits) flag_status(status, r, bits);
        __syncthreads();
    }
}

template <int IPT_Q, int IPT_S>
int launch_lru(cudaStream_t s, int32_t* t2s, int32_t* s2t, int32_t* order, int32_t* stack, int32_t* count,
               const int32_t* query, int32_t* slot_out, uint8_t* hit, uint8_t* inst, int32_t* evicted,
               uint32_t ev_stride, int32_t* ev_count, int64_t* stats, int32_t* status, uint32_t R, uint32_t K,
               uint32_t S, uint32_t Q, uint32_t target) {
    static unsigned long long configured = 0;  // one bit per device: the attribute is per context
    const int smem = static_cast<int>(S * sizeof(int32_t));
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && !((configured >> dev) & 1ull)) {
        cudaError_t e = cudaFuncSetAttribute(lru_step_kernel<IPT_Q, IPT_S>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             kThreads * IPT_S * static_cast<int>(sizeof(int32_t)));
        if (e != cudaSuccess) return ASU_ERR_CUDA_BASE + static_cast<int>(e);
        configured |= 1ull << dev;
    }
    const uint32_t grid = R < 65535u ? R : 65535u;
    lru_step_kernel<IPT_Q, IPT_S><<<grid, kThreads, smem, s>>>(t2s, s2t, order, stack, count, query, slot_out, hit,
                                                                 inst, evicted, ev_stride, ev_count, stats, status,
                                                                 R, K, S, Q, target);
    return asu_launch_status();
}

template <int IPT_Q>
int dispatch_s(uint32_t S, cudaStream_t s, int32_t* t2s, int32_t* s2t, int32_t* order, int32_t* stack,
               int32_t* count, const int32_t* query, int32_t* slot_out, uint8_t* hit, uint8_t* inst,
               int32_t* evicted, uint32_t ev_stride, int32_t* ev_count, int64_t* stats, int32_t* status, uint32_t R,
               uint32_t K, uint32_t Q, uint32_t target) {
#define ASU_LRU_CASE(N)                                                                                           \
    if (S <= static_cast<uint32_t>(kThreads * N))                                                                 \
        return launch_lru<IPT_Q, N>(s, t2s, s2t, order, stack, count, query, slot_out, hit, inst, evicted, ev_stride, \
                                    ev_count, stats, status, R, K, S, Q, target);
    ASU_LRU_CASE(2)
    ASU_LRU_CASE(4)
    ASU_LRU_CASE(8)
    ASU_LRU_CASE(16)
#undef ASU_LRU_CASE
    return ASU_ERR_ARG;
}

}  // namespace
}  // namespace asu

using namespace asu;

extern "C" int asu_lru_step(void* stream, int32_t* token_to_slot, int32_t* slot_to_token, int32_t* lru_order,
                            int32_t* free_stack, int32_t* free_count, const int32_t* query, int32_t* slot_out,
                            uint8_t* hit_mask, uint8_t* install_mask, int32_t* evicted, uint32_t evicted_stride,
                            int32_t* evicted_count, int64_t* stats, int32_t* status, uint32_t req_num,
                            uint32_t key_space, uint32_t slot_count, uint32_t query_count, uint32_t free_target) {
    if (req_num == 0) return ASU_OK;
    if (!token_to_slot || !slot_to_token || !lru_order || !free_stack || !free_count || !evicted_count ||
        (query_count && (!query || !slot_out || !hit_mask || !install_mask)))
        return ASU_ERR_ARG;
    if (key_space == 0 || key_space > 0x7fffffffu || slot_count == 0 || slot_count > 16384u ||
        query_count > 8192u)
        return ASU_ERR_ARG;
    const uint32_t tgt = free_target < slot_count ? free_target : slot_count;
    if (tgt > 0 && (evicted == nullptr || evicted_stride < tgt)) return ASU_ERR_ARG;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (query_count <= 2048u)
        return dispatch_s<2>(slot_count, s, token_to_slot, slot_to_token, lru_order, free_stack, free_count, query,
                             slot_out, hit_mask, install_mask, evicted, evicted_stride, evicted_count, stats, status,
                             req_num, key_space, query_count, free_target);
    if (query_count <= 4096u)
        return dispatch_s<4>(slot_count, s, token_to_slot, slot_to_token, lru_order, free_stack, free_count, query,
                             slot_out, hit_mask, install_mask, evicted, evicted_stride, evicted_count, stats, status,
                             req_num, key_space, query_count, free_target);
    return dispatch_s<8>(slot_count, s, token_to_slot, slot_to_token, lru_order, free_stack, free_count, query,
                         slot_out, hit_mask, install_mask, evicted, evicted_stride, evicted_count, stats, status,
                         req_num, key_space, query_count, free_target);
}
