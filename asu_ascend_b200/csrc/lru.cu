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
// B200 design: one CTA of 1024 threads per request row, everything in one launch, with
// the global round trips taken off the critical path:
//  * At launch every thread issues its loads together: the free count, the whole order
//    row (coalesced into shared memory) and the token_to_slot gathers of its queries.
//  * Eviction needs no sort: the victims are the head of the order row.  They are marked
//    in shared memory (last_pos = -2), so a query that read a victim's slot before the
//    eviction landed is classified as a miss -- exactly what the serial order (evict,
//    then resolve) gives.  The victims' keys are loaded while the table gathers are in flight
//    and unmapped after the classification (one barrier before any install).
//  * The first occurrence of each missing key is found in a shared-memory hash table
//    (atomicMin of the position per key); a block scan ranks first occurrences in query
//    order and rank k pops the free stack: the victims just pushed (top first), then the
//    older entries, read on demand (none at the steady state).  Later duplicates read the
//    installed slot from the hash entry (serially they are hits).
//  * Every touch records its position in last_pos[slot] (shared-memory atomicMax); the
//    new order is [untouched residents in old order] ++ [touched slots by last touching
//    position] -- the OrderedDict order after the serial loop -- built with two block
//    scans in shared memory and written back with coalesced stores.
// No global scratch; the row is read once and written once.
#include "asu_common.cuh"

namespace asu {
namespace {

constexpr int kThreads = 1024;
constexpr int32_t kVictim = -2;  // last_pos marker of a slot evicted in this step
constexpr int32_t kEmptyKey = -1;

enum : uint8_t { kInvalid = 0, kHit = 1, kMiss = 2, kBad = 3 };

__device__ __forceinline__ uint32_t hash_slot(int32_t key, int log2h) {
    return (static_cast<uint32_t>(key) * 0x9E3779B1u) >> (32 - log2h);
}

// kCopyQuery: `query` may be pinned, mapped host memory (read over the host link, so a host caller
// needs no upload of its own), and every query is also stored to query_copy [R, Q] in HBM for the
// swap-in that follows.
template <int IPT_Q, int IPT_S, bool kCopyQuery>
__global__ void __launch_bounds__(kThreads)
lru_step_kernel(int32_t* __restrict__ t2s, int32_t* __restrict__ s2t, int32_t* __restrict__ order,
                int32_t* __restrict__ stack, int32_t* __restrict__ count, const int32_t* __restrict__ query,
                int32_t* __restrict__ query_copy, int32_t* __restrict__ slot_out, uint8_t* __restrict__ hit_mask,
                uint8_t* __restrict__ install_mask, int32_t* __restrict__ evicted, uint32_t ev_stride,
                int32_t* __restrict__ ev_count, int64_t* __restrict__ stats, int32_t* status, uint32_t req_num,
                uint32_t K, uint32_t S, uint32_t Q, uint32_t target, int log2h) {
    pdl_wait();     // launched with launch_pdl: stream order for every access below
    pdl_trigger();  // the swap-in that consumes this step may be scheduled now
    extern __shared__ int32_t smem[];
    const uint32_t H = 1u << log2h;
    const uint32_t Sp = (S + 3) & ~3u;  // row length rounded up to 16 bytes
    int32_t* s_order = smem;            // [Sp] old order row, later the new one
    int32_t* s_last = s_order + Sp;     // [Sp] last touching position (-1 untouched, -2 victim)
    int32_t* s_hkey = s_last + Sp;      // [H]  hash: key
    int32_t* s_hpos = s_hkey + H;       // [H]  hash: first position of the key
    int32_t* s_hmax = s_hpos + H;       // [H]  hash: last position of the key
    int32_t* s_hval = s_hmax + H;       // [H]  hash: installed slot
    __shared__ int scan_a[32], scan_b[32];  // alternating buffers of the one-barrier block scans
    __shared__ int n_hits, n_valid;
    const int tid = threadIdx.x;
    // victims held in registers per thread (positions tid + i * kThreads); more than
    // kVict * kThreads victims (a free target above 4096) are unmapped at once in P0
    constexpr int kVict = IPT_S < 4 ? IPT_S : 4;

    for (uint32_t r = blockIdx.x; r < req_num; r += gridDim.x) {
        int32_t* trow = t2s + static_cast<uint64_t>(r) * K;
        int32_t* srow = s2t + static_cast<uint64_t>(r) * S;
        int32_t* orow = order + static_cast<uint64_t>(r) * S;
        int32_t* krow = stack + static_cast<uint64_t>(r) * S;
        const int32_t* qrow = query + static_cast<uint64_t>(r) * Q;
        int32_t bits = 0;

        // ---- P0: loads, shared-memory set-up and the eviction's marks, one phase ----
        // Every independent load is issued first: the free count, the order row (16-byte loads
        // into registers), the queries and their token_to_slot gathers.  The victims are the head
        // of the order row, lru_order[0, E), E = min(target - free, residents); each thread loads
        // its victim entries itself as soon as the count is in, marks them in shared memory
        // (last_pos = -2, so a query that reads a victim's slot is classified as a miss -- the
        // serial evict-then-resolve order) and loads their keys, which the unmapping after the
        // classification consumes.  Residents that survive get last_pos = -1 from the thread that
        // loaded their order entry; free slots get theirs when they are popped.
        const int32_t free0 = ld_cg(count + r);
        const bool vec_row = (S % 4 == 0) && (reinterpret_cast<uintptr_t>(orow) % 16 == 0);
        constexpr int kVec = (IPT_S + 3) / 4;
        int4 ov[kVec];
        if (vec_row) {
            const int4* src = reinterpret_cast<const int4*>(orow);
#pragma unroll
            for (int j = 0; j < kVec; ++j)
                if (tid + j * kThreads < S / 4) ov[j] = __ldcg(src + tid + j * kThreads);
        }
        int32_t key[IPT_Q], g[IPT_Q];
#pragma unroll
        for (int j = 0; j < IPT_Q; ++j) {
            const uint32_t pos = tid * IPT_Q + j;
            key[j] = -1;
            g[j] = kNotFound;
            if (pos < Q) {
                key[j] = __ldg(qrow + pos);
                if (static_cast<uint32_t>(key[j]) < K) g[j] = ld_cg(trow + key[j]);
            }
        }
        if constexpr (kCopyQuery) {
#pragma unroll
            for (int j = 0; j < IPT_Q; ++j) {
                const uint32_t pos = tid * IPT_Q + j;
                if (pos < Q) query_copy[static_cast<uint64_t>(r) * Q + pos] = key[j];
            }
        }
        {
            const int4 m1 = make_int4(-1, -1, -1, -1);
            const int4 big = make_int4(INT32_MAX, INT32_MAX, INT32_MAX, INT32_MAX);
            for (uint32_t i = tid; i < H / 4; i += kThreads) {
                reinterpret_cast<int4*>(s_hkey)[i] = m1;
                reinterpret_cast<int4*>(s_hpos)[i] = big;
                reinterpret_cast<int4*>(s_hmax)[i] = m1;
            }
        }
        if (tid == 0) {
            n_hits = 0;
            n_valid = 0;
        }
        if (free0 < 0 || free0 > static_cast<int32_t>(S)) {  // uniform across the block
            if (tid == 0) flag_status(status, r, ASU_ST_BAD_STATE);
            __syncthreads();
            continue;
        }
        const int32_t resident0 = static_cast<int32_t>(S) - free0;
        const int32_t tgt = static_cast<int32_t>(target < S ? target : S);
        int32_t E = 0;
        if (free0 < tgt) E = (tgt - free0) < resident0 ? (tgt - free0) : resident0;
        const int32_t free1 = free0 + E;

        int32_t vslot[kVict], vkey[kVict];
#pragma unroll
        for (int i = 0; i < kVict; ++i) {
            const int32_t k = tid + i * kThreads;
            vslot[i] = k < E ? ld_cg(orow + k) : kNotFound;
        }
        // the order row into shared memory; last_pos of the surviving residents
        if (vec_row) {
            int4* dst = reinterpret_cast<int4*>(s_order);
#pragma unroll
            for (int j = 0; j < kVec; ++j) {
                const int32_t i4 = tid + j * kThreads;
                if (i4 >= static_cast<int32_t>(S / 4)) continue;
                dst[i4] = ov[j];
                const int32_t v[4] = {ov[j].x, ov[j].y, ov[j].z, ov[j].w};
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    const int32_t k = 4 * i4 + c;
                    if (k >= E && k < resident0 && static_cast<uint32_t>(v[c]) < S) s_last[v[c]] = -1;
                }
            }
        } else {
            for (int32_t k = tid; k < static_cast<int32_t>(S); k += kThreads) {
                const int32_t v = ld_cg(orow + k);
                s_order[k] = v;
                if (k >= E && k < resident0 && static_cast<uint32_t>(v) < S) s_last[v] = -1;
            }
        }
#pragma unroll
        for (int i = 0; i < kVict; ++i) {
            vkey[i] = kNotFound;
            if (tid + i * kThreads >= E) continue;
            if (static_cast<uint32_t>(vslot[i]) < S) {
                s_last[vslot[i]] = kVictim;
                vkey[i] = ld_cg(srow + vslot[i]);
            } else {
                bits |= ASU_ST_BAD_STATE;
            }
        }
        // victims beyond the registers: marked and unmapped here (a racing gather of such a key
        // reads either the victim slot, marked, or -1: a miss either way)
        for (int32_t k = tid + kVict * kThreads; k < E; k += kThreads) {
            const int32_t v = ld_cg(orow + k);
            int32_t vk = kNotFound;
            if (static_cast<uint32_t>(v) < S) {
                s_last[v] = kVictim;
                vk = ld_cg(srow + v);
                if (static_cast<uint32_t>(vk) < K) st_cg(trow + vk, kNotFound);
                else bits |= ASU_ST_BAD_STATE;
                st_cg(srow + v, kNotFound);
                st_cg(krow + free0 + k, v);
            } else {
                bits |= ASU_ST_BAD_STATE;
            }
            if (static_cast<uint32_t>(k) < ev_stride) evicted[static_cast<uint64_t>(r) * ev_stride + k] = vk;
        }
        if (tid == 0) ev_count[r] = E;
        __syncthreads();  // order row, marks and hash set up

        // ---- P2: classify; hits record their position, misses enter the hash ----
        uint8_t st[IPT_Q];
        int32_t hidx[IPT_Q];
        int valid_local = 0;
#pragma unroll
        for (int j = 0; j < IPT_Q; ++j) {
            const int32_t pos = tid * IPT_Q + j;
            st[j] = kInvalid;
            hidx[j] = -1;
            if (static_cast<uint32_t>(pos) >= Q) continue;
            if (static_cast<uint32_t>(key[j]) >= K) {
                bits |= ASU_ST_BAD_QUERY;
                continue;
            }
            ++valid_local;
            const int32_t s = g[j];
            if (s >= 0 && static_cast<uint32_t>(s) < S && s_last[s] != kVictim) {
                st[j] = kHit;
                atomicMax(&s_last[s], pos);
            } else if (s == kNotFound || (s >= 0 && static_cast<uint32_t>(s) < S)) {
                st[j] = kMiss;
                uint32_t h = hash_slot(key[j], log2h);
                while (true) {  // terminates: at most Q <= H distinct keys
                    const int32_t old = atomicCAS(&s_hkey[h], kEmptyKey, key[j]);
                    if (old == kEmptyKey || old == key[j]) break;
                    h = (h + 1) & (H - 1);
                }
                hidx[j] = static_cast<int32_t>(h);
                atomicMin(&s_hpos[h], pos);  // the first position of the key installs
                atomicMax(&s_hmax[h], pos);  // the last one is its slot's last touch
            } else {
                st[j] = kBad;
                bits |= ASU_ST_BAD_STATE;
            }
        }
        // victim unmapping, ordered before any install by the barrier below
#pragma unroll
        for (int i = 0; i < kVict; ++i) {
            const int32_t k = tid + i * kThreads;
            if (k >= E) continue;
            const int32_t v = vslot[i];
            if (static_cast<uint32_t>(v) < S) {
                if (static_cast<uint32_t>(vkey[i]) < K) st_cg(trow + vkey[i], kNotFound);
                else bits |= ASU_ST_BAD_STATE;
                st_cg(srow + v, kNotFound);
                st_cg(krow + free0 + k, v);
            }
            if (static_cast<uint32_t>(k) < ev_stride) evicted[static_cast<uint64_t>(r) * ev_stride + k] = vkey[i];
        }
        __syncthreads();  // every claim made; victims unmapped

        // ---- P3: first occurrences pop the stack in query order ----
        int canon[IPT_Q];
        int local = 0;
#pragma unroll
        for (int j = 0; j < IPT_Q; ++j) {
            canon[j] = st[j] == kMiss && s_hpos[hidx[j]] == static_cast<int32_t>(tid * IPT_Q + j);
            local += canon[j];
        }
        int n_canon = 0;
        int rank = block_exclusive_scan_1b(local, scan_a, &n_canon);
        int32_t slot[IPT_Q];
        uint8_t inst[IPT_Q];
#pragma unroll
        for (int j = 0; j < IPT_Q; ++j) {
            slot[j] = st[j] == kHit ? g[j] : kNotFound;
            inst[j] = 0;
            if (!canon[j]) continue;
            const int32_t k = rank++;
            int32_t s = kNotFound;
            if (k < free1) {
                // the victims just pushed (top first), then the older entries below them,
                // read on demand: at the steady state every pop takes a victim
                s = k < E ? s_order[E - 1 - k] : ld_cg(krow + (free0 - 1 - (k - E)));
                if (static_cast<uint32_t>(s) >= S) {
                    bits |= ASU_ST_BAD_STATE;
                    s = kNotFound;
                }
            }
            s_hval[hidx[j]] = s;
            if (s >= 0) {
                st_cg(trow + key[j], s);
                st_cg(srow + s, key[j]);
                // only this thread touches a popped slot before the next barrier
                s_last[s] = s_hmax[hidx[j]];
                inst[j] = 1;
            } else {
                bits |= ASU_ST_SHORTAGE;
            }
            slot[j] = s;
        }
        const int32_t n_inst = n_canon < free1 ? n_canon : free1;
        const int32_t free2 = free1 - n_inst;
        __syncthreads();  // installed slots and their last touches visible

        // ---- P4: later duplicates of a missing key read its slot; outputs ----
        int hits_local = 0;
#pragma unroll
        for (int j = 0; j < IPT_Q; ++j) {
            const int32_t pos = tid * IPT_Q + j;
            bool hit = st[j] == kHit;
            if (st[j] == kMiss && !canon[j]) {
                const int32_t v = s_hval[hidx[j]];
                if (v >= 0) {
                    slot[j] = v;
                    hit = true;
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
        // one shared-memory atomic per warp, not per thread (1024 adds to one address serialise)
        hits_local = __reduce_add_sync(0xffffffffu, hits_local);
        valid_local = __reduce_add_sync(0xffffffffu, valid_local);
        if ((tid & 31) == 0) {
            if (hits_local) atomicAdd(&n_hits, hits_local);
            if (valid_local) atomicAdd(&n_valid, valid_local);
        }

        // ---- P5: new LRU order ----
        // thread t owns s_order[t*IPT_S, (t+1)*IPT_S); entries in [E, resident0) are the
        // residents that survived the eviction, in LRU order
        int32_t oldv[IPT_S];
        bool keep[IPT_S];
        int keep_local = 0;
        if (tid * IPT_S < static_cast<int>(Sp)) {
            if constexpr (IPT_S % 4 == 0) {
#pragma unroll
                for (int j = 0; j < IPT_S; j += 4) {
                    const int4 v4 = reinterpret_cast<const int4*>(s_order)[(tid * IPT_S + j) / 4];
                    oldv[j] = v4.x;
                    oldv[j + 1] = v4.y;
                    oldv[j + 2] = v4.z;
                    oldv[j + 3] = v4.w;
                }
            } else {
#pragma unroll
                for (int j = 0; j < IPT_S; ++j) oldv[j] = s_order[tid * IPT_S + j];
            }
        } else {
#pragma unroll
            for (int j = 0; j < IPT_S; ++j) oldv[j] = -1;
        }
#pragma unroll
        for (int j = 0; j < IPT_S; ++j) {
            const int32_t idx = tid * IPT_S + j;
            const bool live = idx >= E && idx < resident0;
            keep[j] = live && static_cast<uint32_t>(oldv[j]) < S && s_last[oldv[j]] == -1;
            if (live && static_cast<uint32_t>(oldv[j]) >= S) bits |= ASU_ST_BAD_STATE;
            keep_local += keep[j];
        }
        bool touched[IPT_Q];
        int touched_local = 0;
#pragma unroll
        for (int j = 0; j < IPT_Q; ++j) {
            touched[j] = slot[j] >= 0 && s_last[slot[j]] == static_cast<int32_t>(tid * IPT_Q + j);
            touched_local += touched[j];
        }
        // one scan for both counts: kept residents in the low 16 bits (<= S <= 16384), touched
        // slots in the high bits (<= Q <= 4096); its barrier ends all reads of the old order
        int packed_total = 0;
        const int packed = block_exclusive_scan_1b(keep_local | (touched_local << 16), scan_b, &packed_total);
        int a = packed & 0xffff;
        int b = packed >> 16;
        const int n_keep = packed_total & 0xffff;
        const int n_touched = packed_total >> 16;
        // A consistent state has n_keep + n_touched == S - free2 <= S; the guards only matter
        // for corrupt input (duplicate slots across the maps), which is flagged below.
#pragma unroll
        for (int j = 0; j < IPT_S; ++j) {
            if (keep[j]) {
                if (a < static_cast<int>(S)) s_order[a] = oldv[j];
                ++a;
            }
        }
#pragma unroll
        for (int j = 0; j < IPT_Q; ++j) {
            if (touched[j]) {
                const int o = n_keep + b++;
                if (o < static_cast<int>(S)) s_order[o] = slot[j];
            }
        }
        __syncthreads();
        const int n_new = min(n_keep + n_touched, static_cast<int>(S));
        if (vec_row) {
            const int n4 = n_new / 4;
            for (int i = tid; i < n4; i += kThreads)
                __stcg(reinterpret_cast<int4*>(orow) + i, reinterpret_cast<const int4*>(s_order)[i]);
            for (int i = n4 * 4 + tid; i < n_new; i += kThreads) st_cg(orow + i, s_order[i]);
        } else {
            for (int i = tid; i < n_new; i += kThreads) st_cg(orow + i, s_order[i]);
        }
        if (tid == 0) {
            st_cg(count + r, free2);
            if (n_keep + n_touched != static_cast<int>(S) - free2) bits |= ASU_ST_BAD_STATE;
            if (stats != nullptr) {  // reductions without a return value: nothing to wait for
                unsigned long long* row =
                    reinterpret_cast<unsigned long long*>(stats + static_cast<uint64_t>(r) * ASU_LRU_STAT_COLS);
                atomicAdd(row + ASU_LRU_STAT_HITS, static_cast<unsigned long long>(n_hits));
                atomicAdd(row + ASU_LRU_STAT_MISSES, static_cast<unsigned long long>(n_valid - n_hits));
                atomicAdd(row + ASU_LRU_STAT_INSTALLS, static_cast<unsigned long long>(n_inst));
                atomicAdd(row + ASU_LRU_STAT_SHORTAGES, static_cast<unsigned long long>(n_valid - n_hits - n_inst));
                atomicAdd(row + ASU_LRU_STAT_EVICTIONS, static_cast<unsigned long long>(E));
            }
        }
        if (bits) flag_status(status, r, bits);
        if (r + gridDim.x < req_num) __syncthreads();  // shared memory is reused by the next request
    }
}

inline uint32_t pow2ceil(uint32_t x) {
    uint32_t p = 1;
    while (p < x) p <<= 1;
    return p;
}

// Dynamic shared memory of one launch: order + last_pos rows and the hash table.
inline size_t lru_smem_bytes(uint32_t S, uint32_t Q, int* log2h_out) {
    const uint64_t Sp = (S + 3) & ~3u;
    uint32_t h = 2 * pow2ceil(Q < 16 ? 16 : Q);
    size_t bytes = (2ull * Sp + 4ull * h) * sizeof(int32_t);
    if (bytes > 200u * 1024u) {  // large S and Q together: load factor up to 1 (still terminates)
        h /= 2;
        bytes = (2ull * Sp + 4ull * h) * sizeof(int32_t);
    }
    int l = 0;
    while ((1u << l) < h) ++l;
    *log2h_out = l;
    return bytes;
}

template <int IPT_Q, int IPT_S, bool kCopyQuery>
int launch_lru(cudaStream_t s, int32_t* t2s, int32_t* s2t, int32_t* order, int32_t* stack, int32_t* count,
               const int32_t* query, int32_t* query_copy, int32_t* slot_out, uint8_t* hit, uint8_t* inst,
               int32_t* evicted, uint32_t ev_stride, int32_t* ev_count, int64_t* stats, int32_t* status, uint32_t R,
               uint32_t K, uint32_t S, uint32_t Q, uint32_t target) {
    int log2h = 0;
    const size_t smem = lru_smem_bytes(S, Q, &log2h);
    int max_dynamic = 0;
    const int rc = asu_max_dynamic_smem(reinterpret_cast<const void*>(lru_step_kernel<IPT_Q, IPT_S, kCopyQuery>),
                                        &max_dynamic);
    if (rc != ASU_OK) return rc;
    if (smem > static_cast<size_t>(max_dynamic)) return ASU_ERR_ARG;
    const uint32_t grid = R < 65535u ? R : 65535u;
    return launch_pdl(lru_step_kernel<IPT_Q, IPT_S, kCopyQuery>, dim3(grid), dim3(kThreads), smem, s, t2s, s2t,
                      order, stack, count, query, query_copy, slot_out, hit, inst, evicted, ev_stride, ev_count, stats,
                      status, R, K, S, Q, target, log2h);
}

template <int IPT_Q, bool kCopyQuery>
int dispatch_s(uint32_t S, cudaStream_t s, int32_t* t2s, int32_t* s2t, int32_t* order, int32_t* stack,
               int32_t* count, const int32_t* query, int32_t* query_copy, int32_t* slot_out, uint8_t* hit,
               uint8_t* inst, int32_t* evicted, uint32_t ev_stride, int32_t* ev_count, int64_t* stats, int32_t* status,
               uint32_t R, uint32_t K, uint32_t Q, uint32_t target) {
#define ASU_LRU_CASE(N)                                                                                           \
    if (S <= static_cast<uint32_t>(kThreads * N))                                                                 \
        return launch_lru<IPT_Q, N, kCopyQuery>(s, t2s, s2t, order, stack, count, query, query_copy, slot_out, hit,   \
                                                inst, evicted, ev_stride, ev_count, stats, status, R, K, S, Q, target);
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

namespace {

template <bool kCopyQuery>
int lru_step(void* stream, int32_t* token_to_slot, int32_t* slot_to_token, int32_t* lru_order, int32_t* free_stack,
             int32_t* free_count, const int32_t* query, int32_t* query_copy, int32_t* slot_out, uint8_t* hit_mask,
             uint8_t* install_mask, int32_t* evicted, uint32_t evicted_stride, int32_t* evicted_count, int64_t* stats,
             int32_t* status, uint32_t req_num, uint32_t key_space, uint32_t slot_count, uint32_t query_count,
             uint32_t free_target) {
    if (req_num == 0) return ASU_OK;
    if (!token_to_slot || !slot_to_token || !lru_order || !free_stack || !free_count || !evicted_count ||
        (query_count && (!query || !slot_out || !hit_mask || !install_mask)) ||
        (kCopyQuery && query_count && !query_copy))
        return ASU_ERR_ARG;
    if (key_space == 0 || key_space > 0x7fffffffu || slot_count == 0 || slot_count > 16384u ||
        query_count > 4096u)
        return ASU_ERR_ARG;
    const uint32_t tgt = free_target < slot_count ? free_target : slot_count;
    if (tgt > 0 && (evicted == nullptr || evicted_stride < tgt)) return ASU_ERR_ARG;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (query_count <= 2048u)
        return dispatch_s<2, kCopyQuery>(slot_count, s, token_to_slot, slot_to_token, lru_order, free_stack,
                                         free_count, query, query_copy, slot_out, hit_mask, install_mask, evicted,
                                         evicted_stride, evicted_count, stats, status, req_num, key_space,
                                         query_count, free_target);
    return dispatch_s<4, kCopyQuery>(slot_count, s, token_to_slot, slot_to_token, lru_order, free_stack, free_count,
                                     query, query_copy, slot_out, hit_mask, install_mask, evicted, evicted_stride,
                                     evicted_count, stats, status, req_num, key_space, query_count, free_target);
}

}  // namespace

extern "C" int asu_lru_step(void* stream, int32_t* token_to_slot, int32_t* slot_to_token, int32_t* lru_order,
                            int32_t* free_stack, int32_t* free_count, const int32_t* query, int32_t* slot_out,
                            uint8_t* hit_mask, uint8_t* install_mask, int32_t* evicted, uint32_t evicted_stride,
                            int32_t* evicted_count, int64_t* stats, int32_t* status, uint32_t req_num,
                            uint32_t key_space, uint32_t slot_count, uint32_t query_count, uint32_t free_target) {
    return lru_step<false>(stream, token_to_slot, slot_to_token, lru_order, free_stack, free_count, query, nullptr,
                           slot_out, hit_mask, install_mask, evicted, evicted_stride, evicted_count, stats, status,
                           req_num, key_space, slot_count, query_count, free_target);
}

extern "C" int asu_lru_step_host_query(void* stream, int32_t* token_to_slot, int32_t* slot_to_token,
                                       int32_t* lru_order, int32_t* free_stack, int32_t* free_count,
                                       const int32_t* query, int32_t* query_copy, int32_t* slot_out,
                                       uint8_t* hit_mask, uint8_t* install_mask, int32_t* evicted,
                                       uint32_t evicted_stride, int32_t* evicted_count, int64_t* stats,
                                       int32_t* status, uint32_t req_num, uint32_t key_space, uint32_t slot_count,
                                       uint32_t query_count, uint32_t free_target) {
    return lru_step<true>(stream, token_to_slot, slot_to_token, lru_order, free_stack, free_count, query, query_copy,
                          slot_out, hit_mask, install_mask, evicted, evicted_stride, evicted_count, stats, status,
                          req_num, key_space, slot_count, query_count, free_target);
}
