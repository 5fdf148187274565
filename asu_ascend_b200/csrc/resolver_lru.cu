// Single-request KV resolver over a bounded managed pool: the resolver's token-state machine
// fused with exact-LRU eviction, so a layer's managed cache can be far smaller than its context
// (e.g. 8192 resident + 2048 free slots for a 128K-token context).
//
// Reference behaviour (the composition of two reference algorithms):
//   * resolver, patch/0001 vllm_ascend/ops/asu_kv_resolver.py::asu_resolve_kv_slots_single_req
//     (patch lines 954-1039): HBM_RESIDENT -> its slot; ASU_ONLY -> install from
//     asu_record_addr[tok]; TAIL_HBM -> install from block_table[tok / bs] * bs + tok % bs;
//     install = pop free_slot_stack[--free_slot_count], copy the kv0 / kv1 row pair, mark the
//     token resident.  With a pool smaller than the context the reference raises "free_slot_stack
//     does not have enough slots" (patch lines 879-888).
//   * LRUManagedCache, simu/kv_cache_eviction_sim.py:124-150: at the step boundary the least
//     recently used residents are evicted until min(free_target, slots) slots are free (each
//     victim pushed on the free list); a hit moves its slot to the most recently used end, an
//     install enters there.
// An evicted token returns to ASU_ONLY when it has a record address (a prefix token, read from
// the ASU store again) and to TAIL_HBM otherwise (read from the paged cache again); its
// hbm_slot_of_token and the slot's owner are cleared.  The pool's recency order is one more
// state array, lru_order [slots]: the first slots - free_slot_count entries are the resident
// slots, least recently used first.
//
// B200 design: one launch of one 8-CTA thread-block cluster (8 SMs) for the request.  The state
// logic is one serial chain per call -- classify, rank, pop, reorder -- and runs in the leader
// CTA (rank 0) with the exact-LRU kernel's phase structure (lru.cu); the parts bound by how many
// random loads and row copies one SM keeps in flight are spread over the cluster:
//  * gathers: each CTA loads its eighth of the top-k entries and their token state, slot,
//    record address and block-table entry, and stores (token, state, slot, source row) into the
//    leader's shared memory through distributed shared memory (DSMEM);
//  * eviction: the victims are the head of the order row, lru_order[0, E); each CTA takes its
//    share, marks them in the leader's last_pos table (-2: an entry whose slot is a victim is
//    classified as a miss), and restores their tokens (ASU_ONLY with a record address, else
//    TAIL_HBM), clears the slot's owner and pushes the slot on the free stack;
//  * the leader meanwhile loads the order row into shared memory and gives the surviving
//    residents last_pos = -1; a free slot gets its last touch when it is popped;
//  * after a cluster barrier the leader classifies, de-duplicates misses in a shared-memory hash
//    (first and last position per token), ranks first occurrences with a block scan (rank k takes
//    the k-th stack pop: the victims just pushed, top first, then older entries), lists the
//    installs in shared memory and arrives at a second cluster barrier; it then writes the
//    outputs and the new order ([untouched residents in old order] ++ [touched slots by last
//    touching position], the OrderedDict order after the serial loop);
//  * the other seven CTAs wait at that barrier, copy the install list out of the leader's
//    shared memory and copy the installed kv0 / kv1 row pairs (16-, 4- or 1-byte units, several
//    loads in flight per thread) while the leader reorders.  A last cluster barrier keeps the
//    leader's shared memory alive until every CTA has read the list.
#include <cooperative_groups.h>

#include "asu_common.cuh"

namespace cg = cooperative_groups;

namespace asu {
namespace {

constexpr int kThreads = 1024;
constexpr int kCluster = 8;  // CTAs of the cluster; rank 0 is the leader
constexpr int32_t kVictim = -2;  // last_pos marker of a slot evicted in this call
constexpr int32_t kEmptyKey = -1;
constexpr int kCopyUnroll = 8;
constexpr uint32_t kMaxTopk = 4096;
constexpr uint32_t kMaxSlots = 16384;
constexpr int64_t kMaxRowBytes = 1 << 20;  // kv0 + kv1 bytes per token

enum : uint8_t { kNone = 0, kHit = 1, kMiss = 2 };

__device__ __forceinline__ uint32_t hash_key(int32_t key, int log2h) {
    return (static_cast<uint32_t>(key) * 0x9E3779B1u) >> (32 - log2h);
}

// Row pairs of the installs in shared memory (source row, managed slot), copied by the CTA.
template <typename V>
__device__ __forceinline__ void copy_rows(const int32_t* s_src, const int32_t* s_slot, int n,
                                          const uint8_t* __restrict__ kv0_src, const uint8_t* __restrict__ kv1_src,
                                          uint8_t* __restrict__ kv0_dst, uint8_t* __restrict__ kv1_dst, uint32_t c0,
                                          uint32_t c1, uint32_t first_thread, uint32_t threads) {
    const V* s0 = reinterpret_cast<const V*>(kv0_src);
    const V* s1 = reinterpret_cast<const V*>(kv1_src);
    V* d0 = reinterpret_cast<V*>(kv0_dst);
    V* d1 = reinterpret_cast<V*>(kv1_dst);
    const uint64_t cpr = static_cast<uint64_t>(c0) + c1;
    const uint64_t total = static_cast<uint64_t>(n) * cpr;
    for (uint64_t base = first_thread; base < total; base += static_cast<uint64_t>(threads) * kCopyUnroll) {
        V buf[kCopyUnroll];
        V* dst[kCopyUnroll];
#pragma unroll
        for (int k = 0; k < kCopyUnroll; ++k) {
            dst[k] = nullptr;
            const uint64_t u = base + static_cast<uint64_t>(k) * threads;
            if (u >= total) continue;
            const uint64_t e = u / cpr;
            const uint64_t ch = u - e * cpr;
            const int64_t src = s_src[e];
            const int64_t slot = s_slot[e];
            if (src < 0 || slot < 0) continue;  // an unusable pop: nothing to copy
            if (ch < c0) {
                buf[k] = __ldg(s0 + src * c0 + ch);
                dst[k] = d0 + slot * c0 + ch;
            } else {
                buf[k] = __ldg(s1 + src * c1 + (ch - c0));
                dst[k] = d1 + slot * c1 + (ch - c0);
            }
        }
#pragma unroll
        for (int k = 0; k < kCopyUnroll; ++k)
            if (dst[k]) *dst[k] = buf[k];
    }
}

struct LruResolveArgs {
    const int32_t* topk;
    uint32_t Q;  // top-k entries
    int32_t* token_state;
    const int32_t* record;
    int32_t* hbm_slot;
    int32_t* owner;
    int32_t* stack;
    int32_t* count;
    int32_t* order;
    uint32_t S;  // managed slots
    uint32_t target;
    const int32_t* block_table;
    int64_t bt_len;
    int64_t src_rows;
    int64_t limit;    // min(actual_seq_len, max_seq_len): valid top-k token ids are [0, limit)
    int64_t max_seq;  // length of the per-token arrays
    int64_t bs;
    int32_t* resolved;
    int32_t* evicted;  // nullable, >= min(target, S) entries
    int32_t* ev_count;  // nullable
    int64_t* stats;     // nullable, ASU_LRU_STAT_COLS
    int32_t* status;    // nullable
    const uint8_t* kv0_src;
    const uint8_t* kv1_src;
    uint8_t* kv0_dst;
    uint8_t* kv1_dst;
    uint32_t c0, c1;  // copy units per kv0 / kv1 row
    int vec;          // copy unit bytes: 16, 4 or 1 (0: nothing to copy)
    int log2h;
};

__device__ __forceinline__ void cluster_arrive() {
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// A gathered entry's token state and slot, packed for the leader: the state's category in bits
// 16-17 (ASU_ONLY 0, HBM_RESIDENT 1, TAIL_HBM 2, anything else 3) and the slot in bits 0-15
// (0xffff when it is not a slot of the pool).
constexpr int32_t kCodeBadSlot = 0xffff;
constexpr int32_t kCatBad = 3;

template <int IPT_Q, int IPT_S>
__global__ void __cluster_dims__(kCluster, 1, 1) __launch_bounds__(kThreads) resolve_lru_kernel(const LruResolveArgs a) {
    pdl_wait();     // launched with launch_pdl: stream order for every access below
    pdl_trigger();  // the next launch on the stream may be scheduled now; it waits for this grid
    extern __shared__ __align__(16) int32_t smem[];
    cg::cluster_group cluster = cg::this_cluster();
    const unsigned crank = cluster.block_rank();
    const bool leader = crank == 0;
    const uint32_t S = a.S, Q = a.Q;
    const uint32_t H = 1u << a.log2h;
    const uint32_t Sp = (S + 3) & ~3u;
    const uint32_t Qp = (Q + 3) & ~3u;
    // the leader's layout (every CTA allocates it; the others use the front for the install list)
    int32_t* s_order = smem;         // [Sp] old order row, later the new one
    int32_t* s_last = s_order + Sp;  // [Sp] last touching position: -1 untouched, -2 victim
    int32_t* s_hkey = s_last + Sp;   // [H]  hash: token (until the claims are done) ...
    int32_t* s_hval = s_hkey;        //      ... then the installed slot
    int32_t* s_hpos = s_hkey + H;    // [H]  hash: first position of the token
    int32_t* s_hmax = s_hpos + H;    // [H]  hash: last position of the token
    int32_t* g_code = s_hmax + H;    // [Qp] gathered per top-k entry: packed state and slot ...
    int32_t* g_src = g_code + Qp;    // [Qp] ... and the source row should it miss
    int32_t* s_isrc = g_code;        // [Qp] after the classification: installs in rank order, source row
    int32_t* s_islot = g_src;        // [Qp] ... and managed slot
    __shared__ int scan_a[32], scan_b[32];
    __shared__ int n_hits, n_valid, s_ninst;
    const int tid = threadIdx.x;
    int32_t bits = 0;

    // ---- P0 (every CTA): the free count, this CTA's share of the gathers and victims ----
    // Distributed shared memory may be written once every CTA of the cluster has started: this
    // barrier's arrival is here, its wait before the first remote store.
    cluster_arrive();
    const int32_t free0 = ld_cg(a.count);
    if (free0 < 0 || free0 > static_cast<int32_t>(S)) {  // uniform across the cluster
        if (leader && tid == 0) flag_status(a.status, 0, ASU_ST_BAD_STATE);
        cluster_wait();
        return;
    }
    const int32_t resident0 = static_cast<int32_t>(S) - free0;
    const int32_t tgt = static_cast<int32_t>(a.target < S ? a.target : S);
    int32_t E = 0;
    if (free0 < tgt) E = (tgt - free0) < resident0 ? (tgt - free0) : resident0;
    const int32_t free1 = free0 + E;

    // the leader's own top-k entries and order row, issued first
    int32_t tok[IPT_Q];
    constexpr int kVec = (IPT_S + 3) / 4;
    int4 ov[kVec];
    const bool vec_row = (S % 4 == 0) && (reinterpret_cast<uintptr_t>(a.order) % 16 == 0);
    if (leader) {
#pragma unroll
        for (int j = 0; j < IPT_Q; ++j) {
            const uint32_t pos = tid * IPT_Q + j;
            tok[j] = -1;
            if (pos < Q) {
                const int32_t t = __ldg(a.topk + pos);
                if (t >= 0 && t < a.limit) tok[j] = t;
            }
        }
        if (vec_row) {
            const int4* src = reinterpret_cast<const int4*>(a.order);
#pragma unroll
            for (int j = 0; j < kVec; ++j)
                if (tid + j * kThreads < S / 4) ov[j] = __ldcg(src + tid + j * kThreads);
        }
    }
    // gathers: entry e of this CTA's eighth -> (state, slot, source) in the leader's shared memory
    {
        const uint32_t per = (Q + kCluster - 1) / kCluster;  // <= 512 < kThreads
        const uint32_t e = crank * per + tid;
        const bool mine = static_cast<uint32_t>(tid) < per && e < Q;
        int32_t code = (kCatBad << 16) | kCodeBadSlot, src = -1;
        if (mine) {
            const int32_t t = __ldg(a.topk + e);
            if (t >= 0 && t < a.limit) {
                const int32_t st = ld_cg(a.token_state + t);
                const int32_t hs = ld_cg(a.hbm_slot + t);
                const int32_t rec = __ldg(a.record + t);
                int32_t tail = -1;
                const int64_t lb = static_cast<int64_t>(t) / a.bs;
                if (lb < a.bt_len) {
                    const int64_t r = static_cast<int64_t>(__ldg(a.block_table + lb)) * a.bs + static_cast<int64_t>(t) % a.bs;
                    tail = (r >= 0 && r <= INT32_MAX) ? static_cast<int32_t>(r) : -1;
                }
                // the source should the entry miss: a record for ASU_ONLY, the paged-cache row for
                // TAIL_HBM; a resident token evicted by this call takes the state its eviction
                // restores (ASU_ONLY with a record address, else TAIL_HBM)
                const int32_t cat = st == ASU_TOKEN_ASU_ONLY ? 0 : st == ASU_TOKEN_HBM_RESIDENT ? 1
                                    : st == ASU_TOKEN_TAIL_HBM ? 2 : kCatBad;
                src = cat == 0 ? rec : cat == 2 ? tail : (rec >= 0 ? rec : tail);
                code = (cat << 16) | (static_cast<uint32_t>(hs) < S ? hs : kCodeBadSlot);
            }
        }
        cluster_wait();  // every CTA has started
        if (mine) {
            cluster.map_shared_rank(g_code, 0)[e] = code;
            cluster.map_shared_rank(g_src, 0)[e] = src;
        }
    }
    // victims lru_order[0, E): position k belongs to thread k / kCluster of CTA k % kCluster, and
    // a second one to the same thread at k + kCluster * kThreads (E <= 16384).  They are marked
    // now in the leader's last_pos table and restored after the first cluster barrier (the
    // gathers above read the token states unchanged).  The first one's slot and owner stay in
    // registers; the rare second one is read again after the barrier.
    const int32_t ct = tid * kCluster + static_cast<int32_t>(crank);
    constexpr int32_t kSpan = kCluster * kThreads;
    int32_t vslot = kNotFound, vtok = kNotFound;
    if (ct < E) {
        vslot = ld_cg(a.order + ct);
        if (static_cast<uint32_t>(vslot) < S) {
            cluster.map_shared_rank(s_last, 0)[vslot] = kVictim;
            vtok = ld_cg(a.owner + vslot);
        } else {
            bits |= ASU_ST_BAD_STATE;
        }
    }
    if (ct + kSpan < E) {
        const int32_t v = ld_cg(a.order + ct + kSpan);
        if (static_cast<uint32_t>(v) < S) cluster.map_shared_rank(s_last, 0)[v] = kVictim;
        else bits |= ASU_ST_BAD_STATE;
    }
    if (leader) {
        // the order row into shared memory, last_pos of the surviving residents, the hash
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
                const int32_t v = ld_cg(a.order + k);
                s_order[k] = v;
                if (k >= E && k < resident0 && static_cast<uint32_t>(v) < S) s_last[v] = -1;
            }
        }
        const int4 m1 = make_int4(-1, -1, -1, -1);
        const int4 big = make_int4(INT32_MAX, INT32_MAX, INT32_MAX, INT32_MAX);
        for (uint32_t i = tid; i < H / 4; i += kThreads) {
            reinterpret_cast<int4*>(s_hkey)[i] = m1;
            reinterpret_cast<int4*>(s_hpos)[i] = big;
            reinterpret_cast<int4*>(s_hmax)[i] = m1;
        }
        if (tid == 0) {
            n_hits = 0;
            n_valid = 0;
            if (a.ev_count) *a.ev_count = E;
        }
    }
    cluster_arrive();
    cluster_wait();  // A: gathers, victim marks, order row and hash in place

    // ---- restores (every CTA: its victims) | classification (leader) ----
    for (int32_t k = ct; k < E; k += kSpan) {
        int32_t v = vslot, vt = vtok;
        if (k != ct) {  // the second victim of this thread
            v = ld_cg(a.order + k);
            vt = static_cast<uint32_t>(v) < S ? ld_cg(a.owner + v) : kNotFound;
        }
        if (static_cast<uint32_t>(v) < S) {
            if (vt >= 0 && vt < a.max_seq) {
                const int32_t vr = __ldg(a.record + vt);
                st_cg(a.token_state + vt, vr >= 0 ? ASU_TOKEN_ASU_ONLY : ASU_TOKEN_TAIL_HBM);
                st_cg(a.hbm_slot + vt, kNotFound);
            } else {
                bits |= ASU_ST_BAD_STATE;
            }
            st_cg(a.owner + v, kNotFound);
            st_cg(a.stack + free0 + k, v);
        }
        if (a.evicted) a.evicted[k] = static_cast<uint32_t>(v) < S ? vt : kNotFound;
    }
    uint8_t cls[IPT_Q];
    int32_t hidx[IPT_Q], src[IPT_Q], hs[IPT_Q];
    int valid_local = 0;
    if (leader) {
#pragma unroll
        for (int j = 0; j < IPT_Q; ++j) {
            const int32_t pos = tid * IPT_Q + j;
            cls[j] = kNone;
            hidx[j] = -1;
            src[j] = -1;
            hs[j] = kNotFound;
            if (static_cast<uint32_t>(pos) < Q && tok[j] < 0) bits |= ASU_ST_BAD_QUERY;
            if (tok[j] < 0) continue;
            ++valid_local;
            const int32_t code = g_code[pos];
            const int32_t cat = code >> 16;
            const int32_t s = code & 0xffff;
            src[j] = g_src[pos];
            if (cat == 1) {
                if (s == kCodeBadSlot) {
                    bits |= ASU_ST_BAD_STATE;
                    continue;
                }
                if (s_last[s] != kVictim) {
                    cls[j] = kHit;
                    hs[j] = s;
                    atomicMax(&s_last[s], pos);
                    continue;
                }
                // evicted by this call: a miss from the source its restored state names
            } else if (cat == kCatBad) {
                bits |= ASU_ST_BAD_TOKEN_STATE;
                continue;
            }
            if (src[j] < 0 || src[j] >= a.src_rows) {
                bits |= ASU_ST_BAD_SOURCE;  // skipped: the reference raises here
                continue;
            }
            cls[j] = kMiss;
            uint32_t h = hash_key(tok[j], a.log2h);
            while (true) {  // terminates: at most Q <= H distinct tokens
                const int32_t old = atomicCAS(&s_hkey[h], kEmptyKey, tok[j]);
                if (old == kEmptyKey || old == tok[j]) break;
                h = (h + 1) & (H - 1);
            }
            hidx[j] = static_cast<int32_t>(h);
            atomicMin(&s_hpos[h], pos);  // the first position installs
            atomicMax(&s_hmax[h], pos);  // the last one is its slot's last touch
        }
    }
    cluster_arrive();
    cluster_wait();  // A2: every claim made; restores ordered before any install

    int32_t n_inst = 0;
    if (leader) {
        // ---- P3: first occurrences pop the stack in top-k order and install ----
        int canon[IPT_Q];
        int local = 0;
#pragma unroll
        for (int j = 0; j < IPT_Q; ++j) {
            canon[j] = cls[j] == kMiss && s_hpos[hidx[j]] == static_cast<int32_t>(tid * IPT_Q + j);
            local += canon[j];
        }
        int n_canon = 0;
        int rank = block_exclusive_scan_1b(local, scan_a, &n_canon);
        int32_t slot[IPT_Q];
#pragma unroll
        for (int j = 0; j < IPT_Q; ++j) {
            slot[j] = cls[j] == kHit ? hs[j] : kNotFound;
            if (!canon[j]) continue;
            const int32_t k = rank++;
            int32_t s = kNotFound;
            if (k < free1) {
                // the victims just pushed (top first), then the older entries below them
                s = k < E ? s_order[E - 1 - k] : ld_cg(a.stack + (free0 - 1 - (k - E)));
                if (static_cast<uint32_t>(s) >= S) {
                    bits |= ASU_ST_BAD_STATE;
                    s = kNotFound;
                }
            } else {
                bits |= ASU_ST_FREE_EXHAUSTED;
            }
            s_hval[hidx[j]] = s;
            if (k < free1) {
                s_isrc[k] = s >= 0 ? src[j] : -1;
                s_islot[k] = s;
            }
            if (s >= 0) {
                st_cg(a.token_state + tok[j], ASU_TOKEN_HBM_RESIDENT);
                st_cg(a.hbm_slot + tok[j], s);
                st_cg(a.owner + s, tok[j]);
                s_last[s] = s_hmax[hidx[j]];  // only this thread touches a popped slot before the barrier
            }
            slot[j] = s;
        }
        n_inst = n_canon < free1 ? n_canon : free1;
        const int32_t free2 = free1 - n_inst;
        if (tid == 0) s_ninst = n_inst;
        __syncthreads();  // installed slots, their last touches and the install list in place
        cluster_arrive();  // B: the other CTAs copy the rows while the leader reorders

        // ---- P4: later duplicates of a missing token, outputs ----
        int hits_local = 0;
#pragma unroll
        for (int j = 0; j < IPT_Q; ++j) {
            const int32_t pos = tid * IPT_Q + j;
            bool hit = cls[j] == kHit;
            if (cls[j] == kMiss && !canon[j]) {
                const int32_t v = s_hval[hidx[j]];
                if (v >= 0) {
                    slot[j] = v;
                    hit = true;
                }
            }
            hits_local += hit;
            if (static_cast<uint32_t>(pos) < Q) a.resolved[pos] = slot[j];
        }
        hits_local = __reduce_add_sync(0xffffffffu, hits_local);
        valid_local = __reduce_add_sync(0xffffffffu, valid_local);
        if ((tid & 31) == 0) {
            if (hits_local) atomicAdd(&n_hits, hits_local);
            if (valid_local) atomicAdd(&n_valid, valid_local);
        }

        // ---- P5: new recency order ----
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
        int packed_total = 0;  // kept residents in the low 16 bits (<= S), touched slots above (<= Q)
        const int packed = block_exclusive_scan_1b(keep_local | (touched_local << 16), scan_b, &packed_total);
        int ka = packed & 0xffff;
        int kb = packed >> 16;
        const int n_keep = packed_total & 0xffff;
        const int n_touched = packed_total >> 16;
#pragma unroll
        for (int j = 0; j < IPT_S; ++j) {
            if (keep[j]) {
                if (ka < static_cast<int>(S)) s_order[ka] = oldv[j];
                ++ka;
            }
        }
#pragma unroll
        for (int j = 0; j < IPT_Q; ++j) {
            if (touched[j]) {
                const int o = n_keep + kb++;
                if (o < static_cast<int>(S)) s_order[o] = slot[j];
            }
        }
        __syncthreads();
        const int n_new = min(n_keep + n_touched, static_cast<int>(S));
        if (vec_row) {
            const int n4 = n_new / 4;
            for (int i = tid; i < n4; i += kThreads)
                __stcg(reinterpret_cast<int4*>(a.order) + i, reinterpret_cast<const int4*>(s_order)[i]);
            for (int i = n4 * 4 + tid; i < n_new; i += kThreads) st_cg(a.order + i, s_order[i]);
        } else {
            for (int i = tid; i < n_new; i += kThreads) st_cg(a.order + i, s_order[i]);
        }
        if (tid == 0) {
            st_cg(a.count, free2);
            if (n_keep + n_touched != static_cast<int>(S) - free2) bits |= ASU_ST_BAD_STATE;
            if (a.stats != nullptr) {
                unsigned long long* row = reinterpret_cast<unsigned long long*>(a.stats);
                atomicAdd(row + ASU_LRU_STAT_HITS, static_cast<unsigned long long>(n_hits));
                atomicAdd(row + ASU_LRU_STAT_MISSES, static_cast<unsigned long long>(n_valid - n_hits));
                atomicAdd(row + ASU_LRU_STAT_INSTALLS, static_cast<unsigned long long>(n_inst));
                atomicAdd(row + ASU_LRU_STAT_SHORTAGES, static_cast<unsigned long long>(n_valid - n_hits - n_inst));
                atomicAdd(row + ASU_LRU_STAT_EVICTIONS, static_cast<unsigned long long>(E));
            }
        }
        cluster_wait();  // B
    } else {
        cluster_arrive();
        cluster_wait();  // B: the install list is complete
        // ---- P6 (CTAs 1..7): the installed row pairs ----
        // An unusable pop (bad slot) is listed with source -1 and copied by nobody.
        n_inst = *cluster.map_shared_rank(&s_ninst, 0);
        const int32_t* l_src = cluster.map_shared_rank(s_isrc, 0);
        const int32_t* l_slot = cluster.map_shared_rank(s_islot, 0);
        int32_t* c_src = smem;       // this CTA's copy of the list
        int32_t* c_slot = smem + Qp;
        for (int i = tid; i < n_inst; i += kThreads) {
            c_src[i] = l_src[i];
            c_slot[i] = l_slot[i];
        }
        __syncthreads();
        const uint32_t first = (crank - 1) * kThreads + tid, threads = (kCluster - 1) * kThreads;
        if (a.vec == 16)
            copy_rows<int4>(c_src, c_slot, n_inst, a.kv0_src, a.kv1_src, a.kv0_dst, a.kv1_dst, a.c0, a.c1, first,
                            threads);
        else if (a.vec == 4)
            copy_rows<int32_t>(c_src, c_slot, n_inst, a.kv0_src, a.kv1_src, a.kv0_dst, a.kv1_dst, a.c0, a.c1, first,
                               threads);
        else if (a.vec == 1)
            copy_rows<uint8_t>(c_src, c_slot, n_inst, a.kv0_src, a.kv1_src, a.kv0_dst, a.kv1_dst, a.c0, a.c1, first,
                               threads);
    }
    if (bits) flag_status(a.status, 0, bits);
    cluster_arrive();
    cluster_wait();  // C: the leader's shared memory stays until every CTA has read the list
}

inline uint32_t pow2ceil(uint32_t x) {
    uint32_t p = 1;
    while (p < x) p <<= 1;
    return p;
}

// Dynamic shared memory of every CTA (the leader's layout): order + last_pos rows, the hash table
// (three arrays) and the gathered entries (two arrays, later the install list).
inline size_t smem_bytes(uint32_t S, uint32_t Q, int* log2h_out) {
    const uint64_t Sp = (S + 3) & ~3u;
    const uint64_t Qp = (Q + 3) & ~3u;
    uint32_t h = 2 * pow2ceil(Q < 16 ? 16 : Q);
    size_t bytes = (2ull * Sp + 3ull * h + 2ull * Qp) * sizeof(int32_t);
    if (bytes > 200u * 1024u) {  // large S and Q together: load factor up to 1 (still terminates)
        h /= 2;
        bytes = (2ull * Sp + 3ull * h + 2ull * Qp) * sizeof(int32_t);
    }
    int l = 0;
    while ((1u << l) < h) ++l;
    *log2h_out = l;
    return bytes;
}

template <int IPT_Q, int IPT_S>
int launch(cudaStream_t s, LruResolveArgs a) {
    const size_t smem = smem_bytes(a.S, a.Q, &a.log2h);
    int max_dynamic = 0;
    const int rc = asu_max_dynamic_smem(reinterpret_cast<const void*>(resolve_lru_kernel<IPT_Q, IPT_S>), &max_dynamic);
    if (rc != ASU_OK) return rc;
    if (smem > static_cast<size_t>(max_dynamic)) return ASU_ERR_ARG;
    return launch_pdl(resolve_lru_kernel<IPT_Q, IPT_S>, dim3(kCluster), dim3(kThreads), smem, s, a);
}

template <int IPT_Q>
int dispatch_s(cudaStream_t s, const LruResolveArgs& a) {
    if (a.S <= 2u * kThreads) return launch<IPT_Q, 2>(s, a);
    if (a.S <= 4u * kThreads) return launch<IPT_Q, 4>(s, a);
    if (a.S <= 8u * kThreads) return launch<IPT_Q, 8>(s, a);
    // 8192 + 2048 managed slots: 12 order entries on each of 854 threads instead of 16 on 640
    if (a.S <= 12u * kThreads) return launch<IPT_Q, 12>(s, a);
    return launch<IPT_Q, 16>(s, a);
}

}  // namespace
}  // namespace asu

using namespace asu;

extern "C" int asu_kv_resolver_lru(void* stream, const int32_t* topk, int64_t topk_numel, int32_t* token_state,
                                   const int32_t* asu_record_addr, int32_t* hbm_slot_of_token,
                                   int32_t* slot_owner_token, int32_t* free_slot_stack, int32_t* free_slot_count,
                                   int32_t* lru_order, int64_t slot_count, int64_t free_target,
                                   const int32_t* block_table, int64_t block_table_len, const void* kv0_src,
                                   const void* kv1_src, void* kv0_dst, void* kv1_dst, int64_t kv0_row_bytes,
                                   int64_t kv1_row_bytes, int64_t src_rows, int64_t max_seq_len,
                                   int64_t actual_seq_len, int64_t block_size, int32_t* resolved, int32_t* evicted,
                                   int32_t* evicted_count, int64_t* stats, int32_t* status) {
    if (topk_numel < 0 || topk_numel > static_cast<int64_t>(kMaxTopk)) return ASU_ERR_ARG;
    if (!topk || !token_state || !asu_record_addr || !hbm_slot_of_token || !slot_owner_token || !free_slot_stack ||
        !free_slot_count || !lru_order || !resolved)
        return ASU_ERR_ARG;
    if (slot_count <= 0 || slot_count > static_cast<int64_t>(kMaxSlots) || free_target < 0 || block_size <= 0 ||
        actual_seq_len < 0 || max_seq_len <= 0 || src_rows < 0 || src_rows > 0x7fffffff || kv0_row_bytes < 0 ||
        kv1_row_bytes < 0 || (block_table_len > 0 && !block_table) || block_table_len < 0)
        return ASU_ERR_ARG;
    if ((kv0_row_bytes > 0 && (!kv0_src || !kv0_dst)) || (kv1_row_bytes > 0 && (!kv1_src || !kv1_dst)))
        return ASU_ERR_ARG;
    if (kv0_row_bytes + kv1_row_bytes > kMaxRowBytes) return ASU_ERR_ARG;
    const int64_t tgt = free_target < slot_count ? free_target : slot_count;
    if (evicted_count && !evicted && tgt > 0) return ASU_ERR_ARG;
    const uintptr_t align = (kv0_row_bytes > 0 ? reinterpret_cast<uintptr_t>(kv0_src) |
                                                     reinterpret_cast<uintptr_t>(kv0_dst) |
                                                     static_cast<uintptr_t>(kv0_row_bytes)
                                               : 0) |
                            (kv1_row_bytes > 0 ? reinterpret_cast<uintptr_t>(kv1_src) |
                                                     reinterpret_cast<uintptr_t>(kv1_dst) |
                                                     static_cast<uintptr_t>(kv1_row_bytes)
                                               : 0);
    const int vec = (kv0_row_bytes == 0 && kv1_row_bytes == 0) ? 0 : (align & 15) == 0 ? 16 : (align & 3) == 0 ? 4 : 1;
    LruResolveArgs a = {};
    a.topk = topk;
    a.Q = static_cast<uint32_t>(topk_numel);
    a.token_state = token_state;
    a.record = asu_record_addr;
    a.hbm_slot = hbm_slot_of_token;
    a.owner = slot_owner_token;
    a.stack = free_slot_stack;
    a.count = free_slot_count;
    a.order = lru_order;
    a.S = static_cast<uint32_t>(slot_count);
    a.target = static_cast<uint32_t>(tgt);
    a.block_table = block_table;
    a.bt_len = block_table_len;
    a.src_rows = src_rows;
    a.limit = actual_seq_len < max_seq_len ? actual_seq_len : max_seq_len;
    a.max_seq = max_seq_len;
    a.bs = block_size;
    a.resolved = resolved;
    a.evicted = evicted;
    a.ev_count = evicted_count;
    a.stats = stats;
    a.status = status;
    a.kv0_src = static_cast<const uint8_t*>(kv0_src);
    a.kv1_src = static_cast<const uint8_t*>(kv1_src);
    a.kv0_dst = static_cast<uint8_t*>(kv0_dst);
    a.kv1_dst = static_cast<uint8_t*>(kv1_dst);
    a.vec = vec;
    a.c0 = vec ? static_cast<uint32_t>(kv0_row_bytes / vec) : 0;
    a.c1 = vec ? static_cast<uint32_t>(kv1_row_bytes / vec) : 0;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    return a.Q <= 2048u ? dispatch_s<2>(s, a) : dispatch_s<4>(s, a);
}
