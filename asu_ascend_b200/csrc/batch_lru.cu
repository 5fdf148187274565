// Batch-LRU lookup: lookup + unique-miss allocation + victim invalidation + batch LRU rewrite.
//
// Reference behaviour: pta-ops/asu_hbm_index_lookup_simt/python/lookup_lru_reference.py:21-89
// (kernel src/asu_hbm_index_lookup_simt_kernel.cpp:10-219):
//   hits       = slots of resident query tokens; unique misses in query order (first occurrence
//                carries miss_mask); invalid tokens -> slot -1, mask false
//   partition  = lru_slots split stably into hit slots and evictable slots (LRU first)
//   miss i     takes evictable[i]; its old token is unmapped; maps are rebound
//   new lru    = evictable[M:] + evictable[:M] + hit slots
//
// B200 design: one CTA (1024 threads) per request; all scratch in shared memory, so the
// caller's workspace is not needed.  At launch every thread issues its loads together: the
// query gathers from token_to_slot, its part of the LRU row (kept in registers) and the
// slot_to_token row (into shared memory, where the victims' old tokens are read later).
// First occurrences of missing tokens are claimed in a shared-memory hash (the reference
// kernel's CAS winner is scheduling-dependent; the oracle's is the first occurrence, which is
// what this returns); a block scan ranks them in query order.  The stable partition of the
// LRU row is one block scan over packed (hit, evictable) counts, and the row is rewritten in
// place.  Later duplicates read their first occurrence's slot from the hash, so no output
// needs a second global read.
#include "asu_common.cuh"

namespace asu {
namespace {

constexpr int kThreads = 1024;
enum : uint8_t { kInvalid = 0, kHit = 1, kMiss = 2 };

__device__ __forceinline__ int batch_claim(int32_t* keys, int32_t* first, uint32_t H, int32_t key, int32_t pos) {
    uint32_t h = hash32(static_cast<uint32_t>(key)) & (H - 1);
    for (uint32_t probe = 0; probe < H; ++probe) {
        const int32_t prev = atomicCAS(keys + h, -1, key);
        if (prev == -1 || prev == key) {
            atomicMin(first + h, pos);
            return static_cast<int>(h);
        }
        h = (h + 1) & (H - 1);
    }
    return -1;  // unreachable: H >= 2 * Q
}

// Dynamic shared memory: slot_to_token row [Sp], hash keys / first position / slot [3H],
// victim list [Q], hit flags [S] bytes.
inline size_t batch_smem_bytes(uint32_t S, uint32_t Q, uint32_t H) {
    const size_t Sp = (S + 3) & ~3u;
    return (Sp + 3ull * H + Q) * sizeof(int32_t) + S;
}

template <int IPT_Q, int IPT_S>
__global__ void __launch_bounds__(kThreads)
batch_lru_kernel(int32_t* __restrict__ t2s, int32_t* __restrict__ s2t, int16_t* __restrict__ lru,
                 const int32_t* __restrict__ query, int32_t* __restrict__ slot_ids, uint8_t* __restrict__ miss_mask,
                 uint32_t req_num, uint32_t K, uint32_t S, uint32_t Q, uint32_t H, int32_t* status) {
    extern __shared__ int32_t dyn[];
    const uint32_t Sp = (S + 3) & ~3u;
    int32_t* s_owner = dyn;                                     // [Sp] slot_to_token row
    int32_t* h_key = s_owner + Sp;                              // [H]
    int32_t* h_first = h_key + H;                               // [H]
    int32_t* h_slot = h_first + H;                              // [H] slot given to the key
    int32_t* vict = h_slot + H;                                 // [Q]
    uint8_t* hitf = reinterpret_cast<uint8_t*>(vict + Q);       // [S]
    __shared__ int scan_a[32], scan_b[32];
    const int tid = threadIdx.x;
    for (uint32_t r = blockIdx.x; r < req_num; r += gridDim.x) {
        int32_t* trow = t2s + static_cast<uint64_t>(r) * K;
        int32_t* srow = s2t + static_cast<uint64_t>(r) * S;
        int16_t* lrow = lru + static_cast<uint64_t>(r) * S;
        const int32_t* qrow = query + static_cast<uint64_t>(r) * Q;
        int32_t bits = 0;

        // ---- loads: queries -> token_to_slot gathers, LRU row, slot_to_token row ----
        int32_t key[IPT_Q], g[IPT_Q];
#pragma unroll
        for (int j = 0; j < IPT_Q; ++j) {
            const uint32_t pos = tid * IPT_Q + j;
            key[j] = pos < Q ? __ldg(qrow + pos) : -1;
            g[j] = kNotFound;
            if (pos < Q && static_cast<uint32_t>(key[j]) < K) g[j] = ld_cg(trow + key[j]);
        }
        int32_t lv[IPT_S];
        bool vec_lru = false;
        if constexpr (IPT_S % 8 == 0) vec_lru = S % 8 == 0 && (reinterpret_cast<uintptr_t>(lrow) & 15) == 0;
        if constexpr (IPT_S % 8 == 0) {
          if (vec_lru) {
            // 16-byte loads of 8 int16 entries each
#pragma unroll
            for (int j = 0; j < IPT_S; j += 8) {
                const uint32_t idx = tid * IPT_S + j;
                if (idx < S) {
                    const int4 v4 = __ldcg(reinterpret_cast<const int4*>(lrow + idx));
                    const int16_t* e = reinterpret_cast<const int16_t*>(&v4);
#pragma unroll
                    for (int u = 0; u < 8; ++u) lv[j + u] = e[u];
                } else {
#pragma unroll
                    for (int u = 0; u < 8; ++u) lv[j + u] = -1;
                }
            }
          }
        }
        if (!vec_lru) {
#pragma unroll
            for (int j = 0; j < IPT_S; ++j) {
                const uint32_t idx = tid * IPT_S + j;
                lv[j] = idx < S ? static_cast<int32_t>(lrow[idx]) : -1;
            }
        }
        for (uint32_t i = tid; i < S; i += kThreads) s_owner[i] = ld_cg(srow + i);
        for (uint32_t i = tid; i < H; i += kThreads) {
            h_key[i] = -1;
            h_first[i] = INT32_MAX;
        }
        for (uint32_t i = tid; i < S; i += kThreads) hitf[i] = 0;
        __syncthreads();  // tables cleared, slot_to_token row in shared memory

        // ---- classify: hits flag their slot, missing tokens claim their first position ----
        int32_t slot[IPT_Q], h[IPT_Q];
        uint8_t st[IPT_Q];
#pragma unroll
        for (int j = 0; j < IPT_Q; ++j) {
            const int32_t pos = static_cast<int32_t>(tid * IPT_Q + j);
            slot[j] = kNotFound;
            h[j] = -1;
            st[j] = kInvalid;
            if (static_cast<uint32_t>(pos) >= Q || static_cast<uint32_t>(key[j]) >= K) continue;
            const int32_t v = g[j];
            if (v >= 0 && static_cast<uint32_t>(v) < S) {
                st[j] = kHit;
                slot[j] = v;
                hitf[v] = 1;
            } else if (v == kNotFound) {
                h[j] = batch_claim(h_key, h_first, H, key[j], pos);
                if (h[j] >= 0) st[j] = kMiss;
                else bits |= ASU_ST_BAD_STATE;
            } else {
                bits |= ASU_ST_BAD_STATE;  // the oracle raises on these
            }
        }
        __syncthreads();  // claims and hit flags complete
        int canon[IPT_Q];
        int local = 0;
#pragma unroll
        for (int j = 0; j < IPT_Q; ++j) {
            canon[j] = st[j] == kMiss && h_first[h[j]] == static_cast<int32_t>(tid * IPT_Q + j);
            local += canon[j];
        }
        int M = 0;
        int mrank = block_exclusive_scan_1b(local, scan_a, &M);

        // ---- stable partition of the LRU row (held in registers) ----
        bool lh[IPT_S];
        int packed = 0;
#pragma unroll
        for (int j = 0; j < IPT_S; ++j) {
            const uint32_t idx = tid * IPT_S + j;
            lh[j] = false;
            if (idx >= S) continue;
            if (static_cast<uint32_t>(lv[j]) < S) {
                lh[j] = hitf[lv[j]] != 0;
                packed += lh[j] ? (1 << 16) : 1;
            } else {
                bits |= ASU_ST_BAD_STATE;
            }
        }
        int ptotal = 0;
        const int pre = block_exclusive_scan_1b(packed, scan_b, &ptotal);
        const int V = ptotal & 0xffff;
        int hrank = pre >> 16, erank = pre & 0xffff;
#pragma unroll
        for (int j = 0; j < IPT_S; ++j) {
            if (static_cast<uint32_t>(lv[j]) >= S || lh[j]) continue;
            if (erank < M) vict[erank] = lv[j];
            ++erank;
        }
        __syncthreads();  // victim list complete

        if (M > V) {  // block-uniform: not enough evictable slots; nothing was written, change nothing
            if (tid == 0) bits |= ASU_ST_NO_VICTIM;
#pragma unroll
            for (int j = 0; j < IPT_Q; ++j) {
                const uint32_t pos = tid * IPT_Q + j;
                if (pos < Q) {
                    slot_ids[static_cast<uint64_t>(r) * Q + pos] = st[j] == kHit ? slot[j] : kNotFound;
                    miss_mask[static_cast<uint64_t>(r) * Q + pos] = 0;
                }
            }
        } else {
#pragma unroll
            for (int j = 0; j < IPT_Q; ++j) {
                if (!canon[j]) continue;
                const int32_t victim = vict[mrank++];
                const int32_t vt = s_owner[victim];
                if (vt >= 0) {
                    if (static_cast<uint32_t>(vt) < K) st_cg(trow + vt, kNotFound);
                    else bits |= ASU_ST_BAD_STATE;
                }
                st_cg(srow + victim, key[j]);
                st_cg(trow + key[j], victim);
                slot[j] = victim;
                h_slot[h[j]] = victim;
            }
            // new order: stale evictables, then this batch's victims, then hit slots
            erank = pre & 0xffff;
#pragma unroll
            for (int j = 0; j < IPT_S; ++j) {
                if (static_cast<uint32_t>(lv[j]) >= S) continue;
                int dst;
                if (lh[j]) {
                    dst = V + hrank++;
                } else {
                    dst = erank >= M ? erank - M : (V - M) + erank;
                    ++erank;
                }
                lrow[dst] = static_cast<int16_t>(lv[j]);
            }
            __syncthreads();  // first occurrences' slots published
#pragma unroll
            for (int j = 0; j < IPT_Q; ++j) {
                const uint32_t pos = tid * IPT_Q + j;
                if (pos >= Q) continue;
                if (st[j] == kMiss && !canon[j]) slot[j] = h_slot[h[j]];  // later duplicate of a miss
                slot_ids[static_cast<uint64_t>(r) * Q + pos] = slot[j];
                miss_mask[static_cast<uint64_t>(r) * Q + pos] = canon[j] ? 1 : 0;
            }
        }
        if (bits) flag_status(status, r, bits);
        __syncthreads();
    }
}

template <int IPT_Q, int IPT_S>
int launch_batch(cudaStream_t s, int32_t* t2s, int32_t* s2t, int16_t* lru, const int32_t* q, int32_t* slot_ids,
                 uint8_t* mask, uint32_t R, uint32_t K, uint32_t S, uint32_t Q, int32_t* status) {
    int max_dynamic = 0;
    const int rc = asu_max_dynamic_smem(reinterpret_cast<const void*>(batch_lru_kernel<IPT_Q, IPT_S>), &max_dynamic);
    if (rc != ASU_OK) return rc;
    uint32_t H = 32;
    while (H < 2 * (Q ? Q : 1)) H <<= 1;
    const size_t smem = batch_smem_bytes(S, Q, H);
    if (smem > static_cast<size_t>(max_dynamic)) return ASU_ERR_ARG;
    const uint32_t grid = R < 65535u ? R : 65535u;
    batch_lru_kernel<IPT_Q, IPT_S><<<grid, kThreads, smem, s>>>(t2s, s2t, lru, q, slot_ids, mask, R, K, S, Q, H,
                                                                 status);
    return asu_launch_status();
}

}  // namespace
}  // namespace asu

using namespace asu;

extern "C" int asu_hbm_index_lookup_simt_ex(void* stream, int32_t* token_to_slot, int32_t* slot_to_token,
                                            int16_t* lru_slots, const int32_t* query_token_ids, int32_t* slot_ids,
                                            uint8_t* miss_mask, uint32_t req_num, uint32_t index_size,
                                            uint32_t slot_count, uint32_t query_count, int32_t* status) {
    if (req_num == 0) return ASU_OK;
    if (!token_to_slot || !slot_to_token || !lru_slots ||
        (query_count && (!query_token_ids || !slot_ids || !miss_mask)))
        return ASU_ERR_ARG;
    if (index_size == 0 || index_size > 0x7fffffffu || slot_count == 0 || slot_count > 16384u || query_count > 4096u)
        return ASU_ERR_ARG;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
#define ASU_BATCH_CASE(QN, SN)                                                                                   \
    if (query_count <= kThreads * QN && slot_count <= kThreads * SN)                                              \
        return launch_batch<QN, SN>(s, token_to_slot, slot_to_token, lru_slots, query_token_ids, slot_ids, miss_mask, \
                                    req_num, index_size, slot_count, query_count, status);
    ASU_BATCH_CASE(2, 4)
    ASU_BATCH_CASE(2, 16)
    ASU_BATCH_CASE(4, 16)
#undef ASU_BATCH_CASE
    return ASU_ERR_ARG;
}

extern "C" int asu_hbm_index_lookup_simt_do(void* stream, void* token_to_slot, void* slot_to_token, void* lru_slots,
                                            void* query_token_ids, void* slot_ids, void* miss_mask, void* workspace,
                                            uint32_t req_num) {
    (void)workspace;  // scratch lives in shared memory
    return asu_hbm_index_lookup_simt_ex(stream, static_cast<int32_t*>(token_to_slot),
                                        static_cast<int32_t*>(slot_to_token), static_cast<int16_t*>(lru_slots),
                                        static_cast<const int32_t*>(query_token_ids), static_cast<int32_t*>(slot_ids),
                                        static_cast<uint8_t*>(miss_mask), req_num, ASU_HBM_INDEX_SIZE,
                                        ASU_HBM_SLOT_COUNT, ASU_HBM_QUERY_COUNT, nullptr);
}
