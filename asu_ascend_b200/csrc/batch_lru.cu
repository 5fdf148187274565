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
// B200 design: one CTA (1024 threads) per request; all scratch in shared memory (hit flags,
// victim list), so the caller's workspace is not needed.  First occurrences are found with
// the atomicMin claim used by the other lookups (the reference kernel's CAS winner is
// scheduling-dependent; the oracle's is the first occurrence, which is what this returns).
// The stable partition of the LRU row is one block scan over packed (hit, evictable)
// counts with the row held in registers, so the row is rewritten in place.
#include "asu_common.cuh"

namespace asu {
namespace {

constexpr int kThreads = 1024;
enum : uint8_t { kInvalid = 0, kHit = 1, kMiss = 2 };

template <int IPT_Q, int IPT_S>
__global__ void __launch_bounds__(kThreads)
batch_lru_kernel(int32_t* __restrict__ t2s, int32_t* __restrict__ s2t, int16_t* __restrict__ lru,
                 const int32_t* __restrict__ query, int32_t* __restrict__ slot_ids, uint8_t* __restrict__ miss_mask,
                 uint32_t req_num, uint32_t K, uint32_t S, uint32_t Q, int32_t* status) {
    extern __shared__ int32_t dyn[];
    int32_t* vict = dyn;                                        // [Q]
    uint8_t* hitf = reinterpret_cast<uint8_t*>(dyn + Q);        // [S]
    __shared__ int scan_buf[33];
    const int tid = threadIdx.x;
    for (uint32_t r = blockIdx.x; r < req_num; r += gridDim.x) {
        int32_t* trow = t2s + static_cast<uint64_t>(r) * K;
        int32_t* srow = s2t + static_cast<uint64_t>(r) * S;
        int16_t* lrow = lru + static_cast<uint64_t>(r) * S;
        const int32_t* qrow = query + static_cast<uint64_t>(r) * Q;
        int32_t bits = 0;
        for (uint32_t s = tid; s < S; s += kThreads) hitf[s] = 0;
        __syncthreads();

        int32_t key[IPT_Q], slot[IPT_Q];
        uint8_t st[IPT_Q];
#pragma unroll
        for (int j = 0; j < IPT_Q; ++j) {
            const uint32_t pos = tid * IPT_Q + j;
            key[j] = -1;
            slot[j] = kNotFound;
            st[j] = kInvalid;
            if (pos < Q) {
                key[j] = __ldg(qrow + pos);
                if (static_cast<uint32_t>(key[j]) < K) {
                    const int32_t v = ld_cg(trow + key[j]);
                    if (v >= 0 && static_cast<uint32_t>(v) < S) {
                        st[j] = kHit;
                        slot[j] = v;
                        hitf[v] = 1;
                    } else if (v == kNotFound) {
                        st[j] = kMiss;
                    } else {
                        bits |= ASU_ST_BAD_STATE;  // the oracle raises on these
                    }
                }
            }
        }
        __syncthreads();
#pragma unroll
        for (int j = 0; j < IPT_Q; ++j)
            if (st[j] == kMiss) atomicMin(trow + key[j], kClaimBase + static_cast<int32_t>(tid * IPT_Q + j));
        __syncthreads();
        int canon[IPT_Q];
        int local = 0;
#pragma unroll
        for (int j = 0; j < IPT_Q; ++j) {
            canon[j] = st[j] == kMiss && ld_cg(trow + key[j]) == kClaimBase + static_cast<int32_t>(tid * IPT_Q + j);
            local += canon[j];
        }
        int M = 0;
        int mrank = block_exclusive_scan(local, scan_buf, &M);

        // stable partition of the LRU row (held in registers)
        int32_t lv[IPT_S];
        bool lh[IPT_S];
        int packed = 0;
#pragma unroll
        for (int j = 0; j < IPT_S; ++j) {
            const uint32_t idx = tid * IPT_S + j;
            lv[j] = -1;
            lh[j] = false;
            if (idx < S) {
                lv[j] = lrow[idx];
                if (static_cast<uint32_t>(lv[j]) < S) {
                    lh[j] = hitf[lv[j]] != 0;
                    packed += lh[j] ? (1 << 16) : 1;
                } else {
                    bits |= ASU_ST_BAD_STATE;
                }
            }
        }
        int ptotal = 0;
        int pre = block_exclusive_scan(packed, scan_buf, &ptotal);
        const int V = ptotal & 0xffff;
        int hrank = pre >> 16, erank = pre & 0xffff;
#pragma unroll
        for (int j = 0; j < IPT_S; ++j) {
            if (lv[j] < 0 || static_cast<uint32_t>(lv[j]) >= S || lh[j]) continue;
            if (erank < M) vict[erank] = lv[j];
            ++erank;
        }
        __syncthreads();

        if (M > V) {  // block-uniform: not enough evictable slots; undo the claims, change nothing
#pragma unroll
            for (int j = 0; j < IPT_Q; ++j)
                if (canon[j]) st_cg(trow + key[j], kNotFound);
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
                const int32_t vt = ld_cg(srow + victim);
                if (vt >= 0) {
                    if (static_cast<uint32_t>(vt) < K) st_cg(trow + vt, kNotFound);
                    else bits |= ASU_ST_BAD_STATE;
                }
                st_cg(srow + victim, key[j]);
                st_cg(trow + key[j], victim);
            }
            // new order: stale evictables, then this batch's victims, then hit slots
            erank = pre & 0xffff;
#pragma unroll
            for (int j = 0; j < IPT_S; ++j) {
                if (lv[j] < 0 || static_cast<uint32_t>(lv[j]) >= S) continue;
                int dst;
                if (lh[j]) {
                    dst = V + hrank++;
                } else {
                    dst = erank >= M ? erank - M : (V - M) + erank;
                    ++erank;
                }
                lrow[dst] = static_cast<int16_t>(lv[j]);
            }
            __syncthreads();
#pragma unroll
            for (int j = 0; j < IPT_Q; ++j) {
                const uint32_t pos = tid * IPT_Q + j;
                if (pos >= Q) continue;
                int32_t out = kNotFound;
                if (static_cast<uint32_t>(key[j]) < K) out = ld_cg(trow + key[j]);
                slot_ids[static_cast<uint64_t>(r) * Q + pos] = out;
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
    static unsigned long long configured = 0;  // one bit per device
    int dev = 0;
    cudaGetDevice(&dev);
    const int max_smem = kThreads * IPT_Q * 4 + kThreads * IPT_S;
    if (dev < 64 && !((configured >> dev) & 1ull)) {
        cudaError_t e = cudaFuncSetAttribute(batch_lru_kernel<IPT_Q, IPT_S>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
        if (e != cudaSuccess) {
            cudaGetLastError();  // leave no error behind for the caller's runtime checks
            return ASU_ERR_CUDA_BASE + static_cast<int>(e);
        }
        configured |= 1ull << dev;
    }
    const size_t smem = static_cast<size_t>(Q) * 4 + S;
    const uint32_t grid = R < 65535u ? R : 65535u;
    batch_lru_kernel<IPT_Q, IPT_S><<<grid, kThreads, smem, s>>>(t2s, s2t, lru, q, slot_ids, mask, R, K, S, Q, status);
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
