// ops contract: lookup with sequential free-list allocation, and the hash-seeded ring maintain.
//
// Reference behaviour (serial per request):
//   lookup   ops/asu_hbm_index_lookup_aiv.cpp:79-130, oracle ops/scripts/asu_hbm_index_common.py:119-139
//            slot = index[q]; on -1: slot = free_slots[head++], index[q] = slot,
//            slot_to_index[slot] = q.  Later duplicates of q reuse the slot.
//   maintain ops/asu_hbm_index_maintain_aicpu_kernel.aicpu:53-95, oracle asu_hbm_index_common.py:185-214
//            walk slots from hash32(seed ^ req) % SLOT_COUNT around the ring; every occupied,
//            unprotected slot is evicted and stored at free_slots[--head] until head == 0.
//
// B200 design: one CTA (1024 threads) per request row.
//  * lookup: queries are processed in chunks of 2048 (two per thread, thread-contiguous).
//    While the query and index loads are in flight the CTA prefetches the free-list window
//    free_slots[head .. head+2048) into shared memory.  The first occurrence of each missing
//    key is found in a shared-memory hash (atomicMin of the position per key), a block-wide
//    exclusive scan over the first-occurrence flags gives each one its rank in query order,
//    and rank k takes free_slots[head + k] -- the serial free_head++ order.  Later
//    duplicates read the allocated slot from the hash after a barrier.
//  * maintain: the protected set is a shared-memory bitset; the ring is walked in
//    thread-contiguous chunks, a scan over the evictable flags ranks candidates in ring
//    order, and rank k < head is evicted into free_slots[head - 1 - k] -- the serial
//    --head order.  One pass covers every slot; if fewer than head slots are evictable
//    the reference would spin forever, here the row gets ASU_ST_RING_EXHAUSTED.
#include "asu_common.cuh"

namespace asu {
namespace {

constexpr int kThreads = 1024;
constexpr int kItems = 2;                   // queries per thread per chunk
constexpr int kChunk = kThreads * kItems;   // 2048 = the reference QUERY_COUNT

constexpr int kHash = 2 * kChunk;           // shared-memory hash: at most kChunk keys, load <= 1/2

// Claim `key` for chunk position `li` (the smallest position wins); returns the table index,
// -1 only if the table were full, which kHash > kChunk rules out.
__device__ __forceinline__ int claim_first(int32_t* keys, int32_t* first, int32_t key, int32_t li) {
    uint32_t h = hash32(static_cast<uint32_t>(key)) & (kHash - 1);
    for (int probe = 0; probe < kHash; ++probe) {
        const int32_t prev = atomicCAS(keys + h, -1, key);
        if (prev == -1 || prev == key) {
            atomicMin(first + h, li);
            return static_cast<int>(h);
        }
        h = (h + 1) & (kHash - 1);
    }
    return -1;
}

__global__ void __launch_bounds__(kThreads)
ops_lookup_kernel(int32_t* __restrict__ index, int32_t* __restrict__ slot_to_index,
                  const int32_t* __restrict__ free_slots, int32_t* __restrict__ free_head,
                  const int32_t* __restrict__ query, int32_t* __restrict__ slot_out, uint32_t req_num,
                  uint32_t index_size, uint32_t slot_count, uint32_t free_count, uint32_t query_count,
                  int32_t* status) {
    __shared__ int scan_buf[33];
    __shared__ int32_t h_key[kHash];    // missing key; reused for its allocated slot after ranking
    __shared__ int32_t h_first[kHash];  // first chunk position of the key
    __shared__ int32_t s_free[kChunk];  // free_slots[head + k], prefetched
    for (uint32_t r = blockIdx.x; r < req_num; r += gridDim.x) {
        int32_t* irow = index + static_cast<uint64_t>(r) * index_size;
        int32_t* srow = slot_to_index + static_cast<uint64_t>(r) * slot_count;
        const int32_t* frow = free_slots + static_cast<uint64_t>(r) * free_count;
        const int32_t* qrow = query + static_cast<uint64_t>(r) * query_count;
        int32_t* orow = slot_out + static_cast<uint64_t>(r) * query_count;
        int32_t head = ld_cg(free_head + r);
        int32_t bits = 0;
        for (uint32_t base = 0; base < query_count; base += kChunk) {
            for (int i = threadIdx.x; i < kHash; i += kThreads) {
                h_key[i] = -1;
                h_first[i] = INT32_MAX;
            }
            for (int k = threadIdx.x; k < kChunk; k += kThreads) {
                const int64_t f = static_cast<int64_t>(head) + k;
                s_free[k] = (f >= 0 && f < static_cast<int64_t>(free_count)) ? __ldg(frow + f) : kNotFound;
            }
            int32_t key[kItems], slot[kItems];
            bool miss[kItems];
#pragma unroll
            for (int j = 0; j < kItems; ++j) {
                const uint32_t pos = base + threadIdx.x * kItems + j;
                key[j] = -1;
                slot[j] = kNotFound;
                miss[j] = false;
                if (pos < query_count) {
                    key[j] = __ldg(qrow + pos);
                    if (static_cast<uint32_t>(key[j]) < index_size) {
                        slot[j] = ld_cg(irow + key[j]);
                        miss[j] = slot[j] == kNotFound;
                    } else {
                        bits |= ASU_ST_BAD_QUERY;
                        key[j] = -1;
                    }
                }
            }
            __syncthreads();  // tables cleared, free window loaded
            int h[kItems];
#pragma unroll
            for (int j = 0; j < kItems; ++j) {
                h[j] = miss[j] ? claim_first(h_key, h_first, key[j], static_cast<int32_t>(threadIdx.x * kItems + j)) : -1;
                if (miss[j] && h[j] < 0) {
                    bits |= ASU_ST_BAD_STATE;
                    miss[j] = false;
                }
            }
            __syncthreads();  // every claim made
            int canon[kItems];
            int local = 0;
#pragma unroll
            for (int j = 0; j < kItems; ++j) {
                canon[j] = miss[j] && h_first[h[j]] == static_cast<int32_t>(threadIdx.x * kItems + j);
                local += canon[j];
            }
            int total = 0;
            int rank = block_exclusive_scan(local, scan_buf, &total);  // ends with a barrier: h_key is free
#pragma unroll
            for (int j = 0; j < kItems; ++j) {
                if (!canon[j]) continue;
                const int32_t k = rank++;
                int32_t s = kNotFound;
                if (static_cast<int64_t>(head) + k < static_cast<int64_t>(free_count) && head + k >= 0) {
                    s = s_free[k];
                } else {
                    bits |= ASU_ST_FREE_EXHAUSTED;
                }
                if (s >= 0 && static_cast<uint32_t>(s) < slot_count) {
                    st_cg(irow + key[j], s);
                    st_cg(srow + s, key[j]);
                } else if (s != kNotFound) {
                    st_cg(irow + key[j], s);  // the reference stores whatever the free list holds
                    bits |= ASU_ST_BAD_STATE;
                }
                slot[j] = s;
                h_key[h[j]] = s;
            }
            __syncthreads();  // allocated slots published
#pragma unroll
            for (int j = 0; j < kItems; ++j) {
                const uint32_t pos = base + threadIdx.x * kItems + j;
                if (miss[j] && !canon[j]) slot[j] = h_key[h[j]];  // duplicate of an earlier miss
                if (pos < query_count) orow[pos] = slot[j];
            }
            int64_t nh = static_cast<int64_t>(head) + total;
            if (nh > static_cast<int64_t>(free_count)) nh = free_count;
            head = static_cast<int32_t>(nh);
            __syncthreads();  // before the next chunk clears the tables
        }
        if (threadIdx.x == 0) st_cg(free_head + r, head);
        if (bits) flag_status(status, r, bits);
        __syncthreads();
    }
}

constexpr int kMaxSlotsPerThread = 16;  // slot_count <= 16384

__global__ void __launch_bounds__(kThreads)
ops_maintain_kernel(int32_t* __restrict__ index, int32_t* __restrict__ slot_to_index,
                    int32_t* __restrict__ free_slots, int32_t* __restrict__ free_head,
                    const int32_t* __restrict__ last_query_slots, uint32_t req_num, uint32_t seed,
                    uint32_t index_size, uint32_t slot_count, uint32_t free_count, uint32_t query_count,
                    int32_t* status) {
    extern __shared__ uint32_t prot[];  // (slot_count + 31) / 32 words
    __shared__ int scan_buf[33];
    const uint32_t words = (slot_count + 31) / 32;
    const uint32_t per = (slot_count + kThreads - 1) / kThreads;
    for (uint32_t r = blockIdx.x; r < req_num; r += gridDim.x) {
        const int32_t head = ld_cg(free_head + r);
        if (head <= 0) continue;  // uniform across the block
        int32_t* irow = index + static_cast<uint64_t>(r) * index_size;
        int32_t* srow = slot_to_index + static_cast<uint64_t>(r) * slot_count;
        int32_t* frow = free_slots + static_cast<uint64_t>(r) * free_count;
        const int32_t* lrow = last_query_slots + static_cast<uint64_t>(r) * query_count;
        for (uint32_t w = threadIdx.x; w < words; w += kThreads) prot[w] = 0u;
        __syncthreads();
        for (uint32_t i = threadIdx.x; i < query_count; i += kThreads) {
            const uint32_t s = static_cast<uint32_t>(__ldg(lrow + i));
            if (s < slot_count) atomicOr(&prot[s >> 5], 1u << (s & 31));
        }
        __syncthreads();
        const uint32_t start = hash32(seed ^ r) % slot_count;
        int32_t bits = 0;
        int local = 0;
        uint32_t slot_of[kMaxSlotsPerThread];
        int32_t key_of[kMaxSlotsPerThread];
        bool ev[kMaxSlotsPerThread];
#pragma unroll
        for (int j = 0; j < kMaxSlotsPerThread; ++j) {
            const uint32_t off = threadIdx.x * per + j;
            ev[j] = false;
            slot_of[j] = 0;
            key_of[j] = kNotFound;
            if (j < static_cast<int>(per) && off < slot_count) {
                uint32_t s = start + off;
                if (s >= slot_count) s -= slot_count;
                slot_of[j] = s;
                key_of[j] = ld_cg(srow + s);
                ev[j] = key_of[j] != kNotFound && !((prot[s >> 5] >> (s & 31)) & 1u);
                local += ev[j];
            }
        }
        int total = 0;
        int rank = block_exclusive_scan(local, scan_buf, &total);
#pragma unroll
        for (int j = 0; j < kMaxSlotsPerThread; ++j) {
            if (!ev[j]) continue;
            const int k = rank++;
            if (k >= head) break;
            st_cg(srow + slot_of[j], kNotFound);
            if (static_cast<uint32_t>(key_of[j]) < index_size) {
                st_cg(irow + key_of[j], kNotFound);
            } else {
                bits |= ASU_ST_BAD_STATE;
            }
            const int32_t dst = head - 1 - k;
            if (dst < static_cast<int32_t>(free_count)) st_cg(frow + dst, static_cast<int32_t>(slot_of[j]));
            else bits |= ASU_ST_BAD_STATE;
        }
        if (threadIdx.x == 0) {
            const int32_t evicted = total < head ? total : head;
            st_cg(free_head + r, head - evicted);
            if (total < head) bits |= ASU_ST_RING_EXHAUSTED;
        }
        if (bits) flag_status(status, r, bits);
        __syncthreads();
    }
}

inline uint32_t req_grid(uint32_t req_num) {
    const uint32_t cap = static_cast<uint32_t>(asu_sm_count()) * 16u;
    return req_num < cap ? req_num : cap;
}

}  // namespace
}  // namespace asu

using namespace asu;

extern "C" int asu_hbm_index_lookup_ex(void* stream, int32_t* index, int32_t* slot_to_index,
                                       const int32_t* free_slots, int32_t* free_head, const int32_t* query_index,
                                       int32_t* slot_out, uint32_t req_num, uint32_t index_size, uint32_t slot_count,
                                       uint32_t free_slot_count, uint32_t query_count, int32_t* status) {
    if (req_num == 0) return ASU_OK;
    if (!index || !slot_to_index || !free_slots || !free_head || (query_count && (!query_index || !slot_out)))
        return ASU_ERR_ARG;
    if (index_size == 0 || index_size > 0x7fffffffu || slot_count == 0 || query_count > 0x7ffffffeu)
        return ASU_ERR_ARG;
    ops_lookup_kernel<<<req_grid(req_num), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
        index, slot_to_index, free_slots, free_head, query_index, slot_out, req_num, index_size, slot_count,
        free_slot_count, query_count, status);
    return asu_launch_status();
}

extern "C" int asu_hbm_index_lookup_do(uint32_t blockDim, void* stream, void* index, void* slotToIndex,
                                       void* freeSlots, void* freeHead, void* queryIndex, void* slotOut,
                                       uint32_t reqNum) {
    (void)blockDim;  // advisory: the grid is one CTA per request row
    return asu_hbm_index_lookup_ex(stream, static_cast<int32_t*>(index), static_cast<int32_t*>(slotToIndex),
                                   static_cast<const int32_t*>(freeSlots), static_cast<int32_t*>(freeHead),
                                   static_cast<const int32_t*>(queryIndex), static_cast<int32_t*>(slotOut), reqNum,
                                   ASU_HBM_INDEX_SIZE, ASU_HBM_SLOT_COUNT, ASU_HBM_FREE_SLOT_COUNT,
                                   ASU_HBM_QUERY_COUNT, nullptr);
}

extern "C" int asu_hbm_index_maintain_ex(void* stream, int32_t* index, int32_t* slot_to_index, int32_t* free_slots,
                                         int32_t* free_head, const int32_t* last_query_slots, uint32_t req_num,
                                         uint32_t seed, uint32_t index_size, uint32_t slot_count,
                                         uint32_t free_slot_count, uint32_t query_count, int32_t* status) {
    if (req_num == 0) return ASU_OK;
    if (!index || !slot_to_index || !free_slots || !free_head || (query_count && !last_query_slots))
        return ASU_ERR_ARG;
    if (slot_count == 0 || slot_count > static_cast<uint32_t>(kThreads * kMaxSlotsPerThread) || index_size == 0 ||
        index_size > 0x7fffffffu)
        return ASU_ERR_ARG;
    const size_t smem = ((slot_count + 31) / 32) * sizeof(uint32_t);
    ops_maintain_kernel<<<req_grid(req_num), kThreads, smem, static_cast<cudaStream_t>(stream)>>>(
        index, slot_to_index, free_slots, free_head, last_query_slots, req_num, seed, index_size, slot_count,
        free_slot_count, query_count, status);
    return asu_launch_status();
}

extern "C" int asu_hbm_index_maintain_do(uint32_t blockDim, void* stream, void* index, void* slotToIndex,
                                         void* freeSlots, void* freeHead, void* lastQuerySlots, uint32_t reqNum,
                                         uint32_t seed) {
    (void)blockDim;  // the reference AICPU launcher ignores it too (ops/asu_hbm_index_maintain_aicpu.cpp:25)
    return asu_hbm_index_maintain_ex(stream, static_cast<int32_t*>(index), static_cast<int32_t*>(slotToIndex),
                                     static_cast<int32_t*>(freeSlots), static_cast<int32_t*>(freeHead),
                                     static_cast<const int32_t*>(lastQuerySlots), reqNum, seed, ASU_HBM_INDEX_SIZE,
                                     ASU_HBM_SLOT_COUNT, ASU_HBM_FREE_SLOT_COUNT, ASU_HBM_QUERY_COUNT, nullptr);
}
