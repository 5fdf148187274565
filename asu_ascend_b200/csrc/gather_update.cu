// Pure lookup gather and seeded random update of a per-request int32 table.
//
// Reference behaviour: simu/hbm_lookup_update/src/hbm_lookup_update_kernel.cpp
//   gather  :88-133  out[r,i] = table[r, q[r,i]], output rows padded to 64 with zeros
//   update  :176-209 table[r, q[r,pos_t]] = new[r,pos_t], pos_t = (a*t+b) mod Q, serial in t
//
// B200 design: the gather is a latency-bound random 4-byte read per query.  Each
// thread owns four consecutive queries (one 16-byte load of keys, four independent
// table loads in flight, one 16-byte store of results, one 4-byte store of the hit
// mask), and the grid covers all requests at once, so a 64 x 2048 batch keeps
// ~32K threads with 128K loads in flight across the 148 SMs.  The update is one
// CTA per request; updates are applied in chunks of blockDim positions in t order,
// and inside a chunk a shared-memory hash table keeps only the largest t per key,
// which is exactly the serial last-writer result.
#include "asu_common.cuh"

namespace asu {
namespace {

constexpr int kGatherThreads = 256;

__device__ __forceinline__ int32_t gather_one(const int32_t* __restrict__ row, uint32_t index_size, int32_t key,
                                              int32_t not_found, bool& bad) {
    uint32_t k = static_cast<uint32_t>(key);
    if (k >= index_size) {
        bad = true;
        return not_found;
    }
    return __ldg(row + k);
}

// Vector path: query_len % 4 == 0, out_stride % 4 == 0, 16-byte aligned pointers.
__global__ void __launch_bounds__(kGatherThreads)
gather_vec4_kernel(const int32_t* __restrict__ table, uint32_t index_size, const int4* __restrict__ query4,
                   uint32_t query_len, int32_t* __restrict__ out, uint32_t out_stride, uint8_t* __restrict__ hit,
                   uint32_t req_num, int32_t not_found, int32_t* status) {
    const uint32_t q4_per_row = query_len >> 2;
    const uint64_t total = static_cast<uint64_t>(req_num) * q4_per_row;
    for (uint64_t t = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; t < total;
         t += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
        const uint32_t r = static_cast<uint32_t>(t / q4_per_row);
        const uint32_t i = static_cast<uint32_t>(t - static_cast<uint64_t>(r) * q4_per_row) << 2;
        const int4 k = __ldg(query4 + t);
        const int32_t* row = table + static_cast<uint64_t>(r) * index_size;
        bool bad = false;
        int4 v;
        v.x = gather_one(row, index_size, k.x, not_found, bad);
        v.y = gather_one(row, index_size, k.y, not_found, bad);
        v.z = gather_one(row, index_size, k.z, not_found, bad);
        v.w = gather_one(row, index_size, k.w, not_found, bad);
        *reinterpret_cast<int4*>(out + static_cast<uint64_t>(r) * out_stride + i) = v;
        if (hit != nullptr) {
            uchar4 h = make_uchar4(v.x != not_found, v.y != not_found, v.z != not_found, v.w != not_found);
            *reinterpret_cast<uchar4*>(hit + static_cast<uint64_t>(r) * query_len + i) = h;
        }
        if (bad) flag_status(status, r, ASU_ST_BAD_QUERY);
    }
    // zero padding columns [query_len, out_stride)
    if (out_stride > query_len) {
        const uint32_t pad = out_stride - query_len;
        const uint64_t ptotal = static_cast<uint64_t>(req_num) * pad;
        for (uint64_t t = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; t < ptotal;
             t += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
            const uint32_t r = static_cast<uint32_t>(t / pad);
            const uint32_t j = static_cast<uint32_t>(t - static_cast<uint64_t>(r) * pad);
            out[static_cast<uint64_t>(r) * out_stride + query_len + j] = 0;
        }
    }
}

// Scalar path for any row length / stride.
__global__ void __launch_bounds__(kGatherThreads)
gather_scalar_kernel(const int32_t* __restrict__ table, uint32_t index_size, const int32_t* __restrict__ query,
                     uint32_t query_len, int32_t* __restrict__ out, uint32_t out_stride, uint8_t* __restrict__ hit,
                     uint32_t req_num, int32_t not_found, int32_t* status) {
    const uint64_t total = static_cast<uint64_t>(req_num) * out_stride;
    for (uint64_t t = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; t < total;
         t += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
        const uint32_t r = static_cast<uint32_t>(t / out_stride);
        const uint32_t i = static_cast<uint32_t>(t - static_cast<uint64_t>(r) * out_stride);
        if (i >= query_len) {
            out[t] = 0;
            continue;
        }
        bool bad = false;
        const int32_t v = gather_one(table + static_cast<uint64_t>(r) * index_size, index_size,
                                     __ldg(query + static_cast<uint64_t>(r) * query_len + i), not_found, bad);
        out[t] = v;
        if (hit != nullptr) hit[static_cast<uint64_t>(r) * query_len + i] = v != not_found;
        if (bad) flag_status(status, r, ASU_ST_BAD_QUERY);
    }
}

constexpr int kUpdateThreads = 1024;
constexpr int kUpdateHash = 2 * kUpdateThreads;  // power of two, >= 2x the keys of one chunk

__device__ uint32_t gcd_u32(uint32_t a, uint32_t b) {
    while (b != 0U) {
        uint32_t r = a % b;
        a = b;
        b = r;
    }
    return a;
}

// First a coprime with n, scanning upward from hash32(seed) % n (kernel.cpp:41-57).
__device__ uint32_t pick_coprime_a(uint32_t seed, uint32_t n) {
    if (n <= 1U) return 1U;
    uint32_t a = hash32(seed) % n;
    if (a == 0U) a = 1U;
    while (gcd_u32(a, n) != 1U) {
        ++a;
        if (a >= n) a = 1U;
    }
    return a;
}

__global__ void __launch_bounds__(kUpdateThreads)
random_update_kernel(int32_t* __restrict__ table, uint32_t index_size, const int32_t* __restrict__ query,
                     const int32_t* __restrict__ new_states, uint32_t query_len, uint32_t req_num, uint32_t seed,
                     uint32_t update_num, int32_t* status) {
    __shared__ int32_t hkey[kUpdateHash];
    __shared__ int32_t hmax[kUpdateHash];
    __shared__ uint32_t ab[2];
    for (uint32_t r = blockIdx.x; r < req_num; r += gridDim.x) {
        if (threadIdx.x == 0) {
            const uint32_t req_seed = seed ^ hash32(r);
            ab[0] = pick_coprime_a(req_seed ^ 0x9e3779b9U, query_len);
            ab[1] = hash32(req_seed ^ 0x85ebca6bU) % query_len;
        }
        __syncthreads();
        const uint64_t a = ab[0], b = ab[1];
        const int32_t* qrow = query + static_cast<uint64_t>(r) * query_len;
        const int32_t* nrow = new_states + static_cast<uint64_t>(r) * query_len;
        int32_t* trow = table + static_cast<uint64_t>(r) * index_size;
        for (uint32_t base = 0; base < update_num; base += kUpdateThreads) {
            for (int i = threadIdx.x; i < kUpdateHash; i += kUpdateThreads) hkey[i] = -1;
            __syncthreads();
            const uint32_t t = base + threadIdx.x;
            int32_t key = -1, val = 0, hslot = -1;
            if (t < update_num) {
                const uint32_t pos = static_cast<uint32_t>((a * t + b) % query_len);
                key = qrow[pos];
                val = nrow[pos];
                if (static_cast<uint32_t>(key) >= index_size) {
                    flag_status(status, r, ASU_ST_BAD_QUERY);
                    key = -1;
                } else {
                    uint32_t h = hash32(static_cast<uint32_t>(key)) & (kUpdateHash - 1);
                    while (true) {  // terminates: at most 1024 keys in a 2048-entry table
                        const int32_t old = atomicCAS(&hkey[h], -1, key);
                        if (old == -1 || old == key) break;
                        h = (h + 1) & (kUpdateHash - 1);
                    }
                    hslot = static_cast<int32_t>(h);
                    hmax[h] = -1;
                }
            }
            __syncthreads();
            if (hslot >= 0) atomicMax(&hmax[hslot], static_cast<int32_t>(threadIdx.x));
            __syncthreads();
            if (hslot >= 0 && hmax[hslot] == static_cast<int32_t>(threadIdx.x)) trow[key] = val;
            __syncthreads();
        }
    }
}

inline uint32_t grid_for(uint64_t work, int threads) {
    uint64_t g = (work + threads - 1) / threads;
    const uint64_t cap = static_cast<uint64_t>(asu_sm_count()) * 16ull;
    if (g > cap) g = cap;
    return static_cast<uint32_t>(g < 1 ? 1 : g);
}

}  // namespace
}  // namespace asu

using namespace asu;

extern "C" int asu_gather_lookup(void* stream, const int32_t* table, uint32_t index_size, const int32_t* query,
                                 uint32_t query_len, int32_t* out, uint32_t out_stride, uint8_t* hit_mask,
                                 uint32_t req_num, int32_t not_found, int32_t* status) {
    if (req_num == 0) return ASU_OK;
    if (!table || !out || (query_len > 0 && !query) || out_stride < query_len || index_size == 0) return ASU_ERR_ARG;
    if (out_stride == 0) return ASU_OK;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const bool vec = (query_len % 4 == 0) && (out_stride % 4 == 0) &&
                     (reinterpret_cast<uintptr_t>(query) % 16 == 0) && (reinterpret_cast<uintptr_t>(out) % 16 == 0) &&
                     (hit_mask == nullptr || reinterpret_cast<uintptr_t>(hit_mask) % 4 == 0);
    if (vec) {
        const uint64_t work = static_cast<uint64_t>(req_num) * (query_len / 4);
        const uint64_t padw = static_cast<uint64_t>(req_num) * (out_stride - query_len);
        gather_vec4_kernel<<<grid_for(work > padw ? work : padw, kGatherThreads), kGatherThreads, 0, s>>>(
            table, index_size, reinterpret_cast<const int4*>(query), query_len, out, out_stride, hit_mask, req_num,
            not_found, status);
    } else {
        gather_scalar_kernel<<<grid_for(static_cast<uint64_t>(req_num) * out_stride, kGatherThreads), kGatherThreads,
                               0, s>>>(table, index_size, query, query_len, out, out_stride, hit_mask, req_num,
                                       not_found, status);
    }
    return asu_launch_status();
}

extern "C" int asu_random_update(void* stream, int32_t* table, uint32_t index_size, const int32_t* query,
                                 const int32_t* new_states, uint32_t query_len, uint32_t req_num, uint32_t seed,
                                 uint32_t update_percent, int32_t* status) {
    if (req_num == 0 || query_len == 0 || update_percent == 0) return ASU_OK;
    if (!table || !query || !new_states || index_size == 0 || index_size > 0x7fffffffu || update_percent > 100)
        return ASU_ERR_ARG;
    uint64_t update_num = (static_cast<uint64_t>(query_len) * update_percent) / 100u;
    if (update_num > query_len) update_num = query_len;
    if (update_num == 0) return ASU_OK;
    const uint32_t cap = static_cast<uint32_t>(asu_sm_count()) * 8u;
    const uint32_t grid = req_num < cap ? req_num : cap;
    random_update_kernel<<<grid, kUpdateThreads, 0, static_cast<cudaStream_t>(stream)>>>(
        table, index_size, query, new_states, query_len, req_num, seed, static_cast<uint32_t>(update_num), status);
    return asu_launch_status();
}

extern "C" int hbm_lookup_vec_do(uint32_t blockDim, void* stream, void* tableKeys, void* tableStates,
                                 void* queryKeys, void* statesOut, uint32_t reqNum, uint32_t queryLen,
                                 int32_t notFound) {
    (void)blockDim;
    (void)tableKeys;
    // The reference kernel ignores notFound and returns the raw table entry; out-of-range
    // keys (which it reads out of bounds) return -1 here.
    (void)notFound;
    if (queryLen == 0) return ASU_OK;
    const uint32_t padded = (queryLen + ASU_HBM_QUERY_TILE - 1) / ASU_HBM_QUERY_TILE * ASU_HBM_QUERY_TILE;
    return asu_gather_lookup(stream, static_cast<const int32_t*>(tableStates), ASU_HBM_INDEX_SIZE,
                             static_cast<const int32_t*>(queryKeys), queryLen, static_cast<int32_t*>(statesOut),
                             padded, nullptr, reqNum, -1, nullptr);
}

extern "C" int hbm_random_update_do(uint32_t blockDim, void* stream, void* tableKeys, void* tableStates,
                                    void* queryKeys, void* newStates, uint32_t reqNum, uint32_t queryLen,
                                    uint32_t seed, uint32_t updatePercent) {
    (void)blockDim;
    (void)tableKeys;
    return asu_random_update(stream, static_cast<int32_t*>(tableStates), ASU_HBM_INDEX_SIZE,
                             static_cast<const int32_t*>(queryKeys), static_cast<const int32_t*>(newStates), queryLen,
                             reqNum, seed, updatePercent, nullptr);
}
