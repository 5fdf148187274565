// Per-layer resolver state (re)initialisation on the device.
//
// Reference behaviour: patch/0003 vllm_ascend/attention/asu_kv_cache_manager.py
// ASULayerKVCacheContext.reset_state (patch lines 234-292):
//   token_state[:] = INVALID; asu_record_addr[:] = INVALID; hbm_slot_of_token[:] = INVALID
//   slot_owner_token[:] = INVALID; free_slot_stack = arange(slots); free_slot_count = slots
//   prefix p < managed_prefix_len: token_state = ASU_ONLY,
//                                  asu_record_addr = block_table[p / bs] * bs + p % bs
//   managed_prefix_len <= p < actual_seq_len: token_state = TAIL_HBM
// The reference does this with a handful of torch ops per layer; here it is one grid-stride
// launch writing every array once (coalesced 4-byte stores), so a decode step that resets
// all layers costs one small kernel per layer.
#include "asu_common.cuh"

namespace asu {
namespace {

constexpr int kThreads = 256;

__global__ void __launch_bounds__(kThreads)
resolver_reset_kernel(int32_t* __restrict__ token_state, int32_t* __restrict__ record,
                      int32_t* __restrict__ hbm_slot, int64_t max_seq, int32_t* __restrict__ owner,
                      int32_t* __restrict__ stack, int32_t* __restrict__ count, int64_t slots,
                      const int32_t* __restrict__ block_table, int64_t bs, int64_t actual, int64_t prefix) {
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t p = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; p < max_seq; p += stride) {
        int32_t st = ASU_TOKEN_INVALID, rec = ASU_TOKEN_INVALID;
        if (p < prefix) {
            st = ASU_TOKEN_ASU_ONLY;
            rec = static_cast<int32_t>(static_cast<int64_t>(__ldg(block_table + p / bs)) * bs + p % bs);
        } else if (p < actual) {
            st = ASU_TOKEN_TAIL_HBM;
        }
        token_state[p] = st;
        record[p] = rec;
        hbm_slot[p] = kNotFound;
    }
    for (int64_t s = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; s < slots; s += stride) {
        owner[s] = kNotFound;
        stack[s] = static_cast<int32_t>(s);
    }
    if (blockIdx.x == 0 && threadIdx.x == 0) *count = static_cast<int32_t>(slots);
}

}  // namespace
}  // namespace asu

using namespace asu;

extern "C" int asu_resolver_reset(void* stream, int32_t* token_state, int32_t* asu_record_addr,
                                  int32_t* hbm_slot_of_token, int64_t max_seq_len, int32_t* slot_owner_token,
                                  int32_t* free_slot_stack, int32_t* free_slot_count, int64_t slot_count,
                                  const int32_t* block_table, int64_t block_table_len, int64_t block_size,
                                  int64_t actual_seq_len, int64_t managed_prefix_len) {
    if (!token_state || !asu_record_addr || !hbm_slot_of_token || !slot_owner_token || !free_slot_stack ||
        !free_slot_count)
        return ASU_ERR_ARG;
    // the reference's ValueError / RuntimeError conditions (patch lines 241-249, 279-280)
    if (max_seq_len <= 0 || slot_count <= 0 || slot_count > 0x7fffffff || block_size <= 0 || actual_seq_len < 0 ||
        managed_prefix_len < 0 || managed_prefix_len > actual_seq_len || actual_seq_len > max_seq_len)
        return ASU_ERR_ARG;
    if (managed_prefix_len > 0 && (!block_table || (managed_prefix_len - 1) / block_size >= block_table_len))
        return ASU_ERR_ARG;
    int64_t work = max_seq_len > slot_count ? max_seq_len : slot_count;
    int64_t grid = (work + kThreads - 1) / kThreads;
    const int64_t cap = static_cast<int64_t>(asu_sm_count()) * 16;
    if (grid > cap) grid = cap;
    resolver_reset_kernel<<<static_cast<uint32_t>(grid), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
        token_state, asu_record_addr, hbm_slot_of_token, max_seq_len, slot_owner_token, free_slot_stack,
        free_slot_count, slot_count, block_table, block_size, actual_seq_len, managed_prefix_len);
    return asu_launch_status();
}
