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
// launch writing every array once (coalesced 4-byte stores).  A manager that keeps every
// layer's state in [layers, ...] tensors resets all its layers with one launch (the y grid
// dimension walks the layers), and registers a decode token in all of them with one more
// (ASULayerKVCacheContext.mark_decode_token, patch lines 294-298, per layer in the reference).
#include "asu_common.cuh"

namespace asu {
namespace {

constexpr int kThreads = 256;

__global__ void __launch_bounds__(kThreads)
resolver_reset_kernel(int32_t* __restrict__ token_state, int32_t* __restrict__ record,
                      int32_t* __restrict__ hbm_slot, int64_t max_seq, int32_t* __restrict__ owner,
                      int32_t* __restrict__ stack, int32_t* __restrict__ count, int64_t slots,
                      const int32_t* __restrict__ block_table, int64_t bs, int64_t actual, int64_t prefix) {
    // layer blockIdx.y of [layers, max_seq] / [layers, slots] / [layers] state
    const int64_t layer = blockIdx.y;
    token_state += layer * max_seq;
    record += layer * max_seq;
    hbm_slot += layer * max_seq;
    owner += layer * slots;
    stack += layer * slots;
    count += layer;
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

// token_state[l * max_seq + token] = TAIL_HBM for every layer l.
__global__ void __launch_bounds__(kThreads)
mark_token_kernel(int32_t* __restrict__ token_state, int64_t layers, int64_t max_seq, int64_t token) {
    for (int64_t l = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; l < layers;
         l += static_cast<int64_t>(gridDim.x) * blockDim.x)
        token_state[l * max_seq + token] = ASU_TOKEN_TAIL_HBM;
}

}  // namespace
}  // namespace asu

using namespace asu;

extern "C" int asu_resolver_reset_layers(void* stream, int64_t layers, int32_t* token_state,
                                         int32_t* asu_record_addr, int32_t* hbm_slot_of_token, int64_t max_seq_len,
                                         int32_t* slot_owner_token, int32_t* free_slot_stack,
                                         int32_t* free_slot_count, int64_t slot_count, const int32_t* block_table,
                                         int64_t block_table_len, int64_t block_size, int64_t actual_seq_len,
                                         int64_t managed_prefix_len) {
    if (layers == 0) return ASU_OK;
    if (layers < 0 || layers > 65535 || !token_state || !asu_record_addr || !hbm_slot_of_token ||
        !slot_owner_token || !free_slot_stack || !free_slot_count)
        return ASU_ERR_ARG;
    // the reference's ValueError / RuntimeError conditions (patch lines 241-249, 279-280)
    if (max_seq_len <= 0 || slot_count <= 0 || slot_count > 0x7fffffff || block_size <= 0 || actual_seq_len < 0 ||
        managed_prefix_len < 0 || managed_prefix_len > actual_seq_len || actual_seq_len > max_seq_len)
        return ASU_ERR_ARG;
    if (managed_prefix_len > 0 && (!block_table || (managed_prefix_len - 1) / block_size >= block_table_len))
        return ASU_ERR_ARG;
    int64_t work = max_seq_len > slot_count ? max_seq_len : slot_count;
    int64_t grid = (work + kThreads - 1) / kThreads;
    const int64_t cap = (static_cast<int64_t>(asu_sm_count()) * 16 + layers - 1) / layers;  // blocks per layer
    if (grid > cap) grid = cap;
    if (grid < 1) grid = 1;
    resolver_reset_kernel<<<dim3(static_cast<uint32_t>(grid), static_cast<uint32_t>(layers)), kThreads, 0,
                            static_cast<cudaStream_t>(stream)>>>(
        token_state, asu_record_addr, hbm_slot_of_token, max_seq_len, slot_owner_token, free_slot_stack,
        free_slot_count, slot_count, block_table, block_size, actual_seq_len, managed_prefix_len);
    return asu_launch_status();
}

extern "C" int asu_resolver_reset(void* stream, int32_t* token_state, int32_t* asu_record_addr,
                                  int32_t* hbm_slot_of_token, int64_t max_seq_len, int32_t* slot_owner_token,
                                  int32_t* free_slot_stack, int32_t* free_slot_count, int64_t slot_count,
                                  const int32_t* block_table, int64_t block_table_len, int64_t block_size,
                                  int64_t actual_seq_len, int64_t managed_prefix_len) {
    return asu_resolver_reset_layers(stream, 1, token_state, asu_record_addr, hbm_slot_of_token, max_seq_len,
                                     slot_owner_token, free_slot_stack, free_slot_count, slot_count, block_table,
                                     block_table_len, block_size, actual_seq_len, managed_prefix_len);
}

extern "C" int asu_resolver_mark_token(void* stream, int64_t layers, int32_t* token_state, int64_t max_seq_len,
                                       int64_t token_id) {
    if (layers == 0) return ASU_OK;
    if (layers < 0 || !token_state || max_seq_len <= 0 || token_id < 0 || token_id >= max_seq_len)
        return ASU_ERR_ARG;
    const int64_t blocks = (layers + kThreads - 1) / kThreads;
    mark_token_kernel<<<static_cast<uint32_t>(blocks < 65535 ? blocks : 65535), kThreads, 0,
                        static_cast<cudaStream_t>(stream)>>>(token_state, layers, max_seq_len, token_id);
    return asu_launch_status();
}
