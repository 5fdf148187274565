// C++ torch binding of the hot-path operators: npu_asu_resolve_kv_slots_single_req, the op a
// decode step calls once per layer, and the index operators asu_hbm_index_lookup,
// asu_hbm_index_maintain and asu_hbm_index_lookup_simt.
//
// Reference interface: patch/0001 csrc/torch_binding.cpp hunk (patch lines 810-826, schema) and
// csrc/asu_kv_resolver/asu_kv_resolver_torch_adpt.h (patch lines 21-59): TORCH_LIBRARY_FRAGMENT
// registration under _C_ascend, int32 index tensors, resolved = empty(topk.shape, int32).  The
// same schema is registered under `asu` and `_C_ascend` with CUDA, CPU (argument checks only:
// there is no CPU implementation) and Meta kernels.  The argument checks and their error types
// (ValueError / RuntimeError) are the ones the Python reference raises (patch lines 954-994).
//
// Index operators: ascend-ops/torch_binding_asu_hbm_index.cpp:7-25 (schemas under _C_ascend)
// and the adapters asu_hbm_index_lookup/asu_hbm_index_lookup_torch_adpt.h:15-35 and
// asu_hbm_index_maintain/asu_hbm_index_maintain_torch_adpt.h (the int32 dtype checks, then
// req_num > 0, then slot_out = empty_like(query_index)); the device, contiguity and row-width
// checks the raw pointers need follow.  The batch-LRU operator has no torch binding in the
// reference (pta-ops/asu_hbm_index_lookup_simt calls its C launcher through ctypes); it is
// registered here with the same conventions.
//
// Why C++: the ops are on the per-layer decode path, and a Python kernel spends tens of
// microseconds per call on argument handling; here a call costs a few microseconds of host time
// on top of its launches.  The kernels are reached through the C ABI (asu_kv_resolver_do,
// asu_hbm_index_*_ex).  A device status word is allocated, read back and turned into an error
// only while status checks are on; otherwise the launches get no status pointer and the ops stay
// asynchronous, like the NPU ones.
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/library.h>

#include <atomic>
#include <optional>
#include <sstream>
#include <tuple>
#include <string>

#include "../../include/asu_b200.h"

namespace {

std::atomic<bool> g_status_checks{false};

const char* const kStatusNames[] = {"BAD_QUERY",  "FREE_EXHAUSTED", "RING_EXHAUSTED",  "BAD_STATE", "SHORTAGE",
                                    "BAD_SOURCE", "BAD_TOKEN_STATE", "NO_VICTIM", "TIMEOUT"};

std::string status_list(int bits) {
    std::ostringstream os;
    os << "[";
    bool first = true;
    for (int i = 0; i < 9; ++i) {
        if (bits & (1 << i)) {
            os << (first ? "" : ", ") << "'" << kStatusNames[i] << "'";
            first = false;
        }
    }
    os << "]";
    return os.str();
}

// Read-only index inputs: int64 is narrowed to int32 (the NPU op takes int32 only).
at::Tensor as_i32_input(const char* name, const at::Tensor& t, const c10::Device& dev) {
    TORCH_CHECK(t.device() == dev, name, " must be on ", dev);
    at::Tensor r = t.scalar_type() == at::kLong ? t.to(at::kInt) : t;
    TORCH_CHECK(r.scalar_type() == at::kInt, name, " must be int32");
    return r.contiguous();
}

void req_cuda_i32(const char* name, const at::Tensor& t, const c10::Device& dev) {
    TORCH_CHECK(t.scalar_type() == at::kInt, name, " must be int32");
    TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor, got ", t.numel(),
                " elements in host memory (asu_ascend_b200 has no CPU implementation)");
    TORCH_CHECK(t.device() == dev, name, " must be on ", dev, ", got ", t.device());
    TORCH_CHECK(t.is_contiguous(), name, " must be contiguous");
}

bool kv_dtype_ok(const at::Tensor& t) {
    const auto d = t.scalar_type();
    return d == at::kHalf || d == at::kBFloat16 || d == at::kFloat;
}

int64_t row_bytes(const at::Tensor& t) {
    const int64_t rows = t.size(0) > 0 ? t.size(0) : 1;
    return t.numel() / rows * static_cast<int64_t>(t.element_size());
}

// The checks of patch lines 964-994 and the pointer contract, in the order the Python op runs them.
struct Prepared {
    at::Tensor topk, record, stack, block_table;
};

Prepared prepare(const at::Tensor& topk_in, int64_t actual_seq_len, const at::Tensor& token_state,
                 const at::Tensor& asu_record_addr, const at::Tensor& hbm_slot_of_token,
                 const at::Tensor& slot_owner_token, const at::Tensor& free_slot_stack,
                 const at::Tensor& free_slot_count, const at::Tensor& block_table_in, const at::Tensor& o0,
                 const at::Tensor& o1, const at::Tensor& m0, const at::Tensor& m1, int64_t block_size) {
    TORCH_CHECK_VALUE(actual_seq_len >= 0, "actual_seq_len must be non-negative");
    TORCH_CHECK_VALUE(block_size > 0, "block_size must be positive");
    const c10::Device dev = token_state.device();
    req_cuda_i32("token_state", token_state, dev);
    req_cuda_i32("hbm_slot_of_token", hbm_slot_of_token, dev);
    req_cuda_i32("slot_owner_token", slot_owner_token, dev);
    req_cuda_i32("free_slot_count", free_slot_count, dev);
    Prepared p;
    p.topk = as_i32_input("original_topk_indices", topk_in, dev);
    p.record = as_i32_input("asu_record_addr", asu_record_addr, dev);
    p.stack = as_i32_input("free_slot_stack", free_slot_stack, dev);
    p.block_table = as_i32_input("original_block_table", block_table_in, dev);
    const char* names[] = {"original_kv_cache_0", "original_kv_cache_1", "managed_kv_cache_0", "managed_kv_cache_1"};
    const at::Tensor* kv[] = {&o0, &o1, &m0, &m1};
    for (int i = 0; i < 4; ++i) {
        TORCH_CHECK_VALUE(kv[i]->dim() >= 1, names[i], " must have a slot dimension");
        TORCH_CHECK(kv[i]->device() == dev && kv[i]->is_contiguous(), names[i], " must be a contiguous tensor on ",
                    dev);
        TORCH_CHECK(kv_dtype_ok(*kv[i]), names[i], " must be float16, bfloat16 or float32");
    }
    TORCH_CHECK_VALUE(o0.sizes().slice(1) == m0.sizes().slice(1),
                      "original_kv_cache_0 and managed_kv_cache_0 must have matching per-slot shapes");
    TORCH_CHECK_VALUE(o1.sizes().slice(1) == m1.sizes().slice(1),
                      "original_kv_cache_1 and managed_kv_cache_1 must have matching per-slot shapes");
    TORCH_CHECK(o0.scalar_type() == m0.scalar_type() && o1.scalar_type() == m1.scalar_type(),
                "original and managed KV caches must have the same dtype");
    return p;
}

at::Tensor resolve_cuda(const at::Tensor& original_topk_indices, int64_t actual_seq_len, int64_t managed_prefix_len,
                        const at::Tensor& token_state, const at::Tensor& asu_record_addr,
                        const at::Tensor& hbm_slot_of_token, const at::Tensor& slot_owner_token,
                        const at::Tensor& free_slot_stack, const at::Tensor& free_slot_count,
                        const at::Tensor& original_block_table, const at::Tensor& original_kv_cache_0,
                        const at::Tensor& original_kv_cache_1, const at::Tensor& managed_kv_cache_0,
                        const at::Tensor& managed_kv_cache_1, int64_t block_size) {
    (void)managed_prefix_len;  // unused by the reference as well (patch line 970)
    Prepared p = prepare(original_topk_indices, actual_seq_len, token_state, asu_record_addr, hbm_slot_of_token,
                         slot_owner_token, free_slot_stack, free_slot_count, original_block_table,
                         original_kv_cache_0, original_kv_cache_1, managed_kv_cache_0, managed_kv_cache_1,
                         block_size);
    const c10::Device dev = token_state.device();
    const c10::cuda::CUDAGuard guard(dev);
    at::Tensor resolved = at::empty(original_topk_indices.sizes(), token_state.options().dtype(at::kInt));
    const int64_t n = p.topk.numel();
    if (n == 0) return resolved;
    const at::Tensor &o0 = original_kv_cache_0, &o1 = original_kv_cache_1;
    const at::Tensor &m0 = managed_kv_cache_0, &m1 = managed_kv_cache_1;
    const int64_t src_rows = std::min(o0.size(0), o1.size(0));
    const int64_t slot_count = std::min({m0.size(0), m1.size(0), slot_owner_token.numel()});
    const int64_t max_seq = std::min({token_state.numel(), hbm_slot_of_token.numel(), p.record.numel()});
    at::Tensor ws = at::empty({asu_kv_resolver_workspace_bytes(n)}, token_state.options().dtype(at::kByte));
    const bool checks = g_status_checks.load(std::memory_order_relaxed);
    at::Tensor status = checks ? at::zeros({1}, token_state.options()) : at::Tensor();
    const cudaStream_t stream = c10::cuda::getCurrentCUDAStream(dev.index()).stream();
    const int rc = asu_kv_resolver_do(
        stream, p.topk.data_ptr<int32_t>(), n, token_state.data_ptr<int32_t>(), p.record.data_ptr<int32_t>(),
        hbm_slot_of_token.data_ptr<int32_t>(), slot_owner_token.data_ptr<int32_t>(), p.stack.data_ptr<int32_t>(),
        free_slot_count.data_ptr<int32_t>(), p.stack.numel(), p.block_table.data_ptr<int32_t>(),
        p.block_table.numel(), o0.data_ptr(), o1.data_ptr(), m0.data_ptr(), m1.data_ptr(), row_bytes(o0),
        row_bytes(o1), src_rows, slot_count, max_seq, actual_seq_len, block_size, resolved.data_ptr<int32_t>(),
        ws.data_ptr(), checks ? status.data_ptr<int32_t>() : nullptr);
    TORCH_CHECK(rc == ASU_OK, "npu_asu_resolve_kv_slots_single_req failed: ", asu_status_string(rc), " (code ", rc,
                ")");
    if (checks) {
        const int bits = status.item<int32_t>();
        if (bits != 0) {
            std::ostringstream hex;
            hex << std::hex << bits;
            TORCH_CHECK(false, "npu_asu_resolve_kv_slots_single_req: device status ", status_list(bits), " (0x",
                        hex.str(), ")");
        }
    }
    return resolved;
}

// Host tensors: the same argument checks, then the refusal the CUDA-only op gives.
at::Tensor resolve_cpu(const at::Tensor& original_topk_indices, int64_t actual_seq_len, int64_t managed_prefix_len,
                       const at::Tensor& token_state, const at::Tensor& asu_record_addr,
                       const at::Tensor& hbm_slot_of_token, const at::Tensor& slot_owner_token,
                       const at::Tensor& free_slot_stack, const at::Tensor& free_slot_count,
                       const at::Tensor& original_block_table, const at::Tensor& original_kv_cache_0,
                       const at::Tensor& original_kv_cache_1, const at::Tensor& managed_kv_cache_0,
                       const at::Tensor& managed_kv_cache_1, int64_t block_size) {
    (void)managed_prefix_len;
    prepare(original_topk_indices, actual_seq_len, token_state, asu_record_addr, hbm_slot_of_token, slot_owner_token,
            free_slot_stack, free_slot_count, original_block_table, original_kv_cache_0, original_kv_cache_1,
            managed_kv_cache_0, managed_kv_cache_1, block_size);
    TORCH_CHECK(false, "npu_asu_resolve_kv_slots_single_req needs CUDA tensors (asu_ascend_b200 has no CPU "
                       "implementation)");
}

// patch/0001 csrc/torch_binding_meta.cpp hunk (patch lines 592-625): output shape only.
at::Tensor resolve_meta(const at::Tensor& original_topk_indices, int64_t, int64_t, const at::Tensor&,
                        const at::Tensor&, const at::Tensor&, const at::Tensor&, const at::Tensor&, const at::Tensor&,
                        const at::Tensor&, const at::Tensor&, const at::Tensor&, const at::Tensor&, const at::Tensor&,
                        int64_t) {
    return at::empty(original_topk_indices.sizes(), original_topk_indices.options().dtype(at::kInt));
}

// ---------------------------------------------------------------------------------------------
// resolver over a bounded managed pool (exact-LRU eviction); no reference counterpart: it is the
// resolver of patch/0001 composed with simu/kv_cache_eviction_sim.py's LRUManagedCache, so the
// managed cache can be smaller than the context.  Same argument checks as the resolver op, plus
// the recency order row and the free target.

at::Tensor resolve_lru_cuda(const at::Tensor& original_topk_indices, int64_t actual_seq_len,
                            int64_t managed_prefix_len, const at::Tensor& token_state,
                            const at::Tensor& asu_record_addr, const at::Tensor& hbm_slot_of_token,
                            const at::Tensor& slot_owner_token, const at::Tensor& free_slot_stack,
                            const at::Tensor& free_slot_count, const at::Tensor& lru_order, int64_t free_target,
                            const at::Tensor& original_block_table, const at::Tensor& original_kv_cache_0,
                            const at::Tensor& original_kv_cache_1, const at::Tensor& managed_kv_cache_0,
                            const at::Tensor& managed_kv_cache_1, int64_t block_size,
                            const std::optional<at::Tensor>& stats) {
    (void)managed_prefix_len;
    Prepared p = prepare(original_topk_indices, actual_seq_len, token_state, asu_record_addr, hbm_slot_of_token,
                         slot_owner_token, free_slot_stack, free_slot_count, original_block_table,
                         original_kv_cache_0, original_kv_cache_1, managed_kv_cache_0, managed_kv_cache_1,
                         block_size);
    const c10::Device dev = token_state.device();
    req_cuda_i32("free_slot_stack", free_slot_stack, dev);  // written: evictions push on it
    req_cuda_i32("lru_order", lru_order, dev);
    TORCH_CHECK_VALUE(free_target >= 0, "free_target must be non-negative");
    int64_t* stats_ptr = nullptr;
    if (stats.has_value() && stats->defined()) {
        TORCH_CHECK(stats->scalar_type() == at::kLong && stats->device() == dev && stats->is_contiguous() &&
                        stats->numel() == ASU_LRU_STAT_COLS,
                    "stats must be a contiguous int64 tensor of ", ASU_LRU_STAT_COLS, " elements on ", dev);
        stats_ptr = stats->data_ptr<int64_t>();
    }
    const c10::cuda::CUDAGuard guard(dev);
    at::Tensor resolved = at::empty(original_topk_indices.sizes(), token_state.options().dtype(at::kInt));
    const int64_t n = p.topk.numel();
    TORCH_CHECK_VALUE(n <= 4096, "npu_asu_resolve_kv_slots_lru takes at most 4096 top-k entries, got ", n);
    const at::Tensor &o0 = original_kv_cache_0, &o1 = original_kv_cache_1;
    const at::Tensor &m0 = managed_kv_cache_0, &m1 = managed_kv_cache_1;
    const int64_t slot_count = std::min({m0.size(0), m1.size(0), slot_owner_token.numel(), free_slot_stack.numel(),
                                         lru_order.numel()});
    TORCH_CHECK_VALUE(slot_count > 0 && slot_count <= 16384, "managed slot count must be in [1, 16384], got ",
                      slot_count);
    const int64_t src_rows = std::min(o0.size(0), o1.size(0));
    const int64_t max_seq = std::min({token_state.numel(), hbm_slot_of_token.numel(), p.record.numel()});
    const bool checks = g_status_checks.load(std::memory_order_relaxed);
    at::Tensor status = checks ? at::zeros({1}, token_state.options()) : at::Tensor();
    const cudaStream_t stream = c10::cuda::getCurrentCUDAStream(dev.index()).stream();
    const int rc = asu_kv_resolver_lru(
        stream, p.topk.data_ptr<int32_t>(), n, token_state.data_ptr<int32_t>(), p.record.data_ptr<int32_t>(),
        hbm_slot_of_token.data_ptr<int32_t>(), slot_owner_token.data_ptr<int32_t>(),
        free_slot_stack.data_ptr<int32_t>(), free_slot_count.data_ptr<int32_t>(), lru_order.data_ptr<int32_t>(),
        slot_count, free_target, p.block_table.data_ptr<int32_t>(), p.block_table.numel(), o0.data_ptr(),
        o1.data_ptr(), m0.data_ptr(), m1.data_ptr(), row_bytes(o0), row_bytes(o1), src_rows, max_seq,
        actual_seq_len, block_size, resolved.data_ptr<int32_t>(), nullptr, nullptr, stats_ptr,
        checks ? status.data_ptr<int32_t>() : nullptr);
    TORCH_CHECK(rc == ASU_OK, "npu_asu_resolve_kv_slots_lru failed: ", asu_status_string(rc), " (code ", rc, ")");
    if (checks) {
        const int bits = status.item<int32_t>();
        if (bits != 0) {
            std::ostringstream hex;
            hex << std::hex << bits;
            TORCH_CHECK(false, "npu_asu_resolve_kv_slots_lru: device status ", status_list(bits), " (0x", hex.str(),
                        ")");
        }
    }
    return resolved;
}

at::Tensor resolve_lru_cpu(const at::Tensor& original_topk_indices, int64_t actual_seq_len,
                           int64_t managed_prefix_len, const at::Tensor& token_state,
                           const at::Tensor& asu_record_addr, const at::Tensor& hbm_slot_of_token,
                           const at::Tensor& slot_owner_token, const at::Tensor& free_slot_stack,
                           const at::Tensor& free_slot_count, const at::Tensor&, int64_t,
                           const at::Tensor& original_block_table, const at::Tensor& original_kv_cache_0,
                           const at::Tensor& original_kv_cache_1, const at::Tensor& managed_kv_cache_0,
                           const at::Tensor& managed_kv_cache_1, int64_t block_size,
                           const std::optional<at::Tensor>&) {
    (void)managed_prefix_len;
    prepare(original_topk_indices, actual_seq_len, token_state, asu_record_addr, hbm_slot_of_token, slot_owner_token,
            free_slot_stack, free_slot_count, original_block_table, original_kv_cache_0, original_kv_cache_1,
            managed_kv_cache_0, managed_kv_cache_1, block_size);
    TORCH_CHECK(false, "npu_asu_resolve_kv_slots_lru needs CUDA tensors (asu_ascend_b200 has no CPU implementation)");
}

at::Tensor resolve_lru_meta(const at::Tensor& original_topk_indices, int64_t, int64_t, const at::Tensor&,
                            const at::Tensor&, const at::Tensor&, const at::Tensor&, const at::Tensor&,
                            const at::Tensor&, const at::Tensor&, int64_t, const at::Tensor&, const at::Tensor&,
                            const at::Tensor&, const at::Tensor&, const at::Tensor&, int64_t,
                            const std::optional<at::Tensor>&) {
    return at::empty(original_topk_indices.sizes(), original_topk_indices.options().dtype(at::kInt));
}

// ---------------------------------------------------------------------------------------------
// index operators

int64_t row_width(const char* name, const at::Tensor& t, int64_t req_num) {
    TORCH_CHECK(t.numel() % req_num == 0, name, " has ", t.numel(), " elements, not a multiple of req_num=", req_num);
    const int64_t w = t.numel() / req_num;
    TORCH_CHECK(w <= 0x7fffffff, name, " rows are too long (", w, " elements)");
    return w;
}

void check_int32(const char* name, const at::Tensor& t) {
    TORCH_CHECK(t.scalar_type() == at::kInt, name, " must be int32");
}

// Status word of one launch: allocated only while checks are on.
at::Tensor new_status(int64_t req_num, const at::Tensor& like) {
    return g_status_checks.load(std::memory_order_relaxed) ? at::zeros({req_num}, like.options().dtype(at::kInt))
                                                            : at::Tensor();
}

void launch_ok(int rc, const char* what) {
    TORCH_CHECK(rc == ASU_OK, what, " failed: ", asu_status_string(rc), " (code ", rc, ")");
}

// Reads the status words back (a synchronisation) and raises on any bit but SHORTAGE, which the
// statistics count.
void raise_on_status(const at::Tensor& status, const char* what) {
    if (!status.defined()) return;
    const at::Tensor host = status.cpu();
    const int32_t* p = host.data_ptr<int32_t>();
    int bits = 0;
    for (int64_t i = 0; i < host.numel(); ++i) bits |= p[i];
    bits &= ~ASU_ST_SHORTAGE;
    if (bits != 0) {
        std::ostringstream hex;
        hex << std::hex << bits;
        TORCH_CHECK(false, what, ": device status ", status_list(bits), " (0x", hex.str(), ")");
    }
}

int32_t* status_ptr(const at::Tensor& status) { return status.defined() ? status.data_ptr<int32_t>() : nullptr; }

// The reference adapter's checks, in its order, then the pointer contract.
void index_op_checks(const char* const* names, const at::Tensor* const* ts, int n, int64_t req_num) {
    for (int i = 0; i < n; ++i) check_int32(names[i], *ts[i]);
    TORCH_CHECK(req_num > 0, "req_num must be greater than 0");
    TORCH_CHECK(req_num <= 0x7fffffff, "req_num must fit in int32");
    const c10::Device dev = ts[0]->device();
    for (int i = 0; i < n; ++i) req_cuda_i32(names[i], *ts[i], dev);
}

at::Tensor lookup_cuda(at::Tensor& index, at::Tensor& slot_to_index, at::Tensor& free_slots, at::Tensor& free_head,
                       const at::Tensor& query_index, int64_t req_num) {
    const char* names[] = {"index", "slot_to_index", "free_slots", "free_head", "query_index"};
    const at::Tensor* ts[] = {&index, &slot_to_index, &free_slots, &free_head, &query_index};
    index_op_checks(names, ts, 5, req_num);
    TORCH_CHECK(free_head.numel() >= req_num, "free_head must hold req_num entries");
    const c10::cuda::CUDAGuard guard(index.device());
    at::Tensor slot_out = at::empty_like(query_index);
    const at::Tensor status = new_status(req_num, index);
    launch_ok(asu_hbm_index_lookup_ex(
                  c10::cuda::getCurrentCUDAStream(index.device().index()).stream(), index.data_ptr<int32_t>(),
                  slot_to_index.data_ptr<int32_t>(), free_slots.data_ptr<int32_t>(), free_head.data_ptr<int32_t>(),
                  query_index.data_ptr<int32_t>(), slot_out.data_ptr<int32_t>(), static_cast<uint32_t>(req_num),
                  row_width("index", index, req_num), row_width("slot_to_index", slot_to_index, req_num),
                  row_width("free_slots", free_slots, req_num), row_width("query_index", query_index, req_num),
                  status_ptr(status)),
              "asu_hbm_index_lookup");
    raise_on_status(status, "asu_hbm_index_lookup");
    return slot_out;
}

void maintain_cuda(at::Tensor& index, at::Tensor& slot_to_index, at::Tensor& free_slots, at::Tensor& free_head,
                   const at::Tensor& last_query_slots, int64_t req_num, int64_t seed) {
    const char* names[] = {"index", "slot_to_index", "free_slots", "free_head", "last_query_slots"};
    const at::Tensor* ts[] = {&index, &slot_to_index, &free_slots, &free_head, &last_query_slots};
    index_op_checks(names, ts, 5, req_num);
    TORCH_CHECK(free_head.numel() >= req_num, "free_head must hold req_num entries");
    const c10::cuda::CUDAGuard guard(index.device());
    const at::Tensor status = new_status(req_num, index);
    launch_ok(asu_hbm_index_maintain_ex(
                  c10::cuda::getCurrentCUDAStream(index.device().index()).stream(), index.data_ptr<int32_t>(),
                  slot_to_index.data_ptr<int32_t>(), free_slots.data_ptr<int32_t>(), free_head.data_ptr<int32_t>(),
                  last_query_slots.data_ptr<int32_t>(), static_cast<uint32_t>(req_num),
                  static_cast<uint32_t>(seed & 0xFFFFFFFF), row_width("index", index, req_num),
                  row_width("slot_to_index", slot_to_index, req_num), row_width("free_slots", free_slots, req_num),
                  row_width("last_query_slots", last_query_slots, req_num), status_ptr(status)),
              "asu_hbm_index_maintain");
    raise_on_status(status, "asu_hbm_index_maintain");
}

std::tuple<at::Tensor, at::Tensor> simt_cuda(at::Tensor& token_to_slot, at::Tensor& slot_to_token,
                                             at::Tensor& lru_slots, const at::Tensor& query_token_ids,
                                             int64_t req_num) {
    const char* names[] = {"token_to_slot", "slot_to_token", "query_token_ids"};
    const at::Tensor* ts[] = {&token_to_slot, &slot_to_token, &query_token_ids};
    TORCH_CHECK(lru_slots.scalar_type() == at::kShort, "lru_slots must be int16");
    index_op_checks(names, ts, 3, req_num);
    TORCH_CHECK(lru_slots.device() == token_to_slot.device() && lru_slots.is_contiguous(),
                "lru_slots must be a contiguous int16 tensor on the same device");
    const c10::cuda::CUDAGuard guard(token_to_slot.device());
    at::Tensor slot_ids = at::empty_like(query_token_ids);
    at::Tensor miss_mask = at::empty(query_token_ids.sizes(), query_token_ids.options().dtype(at::kBool));
    const at::Tensor status = new_status(req_num, token_to_slot);
    launch_ok(asu_hbm_index_lookup_simt_ex(
                  c10::cuda::getCurrentCUDAStream(token_to_slot.device().index()).stream(),
                  token_to_slot.data_ptr<int32_t>(), slot_to_token.data_ptr<int32_t>(),
                  lru_slots.data_ptr<int16_t>(), query_token_ids.data_ptr<int32_t>(), slot_ids.data_ptr<int32_t>(),
                  reinterpret_cast<uint8_t*>(miss_mask.data_ptr<bool>()), static_cast<uint32_t>(req_num),
                  row_width("token_to_slot", token_to_slot, req_num), row_width("slot_to_token", slot_to_token, req_num),
                  row_width("query_token_ids", query_token_ids, req_num), status_ptr(status)),
              "asu_hbm_index_lookup_simt");
    raise_on_status(status, "asu_hbm_index_lookup_simt");
    return {slot_ids, miss_mask};
}

// Host tensors: the same checks (the first failing one reports host memory), then a refusal.
at::Tensor lookup_cpu(at::Tensor& index, at::Tensor& slot_to_index, at::Tensor& free_slots, at::Tensor& free_head,
                      const at::Tensor& query_index, int64_t req_num) {
    const char* names[] = {"index", "slot_to_index", "free_slots", "free_head", "query_index"};
    const at::Tensor* ts[] = {&index, &slot_to_index, &free_slots, &free_head, &query_index};
    index_op_checks(names, ts, 5, req_num);
    TORCH_CHECK(false, "asu_hbm_index_lookup needs CUDA tensors");
}

void maintain_cpu(at::Tensor& index, at::Tensor& slot_to_index, at::Tensor& free_slots, at::Tensor& free_head,
                  const at::Tensor& last_query_slots, int64_t req_num, int64_t) {
    const char* names[] = {"index", "slot_to_index", "free_slots", "free_head", "last_query_slots"};
    const at::Tensor* ts[] = {&index, &slot_to_index, &free_slots, &free_head, &last_query_slots};
    index_op_checks(names, ts, 5, req_num);
    TORCH_CHECK(false, "asu_hbm_index_maintain needs CUDA tensors");
}

std::tuple<at::Tensor, at::Tensor> simt_cpu(at::Tensor& token_to_slot, at::Tensor& slot_to_token,
                                            at::Tensor& lru_slots, const at::Tensor& query_token_ids,
                                            int64_t req_num) {
    const char* names[] = {"token_to_slot", "slot_to_token", "query_token_ids"};
    const at::Tensor* ts[] = {&token_to_slot, &slot_to_token, &query_token_ids};
    TORCH_CHECK(lru_slots.scalar_type() == at::kShort, "lru_slots must be int16");
    index_op_checks(names, ts, 3, req_num);
    TORCH_CHECK(false, "asu_hbm_index_lookup_simt needs CUDA tensors");
}

at::Tensor lookup_meta(at::Tensor&, at::Tensor&, at::Tensor&, at::Tensor&, const at::Tensor& query_index, int64_t) {
    return at::empty_like(query_index);
}

void maintain_meta(at::Tensor&, at::Tensor&, at::Tensor&, at::Tensor&, const at::Tensor&, int64_t, int64_t) {}

std::tuple<at::Tensor, at::Tensor> simt_meta(at::Tensor&, at::Tensor&, at::Tensor&, const at::Tensor& query_token_ids,
                                             int64_t) {
    return {at::empty_like(query_token_ids), at::empty(query_token_ids.sizes(), query_token_ids.options().dtype(at::kBool))};
}

constexpr const char* kLookupSchema =
    "asu_hbm_index_lookup(Tensor(a!) index, Tensor(b!) slot_to_index, Tensor(c!) free_slots, Tensor(d!) free_head, "
    "Tensor query_index, int req_num) -> Tensor";
constexpr const char* kMaintainSchema =
    "asu_hbm_index_maintain(Tensor(a!) index, Tensor(b!) slot_to_index, Tensor(c!) free_slots, Tensor(d!) free_head, "
    "Tensor last_query_slots, int req_num, int seed) -> ()";
constexpr const char* kSimtSchema =
    "asu_hbm_index_lookup_simt(Tensor(a!) token_to_slot, Tensor(b!) slot_to_token, Tensor(c!) lru_slots, "
    "Tensor query_token_ids, int req_num) -> (Tensor, Tensor)";

// ---------------------------------------------------------------------------------------------

constexpr const char* kSchema =
    "npu_asu_resolve_kv_slots_single_req(Tensor original_topk_indices, int actual_seq_len, int managed_prefix_len, "
    "Tensor! token_state, Tensor asu_record_addr, Tensor! hbm_slot_of_token, Tensor! slot_owner_token, "
    "Tensor free_slot_stack, Tensor! free_slot_count, Tensor original_block_table, Tensor original_kv_cache_0, "
    "Tensor original_kv_cache_1, Tensor! managed_kv_cache_0, Tensor! managed_kv_cache_1, int block_size) -> Tensor";

constexpr const char* kLruSchema =
    "npu_asu_resolve_kv_slots_lru(Tensor original_topk_indices, int actual_seq_len, int managed_prefix_len, "
    "Tensor! token_state, Tensor asu_record_addr, Tensor! hbm_slot_of_token, Tensor! slot_owner_token, "
    "Tensor! free_slot_stack, Tensor! free_slot_count, Tensor! lru_order, int free_target, "
    "Tensor original_block_table, Tensor original_kv_cache_0, Tensor original_kv_cache_1, "
    "Tensor! managed_kv_cache_0, Tensor! managed_kv_cache_1, int block_size, Tensor(s!)? stats=None) -> Tensor";

}  // namespace

#define ASU_DEFINE_OPS(m)    \
    m.def(kSchema);          \
    m.def(kLookupSchema);    \
    m.def(kMaintainSchema);  \
    m.def(kSimtSchema);
#define ASU_IMPL_OPS(m, resolve, lookup, maintain, simt)         \
    m.impl("npu_asu_resolve_kv_slots_single_req", &resolve);     \
    m.impl("asu_hbm_index_lookup", &lookup);                     \
    m.impl("asu_hbm_index_maintain", &maintain);                 \
    m.impl("asu_hbm_index_lookup_simt", &simt);

TORCH_LIBRARY_FRAGMENT(asu, m) { ASU_DEFINE_OPS(m) }
TORCH_LIBRARY_FRAGMENT(_C_ascend, m) { ASU_DEFINE_OPS(m) }

TORCH_LIBRARY_IMPL(asu, CUDA, m) { ASU_IMPL_OPS(m, resolve_cuda, lookup_cuda, maintain_cuda, simt_cuda) }
TORCH_LIBRARY_IMPL(_C_ascend, CUDA, m) { ASU_IMPL_OPS(m, resolve_cuda, lookup_cuda, maintain_cuda, simt_cuda) }
TORCH_LIBRARY_IMPL(asu, CPU, m) { ASU_IMPL_OPS(m, resolve_cpu, lookup_cpu, maintain_cpu, simt_cpu) }
TORCH_LIBRARY_IMPL(_C_ascend, CPU, m) { ASU_IMPL_OPS(m, resolve_cpu, lookup_cpu, maintain_cpu, simt_cpu) }
TORCH_LIBRARY_IMPL(asu, Meta, m) { ASU_IMPL_OPS(m, resolve_meta, lookup_meta, maintain_meta, simt_meta) }
TORCH_LIBRARY_IMPL(_C_ascend, Meta, m) { ASU_IMPL_OPS(m, resolve_meta, lookup_meta, maintain_meta, simt_meta) }

// The bounded-pool resolver is this library's own operator: registered under `asu` only.
TORCH_LIBRARY_FRAGMENT(asu, m) { m.def(kLruSchema); }
TORCH_LIBRARY_IMPL(asu, CUDA, m) { m.impl("npu_asu_resolve_kv_slots_lru", &resolve_lru_cuda); }
TORCH_LIBRARY_IMPL(asu, CPU, m) { m.impl("npu_asu_resolve_kv_slots_lru", &resolve_lru_cpu); }
TORCH_LIBRARY_IMPL(asu, Meta, m) { m.impl("npu_asu_resolve_kv_slots_lru", &resolve_lru_meta); }

// Status checks of the op (synchronise after each call and raise on a device status); the Python
// side's ops.set_status_checks() forwards here.
extern "C" void asu_torch_set_status_checks(int enabled) { g_status_checks.store(enabled != 0); }
extern "C" int asu_torch_status_checks() { return g_status_checks.load() ? 1 : 0; }
