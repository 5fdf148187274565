// C++ torch binding of npu_asu_resolve_kv_slots_single_req, the op a decode step calls once per
// layer.
//
// Reference interface: patch/0001 csrc/torch_binding.cpp hunk (patch lines 810-826, schema) and
// csrc/asu_kv_resolver/asu_kv_resolver_torch_adpt.h (patch lines 21-59): TORCH_LIBRARY_FRAGMENT
// registration under _C_ascend, int32 index tensors, resolved = empty(topk.shape, int32).  The
// same schema is registered under `asu` and `_C_ascend` with CUDA, CPU (argument checks only:
// there is no CPU implementation) and Meta kernels.  The argument checks and their error types
// (ValueError / RuntimeError) are the ones the Python reference raises (patch lines 954-994).
//
// Why C++: the op is on the per-layer decode path, and a Python kernel spends tens of
// microseconds per call on argument handling; here a call costs a few microseconds of host time
// on top of its two launches.  The kernels are reached through the C ABI (asu_kv_resolver_do).
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/library.h>

#include <atomic>
#include <sstream>
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

constexpr const char* kSchema =
    "npu_asu_resolve_kv_slots_single_req(Tensor original_topk_indices, int actual_seq_len, int managed_prefix_len, "
    "Tensor! token_state, Tensor asu_record_addr, Tensor! hbm_slot_of_token, Tensor! slot_owner_token, "
    "Tensor free_slot_stack, Tensor! free_slot_count, Tensor original_block_table, Tensor original_kv_cache_0, "
    "Tensor original_kv_cache_1, Tensor! managed_kv_cache_0, Tensor! managed_kv_cache_1, int block_size) -> Tensor";

}  // namespace

TORCH_LIBRARY_FRAGMENT(asu, m) { m.def(kSchema); }
TORCH_LIBRARY_FRAGMENT(_C_ascend, m) { m.def(kSchema); }

TORCH_LIBRARY_IMPL(asu, CUDA, m) { m.impl("npu_asu_resolve_kv_slots_single_req", &resolve_cuda); }
TORCH_LIBRARY_IMPL(_C_ascend, CUDA, m) { m.impl("npu_asu_resolve_kv_slots_single_req", &resolve_cuda); }
TORCH_LIBRARY_IMPL(asu, CPU, m) { m.impl("npu_asu_resolve_kv_slots_single_req", &resolve_cpu); }
TORCH_LIBRARY_IMPL(_C_ascend, CPU, m) { m.impl("npu_asu_resolve_kv_slots_single_req", &resolve_cpu); }
TORCH_LIBRARY_IMPL(asu, Meta, m) { m.impl("npu_asu_resolve_kv_slots_single_req", &resolve_meta); }
TORCH_LIBRARY_IMPL(_C_ascend, Meta, m) { m.impl("npu_asu_resolve_kv_slots_single_req", &resolve_meta); }

// Status checks of the op (synchronise after each call and raise on a device status); the Python
// side's ops.set_status_checks() forwards here.
extern "C" void asu_torch_set_status_checks(int enabled) { g_status_checks.store(enabled != 0); }
extern "C" int asu_torch_status_checks() { return g_status_checks.load() ? 1 : 0; }
