// Library-level C entry points: version and status-code text.
#include "asu_common.cuh"

extern "C" int asu_version(void) { return 10000; /* 1.0.0 */ }

extern "C" const char* asu_status_string(int code) {
    switch (code) {
        case ASU_OK: return "ok";
        case ASU_ERR_ARG: return "invalid argument (null pointer or size out of range)";
        case ASU_ERR_ALIGN: return "pointer or row size not 16-byte aligned";
        case ASU_ERR_NOALLOC_CAPACITY:
            return "topk_numel exceeds the fixed scratch of asu_kv_resolver_noalloc (ASU_RESOLVER_NOALLOC_MAX_TOPK)";
        default: break;
    }
    if (code >= ASU_ERR_CUDA_BASE) return cudaGetErrorString(static_cast<cudaError_t>(code - ASU_ERR_CUDA_BASE));
    return "unknown status";
}
