"""Torch operators of the resolver hot path, registered with the reference's schemas.

Each operator is defined twice with the same schema: under ``torch.ops.asu`` and under
``torch.ops._C_ascend`` -- the namespace vLLM-Ascend's decode path calls
(ascend-ops/torch_binding_asu_hbm_index.cpp:7-25; patch/0001 csrc/torch_binding.cpp hunk,
patch lines 810-826), so code written against the reference resolves to these CUDA
implementations unchanged.  All four -- asu_hbm_index_lookup, asu_hbm_index_maintain,
asu_hbm_index_lookup_simt and npu_asu_resolve_kv_slots_single_req -- are registered in C++ by
libasu_torch.so (csrc/torch_binding.cpp), which this module loads; their CUDA kernels call
libasu_b200.so through its C ABI on the current stream.  There is no CPU implementation: host
tensors get the reference's argument checks and then an error.

Host-side argument checks mirror the reference adapters' TORCH_CHECKs
(ascend-ops/asu_hbm_index_lookup/asu_hbm_index_lookup_torch_adpt.h:22-27,
asu_hbm_index_maintain_torch_adpt.h:22-27) plus device / contiguity / shape checks that
the raw pointers need.  Device-side problems are written to a status word; with
``set_status_checks(True)`` every op synchronises and raises RuntimeError on a non-zero status
(SHORTAGE excepted: the LRU statistics count it) -- off by default: the ops stay asynchronous
like the NPU ones.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

import torch

NAMESPACES = ("asu", "_C_ascend")

_STATUS_CHECKS = os.environ.get("ASU_CHECK_STATUS", "0") not in ("", "0")

TORCH_LIB_PATH = Path(__file__).resolve().with_name("libasu_torch.so")


def _load_torch_binding() -> ctypes.CDLL:
    """Register the operators from the C++ binding (csrc/torch_binding.cpp)."""
    if not TORCH_LIB_PATH.exists():
        raise ImportError(f"{TORCH_LIB_PATH} is not built: run `python -m asu_ascend_b200.build`; "
                          "asu_ascend_b200 has no CPU fallback")
    if not torch._C._jit_get_schemas_for_operator("asu::asu_hbm_index_lookup"):
        torch.ops.load_library(str(TORCH_LIB_PATH))
    handle = ctypes.CDLL(str(TORCH_LIB_PATH))  # the same loaded image: shares the status-check flag
    handle.asu_torch_set_status_checks.argtypes = [ctypes.c_int]
    handle.asu_torch_set_status_checks.restype = None
    return handle


_torch_binding = _load_torch_binding()


def set_status_checks(enabled: bool) -> None:
    """Synchronise after every op and raise on a device status (debug / tests)."""
    global _STATUS_CHECKS
    _STATUS_CHECKS = bool(enabled)
    _torch_binding.asu_torch_set_status_checks(int(_STATUS_CHECKS))


def status_checks_enabled() -> bool:
    return _STATUS_CHECKS


# Python names of the operators (the reference's ctypes harnesses and tests call these names).
def asu_hbm_index_lookup(index, slot_to_index, free_slots, free_head, query_index, req_num):
    """In-place lookup + sequential free-list allocation; returns slot_out (empty_like(query_index))."""
    return torch.ops.asu.asu_hbm_index_lookup(index, slot_to_index, free_slots, free_head, query_index, req_num)


def asu_hbm_index_maintain(index, slot_to_index, free_slots, free_head, last_query_slots, req_num, seed):
    """In-place hash-seeded ring eviction refilling free_slots[--free_head]."""
    torch.ops.asu.asu_hbm_index_maintain(index, slot_to_index, free_slots, free_head, last_query_slots, req_num, seed)


def asu_hbm_index_lookup_simt(token_to_slot, slot_to_token, lru_slots, query_token_ids, req_num):
    """Batch-LRU lookup (in place); returns (slot_ids int32, miss_mask bool)."""
    return torch.ops.asu.asu_hbm_index_lookup_simt(token_to_slot, slot_to_token, lru_slots, query_token_ids, req_num)


def npu_asu_resolve_kv_slots_single_req(*args, **kwargs):
    """The single-request resolver (patch/0001 schema); see torch.ops.asu.npu_asu_resolve_kv_slots_single_req."""
    return torch.ops.asu.npu_asu_resolve_kv_slots_single_req(*args, **kwargs)


set_status_checks(_STATUS_CHECKS)
