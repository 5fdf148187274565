"""Torch operators of the resolver hot path, registered with the reference's schemas.

Each operator is defined twice with the same schema: under ``torch.ops.asu`` and under
``torch.ops._C_ascend`` -- the namespace vLLM-Ascend's decode path calls
(ascend-ops/torch_binding_asu_hbm_index.cpp:7-25; patch/0001 csrc/torch_binding.cpp hunk,
patch lines 810-826), so code written against the reference resolves to these CUDA
implementations unchanged.  The CUDA implementations call libasu_b200.so through its C
ABI on the current stream; there is no CPU implementation (a CPU tensor raises).  The
lookup / maintain / batch-LRU ops are registered here in Python; the single-request
resolver, which a decode step calls once per layer, is registered in C++ by
libasu_torch.so (csrc/torch_binding.cpp), which this module loads.

Host-side argument checks mirror the reference adapters' TORCH_CHECKs
(ascend-ops/asu_hbm_index_lookup/asu_hbm_index_lookup_torch_adpt.h:22-27,
asu_hbm_index_maintain_torch_adpt.h:22-27) plus device / contiguity / shape checks that
the raw pointers need.  Device-side problems are written to a status word; with
``set_status_checks(True)`` every op synchronises and raises on a non-zero status
(AsuError from the Python ops, RuntimeError from the C++ resolver op; AsuError is a
RuntimeError) -- off by default: the ops stay asynchronous like the NPU ones.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

import torch
from torch.library import Library

from . import _lib
from ._lib import check, lib

NAMESPACES = ("asu", "_C_ascend")

_STATUS_CHECKS = os.environ.get("ASU_CHECK_STATUS", "0") not in ("", "0")
_IGNORED_STATUS = _lib.ST_SHORTAGE  # counted in the stats, not an error


TORCH_LIB_PATH = Path(__file__).resolve().with_name("libasu_torch.so")


def _load_torch_binding() -> ctypes.CDLL:
    """Register npu_asu_resolve_kv_slots_single_req from the C++ binding (csrc/torch_binding.cpp)."""
    if not TORCH_LIB_PATH.exists():
        raise ImportError(f"{TORCH_LIB_PATH} is not built: run `python -m asu_ascend_b200.build`; "
                          "asu_ascend_b200 has no CPU fallback")
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


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _req_cuda_i32(name: str, t: torch.Tensor, device: torch.device | None = None) -> None:
    if t.dtype != torch.int32:
        raise RuntimeError(f"{name} must be int32")
    if t.device.type != "cuda":
        raise RuntimeError(f"{name} must be a CUDA tensor (asu_ascend_b200 has no CPU implementation)")
    if device is not None and t.device != device:
        raise RuntimeError(f"{name} must be on {device}, got {t.device}")
    if not t.is_contiguous():
        raise RuntimeError(f"{name} must be contiguous")


def _row_width(name: str, t: torch.Tensor, req_num: int) -> int:
    if t.numel() % req_num != 0:
        raise RuntimeError(f"{name} has {t.numel()} elements, not a multiple of req_num={req_num}")
    return t.numel() // req_num


def _new_status(n: int, device) -> torch.Tensor:
    return torch.zeros(n, dtype=torch.int32, device=device)


def _raise_on_status(status: torch.Tensor, what: str, ignore: int = _IGNORED_STATUS) -> None:
    if _STATUS_CHECKS:
        _lib.raise_on_status(status, what, ignore)


# ------------------------------------------------------------------ implementations

def asu_hbm_index_lookup(index, slot_to_index, free_slots, free_head, query_index, req_num):
    """In-place lookup + sequential free-list allocation; returns slot_out (empty_like(query_index))."""
    if req_num <= 0:
        raise RuntimeError("req_num must be greater than 0")
    dev = index.device
    for n, t in (("index", index), ("slot_to_index", slot_to_index), ("free_slots", free_slots),
                 ("free_head", free_head), ("query_index", query_index)):
        _req_cuda_i32(n, t, dev)
    if free_head.numel() < req_num:
        raise RuntimeError("free_head must hold req_num entries")
    slot_out = torch.empty_like(query_index)
    status = _new_status(req_num, dev)
    with torch.cuda.device(dev):
        check(lib.asu_hbm_index_lookup_ex(
            _stream(index), index.data_ptr(), slot_to_index.data_ptr(), free_slots.data_ptr(),
            free_head.data_ptr(), query_index.data_ptr(), slot_out.data_ptr(), req_num,
            _row_width("index", index, req_num), _row_width("slot_to_index", slot_to_index, req_num),
            _row_width("free_slots", free_slots, req_num), _row_width("query_index", query_index, req_num),
            status.data_ptr()), "asu_hbm_index_lookup")
    _raise_on_status(status, "asu_hbm_index_lookup")
    return slot_out


def asu_hbm_index_maintain(index, slot_to_index, free_slots, free_head, last_query_slots, req_num, seed):
    """In-place hash-seeded ring eviction refilling free_slots[--free_head]."""
    if req_num <= 0:
        raise RuntimeError("req_num must be greater than 0")
    dev = index.device
    for n, t in (("index", index), ("slot_to_index", slot_to_index), ("free_slots", free_slots),
                 ("free_head", free_head), ("last_query_slots", last_query_slots)):
        _req_cuda_i32(n, t, dev)
    if free_head.numel() < req_num:
        raise RuntimeError("free_head must hold req_num entries")
    status = _new_status(req_num, dev)
    with torch.cuda.device(dev):
        check(lib.asu_hbm_index_maintain_ex(
            _stream(index), index.data_ptr(), slot_to_index.data_ptr(), free_slots.data_ptr(),
            free_head.data_ptr(), last_query_slots.data_ptr(), req_num, seed & 0xFFFFFFFF,
            _row_width("index", index, req_num), _row_width("slot_to_index", slot_to_index, req_num),
            _row_width("free_slots", free_slots, req_num), _row_width("last_query_slots", last_query_slots, req_num),
            status.data_ptr()), "asu_hbm_index_maintain")
    _raise_on_status(status, "asu_hbm_index_maintain")


def asu_hbm_index_lookup_simt(token_to_slot, slot_to_token, lru_slots, query_token_ids, req_num):
    """Batch-LRU lookup (in place); returns (slot_ids int32, miss_mask bool)."""
    if req_num <= 0:
        raise RuntimeError("req_num must be greater than 0")
    dev = token_to_slot.device
    for n, t in (("token_to_slot", token_to_slot), ("slot_to_token", slot_to_token),
                 ("query_token_ids", query_token_ids)):
        _req_cuda_i32(n, t, dev)
    if lru_slots.dtype != torch.int16 or lru_slots.device != dev or not lru_slots.is_contiguous():
        raise RuntimeError("lru_slots must be a contiguous int16 tensor on the same device")
    slot_ids = torch.empty_like(query_token_ids)
    miss_mask = torch.empty(query_token_ids.shape, dtype=torch.bool, device=dev)
    status = _new_status(req_num, dev)
    with torch.cuda.device(dev):
        check(lib.asu_hbm_index_lookup_simt_ex(
            _stream(token_to_slot), token_to_slot.data_ptr(), slot_to_token.data_ptr(), lru_slots.data_ptr(),
            query_token_ids.data_ptr(), slot_ids.data_ptr(), miss_mask.data_ptr(), req_num,
            _row_width("token_to_slot", token_to_slot, req_num), _row_width("slot_to_token", slot_to_token, req_num),
            _row_width("query_token_ids", query_token_ids, req_num), status.data_ptr()),
            "asu_hbm_index_lookup_simt")
    _raise_on_status(status, "asu_hbm_index_lookup_simt")
    return slot_ids, miss_mask


# ------------------------------------------------------------------ registration

_SCHEMAS = {
    "asu_hbm_index_lookup": ("asu_hbm_index_lookup(Tensor(a!) index, Tensor(b!) slot_to_index, "
                             "Tensor(c!) free_slots, Tensor(d!) free_head, Tensor query_index, int req_num) -> Tensor"),
    "asu_hbm_index_maintain": ("asu_hbm_index_maintain(Tensor(a!) index, Tensor(b!) slot_to_index, "
                               "Tensor(c!) free_slots, Tensor(d!) free_head, Tensor last_query_slots, int req_num, "
                               "int seed) -> ()"),
    "asu_hbm_index_lookup_simt": ("asu_hbm_index_lookup_simt(Tensor(a!) token_to_slot, Tensor(b!) slot_to_token, "
                                  "Tensor(c!) lru_slots, Tensor query_token_ids, int req_num) -> (Tensor, Tensor)"),
}
_IMPLS = {
    "asu_hbm_index_lookup": asu_hbm_index_lookup,
    "asu_hbm_index_maintain": asu_hbm_index_maintain,
    "asu_hbm_index_lookup_simt": asu_hbm_index_lookup_simt,
}


def _meta_lookup(index, slot_to_index, free_slots, free_head, query_index, req_num):
    return torch.empty_like(query_index)


def _meta_maintain(index, slot_to_index, free_slots, free_head, last_query_slots, req_num, seed):
    return None


def _meta_simt(token_to_slot, slot_to_token, lru_slots, query_token_ids, req_num):
    return torch.empty_like(query_token_ids), torch.empty(query_token_ids.shape, dtype=torch.bool,
                                                          device=query_token_ids.device)


_METAS = {
    "asu_hbm_index_lookup": _meta_lookup,
    "asu_hbm_index_maintain": _meta_maintain,
    "asu_hbm_index_lookup_simt": _meta_simt,
}

_LIBRARIES: list[Library] = []


def _register() -> None:
    for ns in NAMESPACES:
        libr = Library(ns, "FRAGMENT")
        for name, schema in _SCHEMAS.items():
            if torch._C._jit_get_schemas_for_operator(f"{ns}::{name}"):
                continue  # already defined in this process (module reloaded)
            libr.define(schema)
            libr.impl(name, _IMPLS[name], "CUDA")
            libr.impl(name, _METAS[name], "Meta")
        _LIBRARIES.append(libr)


_register()
set_status_checks(_STATUS_CHECKS)
