"""ctypes binding of libasu_b200.so (the C ABI declared in include/asu_b200.h).

Importing this module loads the library and fails loudly if it is missing: there is no
CPU fallback anywhere in the package.  torch is imported first so that the library's
libcudart.so.12 dependency binds to the CUDA runtime torch already loaded.
"""

from __future__ import annotations

import ctypes
from ctypes import POINTER, c_char_p, c_int, c_int32, c_int64, c_uint32, c_uint64, c_void_p
from pathlib import Path

import torch  # noqa: F401  (must precede the CDLL load, see module docstring)

LIB_PATH = Path(__file__).resolve().with_name("libasu_b200.so")

ASU_OK = 0
ASU_ERR_ARG = -1
ASU_ERR_ALIGN = -2
ASU_ERR_NOALLOC_CAPACITY = -3
ASU_ERR_CUDA_BASE = 1000
RESOLVER_NOALLOC_MAX_TOPK = 16384

STATUS_BITS = {
    0x01: "BAD_QUERY",
    0x02: "FREE_EXHAUSTED",
    0x04: "RING_EXHAUSTED",
    0x08: "BAD_STATE",
    0x10: "SHORTAGE",
    0x20: "BAD_SOURCE",
    0x40: "BAD_TOKEN_STATE",
    0x80: "NO_VICTIM",
    0x100: "TIMEOUT",
}
ST_BAD_QUERY, ST_FREE_EXHAUSTED, ST_RING_EXHAUSTED, ST_BAD_STATE = 0x01, 0x02, 0x04, 0x08
ST_SHORTAGE, ST_BAD_SOURCE, ST_BAD_TOKEN_STATE, ST_NO_VICTIM = 0x10, 0x20, 0x40, 0x80
ST_TIMEOUT = 0x100

LRU_STAT_COLS = 5

_P = c_void_p
# name -> argtypes (restype is int unless listed in _RESTYPE)
_SIGS = {
    "asu_version": [],
    "asu_status_string": [c_int],
    "asu_hbm_index_lookup_do": [c_uint32, _P, _P, _P, _P, _P, _P, _P, c_uint32],
    "asu_hbm_index_lookup_ex": [_P, _P, _P, _P, _P, _P, _P, c_uint32, c_uint32, c_uint32, c_uint32, c_uint32, _P],
    "asu_hbm_index_maintain_do": [c_uint32, _P, _P, _P, _P, _P, _P, c_uint32, c_uint32],
    "asu_hbm_index_maintain_ex": [_P, _P, _P, _P, _P, _P, c_uint32, c_uint32, c_uint32, c_uint32, c_uint32, c_uint32,
                                  _P],
    "hbm_lookup_vec_do": [c_uint32, _P, _P, _P, _P, _P, c_uint32, c_uint32, c_int32],
    "hbm_random_update_do": [c_uint32, _P, _P, _P, _P, _P, c_uint32, c_uint32, c_uint32, c_uint32],
    "asu_gather_lookup": [_P, _P, c_uint32, _P, c_uint32, _P, c_uint32, _P, c_uint32, c_int32, _P],
    "asu_random_update": [_P, _P, c_uint32, _P, _P, c_uint32, c_uint32, c_uint32, c_uint32, _P],
    "asu_hbm_index_lookup_simt_do": [_P, _P, _P, _P, _P, _P, _P, _P, c_uint32],
    "asu_hbm_index_lookup_simt_ex": [_P, _P, _P, _P, _P, _P, _P, c_uint32, c_uint32, c_uint32, c_uint32, _P],
    "asu_lru_step": [_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, c_uint32, _P, _P, _P, c_uint32, c_uint32, c_uint32,
                     c_uint32, c_uint32],
    "asu_lru_step_host_query": [_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, c_uint32, _P, _P, _P, c_uint32,
                                c_uint32, c_uint32, c_uint32, c_uint32],
    "asu_swapin_gather": [_P, _P, c_int64, c_uint32, c_uint32, _P, c_uint32, _P, _P, _P, c_uint32, _P, c_uint32,
                          c_uint32, _P],
    "asu_swapin_gather_to_peer": [_P, _P, c_int64, c_uint32, c_uint32, _P, c_uint32, _P, _P, _P, c_uint32, _P,
                                  c_uint32, c_uint32, _P],
    "asu_host_register": [_P, c_uint64, POINTER(c_void_p)],
    "asu_host_unregister": [_P],
    "asu_ipc_export": [_P, _P, POINTER(c_uint64)],
    "asu_ipc_open": [_P, POINTER(c_void_p)],
    "asu_ipc_close": [_P],
    "asu_host_pool_alloc": [c_uint64, POINTER(c_void_p), POINTER(c_void_p)],
    "asu_host_pool_writeback": [_P, _P, c_int64, c_uint32, c_uint32, _P, c_int64, c_uint64, _P, _P, c_int64, _P],
    "asu_host_pool_free": [_P],
    "asu_host_device_pointer": [_P, POINTER(c_void_p)],
    "asu_mapped_copy": [_P, _P, _P, c_uint64],
    "asu_selftest_bounded_wait": [_P, c_int32, _P],
    "asu_kv_resolver_do": [_P, _P, c_int64, _P, _P, _P, _P, _P, _P, c_int64, _P, c_int64, _P, _P, _P, _P, c_int64,
                           c_int64, c_int64, c_int64, c_int64, c_int64, c_int64, _P, _P, _P],
    "asu_kv_resolver_workspace_bytes": [c_int64],
    "asu_resolver_reset": [_P, _P, _P, _P, c_int64, _P, _P, _P, c_int64, _P, c_int64, c_int64, c_int64, c_int64],
    "asu_kv_resolver_noalloc": [_P, _P, c_int64, _P, _P, _P, _P, _P, _P, c_int64, _P, c_int64, _P, _P, _P, _P,
                                c_int64, c_int64, c_int64, c_int64, c_int64, c_int64, c_int64, _P, _P],
    "asu_resolver_reset_layers": [_P, c_int64, _P, _P, _P, c_int64, _P, _P, _P, c_int64, _P, c_int64, c_int64,
                                  c_int64, c_int64],
    "asu_resolver_mark_token": [_P, c_int64, _P, c_int64, c_int64],
    "asu_kv_resolver_lru": [_P, _P, c_int64, _P, _P, _P, _P, _P, _P, _P, c_int64, c_int64, _P, c_int64, _P, _P, _P,
                            _P, c_int64, c_int64, c_int64, c_int64, c_int64, c_int64, _P, _P, _P, _P, _P],
}
_RESTYPE = {"asu_status_string": c_char_p, "asu_kv_resolver_workspace_bytes": c_int64}


class AsuError(RuntimeError):
    """A C-ABI call rejected its arguments or failed to launch, or a kernel reported a status."""


def _load() -> ctypes.CDLL:
    if not LIB_PATH.exists():
        raise ImportError(
            f"{LIB_PATH} is not built: run `python -m asu_ascend_b200.build` (needs nvcc); "
            "asu_ascend_b200 has no CPU fallback")
    lib = ctypes.CDLL(str(LIB_PATH))
    for name, argtypes in _SIGS.items():
        fn = getattr(lib, name)
        fn.argtypes = argtypes
        fn.restype = _RESTYPE.get(name, c_int)
    return lib


lib = _load()


def exported_symbols() -> list[str]:
    return list(_SIGS)


def check(rc: int, what: str) -> None:
    if rc != ASU_OK:
        msg = lib.asu_status_string(rc)
        raise AsuError(f"{what} failed: {msg.decode() if msg else rc} (code {rc})")


def status_names(bits: int) -> list[str]:
    return [name for bit, name in STATUS_BITS.items() if bits & bit]


def status_bits(status: torch.Tensor) -> int:
    bits = 0
    for v in status.cpu().tolist():
        bits |= int(v)
    return bits


def raise_on_status(status: torch.Tensor, what: str, ignore: int = 0) -> None:
    bits = status_bits(status) & ~ignore
    if bits:
        raise AsuError(f"{what}: device status {status_names(bits)} (0x{bits:x})")
