"""Python mirror of the reference's ``hbm_lookup_update`` extension module.

Same functions, arguments, defaults, checks and output layout as
simu/hbm_lookup_update/pybind/pybind_hbm_lookup_update.cpp:119-270 (lookup_random_update,
lookup_only, update_only), backed by the CUDA gather / update kernels.  Tables are
1-D [128K] or 2-D [req_num, 128K] int32; queries 1-D [query_len] or 2-D
[req_num, query_len].  The lookup returns the PRE-update states (the update is launched
after the lookup on the same stream, :167-181).  ``lookup`` is the extension used by the
lookup-only benchmark: any table width, plus the hit mask (entry != not_found).
"""

from __future__ import annotations

import ctypes

import torch

from ._lib import check, lib

INDEX_SIZE = 128 * 1024
QUERY_TILE = 64


def _check_i32(t: torch.Tensor, name: str) -> None:
    if t is None:
        raise RuntimeError(f"{name} must be defined")
    if t.device.type != "cuda":
        raise RuntimeError(f"{name} must be a CUDA tensor")
    if t.dtype != torch.int32:
        raise RuntimeError(f"{name} must be torch.int32")
    if not t.is_contiguous():
        raise RuntimeError(f"{name} must be contiguous")


def _shapes(table_keys, table_states, query_keys, new_states):
    """CheckLookupShapes, pybind_hbm_lookup_update.cpp:63-116."""
    if table_keys.dim() not in (1, 2):
        raise RuntimeError("table_keys must be 1-D [128K] or 2-D [req_num, 128K]")
    if table_states.shape != table_keys.shape:
        raise RuntimeError("table_states must have the same shape as table_keys")
    if new_states.shape != query_keys.shape:
        raise RuntimeError("new_states must have the same shape as query_keys")
    if table_keys.dim() == 1:
        if table_keys.numel() != INDEX_SIZE:
            raise RuntimeError("table_keys must have exactly 128K elements")
        if query_keys.dim() != 1:
            raise RuntimeError("query_keys must be 1-D when table_keys is 1-D")
        return 1, query_keys.numel(), True
    if table_keys.shape[1] != INDEX_SIZE:
        raise RuntimeError("table_keys shape must be [req_num, 128K]")
    if query_keys.dim() != 2:
        raise RuntimeError("query_keys must be 2-D [req_num, query_len] when table_keys is 2-D")
    if query_keys.shape[0] != table_keys.shape[0]:
        raise RuntimeError("query_keys dim 0 must match table_keys dim 0")
    if table_keys.shape[0] < 1:
        raise RuntimeError("req_num must be at least 1")
    return table_keys.shape[0], query_keys.shape[1], False


def lookup_random_update(table_keys, table_states, query_keys, new_states, seed, update_percent=5, block_dim=8,
                         not_found=-1, do_update=True):
    for t, n in ((table_keys, "table_keys"), (table_states, "table_states"), (query_keys, "query_keys"),
                 (new_states, "new_states")):
        _check_i32(t, n)
    req_num, qlen, single = _shapes(table_keys, table_states, query_keys, new_states)
    if not 0 <= update_percent <= 100:
        raise RuntimeError("update_percent must be in [0, 100]")
    padded = (max(qlen, 1) + QUERY_TILE - 1) // QUERY_TILE * QUERY_TILE
    out_full = torch.empty((padded,) if single else (req_num, padded), dtype=torch.int32, device=query_keys.device)
    stream = torch.cuda.current_stream(query_keys.device).cuda_stream
    with torch.cuda.device(query_keys.device):
        if qlen > 0:
            check(lib.hbm_lookup_vec_do(block_dim, stream, table_keys.data_ptr(), table_states.data_ptr(),
                                        query_keys.data_ptr(), out_full.data_ptr(), req_num, qlen, not_found),
                  "hbm_lookup_vec_do")
            if do_update and update_percent > 0:
                check(lib.hbm_random_update_do(block_dim, stream, table_keys.data_ptr(), table_states.data_ptr(),
                                               query_keys.data_ptr(), new_states.data_ptr(), req_num, qlen,
                                               seed & 0xFFFFFFFF, update_percent), "hbm_random_update_do")
    return out_full.narrow(0, 0, qlen) if single else out_full.narrow(1, 0, qlen)


def lookup_only(table_keys, table_states, query_keys, block_dim=8, not_found=-1):
    dummy = torch.empty_like(query_keys)
    return lookup_random_update(table_keys, table_states, query_keys, dummy, seed=0, update_percent=0,
                                block_dim=block_dim, not_found=not_found, do_update=False)


def update_only(table_keys, table_states, query_keys, new_states, seed, update_percent=5, block_dim=8):
    for t, n in ((table_keys, "table_keys"), (table_states, "table_states"), (query_keys, "query_keys"),
                 (new_states, "new_states")):
        _check_i32(t, n)
    req_num, qlen, _ = _shapes(table_keys, table_states, query_keys, new_states)
    if not 0 <= update_percent <= 100:
        raise RuntimeError("update_percent must be in [0, 100]")
    if qlen == 0 or update_percent == 0:
        return
    with torch.cuda.device(query_keys.device):
        check(lib.hbm_random_update_do(block_dim, torch.cuda.current_stream(query_keys.device).cuda_stream,
                                       table_keys.data_ptr(), table_states.data_ptr(), query_keys.data_ptr(),
                                       new_states.data_ptr(), req_num, qlen, seed & 0xFFFFFFFF, update_percent),
              "hbm_random_update_do")


def _kernel_ptr(t: torch.Tensor, name: str, dtype: torch.dtype, dev: torch.device) -> int:
    """Address a kernel on ``dev`` can use for ``t``: a CUDA tensor on ``dev``, or pinned host
    memory, which the kernel reads / writes over the host link directly (no staging copy)."""
    if t.dtype != dtype:
        raise RuntimeError(f"{name} must be {dtype}")
    if not t.is_contiguous():
        raise RuntimeError(f"{name} must be contiguous")
    if t.device.type == "cuda":
        if t.device != dev:
            raise RuntimeError(f"{name} must be on {dev}")
        return t.data_ptr()
    if not t.is_pinned():
        raise RuntimeError(f"{name} must be a CUDA tensor or pinned host memory")
    d = ctypes.c_void_p()
    check(lib.asu_host_device_pointer(t.data_ptr(), ctypes.byref(d)), f"{name}: device address of pinned memory")
    return d.value


def lookup(table: torch.Tensor, query: torch.Tensor, not_found: int = -1, status: torch.Tensor | None = None,
           out: torch.Tensor | None = None, hit: torch.Tensor | None = None):
    """Gather ``table[r, query[r, i]]`` for a [R, T] table and [R, Q] queries; returns (out, hit_mask).

    ``table`` lives in HBM.  ``query``, ``out`` and ``hit`` may be CUDA tensors or pinned host
    tensors: the kernel then reads the queries from, and writes the results to, host memory
    itself (zero-copy; synchronise the stream before reading host results).  Outputs default to
    the query's placement."""
    _check_i32(table, "table")
    dev = table.device
    if table.dim() != 2 or query.dim() != 2 or table.shape[0] != query.shape[0]:
        raise RuntimeError("table must be [R, T] and query [R, Q]")
    R, Q = query.shape
    on_host = query.device.type == "cpu"
    if out is None:
        out = torch.empty(query.shape, dtype=torch.int32, pin_memory=True) if on_host else torch.empty_like(query)
    if hit is None:
        hit = (torch.empty(query.shape, dtype=torch.bool, pin_memory=True) if on_host
               else torch.empty(query.shape, dtype=torch.bool, device=dev))
    if out.shape != query.shape or hit.shape != query.shape:
        raise RuntimeError("out and hit must have the query's shape")
    qp = _kernel_ptr(query, "query", torch.int32, dev)
    op = _kernel_ptr(out, "out", torch.int32, dev)
    hp = _kernel_ptr(hit, "hit", torch.bool, dev)
    with torch.cuda.device(dev):
        check(lib.asu_gather_lookup(torch.cuda.current_stream(dev).cuda_stream, table.data_ptr(),
                                    table.shape[1], qp, Q, op, Q, hp, R,
                                    not_found, None if status is None else status.data_ptr()), "asu_gather_lookup")
    return out, hit
