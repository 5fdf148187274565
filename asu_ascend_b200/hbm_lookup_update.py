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


def lookup(table: torch.Tensor, query: torch.Tensor, not_found: int = -1, status: torch.Tensor | None = None,
           out: torch.Tensor | None = None, hit: torch.Tensor | None = None):
    """Gather ``table[r, query[r, i]]`` for a [R, T] table and [R, Q] queries; returns (out, hit_mask)."""
    _check_i32(table, "table")
    _check_i32(query, "query")
    if table.dim() != 2 or query.dim() != 2 or table.shape[0] != query.shape[0]:
        raise RuntimeError("table must be [R, T] and query [R, Q]")
    R, Q = query.shape
    out = torch.empty_like(query) if out is None else out
    hit = torch.empty(query.shape, dtype=torch.bool, device=query.device) if hit is None else hit
    with torch.cuda.device(query.device):
        check(lib.asu_gather_lookup(torch.cuda.current_stream(query.device).cuda_stream, table.data_ptr(),
                                    table.shape[1], query.data_ptr(), Q, out.data_ptr(), Q, hit.data_ptr(), R,
                                    not_found, None if status is None else status.data_ptr()), "asu_gather_lookup")
    return out, hit
