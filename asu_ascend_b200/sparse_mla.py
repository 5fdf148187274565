"""Resolver slots for vLLM's FlashMLA-sparse decode (the B200 counterpart of patch/0003).

vLLM's sparse-MLA decode turns each request's top-k token positions into global slots of the
paged cache with ``triton_convert_req_index_to_global_index``
(vllm/v1/attention/backends/mla/flashmla_sparse.py:755-776, sparse_utils.py:85-118):
``slot = block_table[tok // block_size] * block_size + tok % block_size`` and -1 stays -1.
The reference's decode path instead resolves the top-k through the ASU manager and the
single-request resolver and hands the managed cache plus the resolved slots to its sparse
attention (patch/0003 vllm_ascend/attention/sfa_v1.py hunk, patch lines 505-575).

Here the same wiring feeds FlashMLA-sparse: ``resolve_topk`` is the drop-in for the index
conversion of one request (same input, same -1 convention), and ``managed_kv_view`` is the
``[slots, 1, 576]`` cache FlashMLA-sparse reads through those slots.  vLLM keeps the latent
and rope parts of a token in one row (bf16 576 = 512 + 64, or the 656-byte fp8_ds_mla row),
so a layer's managed state has a single cache; the manager's second cache is empty.
"""

from __future__ import annotations

import torch

from . import manager as _manager
from ._lib import ST_BAD_QUERY, check, lib, raise_on_status
from .ops import status_checks_enabled


def contexts_for_mla(kv_caches: dict[str, torch.Tensor], max_seq_len: int, block_size: int,
                     managed_slot_count: int | None = None, enabled: bool | None = None,
                     free_target: int | None = None) -> _manager.ASUFullKVCacheManagerFunctional:
    """Manager over vLLM MLA caches ``[num_blocks, block_size, row]`` (one per layer); a
    ``free_target`` makes every layer's pool an exact-LRU cache."""
    pairs = {name: (c, c.new_empty((*c.shape[:2], 0))) for name, c in kv_caches.items()
             if isinstance(c, torch.Tensor) and c.dim() == 3}
    mgr = _manager.ASUFullKVCacheManagerFunctional.from_kv_caches(pairs, max_seq_len, block_size,
                                                                  managed_slot_count, enabled, free_target)
    for name in pairs:
        if mgr.has_layer(name):  # whole pages, so FlashMLA's paged fp8 decode can read it (rows past the slots unused)
            ctx = mgr.get_layer_context(name)
            m = ctx.managed_kv_cache_0
            rows = -(-m.shape[0] // block_size) * block_size
            if rows != m.shape[0]:
                ctx.managed_kv_cache_0 = m.new_empty((rows, *m.shape[1:]))
    return mgr


def managed_kv_view(ctx: _manager.ASULayerKVCacheContext) -> torch.Tensor:
    """The managed cache as FlashMLA-sparse's ``kv`` operand: ``[slots, 1, row]``."""
    m = ctx.managed_kv_cache_0
    return m.view(m.shape[0], 1, -1)


def managed_paged_view(ctx: _manager.ASULayerKVCacheContext) -> torch.Tensor:
    """The managed cache as a paged ``[pages, block_size, row]`` cache (slot s = page * block_size
    + offset), the layout FlashMLA's fp8 sparse decode reads through global slot indices."""
    m = ctx.managed_kv_cache_0
    return m.view(-1, ctx.block_size, m.shape[-1])


def resolve_topk(ctx: _manager.ASULayerKVCacheContext, topk_indices: torch.Tensor, block_table: torch.Tensor,
                 kv_cache: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """Managed slots of one request's top-k ``[num_tokens, topk]`` (-1 entries stay -1).

    Missing tokens are installed into the managed cache (rows copied from the paged
    ``kv_cache``) exactly as ``npu_asu_resolve_kv_slots_single_req`` does -- through its
    exact-LRU variant (``asu_kv_resolver_lru``) when the layer's pool evicts; the call is
    asynchronous on the current stream.
    """
    dev = ctx.token_state.device
    if topk_indices.dtype != torch.int32 or topk_indices.device != dev or not topk_indices.is_contiguous():
        raise RuntimeError("topk_indices must be a contiguous int32 tensor on the manager's device")
    if kv_cache.dim() != 3 or kv_cache.device != dev or not kv_cache.is_contiguous():
        raise RuntimeError("kv_cache must be a contiguous [num_blocks, block_size, row] tensor")
    m = ctx.managed_kv_cache_0
    if kv_cache.dtype != m.dtype or kv_cache.shape[2:] != m.shape[1:]:
        raise RuntimeError("kv_cache rows must match the managed cache rows")
    bt = block_table.reshape(-1)
    if bt.dtype != torch.int32 or bt.device != dev or not bt.is_contiguous():
        raise RuntimeError("block_table must be a contiguous int32 tensor on the manager's device")
    if out is None:
        out = torch.empty_like(topk_indices)
    n = topk_indices.numel()
    if n == 0:
        return out
    row_bytes = kv_cache.shape[2] * kv_cache.element_size()
    src_rows = kv_cache.shape[0] * kv_cache.shape[1]
    status = torch.zeros(1, dtype=torch.int32, device=dev) if status_checks_enabled() else None
    if ctx.bounded:
        with torch.cuda.device(dev):
            check(lib.asu_kv_resolver_lru(
                torch.cuda.current_stream(dev).cuda_stream, topk_indices.data_ptr(), n, ctx.token_state.data_ptr(),
                ctx.asu_record_addr.data_ptr(), ctx.hbm_slot_of_token.data_ptr(), ctx.slot_owner_token.data_ptr(),
                ctx.free_slot_stack.data_ptr(), ctx.free_slot_count.data_ptr(), ctx.lru_order.data_ptr(),
                ctx.managed_slot_count, ctx.free_target, bt.data_ptr(), bt.numel(), kv_cache.data_ptr(), None,
                m.data_ptr(), None, row_bytes, 0, src_rows, ctx.max_seq_len, ctx.actual_seq_len, ctx.block_size,
                out.data_ptr(), None, None, ctx.lru_stats.data_ptr(), None if status is None else status.data_ptr()),
                "resolve_topk")
        if status is not None:
            raise_on_status(status, "resolve_topk", ST_BAD_QUERY)
        return out
    ws = torch.empty(int(lib.asu_kv_resolver_workspace_bytes(n)), dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        check(lib.asu_kv_resolver_do(
            torch.cuda.current_stream(dev).cuda_stream, topk_indices.data_ptr(), n, ctx.token_state.data_ptr(),
            ctx.asu_record_addr.data_ptr(), ctx.hbm_slot_of_token.data_ptr(), ctx.slot_owner_token.data_ptr(),
            ctx.free_slot_stack.data_ptr(), ctx.free_slot_count.data_ptr(), ctx.free_slot_stack.numel(),
            bt.data_ptr(), bt.numel(), kv_cache.data_ptr(), None, m.data_ptr(), None, row_bytes, 0, src_rows,
            min(m.shape[0], ctx.slot_owner_token.numel()), ctx.max_seq_len, ctx.actual_seq_len, ctx.block_size,
            out.data_ptr(), ws.data_ptr(), None if status is None else status.data_ptr()), "resolve_topk")
    if status is not None:
        raise_on_status(status, "resolve_topk", ST_BAD_QUERY)  # -1 padding is expected here
    return out


def sparse_mla_decode(q: torch.Tensor, ctx: _manager.ASULayerKVCacheContext, topk_indices: torch.Tensor,
                      block_table: torch.Tensor, kv_cache: torch.Tensor, softmax_scale: float,
                      head_padding: int = 128) -> torch.Tensor:
    """One request's sparse-MLA decode over the managed cache: resolve, then FlashMLA-sparse.

    q: ``[num_tokens, num_heads, 576]`` bf16; returns ``[num_tokens, num_heads, 512]``.  Heads are
    padded to a multiple of ``head_padding`` (128 on Blackwell) as vLLM's bf16 path does
    (flashmla_sparse.py:961-990).
    """
    from vllm.third_party.flashmla.flash_mla_interface import flash_mla_sparse_fwd

    slots = resolve_topk(ctx, topk_indices, block_table, kv_cache)
    t, h, d = q.shape
    if h % head_padding:
        hp = (h + head_padding - 1) // head_padding * head_padding
        qp = q.new_zeros((t, hp, d))
        qp[:, :h] = q
        q = qp
    out = flash_mla_sparse_fwd(q, managed_kv_view(ctx), slots.view(t, 1, -1), softmax_scale)[0]
    return out[:, :h]
