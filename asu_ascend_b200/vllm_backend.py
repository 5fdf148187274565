"""vLLM FlashMLA-sparse attention implementation that decodes over the ASU managed cache.

The reference wires its manager into vLLM-Ascend's sparse-attention decode
(patch/0003 vllm_ascend/attention/sfa_v1.py hunk, patch lines 461-575): a layer whose
manager holds it, in a decode-only batch of one request and one token, prepares its context
(reset on a new request, mark the new decode token otherwise), resolves the indexer's top-k
through ``npu_asu_resolve_kv_slots_single_req`` and runs sparse attention over the managed
cache with the resolved slots; every other batch takes the original path.

`asu_flashmla_sparse_impl()` returns the same thing for vLLM's FlashMLA-sparse backend on
B200: a subclass of vLLM's `FlashMLASparseImpl` that, under the reference's conditions,
replaces the block-table conversion (``triton_convert_req_index_to_global_index``,
flashmla_sparse.py:755-776, 803-812, 898-904) with `sparse_mla.resolve_topk` and points the
attention kernel at the managed cache: FlashMLA-sparse over ``[slots, 1, 576]`` for bf16
caches, FlashMLA's fp8 sparse decode over the managed cache seen as pages of ``block_size``
656-byte fp8_ds_mla rows (both fp8 batch layouts: mixed, and separate prefill/decode).
The manager comes from ``attn_metadata.asu_kv_cache_manager`` as in the reference,
else from the class attribute ``asu_manager``; the request id from
``attn_metadata.asu_req_id``, else ``"__single_req__"``::

    register_flashmla_sparse_override()   # before the model is built: vLLM's FLASHMLA_SPARSE
                                          # backend then resolves to ASUFlashMLASparseBackend
    attach_manager(sparse_mla.contexts_for_mla(kv_caches, max_model_len, block_size))
"""

from __future__ import annotations

import functools

import torch

from . import sparse_mla

SINGLE_REQ_ID = "__single_req__"  # patch line 486


def asu_manager_of(impl, attn_metadata):
    m = getattr(attn_metadata, "asu_kv_cache_manager", None)
    return m if m is not None else getattr(impl, "asu_manager", None)


def use_asu_kv_cache(manager, layer_name: str | None, attn_metadata) -> bool:
    """patch lines 461-473, with FlashMLA-sparse's metadata: one request, one decode token."""
    if manager is None or not manager.enabled or layer_name is None or not manager.has_layer(layer_name):
        return False
    if getattr(attn_metadata, "max_query_len", None) != 1:
        return False  # not decode-only
    if getattr(attn_metadata, "num_reqs", 0) != 1:
        return False
    return getattr(attn_metadata, "num_actual_tokens", 0) == 1


def prepare_asu_layer_context(manager, layer_name: str, attn_metadata):
    """patch lines 480-499: reset the manager on a new or shorter request, else mark the token.

    The request's length is ``attn_metadata.max_seq_len`` (a host int: one request).
    """
    ctx = manager.get_layer_context(layer_name)
    actual_seq_len = int(attn_metadata.max_seq_len)
    req_id = getattr(attn_metadata, "asu_req_id", None) or SINGLE_REQ_ID
    if ctx.req_id != req_id or ctx.actual_seq_len == 0 or actual_seq_len < ctx.actual_seq_len:
        managed_prefix_len = max(0, actual_seq_len - attn_metadata.num_actual_tokens)
        manager.reset_single_request(req_id=req_id, actual_seq_len=actual_seq_len,
                                     managed_prefix_len=managed_prefix_len,
                                     original_block_table=attn_metadata.block_table[:1])
    elif actual_seq_len > ctx.actual_seq_len:
        manager.mark_decode_token(actual_seq_len - 1)
    return ctx


@functools.lru_cache(maxsize=1)
def asu_flashmla_sparse_impl():
    """The subclass, built on first use (vLLM is imported only then)."""
    from vllm.v1.attention.backends.mla.flashmla_sparse import FlashMLASparseImpl

    class ASUFlashMLASparseImpl(FlashMLASparseImpl):
        """FlashMLASparseImpl whose single-request bf16 decode reads the ASU managed cache."""

        asu_manager = None

        def forward_mqa(self, q, kv_c_and_k_pe_cache, attn_metadata, layer):
            self._asu_layer_name = getattr(layer, "layer_name", None)
            return super().forward_mqa(q, kv_c_and_k_pe_cache, attn_metadata, layer)

        def _asu_resolve(self, kv_c_and_k_pe_cache, topk_indices, attn_metadata):
            """(context, resolved slots) when this batch takes the ASU path, else None."""
            manager = asu_manager_of(self, attn_metadata)
            name = getattr(self, "_asu_layer_name", None)
            if not use_asu_kv_cache(manager, name, attn_metadata):
                return None
            if torch.cuda.is_available() and torch.cuda.is_current_stream_capturing():
                raise RuntimeError(
                    "the ASU decode path cannot be captured in a CUDA graph: it decides on the host, "
                    "every step, whether to reset or extend the request and passes its length to the "
                    "resolver; run attention eagerly (vLLM cudagraph mode PIECEWISE or NONE)")
            ctx = prepare_asu_layer_context(manager, name, attn_metadata)
            kv = kv_c_and_k_pe_cache.reshape(*kv_c_and_k_pe_cache.shape[:2], -1)
            slots = sparse_mla.resolve_topk(ctx, topk_indices.contiguous(), attn_metadata.block_table[0], kv)
            return ctx, slots

        def _asu_fp8_decode(self, q, ctx, slots, kernel_metadata):
            """One decode token: FlashMLA's fp8 sparse decode over the managed pages."""
            out, _ = self._fp8_flash_mla_kernel(q=q.view(1, 1, *q.shape[1:]),
                                                kv_c_and_k_pe_cache=sparse_mla.managed_paged_view(ctx),
                                                topk_indices=slots.view(1, 1, -1), kernel_metadata=kernel_metadata)
            return out.reshape(q.shape[0], *out.shape[2:])

        def _forward_bf16_kv(self, q, kv_c_and_k_pe_cache, topk_indices, attn_metadata):
            r = self._asu_resolve(kv_c_and_k_pe_cache, topk_indices, attn_metadata)
            if r is None:
                return super()._forward_bf16_kv(q, kv_c_and_k_pe_cache, topk_indices, attn_metadata)
            ctx, slots = r
            return self._bf16_flash_mla_kernel(q, sparse_mla.managed_kv_view(ctx), slots)

        def _forward_fp8_kv_mixed_batch(self, q, kv_c_and_k_pe_cache, topk_indices, attn_metadata):
            r = self._asu_resolve(kv_c_and_k_pe_cache, topk_indices, attn_metadata)
            if r is None:
                return super()._forward_fp8_kv_mixed_batch(q, kv_c_and_k_pe_cache, topk_indices, attn_metadata)
            return self._asu_fp8_decode(q, *r, attn_metadata.fp8_extra_metadata)

        def _forward_fp8_kv_separate_prefill_decode(self, q, kv_c_and_k_pe_cache, topk_indices, attn_metadata):
            meta = attn_metadata.fp8_extra_metadata
            r = None
            if getattr(meta, "decode", None) is not None and getattr(meta, "num_prefill_tokens", 1) == 0:
                r = self._asu_resolve(kv_c_and_k_pe_cache, topk_indices, attn_metadata)
            if r is None:
                return super()._forward_fp8_kv_separate_prefill_decode(q, kv_c_and_k_pe_cache, topk_indices,
                                                                       attn_metadata)
            return self._asu_fp8_decode(q, *r, meta.decode.kernel_metadata)

    return ASUFlashMLASparseImpl


@functools.lru_cache(maxsize=1)
def asu_flashmla_sparse_builder():
    """vLLM's FlashMLA-sparse metadata builder, declared without CUDA-graph support.

    The ASU decode path decides on the host, every step, whether the request is new (reset) or one
    token longer (mark) and passes the request's length to the resolver as a scalar, as the
    reference does (patch/0003, patch lines 480-499).  A full CUDA graph of attention would replay
    the first step's decisions and length forever, so vLLM must keep attention out of its graphs
    (it then captures the rest of the model piecewise)."""
    from vllm.v1.attention.backend import AttentionCGSupport
    from vllm.v1.attention.backends.mla.flashmla_sparse import FlashMLASparseMetadataBuilder

    class ASUFlashMLASparseMetadataBuilder(FlashMLASparseMetadataBuilder):
        _cudagraph_support = AttentionCGSupport.NEVER

    return ASUFlashMLASparseMetadataBuilder


@functools.lru_cache(maxsize=1)
def asu_flashmla_sparse_backend():
    """vLLM's FlashMLASparseBackend with ASUFlashMLASparseImpl as its implementation class and a
    metadata builder without CUDA-graph support (``asu_flashmla_sparse_builder``); the name,
    metadata, cache shape and kernel-block sizes stay vLLM's."""
    from vllm.v1.attention.backends.mla.flashmla_sparse import FlashMLASparseBackend

    impl = asu_flashmla_sparse_impl()
    builder = asu_flashmla_sparse_builder()

    class ASUFlashMLASparseBackend(FlashMLASparseBackend):
        @staticmethod
        def get_impl_cls():
            return impl

        @staticmethod
        def get_builder_cls():
            return builder

    for cls in (ASUFlashMLASparseBackend, impl, builder):  # importable by name (vLLM resolves class paths)
        cls.__module__ = __name__
        cls.__qualname__ = cls.__name__
    return ASUFlashMLASparseBackend


def __getattr__(name):
    """Module attributes built on first use, so importing this module does not import vLLM."""
    if name == "ASUFlashMLASparseBackend":
        return asu_flashmla_sparse_backend()
    if name == "ASUFlashMLASparseImpl":
        return asu_flashmla_sparse_impl()
    if name == "ASUFlashMLASparseMetadataBuilder":
        return asu_flashmla_sparse_builder()
    raise AttributeError(name)


def register_flashmla_sparse_override() -> None:
    """Point vLLM's FLASHMLA_SPARSE attention backend at ASUFlashMLASparseBackend (vLLM's
    ``register_backend`` override).  Call it before vLLM builds the model; batches the ASU path
    does not take still run vLLM's own code."""
    from vllm.v1.attention.backends.registry import AttentionBackendEnum, register_backend

    register_backend(AttentionBackendEnum.FLASHMLA_SPARSE, f"{__name__}.ASUFlashMLASparseBackend")


def attach_manager(manager) -> None:
    """The manager every ASUFlashMLASparseImpl uses when the attention metadata carries none."""
    asu_flashmla_sparse_impl().asu_manager = manager
