"""Per-layer resolver state for single-request decode (the reference's ASU KV-cache manager).

Same API, fields, environment flags and error behaviour as patch/0003
vllm_ascend/attention/asu_kv_cache_manager.py (patch lines 175-432):
``ASUFullKVCacheManagerFunctional.from_kv_caches`` allocates, per attention layer, the
managed KV caches ``[slots, ...]`` and the int32 state tensors that
``npu_asu_resolve_kv_slots_single_req`` mutates; ``reset_single_request`` rebuilds the state
for a new request (prefix tokens read from the paged cache, tail tokens from the tail
blocks); ``mark_decode_token`` registers the token a decode step appended.  The state reset
runs on the GPU as one kernel per layer (``asu_resolver_reset``) instead of a sequence of
tensor ops.
"""

from __future__ import annotations

import os
from dataclasses import dataclass

import torch

INVALID = -1
ASU_ONLY = 0
HBM_RESIDENT = 1
TAIL_HBM = 2

ASU_KV_CACHE_ENABLE_ENV = "VLLM_ASCEND_ENABLE_ASU_KV_CACHE"
ASU_KV_CACHE_SLOT_COUNT_ENV = "VLLM_ASCEND_ASU_KV_CACHE_SLOTS"


def is_asu_kv_cache_enabled() -> bool:
    """patch line 194: the feature gate defaults off."""
    return os.getenv(ASU_KV_CACHE_ENABLE_ENV, "").lower() in {"1", "true", "yes", "on"}


def get_configured_managed_slot_count() -> int | None:
    value = os.getenv(ASU_KV_CACHE_SLOT_COUNT_ENV)
    if value is None or value == "":
        return None
    slot_count = int(value)
    if slot_count <= 0:
        raise ValueError(f"{ASU_KV_CACHE_SLOT_COUNT_ENV} must be positive")
    return slot_count


def _flatten_pa_cache(cache: torch.Tensor) -> torch.Tensor:
    """Paged cache [blocks, block_size, ...] -> [blocks * block_size, ...] (patch lines 211-214)."""
    if cache.dim() < 2:
        raise ValueError("PA cache must have block and block-size dimensions")
    return cache.reshape(cache.shape[0] * cache.shape[1], *cache.shape[2:])


@dataclass
class ASULayerKVCacheContext:
    layer_name: str
    managed_kv_cache_0: torch.Tensor
    managed_kv_cache_1: torch.Tensor
    token_state: torch.Tensor
    asu_record_addr: torch.Tensor
    hbm_slot_of_token: torch.Tensor
    slot_owner_token: torch.Tensor
    free_slot_stack: torch.Tensor
    free_slot_count: torch.Tensor
    max_seq_len: int
    managed_slot_count: int
    block_size: int
    req_id: str | None = None
    actual_seq_len: int = 0
    managed_prefix_len: int = 0

    def original_kv_cache_views(self, kv_cache: tuple[torch.Tensor, ...]) -> tuple[torch.Tensor, torch.Tensor]:
        return _flatten_pa_cache(kv_cache[0]), _flatten_pa_cache(kv_cache[1])

    def reset_state(self, req_id: str, actual_seq_len: int, managed_prefix_len: int,
                    original_block_table: torch.Tensor) -> None:
        """patch lines 234-292; the errors are the reference's, the fill is one CUDA launch."""
        if actual_seq_len < 0:
            raise ValueError("actual_seq_len must be non-negative")
        if managed_prefix_len < 0:
            raise ValueError("managed_prefix_len must be non-negative")
        if managed_prefix_len > actual_seq_len:
            raise ValueError("managed_prefix_len must not exceed actual_seq_len")
        if actual_seq_len > self.max_seq_len:
            raise RuntimeError("ASU max_seq_len does not cover actual_seq_len")
        dev = self.token_state.device
        if dev.type != "cuda":
            raise RuntimeError("ASU state lives in HBM: the manager's tensors must be CUDA tensors")
        block_table = original_block_table.reshape(-1).to(device=dev, dtype=torch.int32).contiguous()
        if managed_prefix_len > 0 and (managed_prefix_len - 1) // self.block_size >= block_table.numel():
            raise RuntimeError("original_block_table does not cover ASU prefix")
        from ._lib import check, lib

        with torch.cuda.device(dev):
            check(lib.asu_resolver_reset(
                torch.cuda.current_stream(dev).cuda_stream, self.token_state.data_ptr(),
                self.asu_record_addr.data_ptr(), self.hbm_slot_of_token.data_ptr(), self.max_seq_len,
                self.slot_owner_token.data_ptr(), self.free_slot_stack.data_ptr(), self.free_slot_count.data_ptr(),
                self.managed_slot_count, block_table.data_ptr(), block_table.numel(), self.block_size,
                actual_seq_len, managed_prefix_len), "asu_resolver_reset")
        self.req_id = req_id
        self.actual_seq_len = actual_seq_len
        self.managed_prefix_len = managed_prefix_len

    def mark_decode_token(self, token_id: int) -> None:
        """patch lines 294-298."""
        if token_id < 0 or token_id >= self.max_seq_len:
            raise RuntimeError("decode token_id is outside ASU max_seq_len")
        self.actual_seq_len = max(self.actual_seq_len, token_id + 1)
        self.token_state[token_id] = TAIL_HBM


class ASUFullKVCacheManagerFunctional:
    def __init__(self, enabled: bool, max_seq_len: int, block_size: int,
                 contexts: dict[str, ASULayerKVCacheContext]) -> None:
        self.enabled = enabled
        self.max_seq_len = max_seq_len
        self.block_size = block_size
        self._contexts = contexts

    @classmethod
    def from_kv_caches(cls, kv_caches: dict[str, tuple[torch.Tensor, ...]], max_seq_len: int, block_size: int,
                       managed_slot_count: int | None = None,
                       enabled: bool | None = None) -> "ASUFullKVCacheManagerFunctional":
        """patch lines 314-403: one context per layer whose kv_cache is a tuple of >= 2 PA caches."""
        is_enabled = is_asu_kv_cache_enabled() if enabled is None else enabled
        if not is_enabled:
            return cls(False, max_seq_len, block_size, {})
        if max_seq_len <= 0:
            raise ValueError("max_seq_len must be positive")
        if block_size <= 0:
            raise ValueError("block_size must be positive")
        slot_count = managed_slot_count or get_configured_managed_slot_count() or max_seq_len
        if slot_count <= 0:
            raise ValueError("managed_slot_count must be positive")
        contexts: dict[str, ASULayerKVCacheContext] = {}
        for layer_name, kv_cache in kv_caches.items():
            if not isinstance(kv_cache, tuple) or len(kv_cache) < 2:
                continue
            c0, c1 = kv_cache[0], kv_cache[1]
            if c0.dim() < 3 or c1.dim() < 3:
                continue
            dev = c0.device

            def full(n, value, _dev=dev):
                return torch.full((n,), value, device=_dev, dtype=torch.int32)

            contexts[layer_name] = ASULayerKVCacheContext(
                layer_name=layer_name,
                managed_kv_cache_0=torch.empty((slot_count, *c0.shape[2:]), device=dev, dtype=c0.dtype),
                managed_kv_cache_1=torch.empty((slot_count, *c1.shape[2:]), device=c1.device, dtype=c1.dtype),
                token_state=full(max_seq_len, INVALID),
                asu_record_addr=full(max_seq_len, INVALID),
                hbm_slot_of_token=full(max_seq_len, INVALID),
                slot_owner_token=full(slot_count, INVALID),
                free_slot_stack=torch.arange(slot_count, device=dev, dtype=torch.int32),
                free_slot_count=torch.tensor(slot_count, device=dev, dtype=torch.int32),
                max_seq_len=max_seq_len,
                managed_slot_count=slot_count,
                block_size=block_size,
            )
        return cls(True, max_seq_len, block_size, contexts)

    def has_layer(self, layer_name: str) -> bool:
        return layer_name in self._contexts

    def get_layer_context(self, layer_name: str) -> ASULayerKVCacheContext:
        return self._contexts[layer_name]

    def reset_single_request(self, req_id: str, actual_seq_len: int, managed_prefix_len: int,
                             original_block_table: torch.Tensor) -> None:
        if not self.enabled:
            return
        for context in self._contexts.values():
            context.reset_state(req_id, actual_seq_len, managed_prefix_len, original_block_table)

    def mark_decode_token(self, token_id: int) -> None:
        if not self.enabled:
            return
        for context in self._contexts.values():
            context.mark_decode_token(token_id)
