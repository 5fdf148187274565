"""Resolver state of every managed attention layer, for single-request decode.

The decode path that uses the resolver (vLLM-Ascend's SFA decode as patch/0003 wires it,
patch lines 461-575; here ``vllm_backend.py`` / ``sparse_mla.py``) talks to a manager and its
per-layer contexts by name: ``enabled``, ``has_layer``, ``get_layer_context``,
``reset_single_request``, ``mark_decode_token``, and on a context the state tensors, the
managed caches, ``req_id`` / ``actual_seq_len`` / ``managed_prefix_len`` and
``original_kv_cache_views``.  Those names, the feature-gate environment variables and the
argument errors follow patch/0003 vllm_ascend/attention/asu_kv_cache_manager.py (patch lines
175-432), so that path runs unchanged.  The storage is designed for the GPU:

* ``LayerStateBank`` keeps the resolver state of all layers on one device as [layers, ...]
  int32 tensors (one allocation per array).  A context is a set of row views into its bank
  plus the layer's managed caches.
* A new request resets every layer with ONE launch (``asu_resolver_reset_layers``), and a
  decode token is registered in every layer with ONE launch (``asu_resolver_mark_token``);
  the reference runs several tensor ops per layer for each.
* Managed caches of layers with the same row shape and dtype are one [layers, slots, ...]
  allocation.
* A free target (``free_target=`` or ``VLLM_ASCEND_ASU_KV_CACHE_FREE_TARGET``; e.g. 2048, one
  DeepSeek-V3.2 top-k, with 8192 + 2048 managed slots) makes the pool an exact-LRU cache: the
  bank then also keeps a recency order row per layer, and the layer resolves through the LRU
  variant of the resolver (``npu_asu_resolve_kv_slots_lru``), which evicts the least recently
  used tokens until that many slots are free before each resolve, so the managed cache can be
  far smaller than the context.  Without one, the pool never evicts and resolves exactly like
  the reference, which fails once the pool is full (patch/0001, patch lines 879-888).
"""

from __future__ import annotations

import os
from dataclasses import dataclass, field

import torch

# token states shared with the resolver kernels (include/asu_b200.h ASU_TOKEN_*)
INVALID = -1
ASU_ONLY = 0
HBM_RESIDENT = 1
TAIL_HBM = 2

ASU_KV_CACHE_ENABLE_ENV = "VLLM_ASCEND_ENABLE_ASU_KV_CACHE"
ASU_KV_CACHE_SLOT_COUNT_ENV = "VLLM_ASCEND_ASU_KV_CACHE_SLOTS"
ASU_KV_CACHE_FREE_TARGET_ENV = "VLLM_ASCEND_ASU_KV_CACHE_FREE_TARGET"

_TRUE = frozenset(("1", "true", "yes", "on"))


def _env_positive_int(name: str) -> int | None:
    raw = os.getenv(name, "")
    if raw == "":
        return None
    value = int(raw)
    if value <= 0:
        raise ValueError(f"{name} must be positive")
    return value


def is_asu_kv_cache_enabled() -> bool:
    """The feature gate (off unless the environment turns it on)."""
    return os.getenv(ASU_KV_CACHE_ENABLE_ENV, "").strip().lower() in _TRUE


def get_configured_managed_slot_count() -> int | None:
    """Managed slots per layer from the environment (None: one per context position)."""
    return _env_positive_int(ASU_KV_CACHE_SLOT_COUNT_ENV)


def get_configured_free_target() -> int | None:
    """Free slots an exact-LRU pool keeps before each resolve (None: the pool never evicts)."""
    return _env_positive_int(ASU_KV_CACHE_FREE_TARGET_ENV)


def _paged_rows(cache: torch.Tensor) -> torch.Tensor:
    """A paged cache [blocks, block_size, ...] seen as rows [blocks * block_size, ...]."""
    if cache.dim() < 2:
        raise ValueError("PA cache must have block and block-size dimensions")
    return cache.flatten(0, 1)


def _launch(fn_name: str, device: torch.device, *args) -> None:
    from ._lib import check, lib

    with torch.cuda.device(device):
        check(getattr(lib, fn_name)(torch.cuda.current_stream(device).cuda_stream, *args), fn_name)


def _check_request_lengths(actual_seq_len: int, managed_prefix_len: int, max_seq_len: int) -> None:
    """The reference's argument errors for a reset (patch lines 241-249)."""
    if actual_seq_len < 0:
        raise ValueError("actual_seq_len must be non-negative")
    if managed_prefix_len < 0:
        raise ValueError("managed_prefix_len must be non-negative")
    if managed_prefix_len > actual_seq_len:
        raise ValueError("managed_prefix_len must not exceed actual_seq_len")
    if actual_seq_len > max_seq_len:
        raise RuntimeError("ASU max_seq_len does not cover actual_seq_len")


class LayerStateBank:
    """The resolver state of the managed layers that live on one device, as [layers, ...] int32
    tensors, plus each layer's request bookkeeping."""

    def __init__(self, names: list[str], device: torch.device, max_seq_len: int, slot_count: int,
                 block_size: int, free_target: int | None) -> None:
        n = len(names)
        self.names = list(names)
        self.device = device
        self.max_seq_len, self.slot_count, self.block_size = max_seq_len, slot_count, block_size
        self.free_target = free_target  # None: the pool never evicts
        opts = {"dtype": torch.int32, "device": device}
        self.token_state = torch.full((n, max_seq_len), INVALID, **opts)
        self.asu_record_addr = torch.full((n, max_seq_len), INVALID, **opts)
        self.hbm_slot_of_token = torch.full((n, max_seq_len), INVALID, **opts)
        self.slot_owner_token = torch.full((n, slot_count), INVALID, **opts)
        self.free_slot_stack = torch.arange(slot_count, **opts).expand(n, slot_count).contiguous()
        self.free_slot_count = torch.full((n,), slot_count, **opts)
        self.lru_order = torch.full((n, slot_count), INVALID, **opts) if free_target is not None else None
        # exact-LRU pools count hits, misses, installs, shortages and evictions per layer (+=)
        self.lru_stats = torch.zeros((n, 5), dtype=torch.int64, device=device) if free_target is not None else None
        self.req_id: list[str | None] = [None] * n
        self.actual_seq_len = [0] * n
        self.managed_prefix_len = [0] * n

    @property
    def bounded(self) -> bool:
        return self.lru_order is not None

    def _block_table(self, original_block_table: torch.Tensor, managed_prefix_len: int) -> torch.Tensor:
        if self.device.type != "cuda":
            raise RuntimeError("ASU state lives in HBM: the manager's tensors must be CUDA tensors")
        bt = original_block_table.reshape(-1).to(device=self.device, dtype=torch.int32).contiguous()
        if managed_prefix_len > 0 and (managed_prefix_len - 1) // self.block_size >= bt.numel():
            raise RuntimeError("original_block_table does not cover ASU prefix")
        return bt

    def reset(self, first: int, count: int, req_id: str, actual_seq_len: int, managed_prefix_len: int,
              original_block_table: torch.Tensor) -> None:
        """Fresh state for rows [first, first + count): one launch."""
        _check_request_lengths(actual_seq_len, managed_prefix_len, self.max_seq_len)
        bt = self._block_table(original_block_table, managed_prefix_len)
        _launch("asu_resolver_reset_layers", self.device, count, self.token_state[first].data_ptr(),
                self.asu_record_addr[first].data_ptr(), self.hbm_slot_of_token[first].data_ptr(), self.max_seq_len,
                self.slot_owner_token[first].data_ptr(), self.free_slot_stack[first].data_ptr(),
                self.free_slot_count[first:].data_ptr(), self.slot_count, bt.data_ptr(), bt.numel(),
                self.block_size, actual_seq_len, managed_prefix_len)
        for i in range(first, first + count):
            self.req_id[i] = req_id
            self.actual_seq_len[i] = actual_seq_len
            self.managed_prefix_len[i] = managed_prefix_len

    def mark(self, first: int, count: int, token_id: int) -> None:
        """The decode token `token_id` becomes TAIL_HBM in rows [first, first + count): one launch."""
        if token_id < 0 or token_id >= self.max_seq_len:
            raise RuntimeError("decode token_id is outside ASU max_seq_len")
        if self.device.type != "cuda":
            raise RuntimeError("ASU state lives in HBM: the manager's tensors must be CUDA tensors")
        _launch("asu_resolver_mark_token", self.device, count, self.token_state[first].data_ptr(), self.max_seq_len,
                token_id)
        for i in range(first, first + count):
            self.actual_seq_len[i] = max(self.actual_seq_len[i], token_id + 1)


class ASULayerKVCacheContext:
    """One managed layer: row views into its bank, the layer's managed caches, and the fields the
    decode path reads by name."""

    def __init__(self, layer_name: str, bank: LayerStateBank, row: int, managed_kv_cache_0: torch.Tensor,
                 managed_kv_cache_1: torch.Tensor) -> None:
        self.layer_name = layer_name
        self.bank, self.row = bank, row
        self.managed_kv_cache_0 = managed_kv_cache_0
        self.managed_kv_cache_1 = managed_kv_cache_1
        self.token_state = bank.token_state[row]
        self.asu_record_addr = bank.asu_record_addr[row]
        self.hbm_slot_of_token = bank.hbm_slot_of_token[row]
        self.slot_owner_token = bank.slot_owner_token[row]
        self.free_slot_stack = bank.free_slot_stack[row]
        self.free_slot_count = bank.free_slot_count[row]
        self.lru_order = bank.lru_order[row] if bank.bounded else None
        self.lru_stats = bank.lru_stats[row] if bank.bounded else None
        self.max_seq_len, self.managed_slot_count, self.block_size = bank.max_seq_len, bank.slot_count, bank.block_size
        self.free_target = bank.free_target

    # request bookkeeping lives in the bank, one entry per layer
    req_id = property(lambda self: self.bank.req_id[self.row],
                      lambda self, v: self.bank.req_id.__setitem__(self.row, v))
    actual_seq_len = property(lambda self: self.bank.actual_seq_len[self.row],
                              lambda self, v: self.bank.actual_seq_len.__setitem__(self.row, v))
    managed_prefix_len = property(lambda self: self.bank.managed_prefix_len[self.row],
                                  lambda self, v: self.bank.managed_prefix_len.__setitem__(self.row, v))

    @property
    def bounded(self) -> bool:
        """True when the managed pool is an exact-LRU cache (it evicts to keep free_target slots free)."""
        return self.lru_order is not None

    def original_kv_cache_views(self, kv_cache: tuple[torch.Tensor, ...]) -> tuple[torch.Tensor, torch.Tensor]:
        return _paged_rows(kv_cache[0]), _paged_rows(kv_cache[1])

    def reset_state(self, req_id: str, actual_seq_len: int, managed_prefix_len: int,
                    original_block_table: torch.Tensor) -> None:
        """Fresh state for a new request in this layer only (one launch)."""
        self.bank.reset(self.row, 1, req_id, actual_seq_len, managed_prefix_len, original_block_table)

    def mark_decode_token(self, token_id: int) -> None:
        """The appended decode token becomes TAIL_HBM in this layer only (one launch)."""
        self.bank.mark(self.row, 1, token_id)


@dataclass
class _CacheGroup:
    """Layers whose managed caches share a row shape and dtype: one [layers, slots, ...] block."""
    names: list[str] = field(default_factory=list)
    caches: tuple[torch.Tensor, torch.Tensor] | None = None


class ASUFullKVCacheManagerFunctional:
    """The managed layers of one model, grouped into one state bank per device."""

    def __init__(self, enabled: bool, max_seq_len: int, block_size: int,
                 contexts: dict[str, ASULayerKVCacheContext], banks: list[LayerStateBank] | None = None) -> None:
        self.enabled = enabled
        self.max_seq_len = max_seq_len
        self.block_size = block_size
        self._contexts = contexts
        self._banks = banks if banks is not None else []

    @classmethod
    def from_kv_caches(cls, kv_caches: dict[str, tuple[torch.Tensor, ...]], max_seq_len: int, block_size: int,
                       managed_slot_count: int | None = None, enabled: bool | None = None,
                       free_target: int | None = None) -> "ASUFullKVCacheManagerFunctional":
        """Contexts for every layer whose cache is a tuple of >= 2 paged caches [blocks, block_size, ...].

        Managed slots per layer: ``managed_slot_count``, else the environment's, else
        ``max_seq_len`` (a slot per context position).  ``free_target`` (else the environment's)
        makes every layer's pool an exact-LRU cache that keeps that many slots free.
        """
        on = is_asu_kv_cache_enabled() if enabled is None else enabled
        if not on:
            return cls(False, max_seq_len, block_size, {})
        if max_seq_len <= 0:
            raise ValueError("max_seq_len must be positive")
        if block_size <= 0:
            raise ValueError("block_size must be positive")
        slots = managed_slot_count or get_configured_managed_slot_count() or max_seq_len
        if slots <= 0:
            raise ValueError("managed_slot_count must be positive")
        target = free_target if free_target is not None else get_configured_free_target()
        if target is not None and target < 0:
            raise ValueError("free_target must be non-negative")
        managed = {name: (kv[0], kv[1]) for name, kv in kv_caches.items()
                   if isinstance(kv, tuple) and len(kv) >= 2 and kv[0].dim() >= 3 and kv[1].dim() >= 3}
        by_device: dict[torch.device, list[str]] = {}
        for name, (c0, _) in managed.items():
            by_device.setdefault(c0.device, []).append(name)
        contexts: dict[str, ASULayerKVCacheContext] = {}
        banks = []
        for dev, names in by_device.items():
            bank = LayerStateBank(names, dev, max_seq_len, slots, block_size, target)
            banks.append(bank)
            groups: dict[tuple, _CacheGroup] = {}
            for name in names:
                c0, c1 = managed[name]
                key = (tuple(c0.shape[2:]), c0.dtype, c1.device, tuple(c1.shape[2:]), c1.dtype)
                groups.setdefault(key, _CacheGroup()).names.append(name)
            for (row0, dt0, dev1, row1, dt1), g in groups.items():
                n = len(g.names)
                block0 = torch.empty((n, slots, *row0), dtype=dt0, device=dev)
                block1 = torch.empty((n, slots, *row1), dtype=dt1, device=dev1)
                for i, name in enumerate(g.names):
                    contexts[name] = ASULayerKVCacheContext(name, bank, bank.names.index(name), block0[i], block1[i])
        return cls(True, max_seq_len, block_size, contexts, banks)

    def has_layer(self, layer_name: str) -> bool:
        return layer_name in self._contexts

    def get_layer_context(self, layer_name: str) -> ASULayerKVCacheContext:
        return self._contexts[layer_name]

    def reset_single_request(self, req_id: str, actual_seq_len: int, managed_prefix_len: int,
                             original_block_table: torch.Tensor) -> None:
        """Fresh state for a new request in every layer: one launch per device."""
        if not self.enabled:
            return
        for bank in self._banks:
            bank.reset(0, len(bank.names), req_id, actual_seq_len, managed_prefix_len, original_block_table)

    def mark_decode_token(self, token_id: int) -> None:
        """Register the appended decode token in every layer: one launch per device."""
        if not self.enabled:
            return
        for bank in self._banks:
            bank.mark(0, len(bank.names), token_id)
