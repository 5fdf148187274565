"""Per-request exact-LRU slot pools on the GPU (host-side owner of the state tensors).

One ``LruSlotPools`` object holds, for ``req_num`` independent requests, the state of
LRUManagedCache (simu/kv_cache_eviction_sim.py:99-150) in HBM and advances every request
by one decode step per ``step()`` call: the step-boundary maintain
(prepare_free_slots, :124-131) followed by the resolve of that step's top-k keys
(resolve_query, :133-150), in one kernel launch.  Keys are per-request logical positions
in ``[0, key_space)``; multi-layer use folds the layer into the key
(key = layer * tokens + token), which gives every request one slot pool shared by its
layers.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from ._lib import LRU_STAT_COLS, ST_SHORTAGE, check, lib, raise_on_status


@dataclass
class LruStepOutput:
    slot: torch.Tensor           # [R, Q] int32, -1 on shortage / invalid key
    hit: torch.Tensor            # [R, Q] bool, serial-order hit
    install: torch.Tensor        # [R, Q] bool, position took a slot (owes one swap-in)
    evicted: torch.Tensor        # [R, target] int32, first evicted_count[r] valid, LRU first
    evicted_count: torch.Tensor  # [R] int32


class LruSlotPools:
    STAT_NAMES = ("hits", "misses", "installs", "shortages", "evictions")

    def __init__(self, req_num: int, key_space: int, slot_count: int, free_target: int, query_count: int,
                 device: torch.device | str = "cuda"):
        if req_num <= 0 or key_space <= 0 or slot_count <= 0 or query_count <= 0 or free_target < 0:
            raise ValueError("req_num, key_space, slot_count, query_count must be positive; free_target >= 0")
        if slot_count > 16384 or query_count > 4096 or key_space >= 2**31:
            raise ValueError("supported: slot_count <= 16384, query_count <= 4096, key_space < 2**31")
        self.req_num, self.key_space, self.slot_count = req_num, key_space, slot_count
        self.free_target, self.query_count = min(free_target, slot_count), query_count
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise RuntimeError("LruSlotPools lives in HBM: device must be CUDA")
        d, i32 = self.device, torch.int32
        self.token_to_slot = torch.full((req_num, key_space), -1, dtype=i32, device=d)
        self.slot_to_token = torch.full((req_num, slot_count), -1, dtype=i32, device=d)
        self.lru_order = torch.full((req_num, slot_count), -1, dtype=i32, device=d)
        self.free_stack = torch.arange(slot_count - 1, -1, -1, dtype=i32, device=d).repeat(req_num, 1)
        self.free_count = torch.full((req_num,), slot_count, dtype=i32, device=d)
        self.stats = torch.zeros((req_num, LRU_STAT_COLS), dtype=torch.int64, device=d)
        self.status = torch.zeros((req_num,), dtype=i32, device=d)
        self._out = self.new_output()

    def new_output(self) -> LruStepOutput:
        """Output buffers for one step (step() reuses its own set unless given one)."""
        d, R, Q = self.device, self.req_num, self.query_count
        return LruStepOutput(
            slot=torch.empty((R, Q), dtype=torch.int32, device=d),
            hit=torch.empty((R, Q), dtype=torch.bool, device=d),
            install=torch.empty((R, Q), dtype=torch.bool, device=d),
            evicted=torch.full((R, max(self.free_target, 1)), -1, dtype=torch.int32, device=d),
            evicted_count=torch.zeros((R,), dtype=torch.int32, device=d),
        )

    def load_state(self, token_to_slot, slot_to_token, lru_order, free_stack, free_count) -> None:
        for dst, src in ((self.token_to_slot, token_to_slot), (self.slot_to_token, slot_to_token),
                         (self.lru_order, lru_order), (self.free_stack, free_stack), (self.free_count, free_count)):
            dst.copy_(torch.as_tensor(src).reshape(dst.shape))

    def step(self, query: torch.Tensor, out: LruStepOutput | None = None, stream: torch.cuda.Stream | None = None
             ) -> LruStepOutput:
        """Advance every request by one step with ``query`` [R, Q] int32 (CUDA, contiguous)."""
        if query.dtype != torch.int32 or query.device != self.device or not query.is_contiguous():
            raise RuntimeError("query must be a contiguous int32 tensor on the pool's device")
        if tuple(query.shape) != (self.req_num, self.query_count):
            raise RuntimeError(f"query must be [{self.req_num}, {self.query_count}], got {tuple(query.shape)}")
        o = out or self._out
        s = (stream or torch.cuda.current_stream(self.device)).cuda_stream
        with torch.cuda.device(self.device):
            check(lib.asu_lru_step(
                s, self.token_to_slot.data_ptr(), self.slot_to_token.data_ptr(), self.lru_order.data_ptr(),
                self.free_stack.data_ptr(), self.free_count.data_ptr(), query.data_ptr(), o.slot.data_ptr(),
                o.hit.data_ptr(), o.install.data_ptr(), o.evicted.data_ptr(), o.evicted.shape[1],
                o.evicted_count.data_ptr(), self.stats.data_ptr(), self.status.data_ptr(), self.req_num,
                self.key_space, self.slot_count, self.query_count, self.free_target), "asu_lru_step")
        return o

    def step_from_host(self, query: torch.Tensor, query_copy: torch.Tensor, out: LruStepOutput | None = None,
                       stream: torch.cuda.Stream | None = None) -> LruStepOutput:
        """``step`` for a top-k in pinned host memory: ``query`` [R, Q] int32 is read by the step
        itself over the host link (no upload), and copied to ``query_copy`` [R, Q] int32 in HBM for
        the swap-in that follows.  Asynchronous: keep ``query`` unchanged until the step is done."""
        if query.dtype != torch.int32 or query.device.type != "cpu" or not query.is_contiguous():
            raise RuntimeError("query must be a contiguous int32 tensor in pinned host memory")
        if query_copy.dtype != torch.int32 or query_copy.device != self.device or not query_copy.is_contiguous():
            raise RuntimeError("query_copy must be a contiguous int32 tensor on the pool's device")
        shape = (self.req_num, self.query_count)
        if tuple(query.shape) != shape or tuple(query_copy.shape) != shape:
            raise RuntimeError(f"query and query_copy must be [{self.req_num}, {self.query_count}]")
        qdev = ctypes.c_void_p()
        check(lib.asu_host_device_pointer(query.data_ptr(), ctypes.byref(qdev)),
              "query: device address of pinned memory")
        o = out or self._out
        s = (stream or torch.cuda.current_stream(self.device)).cuda_stream
        with torch.cuda.device(self.device):
            check(lib.asu_lru_step_host_query(
                s, self.token_to_slot.data_ptr(), self.slot_to_token.data_ptr(), self.lru_order.data_ptr(),
                self.free_stack.data_ptr(), self.free_count.data_ptr(), qdev.value, query_copy.data_ptr(),
                o.slot.data_ptr(), o.hit.data_ptr(), o.install.data_ptr(), o.evicted.data_ptr(), o.evicted.shape[1],
                o.evicted_count.data_ptr(), self.stats.data_ptr(), self.status.data_ptr(), self.req_num,
                self.key_space, self.slot_count, self.query_count, self.free_target), "asu_lru_step_host_query")
        return o

    def check_status(self, ignore: int = ST_SHORTAGE) -> None:
        raise_on_status(self.status, "asu_lru_step", ignore)

    def totals(self) -> dict:
        return dict(zip(self.STAT_NAMES, self.stats.sum(0).cpu().tolist()))
