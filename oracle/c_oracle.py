"""ctypes wrapper of oracle/libasu_oracle.so (TEST INFRASTRUCTURE ONLY: tests and the timed
CPU baseline of bench.py).  See asu_oracle.c for what each function restates."""

from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_int32, c_int64, c_uint32, c_void_p

import numpy as np

from . import build_oracle

_lib = None


def lib():
    global _lib
    if _lib is None:
        if not build_oracle.LIB.exists():
            build_oracle.build()
        L = ctypes.CDLL(str(build_oracle.LIB))
        L.lru_create.restype = c_void_p
        L.lru_create.argtypes = [c_int32, c_int32, c_int32]
        L.lru_destroy.argtypes = [c_void_p]
        L.lru_step.restype = c_int32
        L.lru_step.argtypes = [c_void_p, c_void_p, c_int32, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p]
        L.lru_export.argtypes = [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p]
        L.lru_step_all.restype = c_int32
        L.lru_step_all.argtypes = [POINTER(c_void_p), c_int32, c_int32, c_void_p, c_void_p, c_void_p, c_void_p,
                                   c_void_p, c_int32, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_void_p,
                                   c_int64, c_void_p, c_int32, c_int32]
        L.ops_lookup.argtypes = [c_void_p] * 6 + [c_int32] * 5
        L.ops_maintain.restype = c_int32
        L.ops_maintain.argtypes = [c_void_p] * 5 + [c_int32, c_uint32] + [c_int32] * 4
        L.gather_lookup.argtypes = [c_void_p, c_int32, c_void_p, c_int32, c_void_p, c_void_p, c_int32]
        _lib = L
    return _lib


def _p(a: np.ndarray | None):
    return None if a is None else a.ctypes.data


class LruPools:
    """req_num independent exact-LRU pools on the host (serial algorithm per pool)."""

    def __init__(self, req_num: int, key_space: int, slots: int, target: int):
        L = lib()
        self.req_num, self.key_space, self.slots, self.target = req_num, key_space, slots, min(target, slots)
        self._pools = (c_void_p * req_num)(*[L.lru_create(slots, target, key_space) for _ in range(req_num)])
        self.stats = np.zeros((req_num, 5), np.int64)

    def step_all(self, keys: np.ndarray, threads: int | None = None, want_outputs: bool = True,
                 host_pool: np.ndarray | None = None, record: np.ndarray | None = None,
                 slot_pool: np.ndarray | None = None):
        """One step for every request.  Returns (slot, hit, install, evicted, evicted_n) or None."""
        R, Q = keys.shape
        keys = np.ascontiguousarray(keys, np.int32)
        slot = np.empty((R, Q), np.int32) if want_outputs else None
        hit = np.empty((R, Q), np.uint8) if want_outputs else None
        inst = np.empty((R, Q), np.uint8) if want_outputs else None
        ev_stride = max(self.target, 1)
        ev = np.empty((R, ev_stride), np.int32) if want_outputs else None
        evn = np.empty(R, np.int32) if want_outputs else None
        threads = threads or os.cpu_count() or 1
        lib().lru_step_all(self._pools, R, Q, _p(keys), _p(slot), _p(hit), _p(inst), _p(ev), ev_stride, _p(evn),
                           _p(self.stats), _p(host_pool), 0 if host_pool is None else host_pool.shape[0],
                           0 if host_pool is None else host_pool.shape[1], _p(record),
                           0 if record is None else record.shape[1], _p(slot_pool), self.slots, threads)
        if not want_outputs:
            return None
        return slot, hit.astype(bool), inst.astype(bool), ev, evn

    def export(self, r: int):
        t2s = np.empty(self.key_space, np.int32)
        s2t = np.empty(self.slots, np.int32)
        order = np.empty(self.slots, np.int32)
        stack = np.empty(self.slots, np.int32)
        cnt = c_int32()
        lib().lru_export(self._pools[r], _p(t2s), _p(s2t), _p(order), _p(stack), ctypes.byref(cnt))
        return t2s, s2t, order, stack, cnt.value

    def close(self):
        if getattr(self, "_pools", None) is not None:
            for p in self._pools:
                lib().lru_destroy(p)
            self._pools = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def ops_lookup(index, s2i, free_slots, free_head, query):
    index, s2i, free_head = index.copy(), s2i.copy(), free_head.copy()
    R, Q = query.shape
    out = np.empty((R, Q), np.int32)
    lib().ops_lookup(_p(index), _p(s2i), _p(np.ascontiguousarray(free_slots)), _p(free_head),
                     _p(np.ascontiguousarray(query)), _p(out), R, index.shape[1], s2i.shape[1], free_slots.shape[1], Q)
    return out, index, s2i, free_head


def ops_maintain(index, s2i, free_slots, free_head, lq, seed):
    index, s2i, free_slots, free_head = index.copy(), s2i.copy(), free_slots.copy(), free_head.copy()
    R = index.shape[0]
    rc = lib().ops_maintain(_p(index), _p(s2i), _p(free_slots), _p(free_head), _p(np.ascontiguousarray(lq)), R,
                            seed & 0xFFFFFFFF, index.shape[1], s2i.shape[1], free_slots.shape[1], lq.shape[1])
    return index, s2i, free_slots, free_head, rc


def gather_lookup(table, query):
    R, Q = query.shape
    out = np.empty((R, Q), np.int32)
    hit = np.empty((R, Q), np.uint8)
    lib().gather_lookup(_p(np.ascontiguousarray(table)), table.shape[1], _p(np.ascontiguousarray(query)), Q,
                        _p(out), _p(hit), R)
    return out, hit.astype(bool)
