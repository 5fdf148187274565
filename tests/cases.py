"""Test-case builders restated from the reference's own harnesses (shared by CPU and GPU tests)."""

from __future__ import annotations

import numpy as np

INDEX_SIZE = 128 * 1024
SLOT_COUNT = 10 * 1024
RESIDENT_SLOT_COUNT = 8 * 1024
FREE_SLOT_COUNT = 2 * 1024
QUERY_COUNT = 2 * 1024
NOT_FOUND = -1


def make_query(pattern: str, req_id: int) -> np.ndarray:
    """ops/scripts/asu_hbm_index_common.py:100-116 (the 'mixed' pattern plants duplicates at 1025, 1027)."""
    hit_query = np.arange(QUERY_COUNT, dtype=np.int32) % RESIDENT_SLOT_COUNT
    miss_base = 20_000 + req_id * 3_000
    miss_query = ((miss_base + np.arange(QUERY_COUNT, dtype=np.int32)) % INDEX_SIZE).astype(np.int32)
    if pattern == "hit":
        return hit_query
    if pattern == "miss":
        return miss_query
    if pattern == "mixed":
        q = hit_query.copy()
        q[QUERY_COUNT // 2:] = miss_query[: QUERY_COUNT // 2]
        q[QUERY_COUNT // 2 + 1] = q[QUERY_COUNT // 2]
        q[QUERY_COUNT // 2 + 3] = q[QUERY_COUNT // 2 + 2]
        return q
    raise ValueError(pattern)


def make_index_case(req_num: int, pattern: str):
    """ops/scripts/asu_hbm_index_common.py:80-97 -> (index, slot_to_index, free_slots, free_head, query)."""
    index = np.full((req_num, INDEX_SIZE), NOT_FOUND, np.int32)
    s2i = np.full((req_num, SLOT_COUNT), NOT_FOUND, np.int32)
    free_slots = np.empty((req_num, FREE_SLOT_COUNT), np.int32)
    free_head = np.zeros(req_num, np.int32)
    query = np.empty((req_num, QUERY_COUNT), np.int32)
    keys = np.arange(RESIDENT_SLOT_COUNT, dtype=np.int32)
    for r in range(req_num):
        index[r, keys] = keys
        s2i[r, keys] = keys
        free_slots[r] = np.arange(RESIDENT_SLOT_COUNT, SLOT_COUNT, dtype=np.int32)
        query[r] = make_query(pattern, r)
    return index, s2i, free_slots, free_head, query


def make_maintain_case(req_num: int, evict_ratio: float):
    """ops/scripts/asu_hbm_index_common.py:148-176 -> (index, s2i, free_slots, free_head, last_query_slots)."""
    evict = int(round(FREE_SLOT_COUNT * evict_ratio))
    index = np.full((req_num, INDEX_SIZE), NOT_FOUND, np.int32)
    s2i = np.full((req_num, SLOT_COUNT), NOT_FOUND, np.int32)
    free_slots = np.empty((req_num, FREE_SLOT_COUNT), np.int32)
    free_head = np.full(req_num, evict, np.int32)
    lq = np.empty((req_num, QUERY_COUNT), np.int32)
    keys = np.arange(RESIDENT_SLOT_COUNT, dtype=np.int32)
    miss_keys = 20_000 + np.arange(evict, dtype=np.int32)
    alloc = RESIDENT_SLOT_COUNT + np.arange(evict, dtype=np.int32)
    hit_count = QUERY_COUNT - evict
    for r in range(req_num):
        index[r, keys] = keys
        s2i[r, keys] = keys
        free_slots[r] = np.arange(RESIDENT_SLOT_COUNT, SLOT_COUNT, dtype=np.int32)
        if evict:
            index[r, miss_keys] = alloc
            s2i[r, alloc] = miss_keys
        if hit_count:
            lq[r, :hit_count] = np.arange(hit_count, dtype=np.int32)
        if evict:
            lq[r, hit_count:] = alloc
    return index, s2i, free_slots, free_head, lq


def apply_changes(base: np.ndarray, idx: np.ndarray, val: np.ndarray) -> np.ndarray:
    out = base.copy().reshape(-1)
    out[idx] = val
    return out.reshape(base.shape)


def gather_single_case():
    """simu/hbm_lookup_update/scripts/test_lookup_update.py:89-104 inputs."""
    tok = np.arange(INDEX_SIZE, dtype=np.int32)
    states = (tok.astype(np.int64) * 10 + 7).astype(np.int32)
    q = ((np.arange(512, dtype=np.int64) * 17 + 23) % INDEX_SIZE).astype(np.int32)
    new = (100000 + np.arange(512, dtype=np.int32)).astype(np.int32)
    return states[None, :], q[None, :], new[None, :], 42, 5


def gather_multi_case():
    """simu/hbm_lookup_update/scripts/test_lookup_update.py:134-160 inputs."""
    req_num, qlen = 4, 513
    tok = np.arange(INDEX_SIZE, dtype=np.int32)
    states = np.empty((req_num, INDEX_SIZE), np.int32)
    q = np.empty((req_num, qlen), np.int32)
    new = np.empty((req_num, qlen), np.int32)
    for r in range(req_num):
        states[r] = (tok.astype(np.int64) * 13 + 1000 * r + 17).astype(np.int32)
        q[r] = ((np.arange(qlen, dtype=np.int64) * 19 + r * 101 + 7) % INDEX_SIZE).astype(np.int32)
        new[r] = (200000 + 10000 * r + np.arange(qlen, dtype=np.int32)).astype(np.int32)
    return states, q, new, 2026, 7


def gather_dup_case():
    """Duplicate keys inside the updated positions (last writer must win)."""
    rng = np.random.Generator(np.random.PCG64(5))
    q = rng.integers(0, 300, (3, 700)).astype(np.int32)
    new = rng.integers(-(2**31), 2**31 - 1, (3, 700)).astype(np.int32)
    states = rng.integers(-5, 1000, (3, INDEX_SIZE)).astype(np.int32)
    return states, q, new, 77, 100


def simt_full_resident_state():
    """pta-ops/asu_hbm_index_lookup_simt/python/random_workload.py:78-91 for one row."""
    t2s = np.full(INDEX_SIZE, NOT_FOUND, np.int32)
    t2s[:SLOT_COUNT] = np.arange(SLOT_COUNT, dtype=np.int32)
    s2t = np.arange(SLOT_COUNT, dtype=np.int32)
    lru = np.arange(SLOT_COUNT, dtype=np.int16)
    return t2s, s2t, lru
