"""Test-case builders restated from the reference's own harnesses (shared by CPU and GPU tests)."""

from __future__ import annotations

import numpy as np

from asu_ascend_b200.workloads import (  # noqa: F401  (restated reference harness cases)
    FREE_SLOT_COUNT,
    INDEX_SIZE,
    NOT_FOUND,
    QUERY_COUNT,
    RESIDENT_SLOT_COUNT,
    SLOT_COUNT,
    make_index_case,
    make_maintain_case,
    make_query,
)


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
