"""Seeded synthetic workloads for the resolver benchmarks and parity tests.

The reference measures on no public dataset; every input is synthetic.  The
generators below produce the decode-step top-k traces and table states of the
five benchmark configurations with numpy's PCG64 generator:

* ``c0``/``c2`` locality: step 0 draws top-k distinct ids by Zipf(s) over
  positions; every later step keeps ``reuse`` of the previous step's ids
  (sampled without replacement) and draws the rest by Zipf, re-drawing
  duplicates.  The Zipf draw uses the LRU simulator's CDF method: rank r has
  weight 1/r**s and the id is ``searchsorted(cdf, u * total)``
  (simu/kv_cache_eviction_sim.py:186-195,220-235).
* ``c1``: per request a 128K-entry table that is -1 except ``resident``
  uniformly placed entries holding a permutation of slots; queries are
  distinct, ``hit_frac`` drawn from the resident set.
* ``c4``: a fixed fraction reused from the previous step and the rest uniform
  over a 1M-token context.
"""

from __future__ import annotations

import numpy as np

NOT_FOUND = -1


def zipf_cdf(n: int, s: float) -> np.ndarray:
    """Cumulative weights of ranks 1..n with weight 1/rank**s (float64)."""
    return np.cumsum(1.0 / np.arange(1, n + 1, dtype=np.float64) ** s)


class LocalityTrace:
    """Per-request decode-step top-k streams with reuse + Zipf locality."""

    def __init__(self, req_num: int, key_space: int, topk: int = 2048, reuse: float = 0.7,
                 zipf_s: float = 1.1, seed: int = 0):
        if topk > key_space:
            raise ValueError("topk must not exceed key_space")
        self.req_num = req_num
        self.key_space = key_space
        self.topk = topk
        self.n_reuse = int(round(topk * reuse))
        self.rng = np.random.Generator(np.random.PCG64(seed))
        self.cdf = zipf_cdf(key_space, zipf_s)
        self.total = float(self.cdf[-1])
        self.prev: np.ndarray | None = None

    def _zipf(self, n: int) -> np.ndarray:
        u = self.rng.random(n) * self.total
        return np.minimum(np.searchsorted(self.cdf, u, side="left"), self.key_space - 1)

    def _fill(self, keep: np.ndarray, need: int) -> np.ndarray:
        """Draw ``need`` Zipf ids not in ``keep`` and distinct, in draw order."""
        taken = set(keep.tolist())
        out: list[int] = []
        batch = max(4 * need, 64)
        tries = 0
        while len(out) < need:
            for v in self._zipf(batch).tolist():
                if v not in taken:
                    taken.add(v)
                    out.append(v)
                    if len(out) == need:
                        break
            tries += 1
            if tries > 64:  # heavy head: fall back to uniform fill like _fill_unique_tokens
                while len(out) < need:
                    v = int(self.rng.integers(0, self.key_space))
                    if v not in taken:
                        taken.add(v)
                        out.append(v)
        return np.asarray(out, np.int32)

    def step(self) -> np.ndarray:
        """Next step's [req_num, topk] int32 ids (distinct within a row)."""
        rows = np.empty((self.req_num, self.topk), np.int32)
        for r in range(self.req_num):
            if self.prev is None:
                keep = np.zeros(0, np.int32)
            else:
                keep = self.rng.permutation(self.prev[r])[: self.n_reuse]
            fresh = self._fill(keep, self.topk - keep.size)
            row = np.concatenate([keep, fresh])
            rows[r] = self.rng.permutation(row)
        self.prev = rows
        return rows


def lookup_only_case(req_num: int = 64, index_size: int = 128 * 1024, resident: int = 4096,
                     query_len: int = 2048, hit_frac: float = 0.85, seed: int = 1):
    """Table + queries of the lookup-only workload (64 x 128K table, 64 x 2048 queries)."""
    rng = np.random.Generator(np.random.PCG64(seed))
    table = np.full((req_num, index_size), NOT_FOUND, np.int32)
    query = np.empty((req_num, query_len), np.int32)
    n_hit = int(round(query_len * hit_frac))
    for r in range(req_num):
        pos = rng.choice(index_size, size=resident, replace=False).astype(np.int32)
        table[r, pos] = rng.permutation(resident).astype(np.int32)
        hits = rng.choice(pos, size=n_hit, replace=False)
        mask = np.ones(index_size, bool)
        mask[pos] = False
        absent = np.flatnonzero(mask)
        misses = rng.choice(absent, size=query_len - n_hit, replace=False)
        query[r] = rng.permutation(np.concatenate([hits, misses]).astype(np.int32))
    return table, query


class UniformReuseTrace:
    """Stress trace: ``reuse`` of the previous ids kept, the rest uniform over the context."""

    def __init__(self, req_num: int, key_space: int, topk: int = 2048, reuse: float = 0.2, seed: int = 4):
        self.req_num, self.key_space, self.topk = req_num, key_space, topk
        self.n_reuse = int(round(topk * reuse))
        self.rng = np.random.Generator(np.random.PCG64(seed))
        self.prev: np.ndarray | None = None

    def step(self) -> np.ndarray:
        rows = np.empty((self.req_num, self.topk), np.int32)
        for r in range(self.req_num):
            keep = np.zeros(0, np.int32) if self.prev is None else self.rng.permutation(self.prev[r])[: self.n_reuse]
            taken = set(keep.tolist())
            fresh: list[int] = []
            while len(fresh) < self.topk - keep.size:
                for v in self.rng.integers(0, self.key_space, 2 * self.topk).tolist():
                    if v not in taken:
                        taken.add(v)
                        fresh.append(v)
                        if len(fresh) == self.topk - keep.size:
                            break
            rows[r] = self.rng.permutation(np.concatenate([keep, np.asarray(fresh, np.int32)]))
        self.prev = rows
        return rows


RECORD_SALT = 2654435761  # odd 32-bit multiplier
RECORD_OFFSET = 0x7F4A7C15


def record_addresses(req_num: int, key_space: int, pool_rows: int) -> np.ndarray:
    """[req_num, key_space] int32 row index of each (request, key) record in the host pool.

    A multiplicative hash scatters records over a pool of ``pool_rows`` rows so that a bounded
    pinned pool can stand in for a full per-token backing store (several keys may share a
    row; every check uses the same table).  The product stays below 2**63 for
    req_num * key_space < 2**31, so torch on the GPU computes the same values
    (record_addresses_torch).
    """
    r = np.arange(req_num, dtype=np.int64)[:, None]
    k = np.arange(key_space, dtype=np.int64)[None, :]
    return (((r * key_space + k) * RECORD_SALT + RECORD_OFFSET) % pool_rows).astype(np.int32)


def record_addresses_torch(req_num: int, key_space: int, pool_rows: int, device, key_offset: int = 0,
                           row_stride: int | None = None):
    """record_addresses computed on ``device`` (same values), for tables too large for host RAM.

    ``key_offset`` / ``row_stride`` select the columns [key_offset, key_offset + key_space) of a
    wider table with ``row_stride`` keys per request (one layer of a multi-layer record space).
    """
    import torch

    stride = key_space if row_stride is None else row_stride
    out = torch.empty((req_num, key_space), dtype=torch.int32, device=device)
    k = torch.arange(key_space, dtype=torch.int64, device=device) + key_offset
    for r in range(req_num):
        out[r] = ((r * stride + k) * RECORD_SALT + RECORD_OFFSET).remainder(pool_rows).to(torch.int32)
    return out


class FastLocalityTrace:
    """Vectorised reuse + Zipf (or uniform) trace for large request counts.

    Same recipe as LocalityTrace -- keep ``reuse`` of the previous ids, draw the rest by
    Zipf(s) with the CDF method (uniform when ``zipf_s`` is None), distinct within a row, in
    draw order -- but one random stream serves all rows and every draw column is one vector
    operation over the rows, so its ids differ from LocalityTrace's.  Used by the
    multi-layer and stress benchmarks, which need hundreds of rows per step.
    """

    def __init__(self, req_num: int, key_space: int, topk: int = 2048, reuse: float = 0.7,
                 zipf_s: float | None = 1.1, seed: int = 0):
        self.req_num, self.key_space, self.topk = req_num, key_space, topk
        self.n_reuse = int(round(topk * reuse))
        self.rng = np.random.Generator(np.random.PCG64(seed))
        self.cdf = zipf_cdf(key_space, zipf_s) if zipf_s else None
        self.prev: np.ndarray | None = None

    def _draw(self, shape) -> np.ndarray:
        if self.cdf is None:
            return self.rng.integers(0, self.key_space, shape)
        u = self.rng.random(shape) * self.cdf[-1]
        return np.minimum(np.searchsorted(self.cdf, u, side="left"), self.key_space - 1)

    def step(self) -> np.ndarray:
        R, K = self.req_num, self.key_space
        rows = np.arange(R)
        if self.prev is None:
            keep = np.zeros((R, 0), np.int64)
        else:
            perm = np.argsort(self.rng.random(self.prev.shape), axis=1)[:, : self.n_reuse]
            keep = np.take_along_axis(self.prev, perm, axis=1).astype(np.int64)
        need = self.topk - keep.shape[1]
        taken = np.zeros((R, K), bool)
        taken[rows[:, None], keep] = True
        fresh = np.empty((R, need), np.int64)
        filled = np.zeros(R, np.int64)
        rounds = 0
        while True:
            pend = np.flatnonzero(filled < need)
            if pend.size == 0:
                break
            rounds += 1
            uniform = self.cdf is None or rounds > 16  # heavy head: finish with uniform draws
            cand = (self.rng.integers(0, K, (pend.size, 2 * need)) if uniform
                    else self._draw((pend.size, 2 * need)))
            for c in range(cand.shape[1]):
                v = cand[:, c]
                ok = (~taken[pend, v]) & (filled[pend] < need)
                if not ok.any():
                    if (filled[pend] >= need).all():
                        break
                    continue
                rr, vv = pend[ok], v[ok]
                taken[rr, vv] = True
                fresh[rr, filled[rr]] = vv
                filled[rr] += 1
        out = np.concatenate([keep, fresh], axis=1)
        out = np.take_along_axis(out, np.argsort(self.rng.random(out.shape), axis=1), axis=1)
        self.prev = out.astype(np.int32)
        return self.prev


# ------------------------------------------------------------------ ops lookup / maintain cases
# Restated from the reference's op harness (ops/scripts/asu_hbm_index_common.py), which both its
# validation and its benchmark (ops/scripts/bench_hbm_index_ops.py) build their inputs with.

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


# ------------------------------------------------------------------ batch-LRU (SIMT) cases
# Restated from pta-ops/asu_hbm_index_lookup_simt/python/random_workload.py: every slot
# resident (token t in slot t, LRU order = slot order), and per request a unique 2K query with
# exactly `hit_count` resident tokens and the rest drawn from the non-resident range, shuffled.
# The random draws are this project's own (numpy), so the queries differ from the reference's.

SIMT_SLOT_COUNT = 10 * 1024


def simt_case(req_num: int, hit_count: int, seed: int = 0):
    """(token_to_slot [R, 128K] int32, slot_to_token [R, 10K] int32, lru_slots [R, 10K] int16,
    query [R, 2K] int32)."""
    if not 0 <= hit_count <= QUERY_COUNT:
        raise ValueError(f"hit_count must be in [0, {QUERY_COUNT}]")
    rng = np.random.Generator(np.random.PCG64(seed))
    t2s = np.full((req_num, INDEX_SIZE), NOT_FOUND, np.int32)
    t2s[:, :SIMT_SLOT_COUNT] = np.arange(SIMT_SLOT_COUNT, dtype=np.int32)
    s2t = np.tile(np.arange(SIMT_SLOT_COUNT, dtype=np.int32), (req_num, 1))
    lru = np.tile(np.arange(SIMT_SLOT_COUNT, dtype=np.int16), (req_num, 1))
    query = np.empty((req_num, QUERY_COUNT), np.int32)
    for r in range(req_num):
        hits = rng.choice(SIMT_SLOT_COUNT, hit_count, replace=False)
        misses = SIMT_SLOT_COUNT + rng.choice(INDEX_SIZE - SIMT_SLOT_COUNT, QUERY_COUNT - hit_count, replace=False)
        q = np.concatenate([hits, misses]).astype(np.int32)
        rng.shuffle(q)
        query[r] = q
    return t2s, s2t, lru, query
