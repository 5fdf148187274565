"""CPU oracle for the ASU KV-resolver hot path.

TEST INFRASTRUCTURE ONLY. This module restates, in plain Python/numpy, the
reference algorithms that the CUDA kernels in ``asu_ascend_b200`` implement.
Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py`` (its
``cpu_baseline`` leg and ``--impl reference`` arm) may import it, and only as
the checker / the timed CPU baseline.  The product path never calls it and has
no CPU fallback.

Parity is pinned: ``tests/golden/make_golden.py`` runs the reference's own
Python code (the LRU simulator, the ops oracle, the batch-LRU oracle, the
gather/update oracle and the resolver reference extracted from patch 0001) on
seeded inputs and stores the results in ``tests/golden/*.npz``;
``tests/test_oracle_golden.py`` checks every function below against them.

Every function cites the reference file:line it restates (paths relative to
the ASU-Ascend project root).
"""

from __future__ import annotations

import math
from collections import OrderedDict
from dataclasses import dataclass, field

import numpy as np

NOT_FOUND = -1

# Reference constants: ops/asu_hbm_index_lookup_aiv.cpp:7-12,
# ops/scripts/asu_hbm_index_common.py:9-14.
INDEX_SIZE = 128 * 1024
SLOT_COUNT = 10 * 1024
RESIDENT_SLOT_COUNT = 8 * 1024
FREE_SLOT_COUNT = 2 * 1024
QUERY_COUNT = 2 * 1024
QUERY_TILE = 64  # simu/hbm_lookup_update/src/hbm_lookup_update_kernel.cpp:7

# Resolver token states: patch/0001 vllm_ascend/ops/asu_kv_resolver.py (patch lines 834-837).
INVALID = -1
ASU_ONLY = 0
HBM_RESIDENT = 1
TAIL_HBM = 2


def u32(x: int) -> int:
    return x & 0xFFFFFFFF


def hash32(x: int) -> int:
    """ops/scripts/asu_hbm_index_common.py:70-77; ops/asu_hbm_index_maintain_aicpu_kernel.aicpu:25-33."""
    x = u32(x)
    x ^= x >> 16
    x = u32(x * 0x7FEB352D)
    x ^= x >> 15
    x = u32(x * 0x846CA68B)
    x ^= x >> 16
    return u32(x)


# ---------------------------------------------------------------------------
# Pure gather + random update  (simu/hbm_lookup_update)
# ---------------------------------------------------------------------------

def gather_lookup(table: np.ndarray, query: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """out[r, i] = table[r, query[r, i]] and hit = out != -1.

    simu/hbm_lookup_update/scripts/test_lookup_update.py:75-78 (oracle) and
    src/hbm_lookup_update_kernel.cpp:100-126 (kernel).  The hit mask is the
    extra output the lookup-only benchmark asks for.
    """
    r = np.arange(query.shape[0])[:, None]
    out = table[r, query].astype(np.int32)
    return out, out != NOT_FOUND


def pick_coprime_a(seed: int, n: int) -> int:
    """simu/hbm_lookup_update/scripts/test_lookup_update.py:36-46; kernel.cpp:41-57."""
    if n <= 1:
        return 1
    a = hash32(seed) % n
    if a == 0:
        a = 1
    while math.gcd(a, n) != 1:
        a += 1
        if a >= n:
            a = 1
    return a


def update_positions(query_len: int, seed: int, update_percent: int, req_id: int = 0) -> list[int]:
    """simu/hbm_lookup_update/scripts/test_lookup_update.py:49-56; kernel.cpp:182-203."""
    update_num = (query_len * update_percent) // 100
    if update_num <= 0:
        return []
    req_seed = u32(seed) ^ hash32(req_id)
    a = pick_coprime_a(req_seed ^ 0x9E3779B9, query_len)
    b = hash32(req_seed ^ 0x85EBCA6B) % query_len
    return [((a * t + b) % query_len) for t in range(update_num)]


def random_update(table: np.ndarray, query: np.ndarray, new_states: np.ndarray,
                  seed: int, update_percent: int) -> np.ndarray:
    """Serial last-writer-wins scatter, test_lookup_update.py:80-82; kernel.cpp:193-207."""
    out = table.copy()
    for r in range(query.shape[0]):
        for pos in update_positions(query.shape[1], seed, update_percent, r):
            out[r, int(query[r, pos])] = new_states[r, pos]
    return out


# ---------------------------------------------------------------------------
# ops contract: lookup with sequential allocation, hash-seeded ring maintain
# ---------------------------------------------------------------------------

def ops_lookup_allocate(index, slot_to_index, free_slots, free_head, query):
    """ops/scripts/asu_hbm_index_common.py:119-139 (kernel ops/asu_hbm_index_lookup_aiv.cpp:79-130).

    Returns (slot_out, index, slot_to_index, free_head) as new arrays.
    """
    index = index.copy()
    slot_to_index = slot_to_index.copy()
    free_head = free_head.copy()
    slot_out = np.empty_like(query)
    for r in range(query.shape[0]):
        head = int(free_head[r])
        for pos in range(query.shape[1]):
            key = int(query[r, pos])
            slot = int(index[r, key])
            if slot == NOT_FOUND:
                slot = int(free_slots[r, head])
                head += 1
                index[r, key] = slot
                slot_to_index[r, slot] = key
            slot_out[r, pos] = slot
        free_head[r] = head
    return slot_out, index, slot_to_index, free_head


def ops_maintain(index, slot_to_index, free_slots, free_head, last_query_slots, seed: int):
    """ops/scripts/asu_hbm_index_common.py:185-214 (kernel ops/asu_hbm_index_maintain_aicpu_kernel.aicpu:53-95).

    Returns (index, slot_to_index, free_slots, free_head) as new arrays.
    """
    index = index.copy()
    slot_to_index = slot_to_index.copy()
    free_slots = free_slots.copy()
    free_head = free_head.copy()
    slot_count = slot_to_index.shape[1]
    for r in range(index.shape[0]):
        protected = {int(s) for s in last_query_slots[r]}
        head = int(free_head[r])
        start = hash32(seed ^ r) % slot_count
        offset = 0
        while head > 0:
            slot = (start + offset) % slot_count
            key = int(slot_to_index[r, slot])
            if key != NOT_FOUND and slot not in protected:
                slot_to_index[r, slot] = NOT_FOUND
                index[r, key] = NOT_FOUND
                head -= 1
                free_slots[r, head] = slot
            offset += 1
        free_head[r] = head
    return index, slot_to_index, free_slots, free_head


# ---------------------------------------------------------------------------
# Exact LRU pool (simu/kv_cache_eviction_sim.py LRUManagedCache), one per request
# ---------------------------------------------------------------------------

@dataclass
class LruStepResult:
    slot: np.ndarray       # [Q] int32, -1 on shortage / invalid
    hit: np.ndarray        # [Q] bool, serial-order hit (the simulator's `hits`)
    install: np.ndarray    # [Q] bool, this position took a free slot (one swap-in)
    evicted: np.ndarray    # [E] int32 keys evicted by the step-boundary maintain, LRU first
    shortages: int = 0


@dataclass
class LruPool:
    """One request's slot pool, restating LRUManagedCache (simu/kv_cache_eviction_sim.py:99-150).

    free stack  : list, pop() from the end; initial order [S-1 .. 0] (:109)
    residents   : OrderedDict key -> slot, LRU first (:110)
    """

    total_slots: int
    free_slot_target: int
    free: list = field(default_factory=list)
    residents: OrderedDict = field(default_factory=OrderedDict)

    def __post_init__(self):
        if self.total_slots < 0 or self.free_slot_target < 0:
            raise ValueError("total_slots and free_slot_target must be non-negative")
        self.free_slot_target = min(self.free_slot_target, self.total_slots)
        self.free = list(range(self.total_slots - 1, -1, -1))

    def prepare_free_slots(self) -> list:
        """:124-131 -- evict LRU residents until the free target is met."""
        evicted = []
        while len(self.free) < self.free_slot_target and self.residents:
            key, slot = self.residents.popitem(last=False)
            self.free.append(slot)
            evicted.append(key)
        return evicted

    def resolve(self, keys) -> LruStepResult:
        """:133-150 -- hits move to MRU, misses pop the free stack, else shortage."""
        q = len(keys)
        slot = np.full(q, NOT_FOUND, np.int32)
        hit = np.zeros(q, bool)
        install = np.zeros(q, bool)
        shortages = 0
        for pos, key in enumerate(keys):
            key = int(key)
            if key in self.residents:
                hit[pos] = True
                self.residents.move_to_end(key)
                slot[pos] = self.residents[key]
                continue
            if self.free:
                s = self.free.pop()
                self.residents[key] = s
                slot[pos] = s
                install[pos] = True
            else:
                shortages += 1
        return LruStepResult(slot, hit, install, np.zeros(0, np.int32), shortages)

    def step(self, keys) -> LruStepResult:
        """One decode step of run_simulation (:261-268): maintain, then resolve."""
        evicted = self.prepare_free_slots()
        res = self.resolve(keys)
        res.evicted = np.asarray(evicted, np.int32)
        return res

    def export_state(self, key_space: int):
        """State in the GPU layout: token_to_slot[K], slot_to_token[S], lru_order[S]
        (first resident_count entries, LRU first), free_stack[S] (first free_count
        entries, top last), free_count."""
        s = self.total_slots
        t2s = np.full(key_space, NOT_FOUND, np.int32)
        s2t = np.full(s, NOT_FOUND, np.int32)
        order = np.full(s, NOT_FOUND, np.int32)
        for i, (key, slot) in enumerate(self.residents.items()):
            t2s[key] = slot
            s2t[slot] = key
            order[i] = slot
        stack = np.full(s, NOT_FOUND, np.int32)
        stack[: len(self.free)] = self.free
        return t2s, s2t, order, stack, len(self.free)


def lru_initial_state(req_num: int, key_space: int, slots: int):
    """GPU-layout state of LRUManagedCache.__init__ (:102-110) for req_num requests."""
    t2s = np.full((req_num, key_space), NOT_FOUND, np.int32)
    s2t = np.full((req_num, slots), NOT_FOUND, np.int32)
    order = np.full((req_num, slots), NOT_FOUND, np.int32)
    stack = np.tile(np.arange(slots - 1, -1, -1, dtype=np.int32), (req_num, 1))
    count = np.full(req_num, slots, np.int32)
    return t2s, s2t, order, stack, count


# ---------------------------------------------------------------------------
# Batch-LRU (Ascend 950 SIMT contract)
# ---------------------------------------------------------------------------

def batch_lru(query, token_to_slot, slot_to_token, lru_slots):
    """pta-ops/asu_hbm_index_lookup_simt/python/lookup_lru_reference.py:21-89, one request row.

    Mutates token_to_slot / slot_to_token / lru_slots (python lists or 1-D arrays)
    and returns (slot_ids, miss_mask).
    """
    slot_count = len(slot_to_token)
    if len(lru_slots) != slot_count:
        raise ValueError("lru_slots length must match slot_to_token")
    if sorted(int(s) for s in lru_slots) != list(range(slot_count)):
        raise ValueError("lru_slots must be a permutation of all slot ids")
    n_tok = len(token_to_slot)
    slot_ids = [NOT_FOUND] * len(query)
    miss_mask = [False] * len(query)
    hit_set: set = set()
    unique_misses: list = []
    pending: set = set()
    for pos, token in enumerate(query):
        token = int(token)
        if token < 0 or token >= n_tok:
            continue
        slot = int(token_to_slot[token])
        if slot >= 0:
            if slot >= slot_count:
                raise ValueError(f"token {token} maps outside the slot table")
            slot_ids[pos] = slot
            hit_set.add(slot)
        elif slot == NOT_FOUND and token not in pending:
            pending.add(token)
            unique_misses.append((pos, token))
            miss_mask[pos] = True
        elif slot != NOT_FOUND:
            raise ValueError(f"token {token} has transient/invalid slot {slot}")
    lru = [int(s) for s in lru_slots]
    hit_slots = [s for s in lru if s in hit_set]
    evictable = [s for s in lru if s not in hit_set]
    if len(unique_misses) > len(evictable):
        raise ValueError("unique misses exceed evictable slot count")
    for rank, (_, token) in enumerate(unique_misses):
        victim = evictable[rank]
        victim_token = int(slot_to_token[victim])
        if victim_token >= 0:
            if victim_token >= n_tok:
                raise ValueError(f"slot {victim} contains out-of-range token {victim_token}")
            token_to_slot[victim_token] = NOT_FOUND
        slot_to_token[victim] = token
        token_to_slot[token] = victim
    for pos, token in enumerate(query):
        token = int(token)
        if 0 <= token < n_tok:
            slot_ids[pos] = int(token_to_slot[token])
    m = len(unique_misses)
    new_lru = evictable[m:] + evictable[:m] + hit_slots
    for i, s in enumerate(new_lru):
        lru_slots[i] = s
    return slot_ids, miss_mask


# ---------------------------------------------------------------------------
# Resolver (patch 0001 asu_kv_resolver custom op)
# ---------------------------------------------------------------------------

class ResolverError(RuntimeError):
    """Raised where the reference Python resolver raises (patch/0001 lines 879-888, 993-994, 1035-1036)."""


def resolve_kv_slots_single_req(topk, actual_seq_len, token_state, asu_record_addr, hbm_slot_of_token,
                                slot_owner_token, free_slot_stack, free_slot_count, block_table,
                                kv0_src, kv1_src, kv0_dst, kv1_dst, block_size):
    """patch/0001 vllm_ascend/ops/asu_kv_resolver.py::asu_resolve_kv_slots_single_req (patch lines 954-1039).

    numpy arrays, mutated in place exactly as the reference mutates its tensors;
    kv*_src / kv*_dst are [slots, row] arrays copied row by row.  Returns the
    resolved slot array with topk's shape.  ``free_slot_count`` is a 1-element array.
    """
    if actual_seq_len < 0:
        raise ResolverError("actual_seq_len must be non-negative")
    if block_size <= 0:
        raise ResolverError("block_size must be positive")
    flat = np.asarray(topk).reshape(-1)
    out = np.empty(flat.shape, np.int32)
    bt = np.asarray(block_table).reshape(-1)

    def install(token, src):
        count = int(free_slot_count[0])
        if count <= 0:
            raise ResolverError("free_slot_stack does not have enough slots")
        slot = int(free_slot_stack[count - 1])
        free_slot_count[0] = count - 1
        if src < 0 or src >= kv0_src.shape[0] or src >= kv1_src.shape[0]:
            raise ResolverError(f"source_slot {src} is out of range")
        if slot < 0 or slot >= kv0_dst.shape[0] or slot >= kv1_dst.shape[0]:
            raise ResolverError(f"managed_slot {slot} is out of range")
        kv0_dst[slot] = kv0_src[src]
        kv1_dst[slot] = kv1_src[src]
        token_state[token] = HBM_RESIDENT
        hbm_slot_of_token[token] = slot
        slot_owner_token[slot] = token
        return slot

    for i, tok in enumerate(flat):
        tok = int(tok)
        if tok < 0 or tok >= actual_seq_len:
            raise ResolverError(f"token_id {tok} is out of range")
        state = int(token_state[tok])
        if state == HBM_RESIDENT:
            slot = int(hbm_slot_of_token[tok])
        elif state == ASU_ONLY:
            slot = install(tok, int(asu_record_addr[tok]))
        elif state == TAIL_HBM:
            lb = tok // block_size
            if lb >= bt.size:
                raise ResolverError(f"original_block_table does not cover token_id {tok}")
            slot = install(tok, int(bt[lb]) * block_size + tok % block_size)
        else:
            raise ResolverError(f"unsupported token_state {state} for token_id {tok}")
        out[i] = slot
    return out.reshape(np.asarray(topk).shape)


def reset_state(max_seq_len, slot_count, block_size, actual_seq_len, managed_prefix_len, block_table):
    """Fresh per-layer resolver state, patch/0003 asu_kv_cache_manager.py::reset_state (patch lines 234-292)."""
    if actual_seq_len < 0 or managed_prefix_len < 0:
        raise ValueError("lengths must be non-negative")
    if managed_prefix_len > actual_seq_len:
        raise ValueError("managed_prefix_len must not exceed actual_seq_len")
    if actual_seq_len > max_seq_len:
        raise RuntimeError("ASU max_seq_len does not cover actual_seq_len")
    token_state = np.full(max_seq_len, INVALID, np.int32)
    record = np.full(max_seq_len, INVALID, np.int32)
    hbm_slot = np.full(max_seq_len, INVALID, np.int32)
    owner = np.full(slot_count, INVALID, np.int32)
    stack = np.arange(slot_count, dtype=np.int32)
    count = np.array([slot_count], np.int32)
    if managed_prefix_len > 0:
        pos = np.arange(managed_prefix_len)
        bt = np.asarray(block_table).reshape(-1).astype(np.int64)
        if pos[-1] // block_size >= bt.size:
            raise RuntimeError("original_block_table does not cover ASU prefix")
        token_state[:managed_prefix_len] = ASU_ONLY
        record[:managed_prefix_len] = (bt[pos // block_size] * block_size + pos % block_size).astype(np.int32)
    if managed_prefix_len < actual_seq_len:
        token_state[managed_prefix_len:actual_seq_len] = TAIL_HBM
    return token_state, record, hbm_slot, owner, stack, count


def resolve_kv_slots_lru(topk, actual_seq_len, token_state, asu_record_addr, hbm_slot_of_token, slot_owner_token,
                         free_slot_stack, free_slot_count, lru_order, free_target, block_table,
                         kv0_src, kv1_src, kv0_dst, kv1_dst, block_size):
    """The resolver over a bounded managed pool: the exact LRU pool of
    simu/kv_cache_eviction_sim.py (LRUManagedCache, :124-150) composed with the resolver of
    patch/0001 (asu_resolve_kv_slots_single_req, patch lines 954-1039).

    The resident slots are ``lru_order[: S - free_slot_count]``, least recently used first.
    1. Step-boundary maintain (prepare_free_slots, :124-131): while the free count is below
       ``min(free_target, S)`` and slots are resident, the LRU slot is evicted.  Its token goes
       back to ASU_ONLY when it has a record address (a prefix token read from the ASU store),
       else to TAIL_HBM (read from the paged cache again); its hbm_slot_of_token and the slot's
       owner are cleared and the slot is pushed on the free stack.
    2. Resolve (resolve_query, :133-150, with the resolver's install): an HBM_RESIDENT token is a
       hit and its slot becomes the most recently used; an ASU_ONLY / TAIL_HBM token is installed
       exactly as the resolver installs it (pop the stack top, copy the row pair, mark it
       resident), its slot the most recently used.  Errors raise ResolverError where the
       resolver raises.
    Mutates every state array in place; returns (resolved slots with topk's shape, evicted
    tokens in eviction order).
    """
    slots = int(slot_owner_token.shape[0])
    resident = slots - int(free_slot_count[0])
    order = OrderedDict((int(s), None) for s in lru_order[:resident])
    evicted = []
    while int(free_slot_count[0]) < min(int(free_target), slots) and order:
        victim, _ = order.popitem(last=False)
        tok = int(slot_owner_token[victim])
        if 0 <= tok < token_state.shape[0]:
            token_state[tok] = ASU_ONLY if int(asu_record_addr[tok]) >= 0 else TAIL_HBM
            hbm_slot_of_token[tok] = INVALID
        slot_owner_token[victim] = INVALID
        free_slot_stack[int(free_slot_count[0])] = victim
        free_slot_count[0] += 1
        evicted.append(tok)
    flat = np.asarray(topk).reshape(-1)
    out = np.empty(flat.shape, np.int32)
    for i, tok in enumerate(flat):
        # the resolver's per-token semantics, one token at a time, then the touch
        slot = int(resolve_kv_slots_single_req(
            np.array([tok], np.int32), actual_seq_len, token_state, asu_record_addr, hbm_slot_of_token,
            slot_owner_token, free_slot_stack, free_slot_count, block_table, kv0_src, kv1_src, kv0_dst, kv1_dst,
            block_size)[0])
        order[slot] = None
        order.move_to_end(slot)
        out[i] = slot
    lru_order[: len(order)] = np.fromiter(order.keys(), np.int32, len(order))
    return out.reshape(np.asarray(topk).shape), np.asarray(evicted, np.int32)


# ---------------------------------------------------------------------------
# Swap-in gather: host row pool -> HBM slot pool (byte copy)
# ---------------------------------------------------------------------------

def swapin(host_pool: np.ndarray, record_addr: np.ndarray, query: np.ndarray, slot: np.ndarray,
           install: np.ndarray, slot_pool: np.ndarray) -> np.ndarray:
    """For every installing position: slot_pool[r, slot] = host_pool[record_addr[r, key]].

    The reference moves the same bytes through MicroKV (MicroKV/src/server.cpp:220-251,
    docs/v0.1/kv-cache-offload-v0.1-real-ops-design.md:293-312).  host_pool is
    [rows, row_bytes] uint8; slot_pool is [R, S, row_bytes] uint8 (returned copy).
    """
    out = slot_pool.copy()
    rr, pp = np.nonzero(install)
    keys = query[rr, pp]
    rows = record_addr[rr, keys]
    out[rr, slot[rr, pp]] = host_pool[rows]
    return out
