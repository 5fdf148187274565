"""Pin the CPU oracle against the reference's own outputs (tests/golden, made by make_golden.py)
and against the known-answer vectors of the reference's unit tests."""

import hashlib

import numpy as np
import pytest

from oracle import asu_oracle as O
from tests import cases as C


def digest(*arrays):
    h = hashlib.sha256()
    for a in arrays:
        a = np.ascontiguousarray(a)
        h.update(str(a.dtype).encode())
        h.update(str(a.shape).encode())
        h.update(a.tobytes())
    return h.hexdigest()


# ---------------------------------------------------------------- LRU simulator

def test_lru_reference_unit_vectors():
    """simu/test_kv_cache_eviction_sim.py:17-51 restated on the oracle pool."""
    p = O.LruPool(8, 0)
    first = p.resolve(list(range(4)))
    second = p.resolve(list(range(4)))
    assert first.hit.sum() == 0 and first.install.sum() == 4
    assert second.hit.sum() == 4 and second.install.sum() == 0

    p = O.LruPool(4, 2)
    p.resolve([1, 2, 3, 4])
    p.resolve([2])
    ev = p.prepare_free_slots()
    assert len(ev) == 2 and len(p.residents) == 2 and len(p.free) == 2
    assert set(p.residents) == {2, 4}
    assert ev == [1, 3]

    p = O.LruPool(1, 0)
    r = p.resolve([10, 11])
    assert r.hit.sum() == 0 and r.install.sum() == 1 and r.shortages == 1
    assert set(p.residents) == {10}


@pytest.mark.parametrize("name", ["a", "b", "c", "d"])
def test_lru_oracle_matches_reference_simulator(golden, name):
    g = golden("lru_small")
    slots, target, key_space, n, q = (int(v) for v in g[f"{name}_meta"])
    pool = O.LruPool(slots, target)
    for s in range(n):
        res = pool.step(g[f"{name}_query"][s])
        np.testing.assert_array_equal(res.slot, g[f"{name}_slot"][s])
        np.testing.assert_array_equal(res.hit, g[f"{name}_hit"][s])
        np.testing.assert_array_equal(res.install, g[f"{name}_install"][s])
        k = int(g[f"{name}_evicted_n"][s])
        np.testing.assert_array_equal(res.evicted, g[f"{name}_evicted"][s][:k])
    assert list(pool.residents.values()) == g[f"{name}_final_order"].tolist()
    assert list(pool.residents.keys()) == g[f"{name}_final_keys"].tolist()
    assert pool.free == g[f"{name}_final_free"].tolist()


def test_lru_oracle_matches_reference_on_c0_trace(golden):
    """Full c0 workload: 1 request, 131072 keys, 16384 slots, target 2048, 256 steps x 2048 ids."""
    from asu_ascend_b200.workloads import LocalityTrace

    g = golden("lru_c0")
    tr = LocalityTrace(1, 131072, topk=2048, reuse=0.7, zipf_s=1.1, seed=0)
    steps = [tr.step()[0] for _ in range(256)]
    assert digest(*steps) == str(g["trace_digest"][0])
    pool = O.LruPool(16384, 2048)
    for s, keys in enumerate(steps):
        res = pool.step(keys)
        assert digest(keys, res.slot, res.hit, res.install, res.evicted) == str(g["step_digest"][s]), s
    order = np.asarray(list(pool.residents.values()), np.int32)
    keys = np.asarray(list(pool.residents.keys()), np.int32)
    assert digest(order, keys, np.asarray(pool.free, np.int32)) == str(g["final_digest"][0])


def test_lru_oracle_matches_reference_workload_stats(golden):
    """run_simulation totals for the reference's own TopKWorkload traces (uniform/hotset/zipf/sliding)."""
    g = golden("lru_workloads")
    for i, wl in enumerate(("uniform", "hotset", "zipf", "sliding")):
        pool = O.LruPool(3072, 2048)
        tot = np.zeros(5, np.int64)
        for keys in g[f"trace_{wl}"]:
            res = pool.step(keys)
            tot += [res.hit.sum(), (~res.hit).sum(), res.install.sum(), res.shortages, len(res.evicted)]
        np.testing.assert_array_equal(tot, g["stats"][i])


# ---------------------------------------------------------------- ops contract

@pytest.mark.parametrize("pattern", ["hit", "miss", "mixed"])
def test_ops_lookup_oracle(golden, pattern):
    g = golden("ops")
    index, s2i, fs, fh, q = C.make_index_case(2, pattern)
    np.testing.assert_array_equal(q, g[f"lookup_{pattern}_query"])
    so, idx, s2i2, fh2 = O.ops_lookup_allocate(index, s2i, fs, fh, q)
    np.testing.assert_array_equal(so, g[f"lookup_{pattern}_slot_out"])
    np.testing.assert_array_equal(fh2, g[f"lookup_{pattern}_free_head"])
    np.testing.assert_array_equal(idx, C.apply_changes(index, g[f"lookup_{pattern}_index_idx"],
                                                       g[f"lookup_{pattern}_index_val"]))
    np.testing.assert_array_equal(s2i2, C.apply_changes(s2i, g[f"lookup_{pattern}_s2i_idx"],
                                                        g[f"lookup_{pattern}_s2i_val"]))


@pytest.mark.parametrize("ratio", [0.25, 1.0, 0.5])
def test_ops_maintain_oracle(golden, ratio):
    g = golden("ops")
    tag = f"maintain_{int(ratio * 100)}"
    index, s2i, fs, fh, lq = C.make_maintain_case(3, ratio)
    idx, s2i2, fs2, fh2 = O.ops_maintain(index, s2i, fs, fh, lq, int(g[f"{tag}_seed"][0]))
    np.testing.assert_array_equal(fs2, g[f"{tag}_free_slots"])
    np.testing.assert_array_equal(fh2, g[f"{tag}_free_head"])
    np.testing.assert_array_equal(idx, C.apply_changes(index, g[f"{tag}_index_idx"], g[f"{tag}_index_val"]))
    np.testing.assert_array_equal(s2i2, C.apply_changes(s2i, g[f"{tag}_s2i_idx"], g[f"{tag}_s2i_val"]))


def test_ops_chained_rounds_oracle(golden):
    g = golden("ops")
    index, s2i, fs, fh, _ = C.make_index_case(2, "hit")
    for k in range(3):
        q = g[f"chain{k}_query"]
        so, index, s2i, fh = O.ops_lookup_allocate(index, s2i, fs, fh, q)
        np.testing.assert_array_equal(so, g[f"chain{k}_slot_out"])
        np.testing.assert_array_equal(fh, g[f"chain{k}_head_after_lookup"])
        index, s2i, fs, fh = O.ops_maintain(index, s2i, fs, fh, so, int(g[f"chain{k}_seed"][0]))
        np.testing.assert_array_equal(fh, g[f"chain{k}_head_after_maintain"])
        np.testing.assert_array_equal(fs, g[f"chain{k}_free_slots"])
    assert digest(index, s2i) == str(g["chain_final_digest"][0])


# ---------------------------------------------------------------- batch LRU

def _simt_state(slot_tokens, cap=32):
    t2s = [O.NOT_FOUND] * cap
    for s, t in enumerate(slot_tokens):
        if t >= 0:
            t2s[t] = s
    return t2s, list(slot_tokens), list(range(len(slot_tokens)))


def test_batch_lru_reference_unit_vectors():
    """pta-ops/asu_hbm_index_lookup_simt/tests/test_reference.py:37-91 restated."""
    t2s, s2t, lru = _simt_state([0, 1, 2, 3])
    assert O.batch_lru([2, 0], t2s, s2t, lru) == ([2, 0], [False, False])
    assert lru == [1, 3, 0, 2] and s2t == [0, 1, 2, 3]

    t2s, s2t, lru = _simt_state([1, 4, 2, 5])
    assert O.batch_lru([4, 6, 7], t2s, s2t, lru) == ([1, 0, 2], [False, True, True])
    assert s2t == [6, 4, 7, 5] and t2s[1] == -1 and t2s[2] == -1 and t2s[6] == 0 and t2s[7] == 2
    assert lru == [3, 0, 2, 1]

    t2s, s2t, lru = _simt_state([0, 1, 2, 3])
    assert O.batch_lru([4, 4, -1, 1], t2s, s2t, lru) == ([0, 0, -1, 1], [True, False, False, False])
    assert s2t == [4, 1, 2, 3] and lru == [2, 3, 0, 1]

    t2s, s2t, lru = _simt_state([-1, -1, 2, 3])
    assert O.batch_lru([4, 3], t2s, s2t, lru) == ([0, 3], [True, False])
    assert s2t == [4, -1, 2, 3] and t2s[2] == 2 and lru == [1, 2, 0, 3]

    t2s, s2t, lru = _simt_state([0, 1, 2, 3])
    O.batch_lru([4, 1], t2s, s2t, lru)
    assert O.batch_lru([5, 4], t2s, s2t, lru) == ([2, 0], [True, False])


def test_batch_lru_oracle_matches_reference(golden):
    g = golden("batch_lru")
    for r in range(2):
        t2s, s2t, lru = C.simt_full_resident_state()
        t2s, s2t, lru = t2s.tolist(), s2t.tolist(), lru.astype(np.int32).tolist()
        for rnd in range(3):
            slots, mask = O.batch_lru(g[f"r{r}_q{rnd}"].tolist(), t2s, s2t, lru)
            np.testing.assert_array_equal(slots, g[f"r{r}_slot{rnd}"])
            np.testing.assert_array_equal(mask, g[f"r{r}_mask{rnd}"])
            np.testing.assert_array_equal(lru, g[f"r{r}_lru{rnd}"])
            np.testing.assert_array_equal(s2t, g[f"r{r}_s2t{rnd}"])
            assert digest(np.asarray(t2s, np.int32)) == str(g[f"r{r}_t2s_digest{rnd}"][0])


# ---------------------------------------------------------------- gather / update

@pytest.mark.parametrize("name,builder", [("single", C.gather_single_case), ("multi", C.gather_multi_case),
                                          ("dup", C.gather_dup_case)])
def test_gather_update_oracle(golden, name, builder):
    g = golden("gather")
    states, q, new, seed, pct = builder()
    out, _ = O.gather_lookup(states, q)
    np.testing.assert_array_equal(out.reshape(g[f"{name}_out"].shape), g[f"{name}_out"])
    st = O.random_update(states, q, new, seed, pct)
    np.testing.assert_array_equal(st, C.apply_changes(states, g[f"{name}_upd_idx"], g[f"{name}_upd_val"]))


def test_update_positions_oracle(golden):
    g = golden("gather")
    for key in g.files:
        if key.startswith("pos_"):
            _, n, seed, pct, r = key.split("_")
            assert O.update_positions(int(n), int(seed), int(pct), int(r)) == g[key].tolist()


# ---------------------------------------------------------------- resolver

def test_resolver_reference_unit_vectors():
    """patch/0001 tests/ut/ops/test_asu_kv_resolver.py (patch lines 672-765) restated."""
    kv0 = np.arange(16, dtype=np.float32).reshape(8, 2)
    kv1 = np.arange(24, dtype=np.float32).reshape(8, 3)
    m0 = np.full((4, 2), -1.0, np.float32)
    m1 = np.full((4, 3), -1.0, np.float32)
    ts = np.array([0, 0, 0, 0, 2, 2], np.int32)
    rec = np.array([0, 4, 0, 0, -1, -1], np.int32)
    hs = np.full(6, -1, np.int32)
    own = np.full(4, -1, np.int32)
    stack = np.array([0, 1, 2, 3], np.int32)
    cnt = np.array([4], np.int32)
    out = O.resolve_kv_slots_single_req(np.array([[[1, 1, 5]]], np.int32), 6, ts, rec, hs, own, stack, cnt,
                                        np.array([2, 0, 3], np.int32), kv0, kv1, m0, m1, 2)
    assert out.tolist() == [[[3, 3, 2]]]
    assert cnt[0] == 2
    assert ts.tolist() == [0, 1, 0, 0, 2, 1]
    assert hs.tolist() == [-1, 3, -1, -1, -1, 2]
    assert own.tolist() == [-1, -1, 5, 1]
    np.testing.assert_array_equal(m0[3], kv0[4])
    np.testing.assert_array_equal(m1[3], kv1[4])
    np.testing.assert_array_equal(m0[2], kv0[7])
    np.testing.assert_array_equal(m1[2], kv1[7])


def test_resolver_oracle_matches_reference(golden):
    g = golden("resolver")
    max_seq, slots, bs, actual, prefix = (int(v) for v in g["meta"])
    ts, rec, hs, own, stack, cnt = O.reset_state(max_seq, slots, bs, actual, prefix, g["block_table"])
    np.testing.assert_array_equal(ts, g["reset_token_state"])
    np.testing.assert_array_equal(rec, g["reset_record"])
    kv0, kv1 = g["kv0"], g["kv1"]
    m0 = np.zeros((slots,) + kv0.shape[1:], kv0.dtype)
    m1 = np.zeros((slots,) + kv1.shape[1:], kv1.dtype)
    for s in range(3):
        out = O.resolve_kv_slots_single_req(g[f"s{s}_topk"], actual, ts, rec, hs, own, stack, cnt,
                                            g["block_table"], kv0, kv1, m0, m1, bs)
        np.testing.assert_array_equal(out, g[f"s{s}_out"])
        np.testing.assert_array_equal(ts, g[f"s{s}_token_state"])
        np.testing.assert_array_equal(hs, g[f"s{s}_hbm_slot"])
        np.testing.assert_array_equal(own, g[f"s{s}_owner"])
        assert cnt[0] == g[f"s{s}_count"][0]
        assert digest(m0, m1) == str(g[f"s{s}_kv_digest"][0])


def test_resolver_errors_match_reference():
    """The reference raises on an empty free stack and on out-of-range tokens (patch lines 879-888, 993-994)."""
    args = dict(token_state=np.zeros(4, np.int32), asu_record_addr=np.zeros(4, np.int32),
                hbm_slot_of_token=np.full(4, -1, np.int32), slot_owner_token=np.full(1, -1, np.int32),
                free_slot_stack=np.zeros(1, np.int32), free_slot_count=np.array([1], np.int32),
                block_table=np.zeros(2, np.int32), kv0_src=np.zeros((4, 2)), kv1_src=np.zeros((4, 2)),
                kv0_dst=np.zeros((1, 2)), kv1_dst=np.zeros((1, 2)), block_size=2)
    with pytest.raises(O.ResolverError):
        O.resolve_kv_slots_single_req(np.array([0, 1]), 4, **args)
    with pytest.raises(O.ResolverError):
        O.resolve_kv_slots_single_req(np.array([5]), 4, **args)
