"""The oracle of the resolver over an exact-LRU managed pool (asu_oracle.resolve_kv_slots_lru) is
the composition of two pinned oracles: the resolver of patch/0001 and the LRU pool of
simu/kv_cache_eviction_sim.py.  These CPU checks pin the composition to both:

* with a free target of 0 and a pool that never fills, it is the resolver, call for call;
* its hits, installs and evicted tokens are the LRU simulator's on the same token sequence,
  and the recency order holds the same tokens in the same order (slot numbers differ: the
  resolver pops a stack initialised 0..S-1 from the top, the simulator a list S-1..0);
* evicted prefix tokens return to ASU_ONLY with their record kept, evicted tail tokens to
  TAIL_HBM, and the rows of the installed tokens equal their source rows.
"""

import numpy as np

from oracle import asu_oracle as O


def _case(seed, max_seq=4096, slots=512, bs=16, actual=4000, prefix=3900, w0=6, w1=3):
    rng = np.random.Generator(np.random.PCG64(seed))
    nblk = max_seq // bs
    bt = rng.permutation(nblk + 8)[:nblk].astype(np.int32)
    st = list(O.reset_state(max_seq, slots, bs, actual, prefix, bt))
    src0 = rng.integers(0, 256, ((nblk + 8) * bs, w0), dtype=np.uint8)
    src1 = rng.integers(0, 256, ((nblk + 8) * bs, w1), dtype=np.uint8)
    return rng, bt, st, src0, src1


def test_lru_composition_without_eviction_is_the_resolver():
    rng, bt, st, src0, src1 = _case(1, slots=4096)
    ref = [a.copy() for a in st]
    order = np.full(4096, -1, np.int32)
    d0a, d1a = np.zeros((4096, 6), np.uint8), np.zeros((4096, 3), np.uint8)
    d0b, d1b = d0a.copy(), d1a.copy()
    for _ in range(4):
        topk = rng.integers(0, 4000, 300).astype(np.int32)
        got, ev = O.resolve_kv_slots_lru(topk, 4000, *st, order, 0, bt, src0, src1, d0a, d1a, 16)
        want = O.resolve_kv_slots_single_req(topk, 4000, *ref, bt, src0, src1, d0b, d1b, 16)
        np.testing.assert_array_equal(got, want)
        assert ev.size == 0
        for a, b in zip(st, ref):
            np.testing.assert_array_equal(a, b)
        np.testing.assert_array_equal(d0a, d0b)
        np.testing.assert_array_equal(d1a, d1b)


def test_lru_composition_follows_the_lru_simulator():
    slots, target = 512, 128
    rng, bt, st, src0, src1 = _case(2, slots=slots)
    ts, rec, hs, own, stack, cnt = st
    order = np.full(slots, -1, np.int32)
    d0, d1 = np.zeros((slots, 6), np.uint8), np.zeros((slots, 3), np.uint8)
    sim = O.LruPool(slots, target)
    hot = rng.integers(0, 4000, 700)
    for step in range(12):
        topk = np.where(rng.random(128) < 0.7, rng.choice(hot, 128), rng.integers(0, 4000, 128)).astype(np.int32)
        resident_before = ts == O.HBM_RESIDENT
        got, ev = O.resolve_kv_slots_lru(topk, 4000, ts, rec, hs, own, stack, cnt, order, target, bt, src0, src1,
                                         d0, d1, 16)
        res = sim.step(topk)
        np.testing.assert_array_equal(ev, res.evicted, err_msg=f"step {step}")
        # a position installs iff the simulator's position installs; the rest are hits
        installed = np.zeros(topk.size, bool)
        seen = set()
        for i, t in enumerate(topk):
            t = int(t)
            if t not in seen and not (resident_before[t] and t not in set(ev.tolist())):
                installed[i] = True
            seen.add(t)
        np.testing.assert_array_equal(installed, res.install, err_msg=f"step {step}")
        # recency order: the same tokens, least recently used first
        n_res = slots - int(cnt[0])
        np.testing.assert_array_equal(own[order[:n_res]], np.fromiter(sim.residents.keys(), np.int64),
                                      err_msg=f"step {step}")
        np.testing.assert_array_equal(hs[topk], got)
        assert (ts[topk] == O.HBM_RESIDENT).all()
    # every evicted token went back to its source state, its record kept
    gone = np.nonzero((ts != O.HBM_RESIDENT) & (np.arange(ts.size) < 4000))[0]
    assert (ts[gone[gone < 3900]] == O.ASU_ONLY).all() and (ts[gone[gone >= 3900]] == O.TAIL_HBM).all()
    assert (hs[gone] == O.INVALID).all()
    # resident rows equal their source rows
    for s in order[: slots - int(cnt[0])]:
        t = int(own[s])
        src = rec[t] if t < 3900 else bt[t // 16] * 16 + t % 16
        np.testing.assert_array_equal(d0[s], src0[src])
        np.testing.assert_array_equal(d1[s], src1[src])
