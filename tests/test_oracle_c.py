"""The C restatement (oracle/asu_oracle.c: the timed CPU baseline and the fast large-size
checker) against the Python oracle, which is pinned to the reference's outputs."""

import numpy as np
import pytest

from oracle import asu_oracle as O
from oracle import c_oracle as CO
from tests import cases as C


@pytest.mark.parametrize("name", ["a", "b", "c", "d"])
def test_c_lru_matches_reference_golden(golden, name):
    g = golden("lru_small")
    slots, target, key_space, n, q = (int(v) for v in g[f"{name}_meta"])
    pools = CO.LruPools(1, key_space, slots, target)
    for s in range(n):
        slot, hit, inst, ev, evn = pools.step_all(g[f"{name}_query"][s][None, :], threads=1)
        np.testing.assert_array_equal(slot[0], g[f"{name}_slot"][s])
        np.testing.assert_array_equal(hit[0], g[f"{name}_hit"][s])
        np.testing.assert_array_equal(inst[0], g[f"{name}_install"][s])
        k = int(g[f"{name}_evicted_n"][s])
        assert evn[0] == k
        np.testing.assert_array_equal(ev[0, :k], g[f"{name}_evicted"][s][:k])
    _, _, order, stack, cnt = pools.export(0)
    np.testing.assert_array_equal(order[: slots - cnt], g[f"{name}_final_order"])
    np.testing.assert_array_equal(stack[:cnt], g[f"{name}_final_free"])


def test_c_lru_multithreaded_matches_python_oracle_and_copies_rows():
    from asu_ascend_b200.workloads import LocalityTrace, record_addresses

    R, K, S, Q, tgt, row = 12, 8192, 1024, 256, 256, 32
    tr = LocalityTrace(R, K, topk=Q, seed=5)
    pools = CO.LruPools(R, K, S, tgt)
    ref = [O.LruPool(S, tgt) for _ in range(R)]
    rng = np.random.Generator(np.random.PCG64(1))
    host = rng.integers(0, 256, (500, row), dtype=np.uint8)
    rec = record_addresses(R, K, 500)
    slot_pool = np.zeros((R, S, row), np.uint8)
    expect = slot_pool.copy()
    for _ in range(8):
        q = tr.step()
        slot, hit, inst, ev, evn = pools.step_all(q, threads=4, host_pool=host, record=rec, slot_pool=slot_pool)
        for r in range(R):
            res = ref[r].step(q[r])
            np.testing.assert_array_equal(slot[r], res.slot)
            np.testing.assert_array_equal(hit[r], res.hit)
            np.testing.assert_array_equal(inst[r], res.install)
            np.testing.assert_array_equal(ev[r, : evn[r]], res.evicted)
        expect = O.swapin(host, rec, q, slot, inst, expect)
        np.testing.assert_array_equal(slot_pool, expect)
    for r in range(R):
        got = pools.export(r)
        exp = ref[r].export_state(K)
        for a, b in zip(got[:2], exp[:2]):
            np.testing.assert_array_equal(a, b)
        assert got[4] == exp[4]


def test_c_ops_and_gather_match_golden(golden):
    g = golden("ops")
    index, s2i, fs, fh, q = C.make_index_case(2, "mixed")
    so, *_ = CO.ops_lookup(index, s2i, fs, fh, q)
    np.testing.assert_array_equal(so, g["lookup_mixed_slot_out"])
    index, s2i, fs, fh, lq = C.make_maintain_case(3, 0.25)
    _, _, fs2, fh2, rc = CO.ops_maintain(index, s2i, fs, fh, lq, int(g["maintain_25_seed"][0]))
    assert rc == 0
    np.testing.assert_array_equal(fs2, g["maintain_25_free_slots"])
    np.testing.assert_array_equal(fh2, g["maintain_25_free_head"])
    states, qq, _, _, _ = C.gather_multi_case()
    out, _ = CO.gather_lookup(states, qq)
    np.testing.assert_array_equal(out, golden("gather")["multi_out"])
