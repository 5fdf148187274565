"""GPU parity: every CUDA kernel, called through the C ABI (directly or via the torch ops),
against the oracle and the reference-generated golden vectors.  Bit-exact everywhere
(integer / index / byte work)."""

import ctypes
import hashlib

import numpy as np
import pytest
import torch

from oracle import asu_oracle as O
from tests import cases as C

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


@pytest.fixture(scope="module", autouse=True)
def _lib():
    import asu_ascend_b200

    asu_ascend_b200.load()
    from asu_ascend_b200 import ops

    ops.set_status_checks(True)
    yield
    ops.set_status_checks(False)


def T(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def N(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def digest(*arrays):
    h = hashlib.sha256()
    for a in arrays:
        a = np.ascontiguousarray(a)
        h.update(str(a.dtype).encode())
        h.update(str(a.shape).encode())
        h.update(a.tobytes())
    return h.hexdigest()


def stream_ptr():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


# ------------------------------------------------------------------ gather / update

@pytest.mark.parametrize("name,builder", [("single", C.gather_single_case), ("multi", C.gather_multi_case),
                                          ("dup", C.gather_dup_case)])
def test_gather_update_matches_golden(golden, name, builder):
    from asu_ascend_b200 import hbm_lookup_update as H

    g = golden("gather")
    states, q, new, seed, pct = builder()
    single = name == "single"
    st = T(states[0] if single else states)
    qq = T(q[0] if single else q)
    nn = T(new[0] if single else new)
    keys = torch.zeros_like(st)
    out = H.lookup_random_update(keys, st, qq, nn, seed=seed, update_percent=pct)
    np.testing.assert_array_equal(N(out).reshape(g[f"{name}_out"].shape), g[f"{name}_out"])
    exp_states = C.apply_changes(states, g[f"{name}_upd_idx"], g[f"{name}_upd_val"])
    np.testing.assert_array_equal(N(st).reshape(exp_states.shape), exp_states)
    # lookup_only on a fresh copy, update_only on another
    st2 = T(states[0] if single else states)
    out2 = H.lookup_only(keys, st2, qq)
    np.testing.assert_array_equal(N(out2).reshape(g[f"{name}_out"].shape), g[f"{name}_out"])
    H.update_only(keys, st2, qq, nn, seed=seed, update_percent=pct)
    np.testing.assert_array_equal(N(st2).reshape(exp_states.shape), exp_states)


def test_gather_padded_layout_of_the_c_launcher():
    """hbm_lookup_vec_do writes [req, align64(query_len)] rows with zero padding (kernel.cpp:104-131)."""
    from asu_ascend_b200._lib import lib

    states, q, _, _, _ = C.gather_multi_case()   # query_len 513 -> padded 576
    st, qq = T(states), T(q)
    out = torch.full((4, 576), 12345, dtype=torch.int32, device=DEV)
    assert lib.hbm_lookup_vec_do(8, stream_ptr(), None, st.data_ptr(), qq.data_ptr(), out.data_ptr(), 4, 513, -1) == 0
    o = N(out)
    exp, _ = O.gather_lookup(states, q)
    np.testing.assert_array_equal(o[:, :513], exp)
    assert (o[:, 513:] == 0).all()


def test_lookup_only_workload_full_size():
    """Lookup-only workload: 64 x 128K table (4096 resident), 64 x 2048 distinct queries, ~85% hits."""
    from asu_ascend_b200 import hbm_lookup_update as H
    from asu_ascend_b200.workloads import lookup_only_case

    table, query = lookup_only_case()
    out, hit = H.lookup(T(table), T(query))
    exp, exp_hit = O.gather_lookup(table, query)
    np.testing.assert_array_equal(N(out), exp)
    np.testing.assert_array_equal(N(hit), exp_hit)
    assert 0.8 < exp_hit.mean() < 0.9


@pytest.mark.parametrize("pct,dups", [(5, False), (100, False), (100, True)])
def test_lookup_random_update_full_size(pct, dups):
    """The gather + seeded random update on the lookup workload's full size (64 x 128K tables,
    64 x 2048 queries): the gathered values and the whole updated table against the oracle, at
    the benchmark's 5%, at 100% (every query position updated), and at 100% with duplicate query
    keys, where the last writer in update order must win."""
    from asu_ascend_b200 import hbm_lookup_update as H
    from asu_ascend_b200.workloads import lookup_only_case

    table, query = lookup_only_case()
    if dups:
        query = query.copy()
        query[:, 1::2] = query[:, 0::2]  # every key twice
    rng = np.random.Generator(np.random.PCG64(pct))
    new = rng.integers(0, 1 << 20, query.shape, dtype=np.int32)
    states = T(table)
    out = H.lookup_random_update(torch.zeros_like(states), states, T(query), T(new), seed=2026,
                                 update_percent=pct)
    exp_out, _ = O.gather_lookup(table, query)
    np.testing.assert_array_equal(N(out).reshape(exp_out.shape), exp_out)
    np.testing.assert_array_equal(N(states), O.random_update(table, query, new, 2026, pct))


def test_lookup_zero_copy_host_buffers():
    """Queries read from, results written to pinned host memory by the kernel itself."""
    from asu_ascend_b200 import hbm_lookup_update as H
    from asu_ascend_b200.workloads import lookup_only_case

    table, query = lookup_only_case(req_num=8)
    q_host = torch.from_numpy(query).pin_memory()
    out, hit = H.lookup(T(table), q_host)
    torch.cuda.synchronize()
    assert out.device.type == "cpu" and out.is_pinned() and hit.is_pinned()
    exp, exp_hit = O.gather_lookup(table, query)
    np.testing.assert_array_equal(out.numpy(), exp)
    np.testing.assert_array_equal(hit.numpy(), exp_hit)
    # mixed placement: device queries, host results
    out2 = torch.full(query.shape, 7, dtype=torch.int32).pin_memory()
    H.lookup(T(table), T(query), out=out2)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(out2.numpy(), exp)
    with pytest.raises(RuntimeError, match="pinned"):
        H.lookup(T(table), torch.from_numpy(query))  # pageable host memory is refused


def test_gather_out_of_range_keys_flag_status():
    from asu_ascend_b200 import hbm_lookup_update as H

    table = np.arange(64, dtype=np.int32).reshape(2, 32)
    q = np.array([[0, 31, 32, -1], [5, 99, 3, 2]], np.int32)
    status = torch.zeros(2, dtype=torch.int32, device=DEV)
    out, hit = H.lookup(T(table), T(q), status=status)
    assert N(out).tolist() == [[0, 31, -1, -1], [37, -1, 35, 34]]
    assert N(status).tolist() == [1, 1]


# ------------------------------------------------------------------ ops contract

@pytest.mark.parametrize("pattern", ["hit", "miss", "mixed"])
def test_ops_lookup_matches_golden(golden, pattern):
    g = golden("ops")
    index, s2i, fs, fh, q = C.make_index_case(2, pattern)
    ti, ts, tf, th, tq = T(index), T(s2i), T(fs), T(fh), T(q)
    slot_out = torch.ops._C_ascend.asu_hbm_index_lookup(ti, ts, tf, th, tq, 2)
    np.testing.assert_array_equal(N(slot_out), g[f"lookup_{pattern}_slot_out"])
    np.testing.assert_array_equal(N(th), g[f"lookup_{pattern}_free_head"])
    np.testing.assert_array_equal(N(ti), C.apply_changes(index, g[f"lookup_{pattern}_index_idx"],
                                                         g[f"lookup_{pattern}_index_val"]))
    np.testing.assert_array_equal(N(ts), C.apply_changes(s2i, g[f"lookup_{pattern}_s2i_idx"],
                                                         g[f"lookup_{pattern}_s2i_val"]))


def test_ops_lookup_through_reference_c_launcher(golden):
    """The ctypes call shape of ops/scripts/asu_hbm_index_common.py:319-331."""
    from asu_ascend_b200._lib import lib

    g = golden("ops")
    index, s2i, fs, fh, q = C.make_index_case(2, "mixed")
    ti, ts, tf, th, tq = T(index), T(s2i), T(fs), T(fh), T(q)
    so = torch.empty((2, C.QUERY_COUNT), dtype=torch.int32, device=DEV)
    rc = lib.asu_hbm_index_lookup_do(2, stream_ptr(), ti.data_ptr(), ts.data_ptr(), tf.data_ptr(), th.data_ptr(),
                                     tq.data_ptr(), so.data_ptr(), 2)
    assert rc == 0
    np.testing.assert_array_equal(N(so), g["lookup_mixed_slot_out"])
    np.testing.assert_array_equal(N(th), g["lookup_mixed_free_head"])


@pytest.mark.parametrize("ratio", [0.25, 1.0, 0.5])
def test_ops_maintain_matches_golden(golden, ratio):
    g = golden("ops")
    tag = f"maintain_{int(ratio * 100)}"
    index, s2i, fs, fh, lq = C.make_maintain_case(3, ratio)
    ti, ts, tf, th, tl = T(index), T(s2i), T(fs), T(fh), T(lq)
    torch.ops._C_ascend.asu_hbm_index_maintain(ti, ts, tf, th, tl, 3, int(g[f"{tag}_seed"][0]))
    np.testing.assert_array_equal(N(tf), g[f"{tag}_free_slots"])
    np.testing.assert_array_equal(N(th), g[f"{tag}_free_head"])
    np.testing.assert_array_equal(N(ti), C.apply_changes(index, g[f"{tag}_index_idx"], g[f"{tag}_index_val"]))
    np.testing.assert_array_equal(N(ts), C.apply_changes(s2i, g[f"{tag}_s2i_idx"], g[f"{tag}_s2i_val"]))


def test_ops_maintain_through_reference_c_launcher(golden):
    from asu_ascend_b200._lib import lib

    g = golden("ops")
    index, s2i, fs, fh, lq = C.make_maintain_case(3, 0.25)
    ti, ts, tf, th, tl = T(index), T(s2i), T(fs), T(fh), T(lq)
    rc = lib.asu_hbm_index_maintain_do(1, stream_ptr(), ti.data_ptr(), ts.data_ptr(), tf.data_ptr(), th.data_ptr(),
                                       tl.data_ptr(), 3, int(g["maintain_25_seed"][0]))
    assert rc == 0
    np.testing.assert_array_equal(N(tf), g["maintain_25_free_slots"])
    np.testing.assert_array_equal(N(th), g["maintain_25_free_head"])


def test_ops_chained_rounds_match_golden(golden):
    g = golden("ops")
    index, s2i, fs, fh, _ = C.make_index_case(2, "hit")
    ti, ts, tf, th = T(index), T(s2i), T(fs), T(fh)
    for k in range(3):
        so = torch.ops.asu.asu_hbm_index_lookup(ti, ts, tf, th, T(g[f"chain{k}_query"]), 2)
        np.testing.assert_array_equal(N(so), g[f"chain{k}_slot_out"])
        np.testing.assert_array_equal(N(th), g[f"chain{k}_head_after_lookup"])
        torch.ops.asu.asu_hbm_index_maintain(ti, ts, tf, th, so, 2, int(g[f"chain{k}_seed"][0]))
        np.testing.assert_array_equal(N(th), g[f"chain{k}_head_after_maintain"])
        np.testing.assert_array_equal(N(tf), g[f"chain{k}_free_slots"])
    assert digest(N(ti), N(ts)) == str(g["chain_final_digest"][0])


def test_ops_random_small_sizes_against_oracle():
    """Sized entry points on random small states with duplicates: 4 chained lookup -> maintain rounds."""
    rng = np.random.Generator(np.random.PCG64(3))
    R, IS, S, Q = 5, 300, 64, 40
    index = np.full((R, IS), -1, np.int32)
    s2i = np.full((R, S), -1, np.int32)
    for r in range(R):  # 48 residents in slots 0..47, free list 48..63
        keys = rng.choice(IS, 48, replace=False).astype(np.int32)
        index[r, keys] = np.arange(48, dtype=np.int32)
        s2i[r, :48] = keys
    fs = np.tile(np.arange(48, S, dtype=np.int32), (R, 1))
    fh = np.zeros(R, np.int32)
    ti, ts, tf, th = T(index), T(s2i), T(fs), T(fh)
    for rnd in range(4):
        q = np.empty((R, Q), np.int32)
        for r in range(R):
            resident = np.flatnonzero(index[r] >= 0)
            absent = np.setdiff1d(np.arange(IS), resident)
            miss = rng.choice(absent, 10, replace=False)
            row = rng.choice(np.concatenate([resident, miss]), Q)  # duplicates on purpose
            row[:10] = miss
            q[r] = rng.permutation(row)
        so_e, index, s2i, fh = O.ops_lookup_allocate(index, s2i, fs, fh, q)
        so = torch.ops.asu.asu_hbm_index_lookup(ti, ts, tf, th, T(q), R)
        np.testing.assert_array_equal(N(so), so_e)
        np.testing.assert_array_equal(N(ti), index)
        np.testing.assert_array_equal(N(ts), s2i)
        np.testing.assert_array_equal(N(th), fh)
        seed = int(rng.integers(0, 2**32))
        lq = so_e[:, : Q // 2].copy()  # protects <= 20 of >= 58 occupied slots: the ring always terminates
        index, s2i, fs, fh = O.ops_maintain(index, s2i, fs, fh, lq, seed)
        torch.ops.asu.asu_hbm_index_maintain(ti, ts, tf, th, T(lq), R, seed)
        np.testing.assert_array_equal(N(ti), index)
        np.testing.assert_array_equal(N(ts), s2i)
        np.testing.assert_array_equal(N(tf), fs)
        np.testing.assert_array_equal(N(th), fh)


def test_ops_error_status_instead_of_undefined_behaviour():
    """With status checks on, the C++ ops raise RuntimeError naming the status bits."""
    index = np.full((1, 16), -1, np.int32)
    s2i = np.full((1, 8), -1, np.int32)
    fs = np.array([[4, 5]], np.int32)
    # free list overrun: 3 misses, 2 free entries
    with pytest.raises(RuntimeError, match="FREE_EXHAUSTED"):
        torch.ops.asu.asu_hbm_index_lookup(T(index), T(s2i), T(fs), T(np.zeros(1, np.int32)),
                                           T(np.array([[1, 2, 3]], np.int32)), 1)
    # maintain with nothing evictable: the reference would spin forever
    with pytest.raises(RuntimeError, match="RING_EXHAUSTED"):
        torch.ops.asu.asu_hbm_index_maintain(T(index), T(s2i), T(np.zeros((1, 2), np.int32)),
                                             T(np.array([1], np.int32)), T(np.zeros((1, 2), np.int32)), 1, 0)
    # out-of-range query id
    with pytest.raises(RuntimeError, match="BAD_QUERY"):
        torch.ops.asu.asu_hbm_index_lookup(T(index), T(s2i), T(np.array([[4, 5, 6]], np.int32)),
                                           T(np.zeros(1, np.int32)), T(np.array([[16]], np.int32)), 1)


# ------------------------------------------------------------------ batch LRU

def _simt_state(slot_tokens, cap=32):
    t2s = np.full((1, cap), -1, np.int32)
    for s, t in enumerate(slot_tokens):
        if t >= 0:
            t2s[0, t] = s
    return t2s, np.asarray([slot_tokens], np.int32), np.arange(len(slot_tokens), dtype=np.int16)[None, :]


@pytest.mark.parametrize("slots,query,exp_slots,exp_mask,exp_lru,exp_s2t", [
    ([0, 1, 2, 3], [2, 0], [2, 0], [False, False], [1, 3, 0, 2], [0, 1, 2, 3]),
    ([1, 4, 2, 5], [4, 6, 7], [1, 0, 2], [False, True, True], [3, 0, 2, 1], [6, 4, 7, 5]),
    ([0, 1, 2, 3], [4, 4, -1, 1], [0, 0, -1, 1], [True, False, False, False], [2, 3, 0, 1], [4, 1, 2, 3]),
    ([-1, -1, 2, 3], [4, 3], [0, 3], [True, False], [1, 2, 0, 3], [4, -1, 2, 3]),
])
def test_batch_lru_reference_unit_vectors(slots, query, exp_slots, exp_mask, exp_lru, exp_s2t):
    """pta-ops/asu_hbm_index_lookup_simt/tests/test_reference.py:37-80 on the GPU kernel."""
    t2s, s2t, lru = _simt_state(slots)
    tt, ts, tl = T(t2s), T(s2t), T(lru)
    sid, mask = torch.ops._C_ascend.asu_hbm_index_lookup_simt(tt, ts, tl, T(np.asarray([query], np.int32)), 1)
    assert N(sid)[0].tolist() == exp_slots
    assert N(mask)[0].tolist() == exp_mask
    assert N(tl)[0].tolist() == exp_lru
    assert N(ts)[0].tolist() == exp_s2t


def test_batch_lru_matches_golden_full_size(golden):
    g = golden("batch_lru")
    R = 2
    t2s, s2t, lru = C.simt_full_resident_state()
    tt, ts, tl = T(np.stack([t2s] * R)), T(np.stack([s2t] * R)), T(np.stack([lru] * R))
    for rnd in range(3):
        q = np.stack([g[f"r{r}_q{rnd}"] for r in range(R)])
        sid, mask = torch.ops.asu.asu_hbm_index_lookup_simt(tt, ts, tl, T(q), R)
        for r in range(R):
            np.testing.assert_array_equal(N(sid)[r], g[f"r{r}_slot{rnd}"])
            np.testing.assert_array_equal(N(mask)[r], g[f"r{r}_mask{rnd}"])
            np.testing.assert_array_equal(N(tl)[r], g[f"r{r}_lru{rnd}"])
            np.testing.assert_array_equal(N(ts)[r], g[f"r{r}_s2t{rnd}"])
            assert digest(N(tt)[r]) == str(g[f"r{r}_t2s_digest{rnd}"][0])


def test_batch_lru_through_reference_c_launcher():
    from asu_ascend_b200._lib import lib

    t2s, s2t, lru = (np.stack([a]) for a in C.simt_full_resident_state())
    q = (np.arange(C.QUERY_COUNT, dtype=np.int32)[None, :] * 3) % (C.SLOT_COUNT * 2)
    tt, ts, tl, tq = T(t2s), T(s2t), T(lru), T(q)
    sid = torch.empty((1, C.QUERY_COUNT), dtype=torch.int32, device=DEV)
    mask = torch.empty((1, C.QUERY_COUNT), dtype=torch.bool, device=DEV)
    ws = torch.empty(31492, dtype=torch.int32, device=DEV)
    assert lib.asu_hbm_index_lookup_simt_do(stream_ptr(), tt.data_ptr(), ts.data_ptr(), tl.data_ptr(), tq.data_ptr(),
                                            sid.data_ptr(), mask.data_ptr(), ws.data_ptr(), 1) == 0
    e_t2s, e_s2t, e_lru = t2s[0].tolist(), s2t[0].tolist(), lru[0].astype(np.int32).tolist()
    es, em = O.batch_lru(q[0].tolist(), e_t2s, e_s2t, e_lru)
    np.testing.assert_array_equal(N(sid)[0], es)
    np.testing.assert_array_equal(N(mask)[0], em)
    np.testing.assert_array_equal(N(tl)[0], e_lru)


@pytest.mark.parametrize("S,Q,R", [(37, 5, 3), (1000, 300, 4), (4100, 2048, 2), (10240, 1536, 5)])
def test_batch_lru_random_states_against_oracle(S, Q, R):
    """Slot counts from 37 to 10240 (every thread-work shape of the kernel), partly empty slot
    tables, queries with duplicates, -1 and out-of-range ids, four rounds per request."""
    rng = np.random.Generator(np.random.PCG64(S * 7 + Q))
    K = 3 * S
    t2s = np.full((R, K), -1, np.int32)
    s2t = np.full((R, S), -1, np.int32)
    lru = np.empty((R, S), np.int16)
    for r in range(R):
        resident = rng.choice(K, int(S * 0.8), replace=False)
        slots = rng.choice(S, len(resident), replace=False)
        t2s[r, resident] = slots
        s2t[r, slots] = resident
        lru[r] = rng.permutation(S).astype(np.int16)
    tt, ts, tl = T(t2s), T(s2t), T(lru)
    state = [[t2s[r].tolist(), s2t[r].tolist(), lru[r].astype(np.int32).tolist()] for r in range(R)]
    for _ in range(4):
        q = np.empty((R, Q), np.int32)
        for r in range(R):
            res = [t for t, sl in enumerate(state[r][0]) if sl >= 0]
            # at most S // 4 distinct misses: always enough victims
            pool = np.concatenate([rng.choice(res, Q), rng.integers(0, K, max(1, S // 8))])
            q[r] = rng.choice(pool, Q)
            q[r, rng.random(Q) < 0.02] = -1
            q[r, rng.random(Q) < 0.01] = K + 5
        sid, mask = torch.ops.asu.asu_hbm_index_lookup_simt(tt, ts, tl, T(q), R)
        for r in range(R):
            es, em = O.batch_lru(q[r].tolist(), *state[r])
            np.testing.assert_array_equal(N(sid)[r], es)
            np.testing.assert_array_equal(N(mask)[r], em)
            np.testing.assert_array_equal(N(tt)[r], state[r][0])
            np.testing.assert_array_equal(N(ts)[r], state[r][1])
            np.testing.assert_array_equal(N(tl)[r].astype(np.int32), state[r][2])


def test_batch_lru_reference_benchmark_case_64_requests():
    """The SIMT harness's benchmark case at its largest batch: 64 requests, every one of the 10240
    slots resident, 1536 hits and 512 misses of 2048 per request, two rounds (the second on the
    state the first left); every request's outputs and state against the oracle."""
    from asu_ascend_b200.workloads import simt_case

    t2s, s2t, lru, q = simt_case(64, 1536, seed=64)
    tt, ts, tl = T(t2s), T(s2t), T(lru)
    state = [[t2s[r].tolist(), s2t[r].tolist(), lru[r].astype(np.int32).tolist()] for r in range(64)]
    rng = np.random.Generator(np.random.PCG64(65))
    for rnd in range(2):
        if rnd:  # second round: half of the first round's ids again, half fresh
            q = np.stack([np.concatenate([rng.choice(q[r], 1024, replace=False),
                                          rng.choice(131072, 1024, replace=False)]).astype(np.int32)
                          for r in range(64)])
        sid, mask = torch.ops.asu.asu_hbm_index_lookup_simt(tt, ts, tl, T(q), 64)
        for r in range(64):
            es, em = O.batch_lru(q[r].tolist(), *state[r])
            np.testing.assert_array_equal(N(sid)[r], es)
            np.testing.assert_array_equal(N(mask)[r], em)
        np.testing.assert_array_equal(N(ts), np.asarray([st[1] for st in state], np.int32))
        np.testing.assert_array_equal(N(tl).astype(np.int32), np.asarray([st[2] for st in state], np.int32))
        for r in (0, 31, 63):
            np.testing.assert_array_equal(N(tt)[r], state[r][0])


def test_batch_lru_no_victim_leaves_state_unchanged():
    t2s, s2t, lru = _simt_state([0, 1, 2, 3])
    tt, ts, tl = T(t2s), T(s2t), T(lru)
    with pytest.raises(RuntimeError, match="NO_VICTIM"):  # 2 hits + 3 misses on 4 slots
        torch.ops.asu.asu_hbm_index_lookup_simt(tt, ts, tl, T(np.asarray([[0, 1, 9, 10, 11]], np.int32)), 1)
    np.testing.assert_array_equal(N(tt), t2s)
    np.testing.assert_array_equal(N(ts), s2t)
    np.testing.assert_array_equal(N(tl), lru)


# ------------------------------------------------------------------ exact LRU

def _lru_run_and_compare(pools, oracle_pools, steps, check_state_every=1):
    R = len(oracle_pools)
    for i, q in enumerate(steps):
        out = pools.step(T(q))
        slot, hit, inst = N(out.slot), N(out.hit), N(out.install)
        ev, evn = N(out.evicted), N(out.evicted_count)
        for r in range(R):
            res = oracle_pools[r].step(q[r])
            np.testing.assert_array_equal(slot[r], res.slot, err_msg=f"step {i} req {r} slot")
            np.testing.assert_array_equal(hit[r], res.hit, err_msg=f"step {i} req {r} hit")
            np.testing.assert_array_equal(inst[r], res.install, err_msg=f"step {i} req {r} install")
            assert evn[r] == len(res.evicted)
            np.testing.assert_array_equal(ev[r, : evn[r]], res.evicted, err_msg=f"step {i} req {r} evicted")
        if check_state_every and (i % check_state_every == 0 or i == len(steps) - 1):
            t2s, s2t, order, stack, count = (N(x) for x in (pools.token_to_slot, pools.slot_to_token,
                                                             pools.lru_order, pools.free_stack, pools.free_count))
            for r in range(R):
                et2s, es2t, eorder, estack, ecount = oracle_pools[r].export_state(pools.key_space)
                assert count[r] == ecount
                np.testing.assert_array_equal(t2s[r], et2s)
                np.testing.assert_array_equal(s2t[r], es2t)
                nres = pools.slot_count - ecount
                np.testing.assert_array_equal(order[r, :nres], eorder[:nres])
                np.testing.assert_array_equal(stack[r, :ecount], estack[:ecount])
    pools.check_status()


@pytest.mark.parametrize("name", ["a", "b", "c", "d"])
def test_lru_matches_reference_simulator_golden(golden, name):
    from asu_ascend_b200.lru import LruSlotPools

    g = golden("lru_small")
    slots, target, key_space, n, q = (int(v) for v in g[f"{name}_meta"])
    pools = LruSlotPools(1, key_space, slots, target, q, device=DEV)
    for s in range(n):
        out = pools.step(T(g[f"{name}_query"][s][None, :]))
        np.testing.assert_array_equal(N(out.slot)[0], g[f"{name}_slot"][s])
        np.testing.assert_array_equal(N(out.hit)[0], g[f"{name}_hit"][s])
        np.testing.assert_array_equal(N(out.install)[0], g[f"{name}_install"][s])
        k = int(g[f"{name}_evicted_n"][s])
        assert int(N(out.evicted_count)[0]) == k
        np.testing.assert_array_equal(N(out.evicted)[0][:k], g[f"{name}_evicted"][s][:k])
    cnt = int(N(pools.free_count)[0])
    np.testing.assert_array_equal(N(pools.lru_order)[0][: slots - cnt], g[f"{name}_final_order"])
    np.testing.assert_array_equal(N(pools.free_stack)[0][:cnt], g[f"{name}_final_free"])


def test_lru_matches_reference_on_c0_full_trace(golden):
    """1 request, 131072 keys, 16384 slots, target 2048, 256 steps x 2048 ids: per-step digests."""
    from asu_ascend_b200.lru import LruSlotPools
    from asu_ascend_b200.workloads import LocalityTrace

    g = golden("lru_c0")
    tr = LocalityTrace(1, 131072, topk=2048, reuse=0.7, zipf_s=1.1, seed=0)
    steps = [tr.step() for _ in range(256)]
    pools = LruSlotPools(1, 131072, 16384, 2048, 2048, device=DEV)
    for s, q in enumerate(steps):
        out = pools.step(T(q))
        k = int(N(out.evicted_count)[0])
        d = digest(q[0], N(out.slot)[0], N(out.hit)[0], N(out.install)[0], N(out.evicted)[0][:k])
        assert d == str(g["step_digest"][s]), f"step {s}"
    cnt = int(N(pools.free_count)[0])
    order = N(pools.lru_order)[0][: 16384 - cnt]
    keys = N(pools.slot_to_token)[0][order]
    assert digest(order, keys, N(pools.free_stack)[0][:cnt]) == str(g["final_digest"][0])


def test_lru_many_requests_against_oracle():
    """16 independent requests (one pool each) with duplicates and shortages, full state compared."""
    from asu_ascend_b200.lru import LruSlotPools

    rng = np.random.Generator(np.random.PCG64(11))
    R, K, S, Q, tgt = 16, 3000, 300, 160, 64
    pools = LruSlotPools(R, K, S, tgt, Q, device=DEV)
    oracle = [O.LruPool(S, tgt) for _ in range(R)]
    steps = []
    hot = rng.integers(0, K, (R, 400))
    for _ in range(30):
        q = np.empty((R, Q), np.int32)
        for r in range(R):
            q[r] = np.where(rng.random(Q) < 0.7, rng.choice(hot[r], Q), rng.integers(0, K, Q))
        steps.append(q)
    _lru_run_and_compare(pools, oracle, steps, check_state_every=5)


@pytest.mark.parametrize("S,Q", [(4096, 4096), (16384, 3000), (1023, 333), (5001, 2049)])
def test_lru_kernel_shapes_against_oracle(S, Q):
    """Every thread-work shape of the kernel: 2 or 4 queries and 2 to 16 order entries per
    thread, the 16384-slot / 4096-query maxima, and slot and query counts that are not
    multiples of 4 (the order row then moves with 4-byte accesses); duplicates, evictions and
    shortages on the way."""
    from asu_ascend_b200.lru import LruSlotPools

    rng = np.random.Generator(np.random.PCG64(S + Q))
    R, K = 3, 40000
    tgt = S // 4
    pools = LruSlotPools(R, K, S, tgt, Q, device=DEV)
    oracle = [O.LruPool(S, tgt) for _ in range(R)]
    hot = rng.integers(0, K, (R, 2 * S))
    steps = []
    for _ in range(8):
        q = np.empty((R, Q), np.int32)
        for r in range(R):
            q[r] = np.where(rng.random(Q) < 0.8, rng.choice(hot[r], Q), rng.integers(0, K, Q))
        steps.append(q)
    _lru_run_and_compare(pools, oracle, steps, check_state_every=3)


def test_lru_stress_shape_against_oracle():
    """The stress configuration's shape -- a 1M-token key space, 8192 slots, target 2048, uniform
    top-k 2048 with 20% reuse (~80% misses) -- on 8 requests, full state against the oracle."""
    from asu_ascend_b200.lru import LruSlotPools
    from asu_ascend_b200.workloads import FastLocalityTrace

    R, K = 8, 1 << 20
    tr = FastLocalityTrace(R, K, topk=2048, reuse=0.2, zipf_s=None, seed=77)
    steps = [tr.step() for _ in range(6)]
    pools = LruSlotPools(R, K, 8192, 2048, 2048, device=DEV)
    oracle = [O.LruPool(8192, 2048) for _ in range(R)]
    _lru_run_and_compare(pools, oracle, steps, check_state_every=5)


def _c_oracle_compare_step(out, res, tag):
    """One step of every request: GPU outputs against the C oracle's (slot, hit, install,
    evicted ids and counts)."""
    slot, hit, inst, ev, evn = res
    np.testing.assert_array_equal(N(out.slot), slot, err_msg=f"{tag} slot")
    np.testing.assert_array_equal(N(out.hit), hit, err_msg=f"{tag} hit")
    np.testing.assert_array_equal(N(out.install), inst, err_msg=f"{tag} install")
    gev, gevn = N(out.evicted), N(out.evicted_count)
    np.testing.assert_array_equal(gevn, evn, err_msg=f"{tag} evicted count")
    for r in range(gevn.shape[0]):
        np.testing.assert_array_equal(gev[r, : gevn[r]], ev[r, : evn[r]], err_msg=f"{tag} req {r} evicted")


def _c_oracle_compare_state(pools, cpools, tag):
    """Final state of every request against the C oracle: slot_to_token, the resident part of
    the order row, the free part of the stack and the free count.  token_to_slot is checked as
    the inverse of slot_to_token (every resident key maps back to its slot and no other key
    maps anywhere), which with slot_to_token equal to the oracle's makes it equal too, without
    copying the whole [R, key_space] table back."""
    S = pools.slot_count
    s2t, order, stack, count = (N(x) for x in (pools.slot_to_token, pools.lru_order, pools.free_stack,
                                               pools.free_count))
    for r in range(pools.req_num):
        _, es2t, eorder, estack, ecount = cpools.export(r)
        assert count[r] == ecount, f"{tag} req {r} free count"
        np.testing.assert_array_equal(s2t[r], es2t, err_msg=f"{tag} req {r} slot_to_token")
        np.testing.assert_array_equal(order[r, : S - ecount], eorder[: S - ecount], err_msg=f"{tag} req {r} order")
        np.testing.assert_array_equal(stack[r, :ecount], estack[:ecount], err_msg=f"{tag} req {r} free stack")
    gs2t = pools.slot_to_token
    rows, slots = torch.nonzero(gs2t >= 0, as_tuple=True)
    assert torch.equal(pools.token_to_slot[rows, gs2t[rows, slots].long()], slots.int()), tag
    assert int((pools.token_to_slot >= 0).sum()) == rows.numel(), tag


def test_lru_full_stress_size_against_c_oracle():
    """The full stress size (128 requests, 1M-token key space, 8192 slots, target 2048, uniform
    top-k 2048 with 20% reuse, ~80% misses): every request against the multi-threaded C oracle
    for six steps -- per-step outputs and evicted ids, final state -- plus, after every step,
    the map invariants that need no oracle (maps inverse to each other, the order row holding
    exactly the resident slots and the free stack the others, installs to distinct slots)."""
    from asu_ascend_b200.lru import LruSlotPools
    from asu_ascend_b200.workloads import FastLocalityTrace
    from oracle import c_oracle as CO

    R, K, S = 128, 1 << 20, 8192
    tr = FastLocalityTrace(R, K, topk=2048, reuse=0.2, zipf_s=None, seed=78)
    pools = LruSlotPools(R, K, S, 2048, 2048, device=DEV)
    cpools = CO.LruPools(R, K, S, 2048)
    ar = torch.arange(S, device=DEV)
    for step in range(6):
        q = tr.step()
        out = pools.step(T(q))
        _c_oracle_compare_step(out, cpools.step_all(q), f"step {step}")
        free = pools.free_count.long()
        s2t = pools.slot_to_token
        resident = s2t >= 0
        assert torch.equal(resident.sum(1), S - free)
        order_ok = ar[None, :] < (S - free)[:, None]
        ordered = torch.where(order_ok, pools.lru_order, torch.full_like(pools.lru_order, -1))
        marks = torch.zeros((R, S), dtype=torch.int32, device=DEV)
        marks.scatter_add_(1, ordered.clamp(min=0).long(), order_ok.int())
        assert torch.equal(marks > 0, resident) and int(marks.max()) <= 1
        stack_ok = ar[None, :] < free[:, None]
        fmarks = torch.zeros((R, S), dtype=torch.int32, device=DEV)
        fmarks.scatter_add_(1, pools.free_stack.clamp(min=0).long(), stack_ok.int())
        assert torch.equal(fmarks > 0, ~resident) and int(fmarks.max()) <= 1
        inst = out.install
        islots = torch.where(inst, out.slot, torch.full_like(out.slot, -1))
        imarks = torch.zeros((R, S), dtype=torch.int32, device=DEV)
        imarks.scatter_add_(1, islots.clamp(min=0).long(), inst.int())
        assert int(imarks.max()) <= 1
    _c_oracle_compare_state(pools, cpools, "stress final")
    pools.check_status()
    cpools.close()


def test_lru_multilayer_1024_requests_4_layers_against_c_oracle():
    """The request-sharded configuration's batch on one GPU: 1024 requests (several waves of
    CTAs), 4 layers with independent top-k sets, each (layer, request) with its own 8192-slot
    pool over 131072 tokens, top-k 2048, target 2048.  Every (layer, request) against the C
    oracle for four steps: per-step outputs and evicted ids, then the final state."""
    from asu_ascend_b200.lru import LruSlotPools
    from asu_ascend_b200.workloads import FastLocalityTrace
    from oracle import c_oracle as CO

    R, K, S, L = 1024, 131072, 8192, 4
    traces = [FastLocalityTrace(R, K, topk=2048, seed=79 + 7919 * layer) for layer in range(L)]
    pools = [LruSlotPools(R, K, S, 2048, 2048, device=DEV) for _ in range(L)]
    cpools = [CO.LruPools(R, K, S, 2048) for _ in range(L)]
    for step in range(4):
        for layer in range(L):
            q = traces[layer].step()
            out = pools[layer].step(T(q))
            _c_oracle_compare_step(out, cpools[layer].step_all(q), f"step {step} layer {layer}")
    for layer in range(L):
        _c_oracle_compare_state(pools[layer], cpools[layer], f"layer {layer} final")
        pools[layer].check_status()
        cpools[layer].close()


def test_lru_c2_shape_against_oracle():
    """128 requests, 128K keys, 8192 slots, target 2048, top-k 2048 with c0 locality: 6 steps."""
    from asu_ascend_b200.lru import LruSlotPools
    from asu_ascend_b200.workloads import LocalityTrace

    R = 128
    tr = LocalityTrace(R, 131072, topk=2048, seed=42)
    steps = [tr.step() for _ in range(6)]
    pools = LruSlotPools(R, 131072, 8192, 2048, 2048, device=DEV)
    oracle = [O.LruPool(8192, 2048) for _ in range(R)]
    _lru_run_and_compare(pools, oracle, steps, check_state_every=0)


def test_lru_invalid_keys_and_shortage_status():
    from asu_ascend_b200._lib import AsuError
    from asu_ascend_b200.lru import LruSlotPools

    pools = LruSlotPools(1, 10, 2, 0, 4, device=DEV)
    out = pools.step(T(np.array([[1, 2, 3, 1]], np.int32)))
    assert N(out.slot)[0].tolist() == [0, 1, -1, 0]
    assert N(out.hit)[0].tolist() == [False, False, False, True]
    pools.check_status()  # shortage alone is not an error
    assert pools.totals() == {"hits": 1, "misses": 3, "installs": 2, "shortages": 1, "evictions": 0}
    pools.step(T(np.array([[1, 12, -4, 2]], np.int32)))
    with pytest.raises(AsuError, match="BAD_QUERY"):
        pools.check_status()


# ------------------------------------------------------------------ swap-in

@pytest.mark.parametrize("row_bytes,R,S,Q", [(656, 16, 512, 256), (41984, 4, 16, 8)])
def test_swapin_bytes_exact(row_bytes, R, S, Q):
    from asu_ascend_b200.host_pool import HostRowPool, check_status
    from asu_ascend_b200.lru import LruSlotPools
    from asu_ascend_b200.workloads import LocalityTrace, record_addresses

    K = 4096
    pool = HostRowPool(rows=1000, row_bytes=row_bytes)
    pool.fill_random(7)
    rec = record_addresses(R, K, pool.rows)
    tr = LocalityTrace(R, K, topk=Q, seed=3)
    lru = LruSlotPools(R, K, S, Q // 4, Q, device=DEV)
    slot_pool = torch.zeros((R, S, row_bytes), dtype=torch.uint8, device=DEV)
    expect = np.zeros((R, S, row_bytes), np.uint8)
    trec = T(rec)
    status = torch.zeros(R, dtype=torch.int32, device=DEV)
    for _ in range(5):
        q = tr.step()
        tq = T(q)
        out = lru.step(tq)
        pool.swapin(trec, tq, out.slot, out.install, slot_pool, status=status)
        expect = O.swapin(pool.array, rec, q, N(out.slot), N(out.install), expect)
        np.testing.assert_array_equal(N(slot_pool), expect)
    check_status(status, "swapin")
    pool.close()


def test_swapin_full_resolver_workload_bytes():
    """The default benchmark configuration at full size -- 128 requests, 131072 tokens, 8192
    slots, top-k 2048 with reuse + Zipf locality, 656-byte rows in a 2^20-row pinned pool at the
    768-byte pitch: after each of four steps every row installed in that step equals its host
    record byte for byte, and so does a sample of every request's resident rows."""
    from asu_ascend_b200.host_pool import HostRowPool, check_status
    from asu_ascend_b200.lru import LruSlotPools
    from asu_ascend_b200.workloads import LocalityTrace, record_addresses_torch

    R, K, S, Q, row = 128, 131072, 8192, 2048, 656
    pool = HostRowPool(rows=1 << 20, row_bytes=row)
    pool.fill_random(13)
    host = pool.tensor  # CPU view of the pinned rows
    rec = record_addresses_torch(R, K, pool.rows, DEV)
    tr = LocalityTrace(R, K, topk=Q, seed=15)
    lru = LruSlotPools(R, K, S, 2048, Q, device=DEV)
    kv = torch.zeros((R, S, row), dtype=torch.uint8, device=DEV)
    status = torch.zeros(R, dtype=torch.int32, device=DEV)
    g = torch.Generator().manual_seed(3)
    for _ in range(4):
        q = T(tr.step())
        out = lru.step(q)
        pool.swapin(rec, q, out.slot, out.install, kv, status=status)
        torch.cuda.synchronize()
        r_i, p_i = torch.nonzero(out.install, as_tuple=True)
        src = rec[r_i, q[r_i, p_i].long()].long()
        assert r_i.numel() > 0
        np.testing.assert_array_equal(N(kv[r_i, out.slot[r_i, p_i].long()]), host[src.cpu()].numpy())
        # a sample of resident rows of every request: slot s holds the record of slot_to_token[r, s]
        s_pick = torch.randint(0, S, (R, 64), generator=g).to(DEV)
        tok = lru.slot_to_token.gather(1, s_pick)
        ok = tok >= 0
        rr = torch.arange(R, device=DEV)[:, None].expand(R, 64)[ok]
        srcs = rec[rr, tok[ok].long()].long()
        np.testing.assert_array_equal(N(kv[rr, s_pick[ok]]), host[srcs.cpu()].numpy())
    check_status(status, "swapin")
    lru.check_status()
    pool.close()


def test_swapin_full_stress_block_bytes():
    """The block-granular stress configuration at full size: 128 requests, 16384 blocks of 64
    tokens, 128 block slots, top-k 32 blocks with 20% reuse, 41,984-byte block rows (the 16-byte
    load swap-in kernel) in a 16384-row pinned pool: every block installed in each of four steps
    equals its host record byte for byte."""
    from asu_ascend_b200.host_pool import HostRowPool, check_status
    from asu_ascend_b200.lru import LruSlotPools
    from asu_ascend_b200.workloads import FastLocalityTrace, record_addresses_torch

    R, K, S, Q, row = 128, 16384, 128, 32, 41984
    pool = HostRowPool(rows=16384, row_bytes=row)
    pool.fill_random(17)
    host = pool.tensor
    rec = record_addresses_torch(R, K, pool.rows, DEV)
    tr = FastLocalityTrace(R, K, topk=Q, reuse=0.2, zipf_s=None, seed=19)
    lru = LruSlotPools(R, K, S, Q, Q, device=DEV)
    kv = torch.zeros((R, S, row), dtype=torch.uint8, device=DEV)
    status = torch.zeros(R, dtype=torch.int32, device=DEV)
    for _ in range(4):
        q = T(tr.step())
        out = lru.step(q)
        pool.swapin(rec, q, out.slot, out.install, kv, status=status)
        torch.cuda.synchronize()
        r_i, p_i = torch.nonzero(out.install, as_tuple=True)
        assert r_i.numel() > 0
        src = rec[r_i, q[r_i, p_i].long()].long()
        np.testing.assert_array_equal(N(kv[r_i, out.slot[r_i, p_i].long()]), host[src.cpu()].numpy())
    check_status(status, "swapin")
    lru.check_status()
    pool.close()


@pytest.mark.parametrize("row_bytes,pitch", [(656, None), (656, 656), (64, None), (1024, None), (2048, None)])
def test_swapin_direct_masks_errors_and_pitches(row_bytes, pitch):
    """The swap-in alone, on hand-made install masks: query counts that are not multiples of
    32, installs into arbitrary slots, both kernels (bulk copies up to 1 KiB rows, 16-byte
    loads above), packed and padded host rows, and out-of-range keys / slots / record rows,
    which are skipped and reported while every valid row lands byte-exact."""
    from asu_ascend_b200._lib import ST_BAD_QUERY, ST_BAD_SOURCE, ST_BAD_STATE
    from asu_ascend_b200.host_pool import HostRowPool

    rng = np.random.Generator(np.random.PCG64(row_bytes + (pitch or 0)))
    R, Q, S, K = 3, 100, 300, 500
    pool = HostRowPool(rows=700, row_bytes=row_bytes, pitch=pitch)
    pool.fill_random(9)
    rec = rng.integers(0, 700, (R, K)).astype(np.int32)
    query = rng.integers(0, K, (R, Q)).astype(np.int32)
    slot = np.stack([rng.permutation(S)[:Q] for _ in range(R)]).astype(np.int32)
    install = rng.random((R, Q)) < 0.4
    # planted errors (on installing positions only)
    install[0, 5] = install[1, 7] = install[2, 9] = True
    query[0, 5] = K + 3        # bad key
    slot[1, 7] = S + 1         # bad slot
    rec[2, query[2, 9]] = 700  # bad record row
    ok = install.copy()
    ok[0, 5] = ok[1, 7] = ok[2, 9] = False
    # a valid install elsewhere must not share the bad record's key
    same = (query[2] == query[2, 9]) & ok[2]
    ok[2, same] = False
    install[2, same] = False
    base = rng.integers(0, 256, (R, S, row_bytes), dtype=np.uint8)
    slot_pool = T(base)
    status = torch.zeros(R, dtype=torch.int32, device=DEV)
    pool.swapin(T(rec), T(query), T(slot), T(install), slot_pool, status=status)
    expect = O.swapin(pool.array, np.minimum(rec, 699), query, slot, ok, base)
    np.testing.assert_array_equal(N(slot_pool), expect)
    assert N(status).tolist() == [ST_BAD_QUERY, ST_BAD_STATE, ST_BAD_SOURCE]
    pool.close()


# ------------------------------------------------------------------ resolver

def test_resolver_reference_unit_vectors():
    """patch/0001 tests/ut/ops/test_asu_kv_resolver.py (patch lines 672-765) through the torch op."""
    f = torch.ops._C_ascend.npu_asu_resolve_kv_slots_single_req
    kv0 = torch.arange(16, dtype=torch.float32).reshape(8, 2).to(DEV)
    kv1 = torch.arange(24, dtype=torch.float32).reshape(8, 3).to(DEV)
    m0 = torch.full((4, 2), -1.0, device=DEV)
    m1 = torch.full((4, 3), -1.0, device=DEV)
    ts = torch.tensor([0, 0, 0, 0, 2, 2], dtype=torch.int32, device=DEV)
    rec = torch.tensor([0, 4, 0, 0, -1, -1], dtype=torch.int64, device=DEV)
    hs = torch.full((6,), -1, dtype=torch.int32, device=DEV)
    own = torch.full((4,), -1, dtype=torch.int32, device=DEV)
    stack = torch.tensor([0, 1, 2, 3], dtype=torch.int64, device=DEV)
    cnt = torch.tensor(4, dtype=torch.int32, device=DEV)
    bt = torch.tensor([2, 0, 3], dtype=torch.int64, device=DEV)
    out = f(torch.tensor([[[1, 1, 5]]], dtype=torch.int64, device=DEV), 6, 4, ts, rec, hs, own, stack, cnt, bt,
            kv0, kv1, m0, m1, 2)
    assert out.tolist() == [[[3, 3, 2]]]
    assert cnt.item() == 2
    assert ts.tolist() == [0, 1, 0, 0, 2, 1]
    assert hs.tolist() == [-1, 3, -1, -1, -1, 2]
    assert own.tolist() == [-1, -1, 5, 1]
    assert torch.equal(m0[3], kv0[4]) and torch.equal(m1[3], kv1[4])
    assert torch.equal(m0[2], kv0[7]) and torch.equal(m1[2], kv1[7])

    # second case: a resident token reuses its slot without consuming the stack
    kv0 = torch.arange(12, dtype=torch.float32).reshape(6, 2).to(DEV)
    kv1 = torch.arange(18, dtype=torch.float32).reshape(6, 3).to(DEV)
    m0 = torch.full((3, 2), -1.0, device=DEV)
    m1 = torch.full((3, 3), -1.0, device=DEV)
    m0[1] = torch.tensor([101.0, 102.0], device=DEV)
    m1[1] = torch.tensor([201.0, 202.0, 203.0], device=DEV)
    ts = torch.tensor([0, 0, 1], dtype=torch.int32, device=DEV)
    hs = torch.tensor([-1, -1, 1], dtype=torch.int32, device=DEV)
    own = torch.tensor([-1, 2, -1], dtype=torch.int32, device=DEV)
    cnt = torch.tensor(2, dtype=torch.int32, device=DEV)
    out = f(torch.tensor([[2]], dtype=torch.int32, device=DEV), 3, 3, ts,
            torch.tensor([0, 1, 2], dtype=torch.int32, device=DEV), hs, own,
            torch.tensor([0, 2, -1], dtype=torch.int32, device=DEV), cnt,
            torch.tensor([0, 1], dtype=torch.int32, device=DEV), kv0, kv1, m0, m1, 2)
    assert out.tolist() == [[1]]
    assert cnt.item() == 2
    assert m0[1].tolist() == [101.0, 102.0] and m1[1].tolist() == [201.0, 202.0, 203.0]


def test_resolver_matches_golden(golden):
    g = golden("resolver")
    max_seq, slots, bs, actual, prefix = (int(v) for v in g["meta"])
    ts, rec, hs, own, stack, cnt = O.reset_state(max_seq, slots, bs, actual, prefix, g["block_table"])
    np.testing.assert_array_equal(ts, g["reset_token_state"])
    kv0 = T(g["kv0"]).view(torch.bfloat16)
    kv1 = T(g["kv1"]).view(torch.bfloat16)
    m0 = torch.zeros((slots,) + tuple(kv0.shape[1:]), dtype=torch.bfloat16, device=DEV)
    m1 = torch.zeros((slots,) + tuple(kv1.shape[1:]), dtype=torch.bfloat16, device=DEV)
    tts, trec, ths, town, tstack, tcnt, tbt = T(ts), T(rec), T(hs), T(own), T(stack), T(cnt), T(g["block_table"])
    for s in range(3):
        out = torch.ops._C_ascend.npu_asu_resolve_kv_slots_single_req(
            T(g[f"s{s}_topk"]), actual, prefix, tts, trec, ths, town, tstack, tcnt, tbt, kv0, kv1, m0, m1, bs)
        np.testing.assert_array_equal(N(out), g[f"s{s}_out"])
        np.testing.assert_array_equal(N(tts), g[f"s{s}_token_state"])
        np.testing.assert_array_equal(N(ths), g[f"s{s}_hbm_slot"])
        np.testing.assert_array_equal(N(town), g[f"s{s}_owner"])
        assert int(N(tcnt)[0]) == int(g[f"s{s}_count"][0])
        assert digest(N(m0.view(torch.int16)), N(m1.view(torch.int16))) == str(g[f"s{s}_kv_digest"][0])


def test_resolver_second_resolve_is_idempotent():
    """patch/0004 invariant: resolving the same top-k twice consumes no free slots."""
    rng = np.random.Generator(np.random.PCG64(8))
    max_seq, slots, bs, actual, prefix = 8192, 4096, 64, 6000, 5990
    bt = rng.permutation(200)[:128].astype(np.int32)
    ts, rec, hs, own, stack, cnt = O.reset_state(max_seq, slots, bs, actual, prefix, bt)
    kv0 = torch.randn(200 * bs, 1, 512, device=DEV).to(torch.bfloat16)
    kv1 = torch.randn(200 * bs, 1, 64, device=DEV).to(torch.bfloat16)
    m0 = torch.zeros(slots, 1, 512, dtype=torch.bfloat16, device=DEV)
    m1 = torch.zeros(slots, 1, 64, dtype=torch.bfloat16, device=DEV)
    tts, trec, ths, town, tstack, tcnt = T(ts), T(rec), T(hs), T(own), T(stack), T(cnt)
    topk = T(rng.integers(0, actual, (1, 2048)).astype(np.int32))
    f = torch.ops.asu.npu_asu_resolve_kv_slots_single_req
    first = f(topk, actual, prefix, tts, trec, ths, town, tstack, tcnt, T(bt), kv0, kv1, m0, m1, bs)
    c1 = int(tcnt.item())
    second = f(topk, actual, prefix, tts, trec, ths, town, tstack, tcnt, T(bt), kv0, kv1, m0, m1, bs)
    assert int(tcnt.item()) == c1
    assert torch.equal(first, second)
    topk_np, res_np = N(topk)[0], N(first)[0]
    for tok, slot in list(zip(topk_np, res_np))[:64]:
        src = rec[tok] if ts[tok] == 0 else bt[tok // bs] * bs + tok % bs
        assert torch.equal(m0[slot], kv0[src]) and torch.equal(m1[slot], kv1[src])


@pytest.mark.parametrize("n,key_range,seed", [(6000, 3000, 21), (4097, 100000, 22), (2049, 40, 23)])
def test_resolver_multi_chunk_duplicates_match_oracle(n, key_range, seed):
    """Top-k longer than one 2048-entry chunk, duplicates inside and across chunks, all three
    token states in play: outputs, state arrays, free count and managed rows equal the serial
    oracle's."""
    rng = np.random.Generator(np.random.PCG64(seed))
    max_seq, slots, bs = 131072, 8192, 128
    actual = key_range + 500 if key_range + 500 <= max_seq else max_seq
    prefix = actual - 300
    nblk = (max_seq + bs - 1) // bs
    bt = rng.permutation(nblk + 16)[:nblk].astype(np.int32)
    ts, rec, hs, own, stack, cnt = O.reset_state(max_seq, slots, bs, actual, prefix, bt)
    # some tokens already resident
    warm = rng.choice(actual, 500, replace=False).astype(np.int32)
    src0 = rng.integers(0, 256, ((nblk + 16) * bs, 48), dtype=np.uint8)
    src1 = rng.integers(0, 256, ((nblk + 16) * bs, 16), dtype=np.uint8)
    dst0 = np.zeros((slots, 48), np.uint8)
    dst1 = np.zeros((slots, 16), np.uint8)
    O.resolve_kv_slots_single_req(warm.reshape(1, -1), actual, ts, rec, hs, own, stack, cnt, bt, src0, src1, dst0,
                                  dst1, bs)
    tts, trec, ths, town, tstack, tcnt = T(ts), T(rec), T(hs), T(own), T(stack), T(cnt)
    m0, m1 = T(dst0), T(dst1)
    lo = max(0, actual - key_range)
    topk = rng.integers(lo, actual, (1, 3, (n + 2) // 3)).astype(np.int32)
    topk.reshape(-1)[-1] = actual - 1
    exp = O.resolve_kv_slots_single_req(topk, actual, ts, rec, hs, own, stack, cnt, bt, src0, src1, dst0, dst1, bs)
    out = torch.ops._C_ascend.npu_asu_resolve_kv_slots_single_req(
        T(topk), actual, prefix, tts, trec, ths, town, tstack, tcnt, T(bt), T(src0).view(torch.bfloat16),
        T(src1).view(torch.bfloat16), m0.view(torch.bfloat16), m1.view(torch.bfloat16), bs)
    np.testing.assert_array_equal(N(out), exp)
    np.testing.assert_array_equal(N(tts), ts)
    np.testing.assert_array_equal(N(ths), hs)
    np.testing.assert_array_equal(N(town), own)
    assert int(N(tcnt).reshape(-1)[0]) == int(cnt[0])
    np.testing.assert_array_equal(N(m0), dst0)
    np.testing.assert_array_equal(N(m1), dst1)


@pytest.mark.parametrize("w0,w1", [(3, 5), (2, 6), (8, 0), (640, 0), (720, 8)])
def test_resolver_row_widths_match_oracle(w0, w1):
    """fp16 rows of 6/10 bytes (byte copies), 4/12 bytes (4-byte copies), 16 and 1280 bytes with
    an empty second cache (copied by the resolve cluster itself) and 1440 + 16 bytes (16-byte
    copies by the copy kernel): the managed rows equal the oracle's byte for byte."""
    rng = np.random.Generator(np.random.PCG64(w0 * 10 + w1))
    max_seq, slots, bs, actual, prefix = 4096, 3000, 16, 4000, 3900
    nblk = max_seq // bs
    bt = rng.permutation(nblk + 4)[:nblk].astype(np.int32)
    ts, rec, hs, own, stack, cnt = O.reset_state(max_seq, slots, bs, actual, prefix, bt)
    src0 = rng.integers(0, 1 << 16, ((nblk + 4) * bs, w0), dtype=np.uint16)
    src1 = rng.integers(0, 1 << 16, ((nblk + 4) * bs, w1), dtype=np.uint16)
    dst0 = np.zeros((slots, w0), np.uint16)
    dst1 = np.zeros((slots, w1), np.uint16)
    tts, trec, ths, town, tstack, tcnt = T(ts), T(rec), T(hs), T(own), T(stack), T(cnt)
    m0, m1 = T(dst0.view(np.int16)), T(dst1.view(np.int16))
    for step in range(2):
        topk = rng.integers(0, actual, (1, 2500)).astype(np.int32)
        exp = O.resolve_kv_slots_single_req(topk, actual, ts, rec, hs, own, stack, cnt, bt, src0, src1, dst0, dst1,
                                            bs)
        out = torch.ops._C_ascend.npu_asu_resolve_kv_slots_single_req(
            T(topk), actual, prefix, tts, trec, ths, town, tstack, tcnt, T(bt), T(src0.view(np.int16)).view(torch.float16),
            T(src1.view(np.int16)).view(torch.float16), m0.view(torch.float16), m1.view(torch.float16), bs)
        np.testing.assert_array_equal(N(out), exp)
        np.testing.assert_array_equal(N(m0).view(np.uint16), dst0)
        np.testing.assert_array_equal(N(m1).view(np.uint16), dst1)
        assert int(N(tcnt).reshape(-1)[0]) == int(cnt[0])


def test_resolver_errors_are_reported():
    f = torch.ops.asu.npu_asu_resolve_kv_slots_single_req  # the C++ op raises RuntimeError
    z = lambda n: torch.zeros(n, dtype=torch.int32, device=DEV)  # noqa: E731
    kv = torch.zeros(4, 2, device=DEV)
    m = torch.zeros(1, 2, device=DEV)
    with pytest.raises(RuntimeError, match="FREE_EXHAUSTED"):
        f(torch.tensor([0, 1], dtype=torch.int32, device=DEV), 4, 4, z(4), z(4), z(4) - 1, z(1) - 1, z(1),
          torch.ones(1, dtype=torch.int32, device=DEV), z(2), kv, kv, m, m, 2)
    with pytest.raises(RuntimeError, match="BAD_QUERY"):
        f(torch.tensor([5], dtype=torch.int32, device=DEV), 4, 4, z(4), z(4), z(4) - 1, z(1) - 1, z(1),
          torch.ones(1, dtype=torch.int32, device=DEV), z(2), kv, kv, m, m, 2)
