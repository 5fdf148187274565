"""GPU parity of the resolver over an exact-LRU managed pool (asu_kv_resolver_lru and the torch
op npu_asu_resolve_kv_slots_lru) against the oracle (asu_oracle.resolve_kv_slots_lru, the
resolver of patch/0001 composed with LRUManagedCache of simu/kv_cache_eviction_sim.py):
resolved slots, evicted tokens, every state array, the recency order and the managed rows,
bit-exact, call after call."""

import ctypes

import numpy as np
import pytest
import torch

from oracle import asu_oracle as O

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


@pytest.fixture(scope="module")
def L():
    import asu_ascend_b200

    asu_ascend_b200.load()
    from asu_ascend_b200 import _lib

    return _lib


def T(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def N(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


class Pool:
    """One layer's state on the host (oracle) and on the GPU."""

    def __init__(self, rng, max_seq, slots, bs, actual, prefix, w0, w1, src_extra=16):
        nblk = (max_seq + bs - 1) // bs
        self.bt = rng.permutation(nblk + src_extra)[:nblk].astype(np.int32)
        self.st = list(O.reset_state(max_seq, slots, bs, actual, prefix, self.bt))
        self.order = np.full(slots, -1, np.int32)
        self.src0 = rng.integers(0, 256, ((nblk + src_extra) * bs, w0), dtype=np.uint8)
        self.src1 = rng.integers(0, 256, ((nblk + src_extra) * bs, w1), dtype=np.uint8)
        self.dst0 = np.zeros((slots, w0), np.uint8)
        self.dst1 = np.zeros((slots, w1), np.uint8)
        self.g = [T(a) for a in self.st] + [T(self.order)]
        self.gbt, self.gsrc0, self.gsrc1 = T(self.bt), T(self.src0), T(self.src1)
        self.gdst0, self.gdst1 = T(self.dst0), T(self.dst1)
        self.max_seq, self.slots, self.bs = max_seq, slots, bs

    def oracle(self, topk, actual, target):
        return O.resolve_kv_slots_lru(topk, actual, *self.st, self.order, target, self.bt, self.src0, self.src1,
                                      self.dst0, self.dst1, self.bs)

    def gpu(self, L, topk, actual, target, stats=None):
        ts, rec, hs, own, stack, cnt, order = self.g
        t = T(topk)
        out = torch.full(topk.shape, -7, dtype=torch.int32, device=DEV)
        ev = torch.full((max(min(target, self.slots), 1),), -7, dtype=torch.int32, device=DEV)
        evn = torch.full((1,), -7, dtype=torch.int32, device=DEV)
        status = torch.zeros(1, dtype=torch.int32, device=DEV)
        stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        rc = L.lib.asu_kv_resolver_lru(
            stream, t.data_ptr(), t.numel(), ts.data_ptr(), rec.data_ptr(), hs.data_ptr(), own.data_ptr(),
            stack.data_ptr(), cnt.data_ptr(), order.data_ptr(), self.slots, target, self.gbt.data_ptr(),
            self.gbt.numel(), self.gsrc0.data_ptr(), self.gsrc1.data_ptr(), self.gdst0.data_ptr(),
            self.gdst1.data_ptr(), self.src0.shape[1], self.src1.shape[1], self.src0.shape[0], self.max_seq, actual,
            self.bs, out.data_ptr(), ev.data_ptr(), evn.data_ptr(), None if stats is None else stats.data_ptr(),
            status.data_ptr())
        assert rc == 0, L.lib.asu_status_string(rc)
        return out, ev, evn, status

    def compare(self, tag):
        ts, rec, hs, own, stack, cnt, order = (N(x) for x in self.g)
        ets, erec, ehs, eown, estack, ecnt = self.st
        np.testing.assert_array_equal(ts, ets, err_msg=f"{tag} token_state")
        np.testing.assert_array_equal(hs, ehs, err_msg=f"{tag} hbm_slot_of_token")
        np.testing.assert_array_equal(own, eown, err_msg=f"{tag} slot_owner_token")
        assert int(cnt.reshape(-1)[0]) == int(ecnt[0]), f"{tag} free count"
        c = int(ecnt[0])
        np.testing.assert_array_equal(stack[:c], estack[:c], err_msg=f"{tag} free stack")
        np.testing.assert_array_equal(order[: self.slots - c], self.order[: self.slots - c], err_msg=f"{tag} order")
        np.testing.assert_array_equal(N(self.gdst0), self.dst0, err_msg=f"{tag} kv0 rows")
        np.testing.assert_array_equal(N(self.gdst1), self.dst1, err_msg=f"{tag} kv1 rows")


def _run(L, pool, steps, actual, target, tag):
    for i, topk in enumerate(steps):
        exp, eev = pool.oracle(topk, actual, target)
        out, ev, evn, status = pool.gpu(L, topk, actual, target)
        assert int(N(status)[0]) == 0, f"{tag} step {i}: status {int(N(status)[0]):#x}"
        np.testing.assert_array_equal(N(out), exp, err_msg=f"{tag} step {i} resolved")
        n = int(N(evn)[0])
        assert n == eev.size, f"{tag} step {i} evicted count"
        np.testing.assert_array_equal(N(ev)[:n], eev, err_msg=f"{tag} step {i} evicted")
        pool.compare(f"{tag} step {i}")


def _locality_steps(rng, n_steps, topk, actual, hot_n, reuse=0.7, newest=True):
    hot = rng.integers(0, actual, hot_n)
    prev = rng.choice(hot, topk)
    out = []
    for _ in range(n_steps):
        keep = rng.random(topk) < reuse
        q = np.where(keep, prev, rng.integers(0, actual, topk)).astype(np.int32)
        if newest:
            q[-1] = actual - 1
        out.append(q)
        prev = q
    return out


@pytest.mark.parametrize("w0,w1", [(1024, 128), (640, 16), (720, 8), (6, 3), (2048, 0)])
def test_resolver_lru_matches_oracle_row_widths(L, w0, w1):
    """Small pools that evict every call; 16-, 4- and 1-byte copy units; duplicates in the top-k,
    prefix (ASU_ONLY) and tail (TAIL_HBM) tokens, tokens evicted and asked for again."""
    rng = np.random.Generator(np.random.PCG64(w0 * 7 + w1))
    pool = Pool(rng, 8192, 640, 64, 8000, 7800, w0, w1)
    steps = _locality_steps(rng, 8, 256, 8000, 900)
    _run(L, pool, steps, 8000, 256, f"rows ({w0},{w1})")


@pytest.mark.parametrize("slots,target,topk", [(37, 30, 30), (1000, 0, 700), (2048, 2048, 2048),
                                               (16384, 4096, 4096), (10240, 3000, 3000)])
def test_resolver_lru_matches_oracle_shapes(L, slots, target, topk):
    """Every thread-work shape: slot counts from 37 to the 16384 maximum (2 to 16 order entries per
    thread), top-k from 30 to the 4096 maximum (2 or 4 entries per thread), a target of 0 (the pool
    never evicts) and targets of the top-k size up to the whole pool (every resident evicted)."""
    rng = np.random.Generator(np.random.PCG64(slots + topk))
    actual = 60000
    pool = Pool(rng, 65536, slots, 128, actual, actual - 500, 16, 16)
    steps = _locality_steps(rng, 5, topk, actual, 3 * max(slots, topk))
    if target == 0:  # a pool that never evicts must not run out
        steps = [s[: min(topk, slots // 5)] for s in steps]
    _run(L, pool, steps, actual, target, f"slots {slots} target {target} topk {topk}")


def test_resolver_lru_decode_size_against_oracle(L):
    """The decode workload's full size over a bounded pool: 131072-token context (130944 prefix
    tokens in the ASU store, a paged tail), 8192 + 2048 managed slots, free target 2048, top-k
    2048 with 50% reuse and the newest token always asked for, 512 + 64 bf16 rows (1024 + 128
    bytes), one decode token appended per step; sixteen steps (the pool fills after about eight
    and evicts from then on), everything against the oracle."""
    rng = np.random.Generator(np.random.PCG64(131072))
    max_seq, bs = 131072, 128
    actual, prefix = 130944 + 8, 130944
    pool = Pool(rng, max_seq, 10240, bs, actual, prefix, 1024, 128)
    stats = torch.zeros(5, dtype=torch.int64, device=DEV)
    hot = rng.integers(0, actual, 40000)
    prev = rng.choice(hot, 2048)
    for step in range(16):
        # a decode step appends one token (TAIL_HBM in the state, as mark_decode_token does)
        if step:
            pool.st[0][actual] = O.TAIL_HBM
            pool.g[0][actual] = O.TAIL_HBM
            actual += 1
        q = np.where(rng.random(2048) < 0.5, prev, rng.choice(hot, 2048)).astype(np.int32)
        q[-1] = actual - 1
        prev = q
        exp, eev = pool.oracle(q, actual, 2048)
        out, ev, evn, status = pool.gpu(L, q, actual, 2048, stats=stats)
        assert int(N(status)[0]) == 0
        np.testing.assert_array_equal(N(out), exp, err_msg=f"decode step {step}")
        n = int(N(evn)[0])
        np.testing.assert_array_equal(N(ev)[:n], eev, err_msg=f"decode step {step} evicted")
        pool.compare(f"decode step {step}")
    hits, misses, inst, short, evictions = N(stats).tolist()
    assert short == 0 and inst == misses and evictions > 2048 and hits + misses == 16 * 2048


def test_resolver_lru_torch_op_and_bad_entries(L):
    """The torch op (torch.ops.asu.npu_asu_resolve_kv_slots_lru) on padded top-k: -1 entries resolve
    to -1 and change nothing (BAD_QUERY, raised when status checks are on), a tail token the block
    table does not cover takes no slot (BAD_SOURCE)."""
    from asu_ascend_b200 import ops

    rng = np.random.Generator(np.random.PCG64(5))
    pool = Pool(rng, 4096, 300, 64, 4000, 3900, 32, 32)
    ts, rec, hs, own, stack, cnt, order = pool.g
    q = _locality_steps(rng, 1, 200, 4000, 500)[0]
    exp, _ = pool.oracle(q, 4000, 64)
    padded = np.concatenate([q, np.full(56, -1, np.int32)])
    args = (ts, rec, hs, own, stack, cnt, order, 64, pool.gbt, pool.gsrc0.view(torch.bfloat16),
            pool.gsrc1.view(torch.bfloat16), pool.gdst0.view(torch.bfloat16), pool.gdst1.view(torch.bfloat16), 64)
    out = torch.ops.asu.npu_asu_resolve_kv_slots_lru(T(padded[None, :]), 4000, 3900, *args)
    got = N(out)[0]
    np.testing.assert_array_equal(got[:200], exp)
    assert (got[200:] == -1).all()
    pool.compare("torch op")
    ops.set_status_checks(True)
    try:
        with pytest.raises(RuntimeError, match="BAD_QUERY"):
            torch.ops.asu.npu_asu_resolve_kv_slots_lru(T(np.array([[-1]], np.int32)), 4000, 3900, *args)
        pool.compare("after a bad query")
        # a tail token whose block is past the block table: BAD_SOURCE, no slot taken
        tail = next(t for t in range(3900, 4000) if t not in set(q.tolist()))
        short_bt = pool.gbt[: 3900 // 64]
        args2 = args[:8] + (short_bt,) + args[9:]
        free_before = int(N(cnt).reshape(-1)[0])
        with pytest.raises(RuntimeError, match="BAD_SOURCE"):
            torch.ops.asu.npu_asu_resolve_kv_slots_lru(T(np.array([[tail]], np.int32)), 4000, 3900, *args2)
        assert int(N(ts)[tail]) == O.TAIL_HBM and int(N(hs)[tail]) == -1
        assert int(N(cnt).reshape(-1)[0]) == free_before  # nothing installed (and nothing to evict)
    finally:
        ops.set_status_checks(False)


def test_resolver_lru_shortage_reports_free_exhausted(L):
    """Six missing tokens, four slots, a target of 0: the first four take the stack from the top
    (slots 3, 2, 1, 0), the other two resolve to -1 with FREE_EXHAUSTED (the reference raises)."""
    rng = np.random.Generator(np.random.PCG64(9))
    pool = Pool(rng, 256, 4, 16, 200, 100, 16, 0)
    out, ev, evn, status = pool.gpu(L, np.array([5, 6, 5, 7, 8, 9, 10], np.int32), 200, 0)
    assert N(out).tolist() == [3, 2, 3, 1, 0, -1, -1]
    assert int(N(status)[0]) == L.ST_FREE_EXHAUSTED
    assert int(N(evn)[0]) == 0
    ts, _, hs, own, _, cnt, order = (N(x) for x in pool.g)
    assert int(cnt.reshape(-1)[0]) == 0
    assert order.tolist() == [2, 3, 1, 0]  # least recently used first: token 5's slot 3 was touched again
