"""The synthetic inputs behave as the benchmark configurations describe them: distinct top-k ids
per row, the stated share of ids kept from the previous step, Zipf skew toward low positions
(or none for the uniform stress traces), and the lookup and SIMT cases' hit counts."""

import numpy as np

from asu_ascend_b200 import workloads as W


def _check_trace(tr, reuse, key_space, steps=4):
    prev = None
    for _ in range(steps):
        rows = tr.step()
        assert rows.shape == (tr.req_num, tr.topk) and rows.dtype == np.int32
        assert rows.min() >= 0 and rows.max() < key_space
        for r in range(tr.req_num):
            assert np.unique(rows[r]).size == tr.topk  # distinct within a row
            if prev is not None:
                kept = np.intersect1d(rows[r], prev[r]).size
                assert kept >= int(round(tr.topk * reuse))  # at least the reused share
        prev = rows
    return prev


def test_locality_trace_reuse_and_zipf_skew():
    rows = _check_trace(W.LocalityTrace(4, 131072, topk=2048, reuse=0.7, zipf_s=1.1, seed=1), 0.7, 131072)
    assert np.median(rows) < 131072 // 8  # Zipf(1.1) concentrates on low positions


def test_fast_locality_trace_uniform_stress():
    rows = _check_trace(W.FastLocalityTrace(16, 1 << 20, topk=2048, reuse=0.2, zipf_s=None, seed=2), 0.2, 1 << 20)
    assert abs(np.median(rows) / (1 << 20) - 0.5) < 0.05  # uniform over the context


def test_lookup_only_case_hit_share():
    table, query = W.lookup_only_case(req_num=4)
    assert table.shape == (4, 131072) and query.shape == (4, 2048)
    assert ((table >= 0).sum(1) == 4096).all()  # 4096 resident entries per request
    hit = np.take_along_axis(table, query.astype(np.int64), 1) >= 0
    assert 0.8 < hit.mean() < 0.9
    assert all(np.unique(q).size == q.size for q in query)


def test_simt_case_exact_hits():
    t2s, s2t, lru, q = W.simt_case(3, 1536, seed=5)
    hits = (np.take_along_axis(t2s, q.astype(np.int64), 1) >= 0).sum(1)
    assert (hits == 1536).all()
    assert all(sorted(l.tolist()) == list(range(lru.shape[1])) for l in lru)  # permutations
