"""Multi-rank host logic on CPU: request sharding and the end-of-run statistics reduction
run as world-size-2 gloo ranks and must equal one process doing all requests."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from asu_ascend_b200.dist import max_over_ranks, reduce_stats, rows_by_rank, shard_range


def test_shard_range_covers_every_request_once():
    for total in (0, 1, 7, 128, 1024, 1025):
        for world in (1, 2, 3, 8):
            seen = []
            for r in range(world):
                a, b = shard_range(total, world, r)
                seen.extend(range(a, b))
                assert b - a in (total // world, total // world + 1)
            assert seen == list(range(total))
    with pytest.raises(ValueError):
        shard_range(4, 2, 2)


def _trace(total_req, steps):
    from asu_ascend_b200.workloads import LocalityTrace

    tr = LocalityTrace(total_req, 8192, topk=256, seed=77)
    return np.stack([tr.step() for _ in range(steps)])


def _run_rows(trace, rows):
    from oracle import c_oracle

    pools = c_oracle.LruPools(len(rows), 8192, 1024, 256)
    for s in range(trace.shape[0]):
        pools.step_all(trace[s][rows], threads=1, want_outputs=False)
    st = pools.stats.copy()
    pools.close()
    return st


def _worker(rank, world, port, out_path):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        trace = _trace(6, 5)
        a, b = shard_range(6, world, rank)
        st = _run_rows(trace, list(range(a, b)))
        total = reduce_stats(torch.from_numpy(st))
        slowest = max_over_ranks([float(rank + 1)])
        rows = rows_by_rank([float(rank), 10.0 * rank + 0.5])
        if rank == 0:
            assert rows == [[0.0, 0.5], [1.0, 10.5]]
            np.save(out_path, np.concatenate([total.numpy(), np.asarray(slowest, np.int64)]))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_match_one_process(tmp_path):
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    out = tmp_path / "stats.npy"
    mp.spawn(_worker, args=(2, port, str(out)), nprocs=2, join=True)
    got = np.load(out)
    expect = _run_rows(_trace(6, 5), list(range(6))).sum(0)
    np.testing.assert_array_equal(got[:5], expect)
    assert got[5] == 2  # max over ranks of (rank + 1)


class _FakeNvml:
    """NVML stand-in: GPU i is local to CPUs [4i, 4i+4)."""

    def nvmlInit(self):
        pass

    def nvmlDeviceGetHandleByIndex(self, i):
        return i

    def nvmlDeviceGetCpuAffinity(self, handle, words):
        return [0xF << (4 * handle)] + [0] * (words - 1)


def test_gpu_local_cpus_reads_nvml_affinity_within_the_allowed_set():
    import os

    from asu_ascend_b200.dist import bind_to_gpu_local_cpus, gpu_local_cpus

    allowed = os.sched_getaffinity(0)
    expect = sorted({4, 5, 6, 7} & allowed)
    assert gpu_local_cpus(1, _FakeNvml()) == expect
    try:
        bound = bind_to_gpu_local_cpus(1, _FakeNvml())
        if expect and set(expect) != allowed:
            assert bound == expect and os.sched_getaffinity(0) == set(expect)
    finally:
        os.sched_setaffinity(0, allowed)

    class Broken(_FakeNvml):
        def nvmlInit(self):
            raise RuntimeError("no driver")

    assert gpu_local_cpus(0, Broken()) == [] and bind_to_gpu_local_cpus(0, Broken()) == []


def test_host_link_groups_and_spread_placement():
    from asu_ascend_b200.dist import host_link_groups, spread_devices

    # two sockets of four GPUs (NVML levels: 40 within a NUMA node, 50 across the system)
    two = host_link_groups(8, lambda i, j: 40 if (i < 4) == (j < 4) else 50)
    assert two == [[0, 1, 2, 3], [4, 5, 6, 7]]
    assert spread_devices(1, two) == [0]
    assert spread_devices(2, two) == [0, 4]
    assert spread_devices(4, two) == [0, 4, 1, 5]
    assert spread_devices(8, two) == list(range(8))  # as many ranks as GPUs: rank r keeps GPU r
    # switches below the sockets do not split the groups further: only the widest split counts
    nested = host_link_groups(8, lambda i, j: 20 if i // 2 == j // 2 else (40 if (i < 4) == (j < 4) else 50))
    assert nested == two
    # every pair at the same level: one group, identity placement
    flat = host_link_groups(8, lambda i, j: 40)
    assert flat == [list(range(8))] and spread_devices(4, flat) == [0, 1, 2, 3]
    # uneven groups: round-robin while each group has GPUs left, every GPU at most once
    uneven = [[0, 1, 2], [3]]
    assert spread_devices(3, uneven) == [0, 3, 1]
    for n in range(1, 5):
        got = spread_devices(n, uneven)
        assert len(set(got)) == n
    assert host_link_groups(1, lambda i, j: 0) == [[0]]


def test_placement_candidates_and_choice():
    from asu_ascend_b200.dist import choose_placement, placement_candidates

    assert placement_candidates(8, 4) == [[0, 1, 2, 3], [0, 4, 1, 5]]
    assert placement_candidates(8, 1) == [[0]]
    assert placement_candidates(6, 3) == [[0, 1, 2], [0, 3, 1]]
    # NVML groups that agree with the halves add nothing new
    assert placement_candidates(8, 4, [[0, 1, 2, 3], [4, 5, 6, 7]]) == [[0, 1, 2, 3], [0, 4, 1, 5]]
    cands = placement_candidates(8, 4)
    # the 8-GPU box: GPUs 0-3 copying together get ~29 GB/s each, GPUs 0, 1, 4, 5 ~54
    assert choose_placement(cands, [{0: 28.9, 1: 29.0, 2: 28.9, 3: 29.0}, {0: 53.6, 4: 55.3, 1: 53.7, 5: 55.3}]) == 1
    # within the margin the identity stays
    assert choose_placement(cands, [{0: 55.0, 1: 55.0}, {0: 55.5, 4: 56.0}]) == 0


def test_placed_device_shares_local_rank_0s_choice(monkeypatch):
    import json
    import subprocess
    import threading

    from asu_ascend_b200 import dist as D

    monkeypatch.setattr(torch.cuda, "device_count", lambda: 8)
    calls = []

    def fake_run(cmd, **kw):
        calls.append(cmd)
        out = json.dumps({"devices": [0, 4, 1, 5], "candidates": [[0, 1, 2, 3], [0, 4, 1, 5]],
                          "slowest_gbs": [28.9, 53.6]})
        return subprocess.CompletedProcess(cmd, 0, stdout="log line\n" + out + "\n", stderr="")

    monkeypatch.setattr(subprocess, "run", fake_run)
    store = dist.HashStore()
    got = {}

    def rank(lr):
        got[lr] = D.placed_device(lr, 4, store, key="k")

    threads = [threading.Thread(target=rank, args=(lr,)) for lr in (3, 2, 1, 0)]  # readers wait for rank 0
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout=30)
    assert {lr: d for lr, (d, _) in got.items()} == {0: 0, 1: 4, 2: 1, 3: 5}
    assert len(calls) == 1 and "--measure-placement" in calls[0] and calls[0][-1] == "4"
    assert got[2][1]["slowest_gbs"] == [28.9, 53.6] and got[2][1]["rule"].startswith("measured")
    # as many ranks as GPUs, or no store: rank r keeps GPU r and nothing is measured
    assert D.placed_device(5, 8, store)[0] == 5 and D.placed_device(1, 4, None)[0] == 1
    assert len(calls) == 1

    # a failed measurement falls back to the identity for every rank
    monkeypatch.setattr(subprocess, "run", lambda cmd, **kw: subprocess.CompletedProcess(cmd, 1, "", "boom"))
    store2 = dist.HashStore()
    assert D.placed_device(0, 4, store2, key="k")[0] == 0
    d3, info = D.placed_device(3, 4, store2, key="k")
    assert d3 == 3 and "failed" in info["error"]
