"""Swap-in balancing on the GPU: the shared-memory host pool, the peer-store swap-in kernels and,
with two GPUs, the balanced bench path end to end.

* A pool backed by a shared-memory file (what every rank allocates on N > 1 GPUs) swaps in the
  same bytes as the oracle, and so does a second mapping of the same file registered by the same
  process (what a helper rank maps).
* ``asu_swapin_gather_to_peer`` (plain 16-byte stores, system fence) into a slot pool on this GPU
  equals the oracle for TMA-sized rows and for block rows.
* Two GPUs: ``bench.py --gpus 2 --balance-share 32 --verify`` runs rank 1 as the helper of rank 0
  (NCCL messages, a CUDA IPC mapping of rank 0's slot pool, rank 0's host pool mapped in rank 1),
  refines the share from measured steps, and checks every resident row of every request of both
  ranks against its host record.
"""

import json
import os
import socket
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import asu_oracle as O

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]
DEV = torch.device("cuda:0")


def T(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def N(t):
    return t.cpu().numpy()


def _run_steps(pool, row_bytes, R, S, Q, via_peer_kernel=False, steps=4):
    from asu_ascend_b200.host_pool import check_status
    from asu_ascend_b200.lru import LruSlotPools
    from asu_ascend_b200.workloads import LocalityTrace, record_addresses

    K = 4096
    rec = record_addresses(R, K, pool.rows)
    tr = LocalityTrace(R, K, topk=Q, seed=9)
    lru = LruSlotPools(R, K, S, Q // 4, Q, device=DEV)
    slot_pool = torch.zeros((R, S, row_bytes), dtype=torch.uint8, device=DEV)
    expect = np.zeros((R, S, row_bytes), np.uint8)
    trec = T(rec)
    status = torch.zeros(R, dtype=torch.int32, device=DEV)
    for _ in range(steps):
        q = tr.step()
        tq = T(q)
        out = lru.step(tq)
        if via_peer_kernel:
            pool.swapin_to_peer(trec, tq, out.slot, out.install, slot_pool.data_ptr(), S, status=status)
        else:
            pool.swapin(trec, tq, out.slot, out.install, slot_pool, status=status)
        expect = O.swapin(pool.array, rec, q, N(out.slot), N(out.install), expect)
        np.testing.assert_array_equal(N(slot_pool), expect)
    check_status(status, "swapin")


@pytest.mark.parametrize("row_bytes", [656, 1024, 4096])
def test_shared_pool_swapin_matches_oracle(row_bytes):
    from asu_ascend_b200.host_pool import HostRowPool

    pool = HostRowPool(rows=3000, row_bytes=row_bytes, shared=True)
    try:
        pool.fill_random(17)
        _run_steps(pool, row_bytes, R=5, S=256, Q=96)
    finally:
        pool.close()


@pytest.mark.parametrize("row_bytes", [656, 4096])
def test_peer_store_kernels_match_oracle(row_bytes):
    from asu_ascend_b200.host_pool import HostRowPool

    pool = HostRowPool(rows=3000, row_bytes=row_bytes)
    try:
        pool.fill_random(19)
        _run_steps(pool, row_bytes, R=7, S=300, Q=130, via_peer_kernel=True)
    finally:
        pool.close()


def test_second_mapping_of_a_shared_pool_reads_the_same_rows():
    from asu_ascend_b200.host_pool import HostRowPool

    owner = HostRowPool(rows=2000, row_bytes=656, shared=True)
    owner.fill_random(23)
    helper = HostRowPool.attach(os.dup(owner.shared.fd), owner.rows, owner.row_bytes, owner.pitch)
    try:
        assert helper.device_ptr != owner.device_ptr
        assert np.array_equal(helper.array, owner.array)
        _run_steps(helper, 656, R=4, S=200, Q=64, via_peer_kernel=True)
        owner.array[5, :16] = 0xAB  # writes by the owner are seen through the helper's mapping
        assert (helper.array[5, :16] == 0xAB).all()
    finally:
        helper.close()
        owner.close()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_gpu_balanced_bench_rows_verified():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2", "--master-addr",
           "127.0.0.1", "--master-port", str(port), str(ROOT / "bench.py"), "--gpus", "2", "--steps", "3",
           "--warmup", "3", "--balance-share", "32", "--verify"]
    out = subprocess.run(cmd, capture_output=True, text=True, cwd=ROOT, timeout=900, env=env)
    assert out.returncode == 0, out.stderr[-3000:]
    line = json.loads([ln for ln in out.stdout.splitlines() if ln.startswith("{")][-1])
    assert line["n_gpus"] == 2 and [p[:2] for p in line["balance"]["pairs"]] == [[0, 1]]
    assert line["balance"]["history"][0]["pairs"] == [[0, 1, 32]]
    assert line["verified_rows"] > 0
