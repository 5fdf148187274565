"""asu_lru_step_host_query: the exact-LRU step reading its top-k from pinned host memory (and leaving
an HBM copy for the swap-in) gives the same slots, masks, evictions, statistics and state as
asu_lru_step on an identical pool over several steps, at the resolver workload's shape and at a
ragged one, and the HBM copy equals the top-k."""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda:0")


@pytest.mark.parametrize("R,K,S,Q,target,steps", [(128, 131072, 8192, 2048, 2048, 4), (5, 5000, 1001, 333, 300, 6),
                                                  (3, 70000, 16384, 4096, 4096, 3)])
def test_host_query_step_matches_device_step(R, K, S, Q, target, steps):
    import asu_ascend_b200

    asu_ascend_b200.load()
    from asu_ascend_b200.lru import LruSlotPools
    from asu_ascend_b200.workloads import LocalityTrace

    trace = LocalityTrace(R, K, topk=Q, seed=R * 7 + S)
    a = LruSlotPools(R, K, S, target, Q, device=DEV)
    b = LruSlotPools(R, K, S, target, Q, device=DEV)
    copy = torch.full((R, Q), -5, dtype=torch.int32, device=DEV)
    for step in range(steps):
        q = trace.step()
        if step == steps - 1:
            q[0, : min(Q, 40)] = K + 3  # out-of-range ids take the same status path
        qh = torch.from_numpy(np.ascontiguousarray(q)).pin_memory()
        oa = a.step(qh.to(DEV))
        ob = b.step_from_host(qh, copy)
        torch.cuda.synchronize()
        assert torch.equal(copy.cpu(), qh)
        for x, y in ((oa.slot, ob.slot), (oa.hit, ob.hit), (oa.install, ob.install),
                     (oa.evicted_count, ob.evicted_count)):
            assert torch.equal(x, y)
        n = oa.evicted_count.cpu().numpy()
        ea, eb = oa.evicted.cpu().numpy(), ob.evicted.cpu().numpy()
        for r in range(R):
            assert np.array_equal(ea[r, : n[r]], eb[r, : n[r]])
    for x, y in ((a.token_to_slot, b.token_to_slot), (a.slot_to_token, b.slot_to_token), (a.free_count, b.free_count),
                 (a.stats, b.stats), (a.status, b.status)):
        assert torch.equal(x, y)
    fa = a.free_count.cpu().numpy()
    oa_, ob_ = a.lru_order.cpu().numpy(), b.lru_order.cpu().numpy()
    for r in range(R):
        assert np.array_equal(oa_[r, : S - fa[r]], ob_[r, : S - fa[r]])
    assert int(a.stats[:, 2].sum()) > 0  # the steps installed rows


def test_host_query_step_rejects_device_queries():
    import asu_ascend_b200

    asu_ascend_b200.load()
    from asu_ascend_b200.lru import LruSlotPools

    p = LruSlotPools(2, 100, 16, 4, 8, device=DEV)
    with pytest.raises(RuntimeError, match="pinned host memory"):
        p.step_from_host(torch.zeros((2, 8), dtype=torch.int32, device=DEV),
                         torch.zeros((2, 8), dtype=torch.int32, device=DEV))
    with pytest.raises(RuntimeError):  # host memory that is not pinned has no device address
        p.step_from_host(torch.zeros((2, 8), dtype=torch.int32), torch.zeros((2, 8), dtype=torch.int32, device=DEV))
