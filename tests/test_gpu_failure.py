"""Device-side failure detection without a GPU fault: the bounded wait that the TMA swap-in uses
gives up on an mbarrier that nothing arrives at and reports ASU_ST_TIMEOUT in the status word;
the kernel returns and the context stays usable for the next launch."""

import time

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


def test_bounded_wait_reports_timeout_and_the_context_stays_usable():
    import asu_ascend_b200

    asu_ascend_b200.load()
    from asu_ascend_b200 import hbm_lookup_update as H
    from asu_ascend_b200._lib import ST_TIMEOUT, check, lib

    stream = torch.cuda.current_stream(DEV).cuda_stream
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    check(lib.asu_selftest_bounded_wait(stream, 1, status.data_ptr()), "selftest")  # arrives: no timeout
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    t0 = time.perf_counter()
    check(lib.asu_selftest_bounded_wait(stream, 0, status.data_ptr()), "selftest")  # nothing arrives
    torch.cuda.synchronize()
    waited = time.perf_counter() - t0
    assert int(status.item()) == ST_TIMEOUT
    print(f"bounded wait gave up after {waited * 1e3:.1f} ms")
    # the next launch runs normally
    table = torch.arange(64, dtype=torch.int32, device=DEV).reshape(1, 64)
    query = torch.tensor([[5, 63, 0, 7]], dtype=torch.int32, device=DEV)
    out = torch.empty_like(query)
    H.lookup(table, query, out=out)
    np.testing.assert_array_equal(out.cpu().numpy(), [[5, 63, 0, 7]])
