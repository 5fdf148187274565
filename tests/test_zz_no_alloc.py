"""The resolver entry point that allocates nothing (asu_kv_resolver_noalloc).

It exists for callers that cannot allocate device memory while they resolve a layer: an
engine whose HBM is pre-reserved for its KV-block pool and which forbids cudaMalloc inside
the decode loop, or a C / FFI host without a caching allocator.  Instead of a caller-provided
workspace it uses a fixed scratch array inside the library.

These checks call it through the C ABI and compare it with asu_kv_resolver_do (the entry
point with a caller-provided workspace) on identical copies of the same state, for two calls
in a row, bit-exact like every other resolver test.  They hold when this file runs alone in a
fresh process and after the other tests (the first call on the device does the one-time
set-up).  The file name makes pytest collect it last.
"""

import ctypes

import numpy as np
import pytest
import torch

from oracle import asu_oracle as O

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


def _state(rng, max_seq, slots, bs, actual, prefix, nblk):
    bt = rng.permutation(nblk + 16)[:nblk].astype(np.int32)
    ts, rec, hs, own, stack, cnt = O.reset_state(max_seq, slots, bs, actual, prefix, bt)
    return [torch.from_numpy(a).to(DEV) for a in (ts, rec, hs, own, stack, cnt, bt)]


def _call(lib, use_noalloc, topk, st, kv0, kv1, m0, m1, actual, bs, ws=None):
    ts, rec, hs, own, stack, cnt, bt = st
    resolved = torch.full(topk.shape, -7, dtype=torch.int32, device=DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    common = [topk.data_ptr(), topk.numel(), ts.data_ptr(), rec.data_ptr(), hs.data_ptr(), own.data_ptr(),
              stack.data_ptr(), cnt.data_ptr(), stack.numel(), bt.data_ptr(), bt.numel(), kv0.data_ptr(),
              kv1.data_ptr(), m0.data_ptr(), m1.data_ptr(), kv0[0].numel() * kv0.element_size(),
              kv1[0].numel() * kv1.element_size(), min(kv0.shape[0], kv1.shape[0]),
              min(m0.shape[0], m1.shape[0], own.numel()), ts.numel(), actual, bs, resolved.data_ptr()]
    if use_noalloc:
        rc = lib.asu_kv_resolver_noalloc(stream, *common, status.data_ptr())
    else:
        rc = lib.asu_kv_resolver_do(stream, *common, ws.data_ptr(), status.data_ptr())
    assert rc == 0, lib.asu_status_string(rc)
    torch.cuda.synchronize()
    assert status.item() == 0
    return resolved


def test_noalloc_resolver_matches_workspace_resolver_twice_in_a_row():
    import asu_ascend_b200

    asu_ascend_b200.load()
    from asu_ascend_b200._lib import lib

    rng = np.random.Generator(np.random.PCG64(2027))
    max_seq, slots, bs, actual, prefix, nblk = 16384, 4096, 64, 12000, 11990, 188
    st_ref = _state(rng, max_seq, slots, bs, actual, prefix, nblk)
    st_new = [t.clone() for t in st_ref]
    kv0 = torch.randn((nblk + 16) * bs, 1, 512, device=DEV).to(torch.bfloat16)
    kv1 = torch.randn((nblk + 16) * bs, 1, 64, device=DEV).to(torch.bfloat16)
    m_ref = [torch.zeros(slots, 1, 512, dtype=torch.bfloat16, device=DEV),
             torch.zeros(slots, 1, 64, dtype=torch.bfloat16, device=DEV)]
    m_new = [t.clone() for t in m_ref]
    for call in range(2):
        topk = rng.integers(0, actual, (1, 1, 2048)).astype(np.int32)
        topk[0, 0, 500:560] = topk[0, 0, 0:60]  # duplicates
        topk = torch.from_numpy(topk).to(DEV)
        ws = torch.empty(int(lib.asu_kv_resolver_workspace_bytes(topk.numel())), dtype=torch.uint8, device=DEV)
        want = _call(lib, False, topk, st_ref, kv0, kv1, m_ref[0], m_ref[1], actual, bs, ws)
        got = _call(lib, True, topk, st_new, kv0, kv1, m_new[0], m_new[1], actual, bs)
        assert torch.equal(got, want), f"call {call}: resolved slots differ"
        for a, b in zip(st_new, st_ref):
            assert torch.equal(a, b), f"call {call}: resolver state differs"
        assert torch.equal(m_new[0], m_ref[0]) and torch.equal(m_new[1], m_ref[1]), f"call {call}: KV rows differ"
    assert int(st_ref[5].item()) < slots  # the calls did install rows


def test_noalloc_resolver_rejects_calls_above_its_fixed_capacity():
    import asu_ascend_b200

    asu_ascend_b200.load()
    from asu_ascend_b200._lib import ASU_ERR_NOALLOC_CAPACITY, RESOLVER_NOALLOC_MAX_TOPK, lib

    n = RESOLVER_NOALLOC_MAX_TOPK + 1
    topk = torch.zeros(n, dtype=torch.int32, device=DEV)
    one = torch.zeros(4, dtype=torch.int32, device=DEV)
    resolved = torch.full((n,), -7, dtype=torch.int32, device=DEV)
    rc = lib.asu_kv_resolver_noalloc(None, topk.data_ptr(), n, one.data_ptr(), one.data_ptr(), one.data_ptr(),
                                     one.data_ptr(), one.data_ptr(), one.data_ptr(), 4, one.data_ptr(), 1, None,
                                     None, None, None, 0, 0, 4, 4, 4, 4, 1, resolved.data_ptr(), None)
    assert rc == ASU_ERR_NOALLOC_CAPACITY
    assert b"scratch" in lib.asu_status_string(rc)
    torch.cuda.synchronize()
    assert (resolved == -7).all()  # nothing was launched
