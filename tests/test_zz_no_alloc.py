"""The resolver entry point that allocates nothing (asu_kv_resolver_noalloc).

It exists for callers that cannot allocate device memory while they resolve a layer: an
engine whose HBM is pre-reserved for its KV-block pool and which forbids cudaMalloc inside
the decode loop, or a C / FFI host without a caching allocator.  Instead of a caller-provided
workspace it keeps its install list in a fixed scratch array inside the library.

These checks call it through the C ABI and compare it, for two calls in a row on the same
state, bit-exact with both asu_kv_resolver_do (the entry point with a caller-provided
workspace, run on an identical copy of the state) and the serial oracle.  The cases cover
both ways the installed rows are copied:

* row pairs of up to 1280 bytes with 16-byte-aligned starts, which the resolve cluster copies
  itself (the scratch array holds the install list but nothing reads it back);
* larger or only 4-byte-aligned row pairs, which the copy kernel copies after reading the
  install count and the (source row, slot) pairs back from the scratch array -- one copy
  launch per 2048 entries, so top-k sizes above 2048 read entries at later offsets;

with top-k sizes of one chunk, several chunks (duplicates inside and across chunks) and
exactly the fixed capacity.  They hold when this file runs alone in a fresh process and after
the other tests (the first call on the device does the one-time set-up).  The file name makes
pytest collect it last.
"""

import ctypes

import numpy as np
import pytest
import torch

from oracle import asu_oracle as O

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


def _lib():
    import asu_ascend_b200

    asu_ascend_b200.load()
    from asu_ascend_b200 import _lib as L

    return L


def _call(lib, use_noalloc, topk, st, kv, dst, actual, bs):
    """One resolver call through the C ABI; returns the resolved slots."""
    ts, rec, hs, own, stack, cnt, bt = st
    kv0, kv1 = kv
    m0, m1 = dst
    resolved = torch.full(topk.shape, -7, dtype=torch.int32, device=DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    common = [topk.data_ptr(), topk.numel(), ts.data_ptr(), rec.data_ptr(), hs.data_ptr(), own.data_ptr(),
              stack.data_ptr(), cnt.data_ptr(), stack.numel(), bt.data_ptr(), bt.numel(), kv0.data_ptr(),
              kv1.data_ptr(), m0.data_ptr(), m1.data_ptr(), kv0.shape[1], kv1.shape[1],
              min(kv0.shape[0], kv1.shape[0]), min(m0.shape[0], m1.shape[0], own.numel()), ts.numel(), actual, bs,
              resolved.data_ptr()]
    if use_noalloc:
        rc = lib.asu_kv_resolver_noalloc(stream, *common, status.data_ptr())
    else:
        ws = torch.empty(int(lib.asu_kv_resolver_workspace_bytes(topk.numel())), dtype=torch.uint8, device=DEV)
        rc = lib.asu_kv_resolver_do(stream, *common, ws.data_ptr(), status.data_ptr())
    assert rc == 0, lib.asu_status_string(rc)
    torch.cuda.synchronize()
    assert status.item() == 0
    return resolved


def _byte_rows(rng, rows, width):
    return rng.integers(0, 256, (rows, width), dtype=np.uint8)


# (kv0 row bytes, kv1 row bytes, top-k sizes of the two calls)
CASES = [
    (1024, 128, (2048, 2048)),     # 1152-byte 16-aligned pairs: copied in the resolve cluster
    (720, 8, (2048, 6000)),        # 4-byte aligned: copy kernel, 1 then 3 copy launches
    (1024, 512, (6000, 16384)),    # 1536 bytes: copy kernel, 3 then 8 copy launches (the capacity)
    (640, 16, (16384, 16384)),     # 656-byte DSA rows in the cluster, the capacity twice
]


@pytest.mark.parametrize("w0,w1,sizes", CASES)
def test_noalloc_resolver_matches_workspace_resolver_and_oracle(w0, w1, sizes):
    L = _lib()
    lib = L.lib
    assert max(sizes) <= L.RESOLVER_NOALLOC_MAX_TOPK
    rng = np.random.Generator(np.random.PCG64(2027 + w0 + w1))
    max_seq, bs = 65536, 64
    slots = 24576
    actual, prefix = 60000, 59700
    nblk = max_seq // bs
    bt = rng.permutation(nblk + 16)[:nblk].astype(np.int32)
    ts, rec, hs, own, stack, cnt = O.reset_state(max_seq, slots, bs, actual, prefix, bt)
    src0 = _byte_rows(rng, (nblk + 16) * bs, w0)
    src1 = _byte_rows(rng, (nblk + 16) * bs, w1)
    dst0 = np.zeros((slots, w0), np.uint8)
    dst1 = np.zeros((slots, w1), np.uint8)
    # some tokens resident before the first call
    warm = rng.choice(actual, 700, replace=False).astype(np.int32)
    O.resolve_kv_slots_single_req(warm, actual, ts, rec, hs, own, stack, cnt, bt, src0, src1, dst0, dst1, bs)

    def dev(a):
        return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)

    st_ws = [dev(a) for a in (ts, rec, hs, own, stack, cnt, bt)]
    st_na = [t.clone() for t in st_ws]
    kv = (dev(src0), dev(src1))
    m_ws = (dev(dst0), dev(dst1))
    m_na = (m_ws[0].clone(), m_ws[1].clone())
    for call, n in enumerate(sizes):
        # a narrow key range for the larger calls gives duplicates inside and across chunks;
        # the newest token is always asked for (a TAIL_HBM token)
        span = min(actual, 3 * n)
        topk = rng.integers(actual - span, actual, n).astype(np.int32)
        topk[n // 2: n // 2 + 40] = topk[:40]
        topk[-1] = actual - 1
        exp = O.resolve_kv_slots_single_req(topk, actual, ts, rec, hs, own, stack, cnt, bt, src0, src1, dst0, dst1,
                                            bs)
        t = dev(topk)
        want = _call(lib, False, t, st_ws, kv, m_ws, actual, bs)
        got = _call(lib, True, t, st_na, kv, m_na, actual, bs)
        ctx = f"rows ({w0},{w1}), call {call}, top-k {n}"
        np.testing.assert_array_equal(got.cpu().numpy(), exp, err_msg=ctx)
        assert torch.equal(got, want), ctx
        for a, b, ref in zip(st_na[:6], st_ws[:6], (ts, rec, hs, own, stack, cnt)):
            assert torch.equal(a, b), ctx
            np.testing.assert_array_equal(a.cpu().numpy(), ref, err_msg=ctx)
        for a, b, ref in zip(m_na, m_ws, (dst0, dst1)):
            assert torch.equal(a, b), ctx
            np.testing.assert_array_equal(a.cpu().numpy(), ref, err_msg=ctx)
    assert int(cnt[0]) < slots - 700  # the calls did install rows


def test_noalloc_resolver_rejects_calls_above_its_fixed_capacity():
    L = _lib()
    lib = L.lib
    n = L.RESOLVER_NOALLOC_MAX_TOPK + 1
    topk = torch.zeros(n, dtype=torch.int32, device=DEV)
    one = torch.zeros(4, dtype=torch.int32, device=DEV)
    resolved = torch.full((n,), -7, dtype=torch.int32, device=DEV)
    rc = lib.asu_kv_resolver_noalloc(None, topk.data_ptr(), n, one.data_ptr(), one.data_ptr(), one.data_ptr(),
                                     one.data_ptr(), one.data_ptr(), one.data_ptr(), 4, one.data_ptr(), 1, None,
                                     None, None, None, 0, 0, 4, 4, 4, 4, 1, resolved.data_ptr(), None)
    assert rc == L.ASU_ERR_NOALLOC_CAPACITY
    assert b"scratch" in lib.asu_status_string(rc)
    torch.cuda.synchronize()
    assert (resolved == -7).all()  # nothing was launched
