"""Host-pool producer on the GPU: the write-back kernel's bytes, and the producer -> swap-in
round trip (rows written back by the GPU come back into the HBM slot pool unchanged)."""

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


def test_writeback_rows_and_skips():
    from asu_ascend_b200.host_pool import HostRowPool

    pool = HostRowPool(rows=5000, row_bytes=656)
    full = np.frombuffer((ctypes.c_uint8 * pool.nbytes).from_address(pool._host), np.uint8).reshape(5000, pool.pitch)
    full[:] = 7  # rows and their padding
    g = torch.Generator(device=DEV).manual_seed(2)
    src = torch.randint(0, 256, (3000, 656), dtype=torch.uint8, device=DEV, generator=g)
    dst = torch.randperm(5000, device=DEV, generator=g)[:3000].to(torch.int32)
    dst[::17] = -1  # skipped items
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    pool.writeback(src, dst, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    d, s = dst.cpu().numpy(), src.cpu().numpy()
    keep = d >= 0
    np.testing.assert_array_equal(pool.array[d[keep]], s[keep])
    untouched = np.setdiff1d(np.arange(5000), d[keep])
    assert (pool.array[untouched] == 7).all()
    # a written row's padding up to the 768-byte pitch is zeroed (rows go out as whole lines);
    # the other rows' padding is untouched
    assert pool.pitch == 768 and (full[d[keep], 656:] == 0).all() and (full[untouched, 656:] == 7).all()
    # gathered sources and out-of-range rows
    idx = torch.tensor([5, 2999, 0, 3000, 1], dtype=torch.int32, device=DEV)
    rows = torch.tensor([10, 11, 5000, 12, -1], dtype=torch.int32, device=DEV)
    status.zero_()
    pool.writeback(src, rows, src_index=idx, status=status)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(pool.array[[10, 11]], s[[5, 2999]])
    from asu_ascend_b200._lib import ST_BAD_SOURCE, ST_BAD_STATE
    assert int(status.item()) == ST_BAD_SOURCE | ST_BAD_STATE
    pool.close()


def test_producer_write_back_then_swap_in_round_trip():
    from asu_ascend_b200 import kv_store as KV
    from asu_ascend_b200.host_pool import HostRowPool
    from asu_ascend_b200.lru import LruSlotPools
    from asu_ascend_b200.workloads import LocalityTrace

    tokens, row, layers = 4096, 656, 2
    pool = HostRowPool(rows=4 * tokens, row_bytes=row)
    store = KV.HostKVStore(pool.array, tokens_per_extent=tokens, pool=pool)
    g = torch.Generator(device=DEV).manual_seed(4)
    prefill = [torch.randint(0, 256, (tokens, row), dtype=torch.uint8, device=DEV, generator=g) for _ in range(layers)]
    for layer in range(layers):  # prefill written back in two ranges per layer
        store.write_back(KV.KV_MLA_TOKEN, "req-a", layer, 0, prefill[layer][:1000])
        store.write_back(KV.KV_MLA_TOKEN, "req-a", layer, 1000, prefill[layer][1000:])
    torch.cuda.synchronize()
    assert store.size(KV.KV_MLA_TOKEN) == layers * tokens
    assert store.get(KV.KV_MLA_TOKEN, KV.make_key("req-a", 1, 1234)) == prefill[1][1234].cpu().numpy().tobytes()

    # decode: layer 1's top-k swapped in from the records the producer wrote
    rec = torch.from_numpy(store.record_rows(KV.KV_MLA_TOKEN, "req-a", 1, tokens)[None, :]).to(DEV)
    lru = LruSlotPools(1, tokens, 1024, 256, 512, device=DEV)
    slot_pool = torch.zeros((1, 1024, row), dtype=torch.uint8, device=DEV)
    tr = LocalityTrace(1, tokens, topk=512, seed=8)
    for _ in range(4):
        q = torch.from_numpy(tr.step()).to(DEV)
        out = lru.step(q)
        pool.swapin(rec, q, out.slot, out.install, slot_pool)
        torch.cuda.synchronize()
        got = slot_pool[0, out.slot[0].long()]
        assert torch.equal(got, prefill[1][q[0].long()])
    pool.close()


def test_writeback_full_prefill_size():
    """The write-back workload's size: a 128K-token prefill of 656-byte rows for each of 4 layers,
    written into consecutive extents of a pinned pool under their MicroKV keys; every row of
    every layer reads back unchanged (the whole pool, not a sample)."""
    from asu_ascend_b200 import kv_store as KV
    from asu_ascend_b200.host_pool import HostRowPool

    tokens, row, layers = 131072, 656, 4
    pool = HostRowPool(rows=layers * tokens, row_bytes=row)
    store = KV.HostKVStore(pool.array, tokens_per_extent=tokens, pool=pool)
    g = torch.Generator(device=DEV).manual_seed(8)
    src = [torch.randint(0, 256, (tokens, row), dtype=torch.uint8, device=DEV, generator=g) for _ in range(layers)]
    for layer in range(layers):
        store.write_back(KV.KV_MLA_TOKEN, "prefill-full", layer, 0, src[layer])
    torch.cuda.synchronize()
    for layer in range(layers):
        base = store.extent_base(KV.KV_MLA_TOKEN, "prefill-full", layer)
        np.testing.assert_array_equal(pool.array[base:base + tokens], src[layer].cpu().numpy())
    for t in (0, 65535, tokens - 1):
        assert store.get(KV.KV_MLA_TOKEN, KV.make_key("prefill-full", 3, t)) == src[3][t].cpu().numpy().tobytes()
    pool.close()
