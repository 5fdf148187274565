"""Resolver state manager on the GPU: the reset kernel against the reference manager's outputs,
and a full single-request decode flow (reset -> resolve -> mark decode token -> resolve)
against the oracle."""

import numpy as np
import pytest
import torch

from oracle import asu_oracle as O

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


def test_reset_matches_reference_unit_vector():
    """patch/0003 test_manager_resets_single_request_state_before_decode (patch lines 124-151)."""
    from asu_ascend_b200 import manager as M

    caches = {"layers.0.self_attn": (torch.zeros((3, 4, 1, 8), dtype=torch.float16, device=DEV),
                                     torch.zeros((3, 4, 1, 2), dtype=torch.float16, device=DEV),
                                     torch.zeros((3, 4, 1, 4), dtype=torch.float16, device=DEV))}
    mgr = M.ASUFullKVCacheManagerFunctional.from_kv_caches(caches, max_seq_len=12, block_size=4,
                                                           managed_slot_count=12, enabled=True)
    mgr.reset_single_request("req-1", 6, 4, torch.tensor([[2, 0, 1]], dtype=torch.int32))
    layer = mgr.get_layer_context("layers.0.self_attn")
    assert layer.req_id == "req-1" and layer.actual_seq_len == 6 and layer.managed_prefix_len == 4
    assert layer.token_state[:8].tolist() == [M.ASU_ONLY] * 4 + [M.TAIL_HBM] * 2 + [M.INVALID] * 2
    assert layer.asu_record_addr[:4].tolist() == [8, 9, 10, 11]
    assert layer.free_slot_count.item() == 12
    assert layer.slot_owner_token[:3].tolist() == [M.INVALID] * 3
    assert layer.free_slot_stack.tolist() == list(range(12))


def test_reset_matches_reference_golden(golden):
    from asu_ascend_b200 import manager as M

    g = golden("resolver")
    max_seq, slots, bs, actual, prefix = (int(v) for v in g["meta"])
    nblk = g["block_table"].size
    caches = {"l": (torch.zeros((nblk + 8, bs, 1, 8), dtype=torch.bfloat16, device=DEV),
                    torch.zeros((nblk + 8, bs, 1, 4), dtype=torch.bfloat16, device=DEV))}
    mgr = M.ASUFullKVCacheManagerFunctional.from_kv_caches(caches, max_seq, bs, managed_slot_count=slots,
                                                           enabled=True)
    mgr.reset_single_request("r", actual, prefix, torch.from_numpy(g["block_table"][None, :]))
    ctx = mgr.get_layer_context("l")
    np.testing.assert_array_equal(ctx.token_state.cpu().numpy(), g["reset_token_state"])
    np.testing.assert_array_equal(ctx.asu_record_addr.cpu().numpy(), g["reset_record"])


def test_decode_flow_against_oracle():
    """Reset, resolve top-k, append a decode token, resolve again -- state, slots and KV rows exact."""
    import asu_ascend_b200

    asu_ascend_b200.load()
    from asu_ascend_b200 import manager as M

    rng = np.random.Generator(np.random.PCG64(12))
    max_seq, slots, bs, actual, prefix = 4096, 2048, 16, 3000, 2999
    nblk = (max_seq + bs - 1) // bs
    bt = rng.permutation(nblk + 8)[:nblk].astype(np.int32)
    kv0 = torch.randn(nblk + 8, bs, 1, 64, device=DEV).to(torch.bfloat16)
    kv1 = torch.randn(nblk + 8, bs, 1, 16, device=DEV).to(torch.bfloat16)
    mgr = M.ASUFullKVCacheManagerFunctional.from_kv_caches({"l": (kv0, kv1)}, max_seq, bs,
                                                           managed_slot_count=slots, enabled=True)
    ctx = mgr.get_layer_context("l")
    ctx.managed_kv_cache_0.zero_()
    ctx.managed_kv_cache_1.zero_()
    mgr.reset_single_request("r", actual, prefix, torch.from_numpy(bt[None, :]))
    o0, o1 = ctx.original_kv_cache_views((kv0, kv1))
    ts, rec, hs, own, stack, cnt = O.reset_state(max_seq, slots, bs, actual, prefix, bt)
    e0 = np.zeros(ctx.managed_kv_cache_0.shape, np.float32)
    e1 = np.zeros(ctx.managed_kv_cache_1.shape, np.float32)
    s0, s1 = o0.float().cpu().numpy(), o1.float().cpu().numpy()
    seq = actual
    for step in range(4):
        topk = rng.integers(0, seq, (1, 1, 512)).astype(np.int32)
        topk[0, 0, -1] = seq - 1  # the newest token is always attended
        out = torch.ops._C_ascend.npu_asu_resolve_kv_slots_single_req(
            torch.from_numpy(topk).to(DEV), ctx.actual_seq_len, ctx.managed_prefix_len, ctx.token_state,
            ctx.asu_record_addr, ctx.hbm_slot_of_token, ctx.slot_owner_token, ctx.free_slot_stack,
            ctx.free_slot_count, torch.from_numpy(bt[None, :]).to(DEV), o0, o1, ctx.managed_kv_cache_0,
            ctx.managed_kv_cache_1, bs)
        exp = O.resolve_kv_slots_single_req(topk, seq, ts, rec, hs, own, stack, cnt, bt, s0, s1, e0, e1, bs)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(out.cpu().numpy(), exp)
        np.testing.assert_array_equal(ctx.token_state.cpu().numpy(), ts)
        np.testing.assert_array_equal(ctx.hbm_slot_of_token.cpu().numpy(), hs)
        np.testing.assert_array_equal(ctx.slot_owner_token.cpu().numpy(), own)
        assert int(ctx.free_slot_count.item()) == int(cnt[0])
        np.testing.assert_array_equal(ctx.managed_kv_cache_0.float().cpu().numpy(), e0)
        np.testing.assert_array_equal(ctx.managed_kv_cache_1.float().cpu().numpy(), e1)
        mgr.mark_decode_token(seq)  # the next decode step appends token `seq`
        ts[seq] = O.TAIL_HBM
        seq += 1


def test_managed_rows_equal_original_rows_decode_case():
    """patch/0004 test_indexer_asu_management_sfa_matches_origin_sfa_decode restated at the
    data level: sparse attention over (managed cache, resolved slots) sees exactly the rows
    that sparse attention over (paged cache, block table, top-k) sees, and a second resolve
    of the same top-k is idempotent (same slots, no slot consumed)."""
    from asu_ascend_b200 import manager as M

    g = torch.Generator().manual_seed(4)
    bs, actual, prefix, blocks = 128, 2048 + 77, 2048, 24
    kv = (torch.randn(blocks, bs, 1, 512, generator=g).to(torch.bfloat16).to(DEV),
          torch.randn(blocks, bs, 1, 64, generator=g).to(torch.bfloat16).to(DEV),
          torch.randn(blocks, bs, 1, 128, generator=g).to(torch.bfloat16).to(DEV))
    bt = torch.randperm(blocks, generator=g)[: (actual + bs - 1) // bs].to(torch.int32)[None, :].to(DEV)
    mgr = M.ASUFullKVCacheManagerFunctional.from_kv_caches({"layers.0.self_attn": kv}, max_seq_len=actual,
                                                           block_size=bs, managed_slot_count=actual, enabled=True)
    mgr.reset_single_request("decode-req-0", actual, prefix, bt)
    ctx = mgr.get_layer_context("layers.0.self_attn")
    o0, o1 = ctx.original_kv_cache_views(kv)
    topk = torch.randperm(actual, generator=g)[:2048].to(torch.int32).reshape(1, 1, 2048).to(DEV)

    def resolve():
        return torch.ops._C_ascend.npu_asu_resolve_kv_slots_single_req(
            original_topk_indices=topk, actual_seq_len=ctx.actual_seq_len, managed_prefix_len=ctx.managed_prefix_len,
            token_state=ctx.token_state, asu_record_addr=ctx.asu_record_addr, hbm_slot_of_token=ctx.hbm_slot_of_token,
            slot_owner_token=ctx.slot_owner_token, free_slot_stack=ctx.free_slot_stack,
            free_slot_count=ctx.free_slot_count, original_block_table=bt, original_kv_cache_0=o0,
            original_kv_cache_1=o1, managed_kv_cache_0=ctx.managed_kv_cache_0,
            managed_kv_cache_1=ctx.managed_kv_cache_1, block_size=ctx.block_size)

    slots = resolve()
    assert slots.shape == topk.shape
    tok = topk.reshape(-1).long()
    paged_row = bt.reshape(-1).long()[tok // bs] * bs + tok % bs
    s = slots.reshape(-1).long()
    assert torch.equal(ctx.managed_kv_cache_0[s], o0[paged_row])
    assert torch.equal(ctx.managed_kv_cache_1[s], o1[paged_row])
    left = int(ctx.free_slot_count.item())
    assert left == actual - 2048
    again = resolve()
    assert int(ctx.free_slot_count.item()) == left
    assert torch.equal(again, slots)


def test_decode_flow_at_full_context_against_oracle():
    """The decode workload's size: a 131072-token context with 130944 ASU-managed prefix tokens and
    a paged tail, the manager's default managed slot count (one per context position), bf16 rows
    of 512 + 64 elements, a 2048-entry top-k with step-to-step reuse and the newest token always
    included; three decode steps, state arrays, slots and every managed row exact."""
    import asu_ascend_b200

    asu_ascend_b200.load()
    from asu_ascend_b200 import manager as M

    rng = np.random.Generator(np.random.PCG64(21))
    max_seq, bs = 131072, 64
    actual, prefix = 131000, 130944
    nblk = max_seq // bs
    bt = rng.permutation(nblk + 16)[:nblk].astype(np.int32)
    kv0 = torch.randn(nblk + 16, bs, 1, 512, device=DEV).to(torch.bfloat16)
    kv1 = torch.randn(nblk + 16, bs, 1, 64, device=DEV).to(torch.bfloat16)
    mgr = M.ASUFullKVCacheManagerFunctional.from_kv_caches({"l": (kv0, kv1)}, max_seq, bs, enabled=True)
    ctx = mgr.get_layer_context("l")
    ctx.managed_kv_cache_0.zero_()
    ctx.managed_kv_cache_1.zero_()
    mgr.reset_single_request("r", actual, prefix, torch.from_numpy(bt[None, :]))
    o0, o1 = ctx.original_kv_cache_views((kv0, kv1))
    slots = ctx.managed_slot_count
    ts, rec, hs, own, stack, cnt = O.reset_state(max_seq, slots, bs, actual, prefix, bt)
    u16 = lambda t: t.view(torch.int16).cpu().numpy().view(np.uint16)  # noqa: E731
    s0, s1 = u16(o0), u16(o1)
    e0 = np.zeros((slots,) + s0.shape[1:], np.uint16)
    e1 = np.zeros((slots,) + s1.shape[1:], np.uint16)
    seq = actual
    prev = rng.choice(seq, 2048, replace=False)
    for step in range(3):
        keep = rng.choice(prev, 1434, replace=False)
        fresh = rng.integers(0, seq, 2048 - keep.size)
        topk = np.concatenate([keep, fresh]).astype(np.int32)[None, None, :]
        topk[0, 0, -1] = seq - 1
        prev = topk.reshape(-1)
        out = torch.ops._C_ascend.npu_asu_resolve_kv_slots_single_req(
            torch.from_numpy(topk).to(DEV), ctx.actual_seq_len, ctx.managed_prefix_len, ctx.token_state,
            ctx.asu_record_addr, ctx.hbm_slot_of_token, ctx.slot_owner_token, ctx.free_slot_stack,
            ctx.free_slot_count, torch.from_numpy(bt[None, :]).to(DEV), o0, o1, ctx.managed_kv_cache_0,
            ctx.managed_kv_cache_1, bs)
        exp = O.resolve_kv_slots_single_req(topk, seq, ts, rec, hs, own, stack, cnt, bt, s0, s1, e0, e1, bs)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(out.cpu().numpy(), exp)
        np.testing.assert_array_equal(ctx.token_state.cpu().numpy(), ts)
        np.testing.assert_array_equal(ctx.hbm_slot_of_token.cpu().numpy(), hs)
        np.testing.assert_array_equal(ctx.slot_owner_token.cpu().numpy(), own)
        assert int(ctx.free_slot_count.item()) == int(cnt[0])
        np.testing.assert_array_equal(u16(ctx.managed_kv_cache_0), e0)
        np.testing.assert_array_equal(u16(ctx.managed_kv_cache_1), e1)
        mgr.mark_decode_token(seq)
        ts[seq] = O.TAIL_HBM
        seq += 1
