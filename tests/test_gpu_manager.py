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


def test_batched_reset_and_mark_cover_every_layer_and_only_the_layer_asked():
    """The manager keeps every layer's state in one [layers, ...] bank: a request reset is one
    launch for all 61 layers and equals the reference reset in each; a decode token is marked in
    all layers at once; a context's own reset_state / mark_decode_token touch its layer only."""
    import asu_ascend_b200

    asu_ascend_b200.load()
    from asu_ascend_b200 import manager as M

    max_seq, bs, slots = 4096, 64, 1024
    nblk = max_seq // bs
    rng = np.random.Generator(np.random.PCG64(61))
    bt = rng.permutation(nblk + 4)[:nblk].astype(np.int32)
    caches = {f"layers.{i}.attn": (torch.zeros((nblk + 4, bs, 1, 8), dtype=torch.bfloat16, device=DEV),
                                   torch.zeros((nblk + 4, bs, 1, 4), dtype=torch.bfloat16, device=DEV))
              for i in range(61)}
    mgr = M.ASUFullKVCacheManagerFunctional.from_kv_caches(caches, max_seq, bs, managed_slot_count=slots,
                                                           enabled=True)
    ctxs = [mgr.get_layer_context(f"layers.{i}.attn") for i in range(61)]
    for c in ctxs:  # dirty every layer first
        c.token_state.fill_(7)
        c.free_slot_count.fill_(3)
        c.free_slot_stack.fill_(9)
    mgr.reset_single_request("req", 4000, 3990, torch.from_numpy(bt[None, :]))
    ts, rec, hs, own, stack, cnt = O.reset_state(max_seq, slots, bs, 4000, 3990, bt)
    for c in ctxs:
        np.testing.assert_array_equal(c.token_state.cpu().numpy(), ts)
        np.testing.assert_array_equal(c.asu_record_addr.cpu().numpy(), rec)
        np.testing.assert_array_equal(c.hbm_slot_of_token.cpu().numpy(), hs)
        np.testing.assert_array_equal(c.slot_owner_token.cpu().numpy(), own)
        np.testing.assert_array_equal(c.free_slot_stack.cpu().numpy(), stack)
        assert int(c.free_slot_count.item()) == slots
        assert (c.req_id, c.actual_seq_len, c.managed_prefix_len) == ("req", 4000, 3990)
    mgr.mark_decode_token(4000)
    assert all(int(c.token_state[4000].item()) == M.TAIL_HBM and c.actual_seq_len == 4001 for c in ctxs)
    ctxs[5].mark_decode_token(4001)
    assert [int(c.token_state[4001].item()) for c in ctxs].count(M.TAIL_HBM) == 1
    assert ctxs[5].actual_seq_len == 4002 and ctxs[6].actual_seq_len == 4001
    ctxs[7].token_state.fill_(7)
    ctxs[7].reset_state("other", 100, 50, torch.from_numpy(bt[None, :]))
    assert ctxs[7].req_id == "other" and ctxs[8].req_id == "req"
    assert int(ctxs[8].token_state[4000].item()) == M.TAIL_HBM
    ts7, rec7, *_ = O.reset_state(max_seq, slots, bs, 100, 50, bt)
    np.testing.assert_array_equal(ctxs[7].token_state.cpu().numpy(), ts7)
    np.testing.assert_array_equal(ctxs[7].asu_record_addr.cpu().numpy(), rec7)


def test_bounded_pool_decode_flow_at_full_context_against_oracle():
    """The decode workload's context over an exact-LRU pool of 8192 + 2048 slots (free target
    2048) through the manager and sparse_mla.resolve_topk: reset, twelve decode steps with a
    marked decode token each (the pool fills and then evicts), every state array, the recency
    order and every managed row against the oracle (the resolver composed with the LRU pool)."""
    import asu_ascend_b200

    asu_ascend_b200.load()
    from asu_ascend_b200 import sparse_mla as S

    rng = np.random.Generator(np.random.PCG64(22))
    max_seq, bs, slots, target = 131072, 64, 10240, 2048
    actual, prefix = 131000, 130944
    nblk = max_seq // bs
    bt = rng.permutation(nblk + 16)[:nblk].astype(np.int32)
    kv = torch.randint(0, 256, (nblk + 16, bs, 656), dtype=torch.uint8, device=DEV)
    mgr = S.contexts_for_mla({"l": kv}, max_seq, bs, managed_slot_count=slots, enabled=True, free_target=target)
    ctx = mgr.get_layer_context("l")
    assert ctx.bounded
    ctx.managed_kv_cache_0.zero_()
    gbt = torch.from_numpy(bt).to(DEV)
    mgr.reset_single_request("r", actual, prefix, gbt[None, :])
    ts, rec, hs, own, stack, cnt = O.reset_state(max_seq, slots, bs, actual, prefix, bt)
    order = np.full(slots, -1, np.int32)
    src = kv.view(-1, 656).cpu().numpy()
    dst = np.zeros((slots, 656), np.uint8)
    e_src, e_dst = np.zeros((src.shape[0], 0), np.uint8), np.zeros((slots, 0), np.uint8)
    seq = actual
    hot = rng.integers(0, seq, 40000)
    prev = rng.choice(hot, 2048)
    for step in range(12):
        q = np.where(rng.random(2048) < 0.5, prev, rng.choice(hot, 2048)).astype(np.int32)
        q[-1] = seq - 1
        prev = q
        exp, _ = O.resolve_kv_slots_lru(q, seq, ts, rec, hs, own, stack, cnt, order, target, bt, src, e_src, dst,
                                        e_dst, bs)
        out = S.resolve_topk(ctx, torch.from_numpy(q[None, :]).to(DEV), gbt, kv)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(out.cpu().numpy()[0], exp, err_msg=f"step {step}")
        np.testing.assert_array_equal(ctx.token_state.cpu().numpy(), ts)
        np.testing.assert_array_equal(ctx.hbm_slot_of_token.cpu().numpy(), hs)
        np.testing.assert_array_equal(ctx.slot_owner_token.cpu().numpy(), own)
        c = int(cnt[0])
        assert int(ctx.free_slot_count.item()) == c
        np.testing.assert_array_equal(ctx.lru_order.cpu().numpy()[: slots - c], order[: slots - c])
        np.testing.assert_array_equal(ctx.managed_kv_cache_0[:slots].cpu().numpy(), dst)
        mgr.mark_decode_token(seq)
        ts[seq] = O.TAIL_HBM
        seq += 1
    assert (own >= 0).sum() == slots - c
    hits, misses, installs, shortages, evictions = ctx.lru_stats.tolist()
    assert evictions > 0 and shortages == 0 and installs == misses and hits + misses == 12 * 2048
