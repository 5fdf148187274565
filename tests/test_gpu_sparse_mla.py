"""FlashMLA-sparse decode fed by resolver slots (the B200 counterpart of the reference's
patch/0004 decode parity case, patch lines 265-293): attention over (managed cache, resolved
slots) equals attention over (paged cache, block-table slots) within 2e-2, and resolving the
same top-k again consumes no slot and returns the same slots."""

import numpy as np
import pytest
import torch

from oracle import asu_oracle as O

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


def _paged_slots(topk, bt, bs):
    """vLLM's triton_convert_req_index_to_global_index for one request (sparse_utils.py:97-105)."""
    t = topk.long()
    return torch.where(t >= 0, bt.long()[t.clamp(min=0) // bs] * bs + t.clamp(min=0) % bs, -1).to(torch.int32)


def _case(seed, seq, bs=64, tokens=2, topk=2048, pad=0, row=576, dtype=torch.bfloat16):
    g = torch.Generator().manual_seed(seed)
    nblk = (seq + bs - 1) // bs
    phys = nblk + 8
    if dtype == torch.uint8:
        kv = torch.randint(0, 256, (phys, bs, row), generator=g, dtype=torch.uint8)
    else:
        kv = (torch.randn(phys, bs, row, generator=g) * 0.5).to(dtype)
    bt = torch.randperm(phys, generator=g)[:nblk].to(torch.int32)
    k = min(seq, topk - pad)  # distinct positions per query token, then -1 padding
    idx = torch.full((tokens, topk), -1, dtype=torch.int32)
    for i in range(tokens):
        idx[i, :k] = torch.randperm(seq, generator=g)[:k].to(torch.int32)
    return kv.to(DEV), bt.to(DEV), idx.to(DEV)


@pytest.mark.parametrize("seq,pad", [(4133, 0), (1500, 2048 - 1500)])
def test_flashmla_sparse_decode_on_managed_cache_matches_paged(seq, pad):
    fm = pytest.importorskip("vllm.third_party.flashmla.flash_mla_interface")
    from asu_ascend_b200 import sparse_mla as S

    kv, bt, topk = _case(3, seq, pad=pad)
    q = (torch.randn(topk.shape[0], 128, 576, generator=torch.Generator().manual_seed(9)) * 0.5).to(torch.bfloat16)
    q = q.to(DEV)
    scale = 576 ** -0.5
    origin = fm.flash_mla_sparse_fwd(q, kv.view(-1, 1, 576), _paged_slots(topk, bt, 64).view(2, 1, -1), scale)[0]

    mgr = S.contexts_for_mla({"layers.0.self_attn": kv}, max_seq_len=seq, block_size=64, managed_slot_count=8192,
                             enabled=True)
    mgr.reset_single_request("decode-req-0", seq, seq - 37, bt)
    ctx = mgr.get_layer_context("layers.0.self_attn")
    out = S.sparse_mla_decode(q, ctx, topk, bt, kv, scale)
    torch.testing.assert_close(out.float(), origin.float(), rtol=2e-2, atol=2e-2)

    slots = S.resolve_topk(ctx, topk, bt, kv)  # all resident now
    left = int(ctx.free_slot_count.item())
    again = S.resolve_topk(ctx, topk, bt, kv)
    assert int(ctx.free_slot_count.item()) == left
    assert torch.equal(again, slots)
    assert bool((slots[topk < 0] == -1).all())
    valid = topk >= 0
    assert torch.equal(ctx.managed_kv_cache_0[slots[valid].long()],
                       kv.view(-1, 576)[_paged_slots(topk, bt, 64)[valid].long()])


def test_resolve_topk_fp8_ds_mla_rows_match_oracle():
    """656-byte fp8_ds_mla rows (uint8 cache): slots, state and row bytes equal the oracle's."""
    from asu_ascend_b200 import sparse_mla as S

    seq, bs = 6000, 64
    kv, bt, topk = _case(5, seq, tokens=1, topk=2048, pad=100, row=656, dtype=torch.uint8)
    mgr = S.contexts_for_mla({"l": kv}, max_seq_len=seq, block_size=bs, managed_slot_count=4096, enabled=True)
    mgr.reset_single_request("r", seq, seq - 20, bt)
    ctx = mgr.get_layer_context("l")
    ctx.managed_kv_cache_0.zero_()
    ts, rec, hs, own, stack, cnt = O.reset_state(seq, 4096, bs, seq, seq - 20, bt.cpu().numpy())
    src = kv.view(-1, 656).cpu().numpy()
    dst = np.zeros((4096, 656), np.uint8)
    empty_src = np.zeros((src.shape[0], 0), np.uint8)
    empty_dst = np.zeros((4096, 0), np.uint8)
    t = topk.cpu().numpy()[0]
    valid = t[t >= 0]
    exp = O.resolve_kv_slots_single_req(valid.reshape(1, -1), seq, ts, rec, hs, own, stack, cnt, bt.cpu().numpy(),
                                        src, empty_src, dst, empty_dst, bs)
    out = S.resolve_topk(ctx, topk, bt, kv)
    got = out.cpu().numpy()[0]
    np.testing.assert_array_equal(got[t >= 0], exp.reshape(-1))
    assert (got[t < 0] == -1).all()
    np.testing.assert_array_equal(ctx.token_state.cpu().numpy(), ts)
    np.testing.assert_array_equal(ctx.slot_owner_token.cpu().numpy(), own)
    assert int(ctx.free_slot_count.item()) == int(cnt[0])
    np.testing.assert_array_equal(ctx.managed_kv_cache_0.cpu().numpy(), dst)


def _impl(cls, heads, scale, topk_buffer):
    """An Impl with the fields its bf16 decode reads (no vLLM config is needed for those)."""
    impl = object.__new__(cls)
    impl.num_heads, impl.prefill_padding, impl.softmax_scale = heads, 128, scale
    impl.kv_cache_dtype, impl.topk_indices_buffer = "auto", topk_buffer
    return impl


# managed pools: one slot per context position (never evicts, the reference's setting), or an
# exact-LRU pool of 2560 slots keeping 2048 free over an 8000-token context (evicts every step)
POOLS = {"full": (None, None, 3000), "lru": (2560, 2048, 8000)}


@pytest.mark.parametrize("heads,pool", [(16, "full"), (128, "full"), (16, "lru"), (128, "lru")])
def test_vllm_subclass_decode_steps_match_stock_flashmla_sparse(heads, pool):
    """Decode steps of one request through ASUFlashMLASparseImpl.forward_mqa: each step's output
    equals vLLM's own FlashMLASparseImpl over the paged cache, the first step resets the manager,
    the next ones mark the new decode token, and a shared manager serves two layers -- over a pool
    with a slot per context position and over an exact-LRU pool smaller than the context."""
    pytest.importorskip("vllm.third_party.flashmla.flash_mla_interface")
    from types import SimpleNamespace

    from vllm.v1.attention.backends.mla.flashmla_sparse import FlashMLASparseImpl

    from asu_ascend_b200 import sparse_mla as S
    from asu_ascend_b200 import vllm_backend as V

    slots, target, seq0 = POOLS[pool]
    steps, bs, scale = (3 if target is None else 5), 64, 576 ** -0.5
    kv, bt, _ = _case(11, seq0 + steps, tokens=1)
    kv2 = kv.flip(0).contiguous()  # a second layer's cache
    g = torch.Generator().manual_seed(12)
    mgr = S.contexts_for_mla({"layers.0.attn": kv, "layers.1.attn": kv2}, max_seq_len=seq0 + steps, block_size=bs,
                             managed_slot_count=slots or seq0 + steps, enabled=True, free_target=target)
    assert mgr.get_layer_context("layers.0.attn").bounded == (target is not None)
    buf = torch.full((1, 2048), -1, dtype=torch.int32, device=DEV)
    asu = _impl(V.asu_flashmla_sparse_impl(), heads, scale, buf)
    stock = _impl(FlashMLASparseImpl, heads, scale, buf)
    for step in range(steps):
        seq = seq0 + step
        md = SimpleNamespace(num_reqs=1, max_query_len=1, num_actual_tokens=1, max_seq_len=seq,
                             block_table=bt.view(1, -1), req_id_per_token=torch.zeros(1, dtype=torch.int32, device=DEV),
                             block_size=bs, asu_kv_cache_manager=mgr, asu_req_id="req-0")
        topk = torch.full((2048,), -1, dtype=torch.int32)
        k = 1900 + 30 * step
        topk[:k] = torch.randperm(seq, generator=g)[:k].to(torch.int32)
        topk[0] = seq - 1  # the token this step decodes
        buf[0].copy_(topk)
        q = (torch.randn(1, heads, 576, generator=g) * 0.5).to(torch.bfloat16).to(DEV)
        for name, cache in (("layers.0.attn", kv), ("layers.1.attn", kv2)):
            got, _ = asu.forward_mqa(q, cache, md, SimpleNamespace(layer_name=name))
            exp, _ = stock.forward_mqa(q, cache, md, SimpleNamespace(layer_name=name))
            assert got.shape == exp.shape == (1, heads, 512)
            torch.testing.assert_close(got.float(), exp.float(), rtol=2e-2, atol=2e-2)
        ctx = mgr.get_layer_context("layers.1.attn")
        assert (ctx.req_id, ctx.actual_seq_len, ctx.managed_prefix_len) == ("req-0", seq, seq0 - 1)
    if target is not None:  # the pool did evict, and every layer keeps `target` slots free at each call
        assert int(ctx.free_slot_count.item()) < target


def _fp8_ds_mla_cache(seed, blocks, bs=64):
    """Valid 656-byte fp8_ds_mla rows: 512 e4m3 values, 4 f32 scales, 64 bf16 rope values."""
    g = torch.Generator().manual_seed(seed)
    n = blocks * bs
    nope = (torch.randn(n, 512, generator=g) * 2).to(torch.float8_e4m3fn).view(torch.uint8)
    scales = (torch.rand(n, 4, generator=g) * 0.5 + 0.25).view(torch.uint8)
    rope = (torch.randn(n, 64, generator=g) * 0.5).to(torch.bfloat16).view(torch.uint8)
    return torch.cat([nope, scales, rope], 1).view(blocks, bs, 656).to(DEV)


@pytest.mark.parametrize("layout,pool", [("mixed", "full"), ("separate", "full"), ("mixed", "lru"),
                                         ("separate", "lru")])
def test_vllm_subclass_fp8_decode_matches_stock_flashmla(layout, pool):
    """fp8_ds_mla caches: the subclass decodes with FlashMLA's fp8 sparse decode over the managed
    pages; each step equals vLLM's stock FlashMLASparseImpl (same kernel over the paged cache) in
    both fp8 batch layouts, with a managed pool that is not a whole number of pages (one slot per
    context position) and with an exact-LRU pool smaller than the context."""
    fi = pytest.importorskip("vllm.third_party.flashmla.flash_mla_interface")
    from types import SimpleNamespace

    from vllm.v1.attention.backends.mla.flashmla_sparse import FlashMLASparseImpl, FlashMLASparseMetadata

    from asu_ascend_b200 import sparse_mla as S
    from asu_ascend_b200 import vllm_backend as V

    slots, target, seq0 = POOLS[pool]
    seq0 = 2500 if target is None else seq0
    steps, bs, heads, scale = (3 if target is None else 5), 64, 16, 576 ** -0.5
    nblk = (seq0 + steps + bs - 1) // bs
    kv = _fp8_ds_mla_cache(21, nblk + 5)
    g = torch.Generator().manual_seed(22)
    bt = torch.randperm(nblk + 5, generator=g)[:nblk].to(torch.int32).to(DEV)
    mgr = S.contexts_for_mla({"layers.0.attn": kv}, max_seq_len=seq0 + steps, block_size=bs,
                             managed_slot_count=slots or seq0 + steps, enabled=True, free_target=target)
    assert mgr.get_layer_context("layers.0.attn").managed_kv_cache_0.shape[0] % bs == 0
    buf = torch.full((1, 2048), -1, dtype=torch.int32, device=DEV)
    impls = []
    for cls in (V.asu_flashmla_sparse_impl(), FlashMLASparseImpl):
        impl = _impl(cls, heads, scale, buf)
        impl.kv_cache_dtype, impl.fp8_decode_padded_heads, impl.kv_lora_rank = "fp8_ds_mla", 64, 512
        impls.append(impl)

    def kernel_meta():
        return FlashMLASparseMetadata.FP8KernelMetadata(
            scheduler_metadata=fi.get_mla_metadata()[0], dummy_block_table=torch.zeros(1, 1, dtype=torch.int32,
                                                                                         device=DEV),
            cache_lens=torch.full((1,), seq0 + steps, dtype=torch.int32, device=DEV))

    def fp8_meta():
        if layout == "mixed":
            return kernel_meta()
        P = FlashMLASparseMetadata.FP8SeparatePrefillDecode
        return P(num_decodes=1, num_decode_tokens=1,
                 decode=P.Decode(seq_lens=None, kernel_metadata=kernel_meta(), decode_query_len=1))

    for step in range(steps):
        seq = seq0 + step
        topk = torch.full((2048,), -1, dtype=torch.int32)
        k = 1800 + 40 * step
        topk[:k] = torch.randperm(seq, generator=g)[:k].to(torch.int32)
        topk[0] = seq - 1
        buf[0].copy_(topk)
        q = (torch.randn(1, heads, 576, generator=g) * 0.5).to(torch.bfloat16).to(DEV)
        outs = []
        for impl in impls:
            md = SimpleNamespace(num_reqs=1, max_query_len=1, num_actual_tokens=1, max_seq_len=seq,
                                 block_table=bt.view(1, -1),
                                 req_id_per_token=torch.zeros(1, dtype=torch.int32, device=DEV), block_size=bs,
                                 asu_kv_cache_manager=mgr, fp8_use_mixed_batch=layout == "mixed",
                                 fp8_extra_metadata=fp8_meta())
            outs.append(impl.forward_mqa(q, kv, md, SimpleNamespace(layer_name="layers.0.attn"))[0])
        got, exp = outs
        assert got.shape == exp.shape == (1, heads, 512)
        assert torch.isfinite(exp.float()).all()
        torch.testing.assert_close(got.float(), exp.float(), rtol=2e-2, atol=2e-2)
    ctx = mgr.get_layer_context("layers.0.attn")
    assert (ctx.actual_seq_len, ctx.managed_prefix_len) == (seq0 + steps - 1, seq0 - 1)
