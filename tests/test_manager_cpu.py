"""Resolver state manager (patch 0003 ASUFullKVCacheManagerFunctional) host-side behaviour on CPU:
feature gate, per-layer allocation, argument errors.  The state reset itself is a CUDA kernel
(tested in test_gpu_manager.py)."""

import pytest
import torch

from asu_ascend_b200 import manager as M


def test_feature_gate_defaults_off(monkeypatch):
    """patch/0003 tests/ut/ops/test_asu_kv_cache_manager.py (patch lines 82-89) restated."""
    monkeypatch.delenv(M.ASU_KV_CACHE_ENABLE_ENV, raising=False)
    assert M.is_asu_kv_cache_enabled() is False
    monkeypatch.setenv(M.ASU_KV_CACHE_ENABLE_ENV, "1")
    assert M.is_asu_kv_cache_enabled() is True
    monkeypatch.setenv(M.ASU_KV_CACHE_SLOT_COUNT_ENV, "0")
    with pytest.raises(ValueError):
        M.get_configured_managed_slot_count()


def _caches(dtype, blocks=2):
    return {
        "layers.0.self_attn": (torch.zeros((blocks, 4, 1, 8), dtype=dtype), torch.zeros((blocks, 4, 1, 2), dtype=dtype),
                               torch.zeros((blocks, 4, 1, 4), dtype=dtype)),
        "layers.1.self_attn": (torch.zeros((blocks, 4, 1, 8), dtype=dtype), torch.zeros((blocks, 4, 1, 2), dtype=dtype),
                               torch.zeros((blocks, 4, 1, 4), dtype=dtype)),
        "not_a_cache": torch.zeros(3),
    }


def test_manager_allocates_per_layer_managed_cache_from_pa_cache():
    """patch lines 92-121 restated."""
    mgr = M.ASUFullKVCacheManagerFunctional.from_kv_caches(_caches(torch.bfloat16), max_seq_len=8, block_size=4,
                                                           managed_slot_count=6, enabled=True)
    l0 = mgr.get_layer_context("layers.0.self_attn")
    l1 = mgr.get_layer_context("layers.1.self_attn")
    assert not mgr.has_layer("not_a_cache")
    assert l0.managed_kv_cache_0.shape == (6, 1, 8)
    assert l0.managed_kv_cache_1.shape == (6, 1, 2)
    assert l0.managed_kv_cache_0.dtype is torch.bfloat16
    assert l1.managed_kv_cache_0.data_ptr() != l0.managed_kv_cache_0.data_ptr()
    assert l0.free_slot_count.item() == 6
    assert l0.free_slot_stack.tolist() == [0, 1, 2, 3, 4, 5]
    assert l0.token_state.dtype == torch.int32 and l0.token_state.tolist() == [-1] * 8
    v0, v1 = l0.original_kv_cache_views(_caches(torch.bfloat16)["layers.0.self_attn"])
    assert v0.shape == (8, 1, 8) and v1.shape == (8, 1, 2)


def test_disabled_manager_is_a_no_op():
    mgr = M.ASUFullKVCacheManagerFunctional.from_kv_caches(_caches(torch.float16), 8, 4, enabled=False)
    assert not mgr.enabled and not mgr.has_layer("layers.0.self_attn")
    mgr.reset_single_request("r", 4, 2, torch.zeros(1, 2, dtype=torch.int32))
    mgr.mark_decode_token(3)


def test_reset_argument_errors_match_the_reference():
    mgr = M.ASUFullKVCacheManagerFunctional.from_kv_caches(_caches(torch.float16), 8, 4, managed_slot_count=6,
                                                           enabled=True)
    ctx = mgr.get_layer_context("layers.0.self_attn")
    bt = torch.tensor([[1, 0]], dtype=torch.int32)
    with pytest.raises(ValueError):
        ctx.reset_state("r", -1, 0, bt)
    with pytest.raises(ValueError):
        ctx.reset_state("r", 4, 5, bt)
    with pytest.raises(RuntimeError):
        ctx.reset_state("r", 9, 2, bt)
    with pytest.raises(RuntimeError, match="CUDA"):  # no CPU implementation of the state reset
        ctx.reset_state("r", 6, 4, bt)
    with pytest.raises(RuntimeError):
        ctx.mark_decode_token(8)


def test_sparse_mla_contexts_have_one_managed_cache():
    from asu_ascend_b200 import sparse_mla as S

    caches = {"layers.0.self_attn": torch.zeros((3, 64, 576), dtype=torch.bfloat16),
              "layers.1.self_attn": torch.zeros((3, 64, 656), dtype=torch.uint8),
              "indexer": torch.zeros((3, 64))}
    mgr = S.contexts_for_mla(caches, max_seq_len=192, block_size=64, managed_slot_count=50, enabled=True)
    assert mgr.has_layer("layers.0.self_attn") and mgr.has_layer("layers.1.self_attn") and not mgr.has_layer("indexer")
    c0 = mgr.get_layer_context("layers.0.self_attn")
    # rows padded to whole 64-row pages for FlashMLA's paged fp8 decode; the state keeps 50 slots
    assert c0.managed_kv_cache_0.shape == (64, 576) and c0.managed_kv_cache_1.numel() == 0
    assert c0.slot_owner_token.numel() == 50 and c0.free_slot_stack.numel() == 50
    assert S.managed_kv_view(c0).shape == (64, 1, 576)
    c1 = mgr.get_layer_context("layers.1.self_attn")
    assert c1.managed_kv_cache_0.dtype == torch.uint8 and c1.managed_kv_cache_0.shape == (64, 656)
    assert S.managed_paged_view(c1).shape == (1, 64, 656)
    with pytest.raises(RuntimeError, match="int32"):
        S.resolve_topk(c0, torch.zeros((1, 8), dtype=torch.int64), torch.zeros(3, dtype=torch.int32),
                       caches["layers.0.self_attn"])
    with pytest.raises(RuntimeError, match="rows"):
        S.resolve_topk(c0, torch.zeros((1, 8), dtype=torch.int32), torch.zeros(3, dtype=torch.int32),
                       caches["layers.1.self_attn"])
