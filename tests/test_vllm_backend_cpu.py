"""Host logic of the FlashMLA-sparse subclass (patch/0003 sfa_v1.py hunk, patch lines 461-499):
which batches take the ASU path, and when a layer resets the manager or marks a decode token."""

from types import SimpleNamespace

import pytest
import torch

from asu_ascend_b200 import vllm_backend as V


class FakeManager:
    def __init__(self, layers=("l0",), enabled=True):
        self.enabled = enabled
        self.ctx = {n: SimpleNamespace(req_id=None, actual_seq_len=0, managed_prefix_len=0) for n in layers}
        self.calls = []

    def has_layer(self, name):
        return name in self.ctx

    def get_layer_context(self, name):
        return self.ctx[name]

    def reset_single_request(self, req_id, actual_seq_len, managed_prefix_len, original_block_table):
        self.calls.append(("reset", req_id, actual_seq_len, managed_prefix_len, tuple(original_block_table.shape)))
        for c in self.ctx.values():
            c.req_id, c.actual_seq_len, c.managed_prefix_len = req_id, actual_seq_len, managed_prefix_len

    def mark_decode_token(self, token_id):
        self.calls.append(("mark", token_id))
        for c in self.ctx.values():
            c.actual_seq_len = max(c.actual_seq_len, token_id + 1)


def _md(**kw):
    base = dict(num_reqs=1, max_query_len=1, num_actual_tokens=1, max_seq_len=100,
                block_table=torch.zeros(3, 8, dtype=torch.int32))
    base.update(kw)
    return SimpleNamespace(**base)


def test_use_asu_kv_cache_conditions():
    m = FakeManager()
    assert V.use_asu_kv_cache(m, "l0", _md())
    assert not V.use_asu_kv_cache(None, "l0", _md())
    assert not V.use_asu_kv_cache(FakeManager(enabled=False), "l0", _md())
    assert not V.use_asu_kv_cache(m, "l1", _md())           # layer not managed
    assert not V.use_asu_kv_cache(m, None, _md())
    assert not V.use_asu_kv_cache(m, "l0", _md(max_query_len=4))   # prefill in the batch
    assert not V.use_asu_kv_cache(m, "l0", _md(num_reqs=2))
    assert not V.use_asu_kv_cache(m, "l0", _md(num_actual_tokens=2))


def test_manager_from_metadata_wins_over_class_attribute():
    impl = SimpleNamespace(asu_manager="class")
    assert V.asu_manager_of(impl, _md()) == "class"
    assert V.asu_manager_of(impl, _md(asu_kv_cache_manager="meta")) == "meta"


def test_prepare_resets_then_marks_then_resets_on_new_request():
    m = FakeManager(layers=("l0", "l1"))
    V.prepare_asu_layer_context(m, "l0", _md(max_seq_len=100))
    assert m.calls == [("reset", V.SINGLE_REQ_ID, 100, 99, (1, 8))]
    V.prepare_asu_layer_context(m, "l1", _md(max_seq_len=100))   # the next layer of the same step
    assert len(m.calls) == 1
    V.prepare_asu_layer_context(m, "l0", _md(max_seq_len=101))
    assert m.calls[-1] == ("mark", 100)
    V.prepare_asu_layer_context(m, "l1", _md(max_seq_len=101))
    assert len(m.calls) == 2
    V.prepare_asu_layer_context(m, "l0", _md(max_seq_len=50))    # shorter: a new request
    assert m.calls[-1] == ("reset", V.SINGLE_REQ_ID, 50, 49, (1, 8))
    V.prepare_asu_layer_context(m, "l0", _md(max_seq_len=50, asu_req_id="req-7"))
    assert m.calls[-1] == ("reset", "req-7", 50, 49, (1, 8))


def test_subclass_routes_single_request_decode_to_the_resolver(monkeypatch):
    pytest.importorskip("vllm")
    Impl = V.asu_flashmla_sparse_impl()
    from vllm.v1.attention.backends.mla.flashmla_sparse import FlashMLASparseImpl

    assert issubclass(Impl, FlashMLASparseImpl)
    impl = object.__new__(Impl)
    impl.kv_cache_dtype = "auto"
    impl.topk_indices_buffer = torch.zeros(4, 16, dtype=torch.int32)
    seen = []
    monkeypatch.setattr(FlashMLASparseImpl, "_forward_bf16_kv", lambda self, *a: seen.append("stock") or "stock")
    monkeypatch.setattr(V.sparse_mla, "resolve_topk", lambda ctx, t, bt, kv: seen.append(("resolve", ctx)) or t)
    monkeypatch.setattr(V.sparse_mla, "managed_kv_view", lambda ctx: "managed")
    monkeypatch.setattr(Impl, "_bf16_flash_mla_kernel", lambda self, q, kv, s: seen.append(("attn", kv)) or "asu")
    q, kv = torch.zeros(1, 2, 8), torch.zeros(4, 2, 8)

    m = FakeManager()
    impl.asu_manager = m
    assert impl.forward_mqa(q, kv, _md(), SimpleNamespace(layer_name="l0")) == ("asu", None)
    assert seen == [("resolve", m.ctx["l0"]), ("attn", "managed")]
    assert impl.forward_mqa(q, kv, _md(), SimpleNamespace(layer_name="other")) == ("stock", None)
    assert impl.forward_mqa(q, kv, _md(num_reqs=2), SimpleNamespace(layer_name="l0")) == ("stock", None)


def test_subclass_routes_fp8_decode_to_the_resolver(monkeypatch):
    pytest.importorskip("vllm")
    Impl = V.asu_flashmla_sparse_impl()
    from vllm.v1.attention.backends.mla.flashmla_sparse import FlashMLASparseImpl, FlashMLASparseMetadata

    impl = object.__new__(Impl)
    impl.kv_cache_dtype = "fp8_ds_mla"
    impl.topk_indices_buffer = torch.zeros(4, 16, dtype=torch.int32)
    seen = []
    monkeypatch.setattr(FlashMLASparseImpl, "_forward_fp8_kv_mixed_batch", lambda self, *a: "stock-mixed")
    monkeypatch.setattr(FlashMLASparseImpl, "_forward_fp8_kv_separate_prefill_decode", lambda self, *a: "stock-sep")
    monkeypatch.setattr(V.sparse_mla, "resolve_topk", lambda ctx, t, bt, kv: t)
    monkeypatch.setattr(V.sparse_mla, "managed_paged_view", lambda ctx: "pages")

    def kernel(self, q, kv_c_and_k_pe_cache, topk_indices, kernel_metadata):
        seen.append((tuple(q.shape), kv_c_and_k_pe_cache, tuple(topk_indices.shape), kernel_metadata))
        return torch.zeros(1, 1, q.shape[2], 5), None

    monkeypatch.setattr(Impl, "_fp8_flash_mla_kernel", kernel)
    q, kv = torch.zeros(1, 2, 8), torch.zeros(4, 2, 8)
    impl.asu_manager = FakeManager()
    layer = SimpleNamespace(layer_name="l0")

    out, _ = impl.forward_mqa(q, kv, _md(fp8_use_mixed_batch=True, fp8_extra_metadata="km"), layer)
    assert out.shape == (1, 2, 5) and seen[-1] == ((1, 1, 2, 8), "pages", (1, 1, 16), "km")
    P = FlashMLASparseMetadata.FP8SeparatePrefillDecode
    sep = P(num_decodes=1, num_decode_tokens=1, decode=P.Decode(seq_lens=None, kernel_metadata="kd",
                                                                 decode_query_len=1))
    out, _ = impl.forward_mqa(q, kv, _md(fp8_use_mixed_batch=False, fp8_extra_metadata=sep), layer)
    assert out.shape == (1, 2, 5) and seen[-1][3] == "kd"
    n = len(seen)
    assert impl.forward_mqa(q, kv, _md(fp8_use_mixed_batch=True, fp8_extra_metadata="km", num_reqs=2),
                            layer)[0] == "stock-mixed"
    with_prefill = P(num_decodes=1, num_decode_tokens=1, num_prefill_tokens=3, decode=sep.decode)
    assert impl.forward_mqa(q, kv, _md(fp8_use_mixed_batch=False, fp8_extra_metadata=with_prefill),
                            layer)[0] == "stock-sep"
    assert len(seen) == n


def test_registered_override_resolves_to_the_asu_backend():
    pytest.importorskip("vllm")
    from vllm.v1.attention.backends.mla.flashmla_sparse import FlashMLASparseBackend, FlashMLASparseImpl
    from vllm.v1.attention.backends.registry import _ATTN_OVERRIDES, AttentionBackendEnum

    before = dict(_ATTN_OVERRIDES)
    try:
        V.register_flashmla_sparse_override()
        cls = AttentionBackendEnum.FLASHMLA_SPARSE.get_class()
        assert cls is V.asu_flashmla_sparse_backend() and issubclass(cls, FlashMLASparseBackend)
        assert cls.get_name() == FlashMLASparseBackend.get_name()
        impl = cls.get_impl_cls()
        assert impl is V.ASUFlashMLASparseImpl and issubclass(impl, FlashMLASparseImpl)
        m = FakeManager()
        V.attach_manager(m)
        assert impl.asu_manager is m
    finally:
        _ATTN_OVERRIDES.clear()
        _ATTN_OVERRIDES.update(before)
        V.asu_flashmla_sparse_impl().asu_manager = None


def test_asu_backend_keeps_attention_out_of_full_cuda_graphs(monkeypatch):
    """The ASU path decides on the host every step (reset or mark, the request's length): its
    builder declares no CUDA-graph support, and a capture that reaches the path anyway is refused."""
    pytest.importorskip("vllm")
    from vllm.v1.attention.backend import AttentionCGSupport
    from vllm.v1.attention.backends.mla.flashmla_sparse import FlashMLASparseMetadataBuilder

    backend = V.asu_flashmla_sparse_backend()
    builder = backend.get_builder_cls()
    assert builder is V.ASUFlashMLASparseMetadataBuilder and issubclass(builder, FlashMLASparseMetadataBuilder)
    assert builder.get_cudagraph_support(None, None) == AttentionCGSupport.NEVER
    assert FlashMLASparseMetadataBuilder.get_cudagraph_support(None, None) != AttentionCGSupport.NEVER

    cls = V.asu_flashmla_sparse_impl()
    impl = cls.__new__(cls)
    impl._asu_layer_name = "l0"
    m = FakeManager()
    monkeypatch.setattr(torch.cuda, "is_available", lambda: True)
    monkeypatch.setattr(torch.cuda, "is_current_stream_capturing", lambda: True)
    with pytest.raises(RuntimeError, match="CUDA graph"):
        impl._asu_resolve(None, None, _md(asu_kv_cache_manager=m))
    assert m.calls == []  # refused before any reset or mark was queued
