"""The hot path under CUDA-graph capture.  A serving engine records its decode step once and
replays it (vLLM does for its decode batches), so every launch on the path has to be
capturable: no host synchronisation, no allocation outside the graph's pool, no launch
parameter read back from the device.  Each test records the calls in a graph and replays it
on fresh inputs next to an eager twin of the same state; outputs, state and copied rows must
stay identical step after step."""

import numpy as np
import pytest
import torch

from oracle import asu_oracle as O

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


@pytest.fixture(scope="module", autouse=True)
def _lib():
    import asu_ascend_b200

    asu_ascend_b200.load()
    from asu_ascend_b200 import ops

    ops.set_status_checks(False)  # a status read-back synchronises, which a graph cannot record
    yield


def T(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def test_lru_step_and_swapin_replay_in_a_cuda_graph():
    """LRU maintain + lookup and the TMA bulk swap-in of 656-byte rows, recorded once."""
    from asu_ascend_b200.host_pool import HostRowPool, check_status
    from asu_ascend_b200.lru import LruSlotPools
    from asu_ascend_b200.workloads import LocalityTrace, record_addresses

    R, K, S, Q, row = 16, 4096, 512, 256, 656
    pool = HostRowPool(rows=2000, row_bytes=row)
    pool.fill_random(5)
    trec = T(record_addresses(R, K, pool.rows))
    tr = LocalityTrace(R, K, topk=Q, seed=9)
    eager, graphed = (LruSlotPools(R, K, S, Q // 4, Q, device=DEV) for _ in range(2))
    kv_e, kv_g = (torch.zeros((R, S, row), dtype=torch.uint8, device=DEV) for _ in range(2))
    st_e, st_g = (torch.zeros(R, dtype=torch.int32, device=DEV) for _ in range(2))
    out_g = graphed.new_output()
    q_buf = torch.empty((R, Q), dtype=torch.int32, device=DEV)
    for _ in range(3):  # identical eager warm-up of both twins (also configures the kernels)
        q = T(tr.step())
        for p, kv, st, o in ((eager, kv_e, st_e, None), (graphed, kv_g, st_g, out_g)):
            o = p.step(q, out=o)
            pool.swapin(trec, q, o.slot, o.install, kv, status=st)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        graphed.step(q_buf, out=out_g)
        pool.swapin(trec, q_buf, out_g.slot, out_g.install, kv_g, status=st_g)
    for _ in range(6):
        q = T(tr.step())
        o_e = eager.step(q)
        pool.swapin(trec, q, o_e.slot, o_e.install, kv_e, status=st_e)
        q_buf.copy_(q)
        g.replay()
        torch.cuda.synchronize()
        for name in ("slot", "hit", "install"):
            assert torch.equal(getattr(o_e, name), getattr(out_g, name)), name
        for name in ("token_to_slot", "slot_to_token", "lru_order", "free_stack", "free_count"):
            assert torch.equal(getattr(eager, name), getattr(graphed, name)), name
        assert torch.equal(kv_e, kv_g)
    assert int(out_g.install.sum()) > 0  # the replays installed rows
    check_status(st_g, "swapin")
    graphed.check_status()
    del g
    pool.close()


@pytest.mark.parametrize("w0,w1", [(512, 64), (720, 8)])
def test_resolver_op_replays_in_a_cuda_graph(w0, w1):
    """npu_asu_resolve_kv_slots_single_req recorded once and replayed on new top-k sets: bf16
    row pairs of 1024 + 128 bytes (copied by the resolve cluster) and 1440 + 16 bytes (the
    programmatic dependent copy kernel); slots, state and managed rows equal the oracle's."""
    rng = np.random.Generator(np.random.PCG64(w0 + w1))
    max_seq, slots, bs, actual, prefix = 16384, 16384, 64, 16000, 15900
    nblk = max_seq // bs
    bt = rng.permutation(nblk + 8)[:nblk].astype(np.int32)
    ts, rec, hs, own, stack, cnt = O.reset_state(max_seq, slots, bs, actual, prefix, bt)
    src0 = rng.integers(0, 1 << 16, ((nblk + 8) * bs, w0), dtype=np.uint16)
    src1 = rng.integers(0, 1 << 16, ((nblk + 8) * bs, w1), dtype=np.uint16)
    dst0 = np.zeros((slots, w0), np.uint16)
    dst1 = np.zeros((slots, w1), np.uint16)
    tts, trec, ths, town, tstack, tcnt, tbt = T(ts), T(rec), T(hs), T(own), T(stack), T(cnt), T(bt)
    kv0, kv1 = (T(x.view(np.int16)).view(torch.bfloat16) for x in (src0, src1))
    m0, m1 = (T(x.view(np.int16)).view(torch.bfloat16) for x in (dst0, dst1))
    f = torch.ops.asu.npu_asu_resolve_kv_slots_single_req
    topk_buf = torch.empty((1, 2048), dtype=torch.int32, device=DEV)

    def call():
        return f(topk_buf, actual, prefix, tts, trec, ths, town, tstack, tcnt, tbt, kv0, kv1, m0, m1, bs)

    def step(topk):
        return O.resolve_kv_slots_single_req(topk, actual, ts, rec, hs, own, stack, cnt, bt, src0, src1, dst0, dst1,
                                             bs)

    topk = rng.integers(0, actual, (1, 2048)).astype(np.int32)
    exp = step(topk)  # one eager call first (kernel attributes, library loading)
    topk_buf.copy_(T(topk))
    np.testing.assert_array_equal(call().cpu().numpy(), exp)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = call()
    for _ in range(4):
        topk = rng.integers(0, actual, (1, 2048)).astype(np.int32)
        exp = step(topk)
        topk_buf.copy_(T(topk))
        g.replay()
        torch.cuda.synchronize()
        np.testing.assert_array_equal(out.cpu().numpy(), exp)
        np.testing.assert_array_equal(tts.cpu().numpy(), ts)
        np.testing.assert_array_equal(ths.cpu().numpy(), hs)
        np.testing.assert_array_equal(town.cpu().numpy(), own)
        assert int(tcnt.reshape(-1)[0]) == int(cnt[0])
        np.testing.assert_array_equal(m0.view(torch.int16).cpu().numpy().view(np.uint16), dst0)
        np.testing.assert_array_equal(m1.view(torch.int16).cpu().numpy().view(np.uint16), dst1)
    del g
