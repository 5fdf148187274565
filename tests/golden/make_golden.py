"""Generate the golden fixtures in tests/golden/ by running the REFERENCE's own Python code.

Run in a container where the ASU-Ascend reference is mounted (default
/root/reference, override with ASU_REFERENCE_ROOT):

    python tests/golden/make_golden.py

What is imported from the reference, unchanged:

* simu/kv_cache_eviction_sim.py            LRUManagedCache, TopKWorkload, run_simulation
* ops/scripts/asu_hbm_index_common.py      make_index_case, make_maintain_case,
                                           expected_lookup_allocate, expected_maintain
* pta-ops/asu_hbm_index_lookup_simt/python lookup_allocate_evict, make_random_case
* simu/hbm_lookup_update/scripts/test_lookup_update.py  expected_lookup_update,
  update_positions (its module-level ``torch_npu`` / ``hbm_lookup_update``
  imports are satisfied with empty stand-in modules; no NPU code runs)
* patch/0001 vllm_ascend/ops/asu_kv_resolver.py and patch/0003
  vllm_ascend/attention/asu_kv_cache_manager.py, extracted from the diffs
  into a temporary directory.

The fixtures hold the reference's outputs (full arrays for small cases,
changed entries / sha256 digests for large ones).  Nothing here is used at
run time by the library.
"""

from __future__ import annotations

import hashlib
import importlib.util
import os
import sys
import tempfile
import types
from collections import OrderedDict
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
REF = Path(os.environ.get("ASU_REFERENCE_ROOT", "/root/reference"))

sys.path.insert(0, str(REPO))
from asu_ascend_b200.workloads import LocalityTrace  # noqa: E402


def _load(name: str, path: Path):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def _extract_patch_file(patch: Path, target: str, out: Path) -> Path:
    """Write the '+' lines of the new-file hunk for ``target`` in a git diff."""
    lines = patch.read_text().splitlines()
    body: list[str] = []
    active = False
    for ln in lines:
        if ln.startswith("diff --git "):
            active = ln.endswith(" " + target)
            continue
        if not active or ln.startswith(("+++", "---", "@@", "new file", "index ")):
            continue
        if ln.startswith("+"):
            body.append(ln[1:])
    out.write_text("\n".join(body) + "\n")
    return out


def digest(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        a = np.ascontiguousarray(a)
        h.update(str(a.dtype).encode())
        h.update(str(a.shape).encode())
        h.update(a.tobytes())
    return h.hexdigest()


# ---------------------------------------------------------------------------
# LRU (simulator)
# ---------------------------------------------------------------------------

class RecordingDict(OrderedDict):
    """OrderedDict that records the keys popitem() removes (eviction order)."""

    def __init__(self, *a, **k):
        super().__init__(*a, **k)
        self.popped: list = []

    def popitem(self, last=True):
        key, value = super().popitem(last=last)
        self.popped.append(key)
        return key, value


def run_reference_lru(sim, slots: int, target: int, steps: list[np.ndarray]):
    """Drive LRUManagedCache one token at a time to record per-query outcomes."""
    cache = sim.LRUManagedCache(total_slots=slots, free_slot_target=target)
    cache._residents = RecordingDict(cache._residents)
    out = []
    for keys in steps:
        cache._residents.popped = []
        n_evicted = cache.prepare_free_slots()
        evicted = [k[1] for k in cache._residents.popped]
        assert len(evicted) == n_evicted
        q = len(keys)
        slot = np.full(q, -1, np.int32)
        hit = np.zeros(q, bool)
        install = np.zeros(q, bool)
        for pos, key in enumerate(keys.tolist()):
            st = cache.resolve_query([(0, key)])
            hit[pos] = st.hits == 1
            install[pos] = st.installs == 1
            if st.hits or st.installs:
                slot[pos] = cache._residents[(0, key)]
        out.append((slot, hit, install, np.asarray(evicted, np.int32)))
    final_order = np.asarray([cache._residents[k] for k in cache._residents], np.int32)
    final_keys = np.asarray([k[1] for k in cache._residents], np.int32)
    final_free = np.asarray(cache._free_slots, np.int32)
    return out, final_order, final_keys, final_free


def lru_fixtures(sim):
    rng = np.random.Generator(np.random.PCG64(20260101))
    cases = {}
    # A: tiny pool, duplicates inside a step, evictions every step
    steps_a = [rng.integers(0, 64, 12).astype(np.int32) for _ in range(40)]
    cases["a"] = (16, 4, 64, steps_a)
    # B: medium pool with zipf locality, distinct ids per step
    tr = LocalityTrace(1, 4096, topk=256, reuse=0.7, seed=7)
    steps_b = [tr.step()[0] for _ in range(24)]
    cases["b"] = (512, 128, 4096, steps_b)
    # C: free target 0 -> the pool fills, then shortages
    steps_c = [rng.integers(0, 40, 12).astype(np.int32) for _ in range(8)]
    cases["c"] = (16, 0, 40, steps_c)
    # D: target above the resident count, duplicates heavy
    steps_d = [rng.integers(0, 20, 30).astype(np.int32) for _ in range(10)]
    cases["d"] = (8, 8, 20, steps_d)
    arrays = {}
    for name, (slots, target, key_space, steps) in cases.items():
        res, order, keys, free = run_reference_lru(sim, slots, target, steps)
        q = len(steps[0])
        n = len(steps)
        arrays[f"{name}_meta"] = np.asarray([slots, target, key_space, n, q], np.int64)
        arrays[f"{name}_query"] = np.stack(steps)
        arrays[f"{name}_slot"] = np.stack([r[0] for r in res])
        arrays[f"{name}_hit"] = np.stack([r[1] for r in res])
        arrays[f"{name}_install"] = np.stack([r[2] for r in res])
        ev = np.full((n, max(1, max(len(r[3]) for r in res))), -1, np.int32)
        evn = np.zeros(n, np.int32)
        for i, r in enumerate(res):
            ev[i, : len(r[3])] = r[3]
            evn[i] = len(r[3])
        arrays[f"{name}_evicted"] = ev
        arrays[f"{name}_evicted_n"] = evn
        arrays[f"{name}_final_order"] = order
        arrays[f"{name}_final_keys"] = keys
        arrays[f"{name}_final_free"] = free
    np.savez_compressed(HERE / "lru_small.npz", **arrays)

    # c0: 1 request, 131072 keys, 16384 slots, target 2048, 256 steps x 2048 ids.
    tr = LocalityTrace(1, 131072, topk=2048, reuse=0.7, zipf_s=1.1, seed=0)
    steps = [tr.step()[0] for _ in range(256)]
    res, order, keys, free = run_reference_lru(sim, 16384, 2048, steps)
    per_step = np.asarray([digest(steps[i], *res[i]) for i in range(256)])
    counts = np.asarray([[r[1].sum(), r[2].sum(), len(r[3]), (r[0] < 0).sum()] for r in res], np.int64)
    np.savez_compressed(
        HERE / "lru_c0.npz",
        trace_digest=np.asarray([digest(*steps)]),
        step_digest=per_step,
        counts=counts,
        first_query=np.stack(steps[:3]),
        first_slot=np.stack([r[0] for r in res[:3]]),
        first_hit=np.stack([r[1] for r in res[:3]]),
        first_evicted=res[1][3],
        final_digest=np.asarray([digest(order, keys, free)]),
    )

    # Reference workloads (TopKWorkload) on one request, aggregated stats of run_simulation.
    stats = []
    for wl in ("uniform", "hotset", "zipf", "sliding"):
        cfg = sim.SimulationConfig(req_num=1, steps=6, managed_tokens_per_req=8192, hbm_slots_per_req=3072,
                                   free_slots_target_per_req=2048, workload=wl, hotset_size=4096, seed=5)
        wk = sim.TopKWorkload(cfg)
        qs = [np.asarray([t for _, t in wk.query(0, s)], np.int32) for s in range(cfg.steps)]
        result = sim.run_simulation(cfg)
        stats.append([result.total.hits, result.total.misses, result.total.installs,
                      result.total.shortages, result.total.cpu_evictions])
        np.save(HERE / f"_tmp_{wl}.npy", np.stack(qs))
    traces = {wl: np.load(HERE / f"_tmp_{wl}.npy") for wl in ("uniform", "hotset", "zipf", "sliding")}
    for wl in traces:
        os.remove(HERE / f"_tmp_{wl}.npy")
    np.savez_compressed(HERE / "lru_workloads.npz", stats=np.asarray(stats, np.int64),
                        **{f"trace_{k}": v for k, v in traces.items()})


# ---------------------------------------------------------------------------
# ops contract
# ---------------------------------------------------------------------------

def changed(before: np.ndarray, after: np.ndarray):
    idx = np.flatnonzero(before.reshape(-1) != after.reshape(-1)).astype(np.int64)
    return idx, after.reshape(-1)[idx].astype(np.int32)


def ops_fixtures(common):
    arrays = {}
    for pattern in ("hit", "miss", "mixed"):
        case = common.make_index_case(2, pattern)
        exp = common.expected_lookup_allocate(case)
        arrays[f"lookup_{pattern}_query"] = case.query_index
        arrays[f"lookup_{pattern}_slot_out"] = exp.slot_out
        arrays[f"lookup_{pattern}_free_head"] = exp.free_head
        i, v = changed(case.index, exp.index)
        arrays[f"lookup_{pattern}_index_idx"], arrays[f"lookup_{pattern}_index_val"] = i, v
        i, v = changed(case.slot_to_index, exp.slot_to_index)
        arrays[f"lookup_{pattern}_s2i_idx"], arrays[f"lookup_{pattern}_s2i_val"] = i, v
    for ratio, seed in ((0.25, 123), (1.0, 7), (0.5, 0xDEADBEEF)):
        case = common.make_maintain_case(3, ratio)
        idx, s2i, fs, fh = common.expected_maintain(case.index, case.slot_to_index, case.free_slots,
                                                    case.free_head, case.last_query_slots, seed)
        tag = f"maintain_{int(ratio * 100)}"
        arrays[f"{tag}_seed"] = np.asarray([seed], np.int64)
        arrays[f"{tag}_free_slots"] = fs
        arrays[f"{tag}_free_head"] = fh
        i, v = changed(case.index, idx)
        arrays[f"{tag}_index_idx"], arrays[f"{tag}_index_val"] = i, v
        i, v = changed(case.slot_to_index, s2i)
        arrays[f"{tag}_s2i_idx"], arrays[f"{tag}_s2i_val"] = i, v
    # chained random rounds at the reference sizes: lookup with duplicates, then maintain
    rng = np.random.Generator(np.random.PCG64(99))
    case = common.make_index_case(2, "hit")
    index, s2i, fs, fh = case.index, case.slot_to_index, case.free_slots, case.free_head
    rounds = []
    for rnd in range(3):
        q = rng.integers(0, common.INDEX_SIZE, (2, common.QUERY_COUNT)).astype(np.int32)
        q[:, ::7] = rng.integers(0, 8192, q[:, ::7].shape)  # some hits
        q[:, 5::11] = q[:, 3::11][:, : q[:, 5::11].shape[1]]  # duplicates
        c = common.IndexCase(index, s2i, fs, fh, q)
        exp = common.expected_lookup_allocate(c)
        seed = int(rng.integers(0, 2**32))
        index2, s2i2, fs2, fh2 = common.expected_maintain(exp.index, exp.slot_to_index, fs, exp.free_head,
                                                          exp.slot_out, seed)
        rounds.append((q, exp.slot_out, exp.free_head, seed, fh2, fs2))
        index, s2i, fs, fh = index2, s2i2, fs2, fh2
    for k, (q, so, fh1, seed, fh2, fs2) in enumerate(rounds):
        arrays[f"chain{k}_query"] = q
        arrays[f"chain{k}_slot_out"] = so
        arrays[f"chain{k}_head_after_lookup"] = fh1
        arrays[f"chain{k}_seed"] = np.asarray([seed], np.int64)
        arrays[f"chain{k}_head_after_maintain"] = fh2
        arrays[f"chain{k}_free_slots"] = fs2
    arrays["chain_final_digest"] = np.asarray([digest(index, s2i)])
    np.savez_compressed(HERE / "ops.npz", **arrays)


# ---------------------------------------------------------------------------
# batch LRU (SIMT)
# ---------------------------------------------------------------------------

def batch_lru_fixtures(ref, wl):
    arrays = {}
    case = wl.make_random_case(np, 2, 1536, seed=17, case_id=3)
    for r in range(2):
        st = ref.LookupState(case.token_to_slot[r].tolist(), case.slot_to_token[r].tolist(),
                             case.lru_slots[r].astype(np.int32).tolist())
        for rnd in range(3):
            q = (case.query_token_ids[r] if rnd == 0 else
                 np.asarray(wl.make_random_query_row(1024 + 256 * rnd, seed=17, case_id=10 + rnd, req_id=r), np.int32))
            if rnd == 2:
                q = q.copy()
                q[100:110] = q[0:10]       # duplicates
                q[200] = -1                # padding
                q[201] = wl.INDEX_SIZE + 5  # out of range padding
            slots, mask = ref.lookup_allocate_evict(q.tolist(), st)
            arrays[f"r{r}_q{rnd}"] = np.asarray(q, np.int32)
            arrays[f"r{r}_slot{rnd}"] = np.asarray(slots, np.int32)
            arrays[f"r{r}_mask{rnd}"] = np.asarray(mask, bool)
            arrays[f"r{r}_lru{rnd}"] = np.asarray(st.lru_slots, np.int16)
            arrays[f"r{r}_s2t{rnd}"] = np.asarray(st.slot_to_token, np.int32)
            arrays[f"r{r}_t2s_digest{rnd}"] = np.asarray([digest(np.asarray(st.token_to_slot, np.int32))])
    np.savez_compressed(HERE / "batch_lru.npz", **arrays)


# ---------------------------------------------------------------------------
# gather / update (simu/hbm_lookup_update)
# ---------------------------------------------------------------------------

def gather_fixtures(tlu):
    index_size = tlu.INDEX_SIZE
    tok = np.arange(index_size, dtype=np.int32)
    arrays = {}
    # single-request case of run_single_req_case
    states = (tok.astype(np.int64) * 10 + 7).astype(np.int32)
    q = ((np.arange(512, dtype=np.int64) * 17 + 23) % index_size).astype(np.int32)
    new = (100000 + np.arange(512, dtype=np.int32)).astype(np.int32)
    out, st = tlu.expected_lookup_update(states, q, new, 42, 5)
    arrays["single_out"] = out
    i, v = changed(states, st)
    arrays["single_upd_idx"], arrays["single_upd_val"] = i, v
    # multi-request case of run_multi_req_case
    req_num, qlen = 4, 513
    states = np.empty((req_num, index_size), np.int32)
    q = np.empty((req_num, qlen), np.int32)
    new = np.empty((req_num, qlen), np.int32)
    for r in range(req_num):
        states[r] = (tok.astype(np.int64) * 13 + 1000 * r + 17).astype(np.int32)
        q[r] = ((np.arange(qlen, dtype=np.int64) * 19 + r * 101 + 7) % index_size).astype(np.int32)
        new[r] = (200000 + 10000 * r + np.arange(qlen, dtype=np.int32)).astype(np.int32)
    out, st = tlu.expected_lookup_update(states, q, new, 2026, 7)
    arrays["multi_out"] = out
    i, v = changed(states, st)
    arrays["multi_upd_idx"], arrays["multi_upd_val"] = i, v
    # duplicates inside the updated positions: last writer wins
    rng = np.random.Generator(np.random.PCG64(5))
    q = rng.integers(0, 300, (3, 700)).astype(np.int32)
    new = rng.integers(-(2**31), 2**31 - 1, (3, 700)).astype(np.int32)
    states = rng.integers(-5, 1000, (3, index_size)).astype(np.int32)
    out, st = tlu.expected_lookup_update(states, q, new, 77, 100)
    arrays["dup_seed_states"] = np.asarray([5], np.int64)
    arrays["dup_out"] = out
    i, v = changed(states, st)
    arrays["dup_upd_idx"], arrays["dup_upd_val"] = i, v
    pos = {}
    for n, seed, pct in ((512, 42, 5), (513, 2026, 7), (2048, 0, 5), (1, 3, 100), (97, 11, 50)):
        for r in range(3):
            pos[f"pos_{n}_{seed}_{pct}_{r}"] = np.asarray(tlu.update_positions(n, seed, pct, r), np.int64)
    arrays.update(pos)
    np.savez_compressed(HERE / "gather.npz", **arrays)


# ---------------------------------------------------------------------------
# resolver (patch 0001) + manager reset (patch 0003)
# ---------------------------------------------------------------------------

def resolver_fixtures(res_mod, mgr_mod):
    import torch

    arrays = {}
    rng = np.random.Generator(np.random.PCG64(31))
    max_seq, slots, bs = 4096, 1024, 64
    actual, prefix = 3000, 2990
    nblk = (max_seq + bs - 1) // bs
    block_table = rng.permutation(nblk + 8)[:nblk].astype(np.int32)
    kv0 = torch.from_numpy(rng.standard_normal(((nblk + 8) * bs, 1, 8)).astype(np.float32)).to(torch.bfloat16)
    kv1 = torch.from_numpy(rng.standard_normal(((nblk + 8) * bs, 1, 4)).astype(np.float32)).to(torch.bfloat16)
    caches = {"layers.0.self_attn": (kv0.reshape(nblk + 8, bs, 1, 8), kv1.reshape(nblk + 8, bs, 1, 4),
                                     torch.zeros(nblk + 8, bs, 1, 2))}
    mgr = mgr_mod.ASUFullKVCacheManagerFunctional.from_kv_caches(caches, max_seq_len=max_seq, block_size=bs,
                                                                   managed_slot_count=slots, enabled=True)
    mgr.reset_single_request("r", actual, prefix, torch.from_numpy(block_table[None, :]))
    ctx = mgr.get_layer_context("layers.0.self_attn")
    arrays["reset_token_state"] = ctx.token_state.numpy().copy()
    arrays["reset_record"] = ctx.asu_record_addr.numpy().copy()
    ctx.managed_kv_cache_0.fill_(0)
    ctx.managed_kv_cache_1.fill_(0)
    o0, o1 = ctx.original_kv_cache_views(caches["layers.0.self_attn"])
    arrays["meta"] = np.asarray([max_seq, slots, bs, actual, prefix], np.int64)
    arrays["block_table"] = block_table
    arrays["kv0"] = o0.view(torch.int16).numpy().copy()
    arrays["kv1"] = o1.view(torch.int16).numpy().copy()
    for step in range(3):
        topk = rng.integers(0, actual, (1, 1, 256)).astype(np.int32)
        topk[0, 0, 100:140] = topk[0, 0, 0:40]  # duplicates
        topk[0, 0, 200] = actual - 1            # tail token
        out = res_mod.asu_resolve_kv_slots_single_req(
            torch.from_numpy(topk), actual_seq_len=actual, managed_prefix_len=prefix,
            token_state=ctx.token_state, asu_record_addr=ctx.asu_record_addr,
            hbm_slot_of_token=ctx.hbm_slot_of_token, slot_owner_token=ctx.slot_owner_token,
            free_slot_stack=ctx.free_slot_stack, free_slot_count=ctx.free_slot_count,
            original_block_table=torch.from_numpy(block_table[None, :]), original_kv_cache_0=o0,
            original_kv_cache_1=o1, managed_kv_cache_0=ctx.managed_kv_cache_0,
            managed_kv_cache_1=ctx.managed_kv_cache_1, block_size=bs)
        arrays[f"s{step}_topk"] = topk
        arrays[f"s{step}_out"] = out.numpy()
        arrays[f"s{step}_token_state"] = ctx.token_state.numpy().copy()
        arrays[f"s{step}_hbm_slot"] = ctx.hbm_slot_of_token.numpy().copy()
        arrays[f"s{step}_owner"] = ctx.slot_owner_token.numpy().copy()
        arrays[f"s{step}_count"] = np.asarray([int(ctx.free_slot_count.item())], np.int32)
        arrays[f"s{step}_kv_digest"] = np.asarray([digest(ctx.managed_kv_cache_0.view(torch.int16).numpy(),
                                                          ctx.managed_kv_cache_1.view(torch.int16).numpy())])
    np.savez_compressed(HERE / "resolver.npz", **arrays)


# ---------------------------------------------------------------------------
# MicroKV keys (MicroKV/python/microkv/client.py make_key)
# ---------------------------------------------------------------------------

MICROKV_KEY_CASES = [
    ("req-phase1", 2, 0, 0), ("req-phase1", 2, 3, 0), ("shared-server", 0, 0, 0), ("mla-req", 12, 34, 0),
    ("type-space", 1, 1, 2), ("", 0, 0, 0), ("\u8bf7\u6c42-7", 61, 131071, 3),
    (0, 0, 0, 0), (1, 2, 3, 1), (0xFFFFFFFFFFFFFFFF, 0xFFFFFFFF, 0xFFFFFFFF, 255), (123456789, 60, 4095, 0),
]


def microkv_fixtures(client):
    keys = [client.make_key(r, layer, pos, t) for r, layer, pos, t in MICROKV_KEY_CASES]
    req_str = np.asarray([r if isinstance(r, str) else "" for r, *_ in MICROKV_KEY_CASES])
    req_int = np.asarray([r if isinstance(r, int) else 0 for r, *_ in MICROKV_KEY_CASES], np.uint64)
    is_str = np.asarray([isinstance(r, str) for r, *_ in MICROKV_KEY_CASES])
    fields = np.asarray([c[1:] for c in MICROKV_KEY_CASES], np.int64)
    np.savez_compressed(HERE / "microkv_keys.npz", keys=np.frombuffer(b"".join(keys), np.uint8).reshape(-1, 32),
                        req_str=req_str, req_int=req_int, is_str=is_str, fields=fields)


def main():
    if not REF.exists():
        raise SystemExit(f"reference not found at {REF}")
    if sys.argv[1:] == ["microkv"]:  # only the MicroKV key fixture
        microkv_fixtures(_load("microkv_client", REF / "MicroKV" / "python" / "microkv" / "client.py"))
        return
    sim = _load("kv_cache_eviction_sim", REF / "simu" / "kv_cache_eviction_sim.py")
    common = _load("asu_hbm_index_common", REF / "ops" / "scripts" / "asu_hbm_index_common.py")
    common.np = np  # the module resolves numpy lazily through require_numpy()
    simt = REF / "pta-ops" / "asu_hbm_index_lookup_simt"
    sys.path.insert(0, str(simt))
    ref_lru = _load("python.lookup_lru_reference", simt / "python" / "lookup_lru_reference.py")
    ref_wl = _load("python.random_workload", simt / "python" / "random_workload.py")
    for stub in ("torch_npu", "hbm_lookup_update"):
        sys.modules.setdefault(stub, types.ModuleType(stub))
    tlu = _load("test_lookup_update", REF / "simu" / "hbm_lookup_update" / "scripts" / "test_lookup_update.py")
    with tempfile.TemporaryDirectory() as tmp:
        tmp = Path(tmp)
        p1 = next((REF / "patch").glob("0001-*.patch"))
        p3 = next((REF / "patch").glob("0003-*.patch"))
        res_mod = _load("asu_kv_resolver_ref", _extract_patch_file(p1, "vllm_ascend/ops/asu_kv_resolver.py",
                                                                    tmp / "asu_kv_resolver.py"))
        mgr_mod = _load("asu_kv_cache_manager_ref", _extract_patch_file(
            p3, "vllm_ascend/attention/asu_kv_cache_manager.py", tmp / "asu_kv_cache_manager.py"))
        resolver_fixtures(res_mod, mgr_mod)
    lru_fixtures(sim)
    ops_fixtures(common)
    batch_lru_fixtures(ref_lru, ref_wl)
    gather_fixtures(tlu)
    microkv_fixtures(_load("microkv_client", REF / "MicroKV" / "python" / "microkv" / "client.py"))
    for f in sorted(HERE.glob("*.npz")):
        print(f.name, f.stat().st_size)


if __name__ == "__main__":
    main()
