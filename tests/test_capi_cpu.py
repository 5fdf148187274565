"""CPU-only checks of the boundary: the C-ABI library loads and exports every symbol that
include/asu_b200.h declares, argument validation rejects bad calls before any launch,
and the torch operators carry the reference schemas (no compute without a GPU)."""

import ctypes
import re
from pathlib import Path

import numpy as np
import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "asu_b200.h"


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\*?\s+\*?((?:asu|hbm)_\w+)\s*\(", text, flags=re.M)))


@pytest.fixture(scope="module")
def lib():
    from asu_ascend_b200 import _lib

    return _lib


def test_header_declares_the_reference_launchers():
    names = declared_functions()
    for ref in ("asu_hbm_index_lookup_do", "asu_hbm_index_maintain_do", "asu_hbm_index_lookup_simt_do",
                "hbm_lookup_vec_do", "hbm_random_update_do"):
        assert ref in names
    assert len(names) >= 18


def test_library_exports_every_declared_symbol(lib):
    raw = ctypes.CDLL(str(lib.LIB_PATH))
    for name in declared_functions():
        assert hasattr(raw, name), name
        assert name in lib.exported_symbols(), name


def test_version_and_status_strings(lib):
    assert lib.lib.asu_version() == 10000
    assert b"invalid argument" in lib.lib.asu_status_string(-1)
    assert b"aligned" in lib.lib.asu_status_string(-2)
    assert lib.status_names(0x03) == ["BAD_QUERY", "FREE_EXHAUSTED"]


def test_argument_validation_rejects_before_launch(lib):
    L = lib.lib
    # zero requests: nothing to do
    assert L.asu_hbm_index_lookup_ex(None, 1, 1, 1, 1, 1, 1, 0, 1, 1, 1, 1, None) == 0
    # null pointers
    assert L.asu_hbm_index_lookup_ex(None, None, 1, 1, 1, 1, 1, 1, 16, 8, 2, 2, None) == lib.ASU_ERR_ARG
    assert L.asu_hbm_index_maintain_ex(None, 1, 1, 1, 1, 1, 1, 0, 16, 0, 2, 2, None) == lib.ASU_ERR_ARG
    # LRU limits
    assert L.asu_lru_step(None, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 2048, 1, None, None, 1, 100, 16385, 16, 0) == \
        lib.ASU_ERR_ARG
    assert L.asu_lru_step(None, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 4, 1, None, None, 1, 100, 64, 16, 8) == \
        lib.ASU_ERR_ARG  # evicted row narrower than the free target
    # swap-in alignment
    assert L.asu_swapin_gather(None, 16, 10, 24, 0, 1, 1, 1, 1, 1, 4, 16, 4, 1, None) == lib.ASU_ERR_ALIGN
    assert L.asu_swapin_gather(None, 8, 10, 32, 0, 1, 1, 1, 1, 1, 4, 16, 4, 1, None) == lib.ASU_ERR_ALIGN
    assert L.asu_swapin_gather(None, 16, 10, 32, 40, 1, 1, 1, 1, 1, 4, 16, 4, 1, None) == lib.ASU_ERR_ALIGN
    assert L.asu_swapin_gather(None, 16, 10, 32, 16, 1, 1, 1, 1, 1, 4, 16, 4, 1, None) == lib.ASU_ERR_ARG
    # the balancing's entry points: the peer-store swap-in checks like the local one; null
    # arguments are rejected (or a no-op for the release calls) before any CUDA call
    assert L.asu_swapin_gather_to_peer(None, 16, 10, 24, 0, 1, 1, 1, 1, 1, 4, 16, 4, 1, None) == lib.ASU_ERR_ALIGN
    assert L.asu_swapin_gather_to_peer(None, 16, 10, 32, 16, 1, 1, 1, 1, 1, 4, 16, 4, 1, None) == lib.ASU_ERR_ARG
    assert L.asu_swapin_gather_to_peer(None, 16, 10, 32, 0, 1, 1, 1, 1, 1, 4, 16, 4, 0, None) == lib.ASU_OK
    assert L.asu_host_register(None, 4096, None) == lib.ASU_ERR_ARG
    assert L.asu_ipc_export(None, None, None) == lib.ASU_ERR_ARG
    assert L.asu_ipc_open(None, None) == lib.ASU_ERR_ARG
    assert L.asu_ipc_close(None) == lib.ASU_OK and L.asu_host_unregister(None) == lib.ASU_OK
    # resolver: block_size 0
    assert L.asu_kv_resolver_do(None, 1, 4, 1, 1, 1, 1, 1, 1, 4, 1, 1, 1, 1, 1, 1, 4, 4, 4, 4, 4, 4, 0, 1, 1,
                                None) == lib.ASU_ERR_ARG
    assert L.asu_kv_resolver_workspace_bytes(2048) == ((1 + 4096) * 4 + 15) // 16 * 16
    # SM-driven host copy: nothing to copy, null pointers, overlapping ranges
    assert L.asu_mapped_copy(None, None, None, 0) == lib.ASU_OK
    assert L.asu_mapped_copy(None, None, 4096, 16) == lib.ASU_ERR_ARG
    assert L.asu_mapped_copy(None, 4096, 4096 + 8, 16) == lib.ASU_ERR_ARG


def test_mapped_copy_wrapper_checks_its_arguments_on_the_host():
    import torch

    from asu_ascend_b200.host_pool import mapped_copy_

    with pytest.raises(RuntimeError, match="same size"):
        mapped_copy_(torch.zeros(4, dtype=torch.uint8), torch.zeros(8, dtype=torch.uint8))
    with pytest.raises(RuntimeError, match="CUDA tensor"):
        mapped_copy_(torch.zeros(4), torch.zeros(4))


def test_torch_ops_carry_reference_schemas():
    import asu_ascend_b200.ops  # noqa: F401

    want = {
        "asu_hbm_index_lookup": "(Tensor(a!) index, Tensor(b!) slot_to_index, Tensor(c!) free_slots, "
                                "Tensor(d!) free_head, Tensor query_index, int req_num) -> Tensor",
        "asu_hbm_index_maintain": "(Tensor(a!) index, Tensor(b!) slot_to_index, Tensor(c!) free_slots, "
                                  "Tensor(d!) free_head, Tensor last_query_slots, int req_num, int seed) -> ()",
    }
    for ns in ("asu", "_C_ascend"):
        for name, sig in want.items():
            schema = str(getattr(getattr(torch.ops, ns), name).default._schema)
            assert schema == f"{ns}::{name}{sig}"
        s = str(getattr(torch.ops, ns).npu_asu_resolve_kv_slots_single_req.default._schema)
        for arg in ("Tensor original_topk_indices", "int actual_seq_len", "int managed_prefix_len",
                    "token_state", "Tensor asu_record_addr", "hbm_slot_of_token", "slot_owner_token",
                    "Tensor free_slot_stack", "free_slot_count", "Tensor original_block_table",
                    "Tensor original_kv_cache_0", "Tensor original_kv_cache_1", "managed_kv_cache_0",
                    "managed_kv_cache_1", "int block_size"):
            assert arg in s


def test_ops_reject_cpu_tensors_and_bad_arguments():
    from asu_ascend_b200 import ops

    z = torch.zeros(4, dtype=torch.int32)
    with pytest.raises(RuntimeError, match="CUDA"):  # the dispatcher has no CPU kernel
        torch.ops.asu.asu_hbm_index_lookup(z, z, z, z, z, 1)
    with pytest.raises(RuntimeError, match="CUDA tensor"):  # and the implementation refuses host memory
        ops.asu_hbm_index_lookup(z, z, z, z, z, 1)
    with pytest.raises(RuntimeError, match="req_num"):
        ops.asu_hbm_index_lookup(z, z, z, z, z, 0)
    with pytest.raises(RuntimeError, match="int32"):
        ops.asu_hbm_index_maintain(z.float(), z, z, z, z, 1, 0)
    f = torch.ops.asu.npu_asu_resolve_kv_slots_single_req  # C++ op: argument checks on host tensors too
    kv = torch.zeros(4, 2)
    with pytest.raises(ValueError, match="block_size"):
        f(z, 4, 4, z, z, z, z, z, z, z, kv, kv, kv, kv, 0)
    with pytest.raises(ValueError, match="actual_seq_len"):
        f(z, -1, 4, z, z, z, z, z, z, z, kv, kv, kv, kv, 2)
    with pytest.raises(RuntimeError, match="CUDA tensor"):
        f(z, 4, 4, z, z, z, z, z, z, z, kv, kv, kv, kv, 2)
    with pytest.raises(RuntimeError, match="int32"):
        f(z, 4, 4, z.float(), z, z, z, z, z, z, kv, kv, kv, kv, 2)


def test_torch_binding_formats_numbers_and_links_the_process_libstdcxx():
    """libasu_torch.so must use the process's libstdc++ (a second, statically linked copy
    crashes on the first formatted number); its host-memory refusal formats an integer."""
    import subprocess

    from asu_ascend_b200 import ops

    z = torch.zeros(7, dtype=torch.int32)
    kv = torch.zeros(4, 2)
    with pytest.raises(RuntimeError, match="got 7 elements in host memory"):
        torch.ops.asu.npu_asu_resolve_kv_slots_single_req(z, 7, 7, z, z, z, z, z, z, z, kv, kv, kv, kv, 2)
    out = subprocess.run(["nm", "-D", "--defined-only", str(ops.TORCH_LIB_PATH)], capture_output=True, text=True)
    if out.returncode == 0:
        assert "codecvt" not in out.stdout and "_txnal_cow_string" not in out.stdout


def test_meta_kernels_give_output_shapes():
    import asu_ascend_b200.ops  # noqa: F401

    m = lambda *s, dt=torch.int32: torch.empty(*s, dtype=dt, device="meta")  # noqa: E731
    out = torch.ops._C_ascend.asu_hbm_index_lookup(m(2, 16), m(2, 8), m(2, 4), m(2), m(2, 5), 2)
    assert out.shape == (2, 5) and out.dtype == torch.int32
    sid, mask = torch.ops.asu.asu_hbm_index_lookup_simt(m(1, 32), m(1, 4), m(1, 4, dt=torch.int16), m(1, 3), 1)
    assert sid.shape == (1, 3) and mask.dtype == torch.bool
    r = torch.ops._C_ascend.npu_asu_resolve_kv_slots_single_req(
        m(1, 1, 7, dt=torch.int64), 6, 4, m(6), m(6), m(6), m(4), m(4), m(()), m(3),
        m(8, 2, dt=torch.float32), m(8, 3, dt=torch.float32), m(4, 2, dt=torch.float32),
        m(4, 3, dt=torch.float32), 2)
    assert r.shape == (1, 1, 7) and r.dtype == torch.int32


def test_workloads_are_deterministic_and_well_formed():
    from asu_ascend_b200.workloads import LocalityTrace, UniformReuseTrace, lookup_only_case, record_addresses

    a = LocalityTrace(3, 131072, seed=9)
    b = LocalityTrace(3, 131072, seed=9)
    for _ in range(3):
        x, y = a.step(), b.step()
        np.testing.assert_array_equal(x, y)
        for row in x:
            assert len(set(row.tolist())) == 2048
    prev = x
    nxt = a.step()
    for r in range(3):
        assert len(set(prev[r].tolist()) & set(nxt[r].tolist())) >= int(round(0.7 * 2048))
    u = UniformReuseTrace(2, 1 << 20, seed=1)
    u1, u2 = u.step(), u.step()
    assert len(set(u1[0].tolist()) & set(u2[0].tolist())) >= int(round(0.2 * 2048))
    table, query = lookup_only_case(req_num=2)
    assert table.shape == (2, 131072) and ((table >= 0).sum(1) == 4096).all()
    assert query.shape == (2, 2048)
    rec = record_addresses(4, 1000, 777)
    assert rec.min() >= 0 and rec.max() < 777 and rec.dtype == np.int32
