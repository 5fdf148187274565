"""B200-native KV-resolver hot path of ASU-Ascend: lookup, slot maintenance, swap-in.

Submodules (importing any of the CUDA-backed ones loads libasu_b200.so and fails loudly
if it is not built -- there is no CPU fallback):

* ``ops``               loads the C++ torch operators with the reference schemas, under
                        torch.ops.asu and torch.ops._C_ascend (asu_hbm_index_lookup / _maintain /
                        _lookup_simt, npu_asu_resolve_kv_slots_single_req)
* ``manager``           per-layer single-request resolver state (patch/0003 manager)
* ``sparse_mla``        resolver slots for vLLM's FlashMLA-sparse decode
* ``vllm_backend``      FlashMLASparseImpl subclass that decodes over the managed cache
* ``kv_store``          MicroKV-keyed view of the host row pool (prefill write-back)
* ``kv_server``         MicroKV socket protocol in front of that store
* ``hbm_lookup_update`` mirror of the reference's gather/update extension module
* ``lru``               per-request exact-LRU slot pools (LruSlotPools)
* ``host_pool``         pinned mapped host row pool + swap-in gather (HostRowPool)
* ``dist``              request sharding, end-of-run statistics, rank placement on a host's GPUs
* ``balance``           swap-in balancing between the ranks of one host (peer stores over NVLink)
* ``workloads``         seeded synthetic traces (no CUDA needed)
* ``build``             nvcc build of the library
"""

__version__ = "1.0.0"


def load():
    """Import every CUDA-backed submodule (registers the torch operators)."""
    from . import _lib, hbm_lookup_update, host_pool, lru, ops  # noqa: F401

    return _lib.lib
