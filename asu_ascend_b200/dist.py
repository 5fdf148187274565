"""Request sharding and end-of-run statistics for multi-GPU runs (one process per GPU).

Requests are independent (each owns its tables, slot pool and host rows), so a job of
``total`` requests is split into contiguous ranges, one per rank, with no collective on the
data path.  The only collectives are the end-of-run reductions below (NCCL on GPUs, gloo in
the CPU tests).
"""

from __future__ import annotations

from typing import Callable

import torch


def shard_range(total: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous [start, end) of ``total`` requests owned by ``rank`` (sizes differ by at most 1)."""
    if world <= 0 or not 0 <= rank < world or total < 0:
        raise ValueError("need world > 0, 0 <= rank < world, total >= 0")
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def _initialized() -> bool:
    return torch.distributed.is_available() and torch.distributed.is_initialized()


def reduce_stats(stats: torch.Tensor) -> torch.Tensor:
    """Sum per-rank int64 counters (hits, misses, installs, shortages, evictions) over ranks."""
    total = stats.reshape(-1, stats.shape[-1]).sum(0).to(torch.int64)
    if _initialized():
        torch.distributed.all_reduce(total, op=torch.distributed.ReduceOp.SUM)
    return total


def rows_by_rank(values: list[float], device: torch.device | str = "cpu") -> list[list[float]]:
    """Every rank's ``values`` (same length on all ranks), indexed by rank: an end-of-run report
    of per-rank figures, one all-reduce of a [world, n] tensor holding this rank's row."""
    if not _initialized():
        return [list(map(float, values))]
    world, rank = torch.distributed.get_world_size(), torch.distributed.get_rank()
    t = torch.zeros((world, len(values)), dtype=torch.float64, device=device)
    t[rank] = torch.tensor(values, dtype=torch.float64)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.SUM)
    return t.cpu().tolist()


def max_over_ranks(values: list[float], device: torch.device | str = "cpu") -> list[float]:
    """Element-wise max over ranks (timings are reported as the slowest rank's)."""
    t = torch.tensor(values, dtype=torch.float64, device=device)
    if _initialized():
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return t.tolist()


def gpu_local_cpus(gpu_index: int, nvml=None) -> list[int]:
    """Host CPUs that NVML reports as local to physical GPU ``gpu_index`` (its NUMA node's
    cores), restricted to the CPUs this process may use; empty when NVML cannot tell."""
    import os

    try:
        if nvml is None:
            import pynvml as nvml
        nvml.nvmlInit()
        handle = nvml.nvmlDeviceGetHandleByIndex(gpu_index)
        words = ((os.cpu_count() or 1) + 63) // 64
        mask = nvml.nvmlDeviceGetCpuAffinity(handle, words)
    except Exception:
        return []
    cpus = {w * 64 + b for w, word in enumerate(mask) for b in range(64) if (int(word) >> b) & 1}
    return sorted(cpus & os.sched_getaffinity(0))


def bind_to_gpu_local_cpus(gpu_index: int, nvml=None) -> list[int]:
    """Run this process on the CPUs local to its GPU before it allocates the pinned host pool.

    Page-locked host memory is placed on the NUMA node of the thread that allocates and first
    touches it, and every swap-in reads that memory over the GPU's host link, so on a
    multi-socket host the pool belongs on the GPU's socket.  Returns the CPUs bound (empty:
    affinity left unchanged, e.g. a single-node host or no NVML)."""
    import os

    cpus = gpu_local_cpus(gpu_index, nvml)
    if cpus and set(cpus) != os.sched_getaffinity(0):
        os.sched_setaffinity(0, cpus)
        return cpus
    return []


# ------------------------------------------------------------------ rank placement over host links

def host_link_groups(count: int, level: Callable[[int, int], int]) -> list[list[int]]:
    """Groups of GPUs (ordinals ``0..count-1``) that share a host attachment.

    ``level(i, j)`` is the NVML topology level of the pair's closest common ancestor (10 same board,
    20 / 30 PCIe switches or one host bridge, 40 same NUMA node, 50 across the system).  GPUs are in
    one group when their level is below the largest level seen between any two of them, so a box
    whose GPUs hang off two sockets (or two host bridges) gives two groups, and a box where every
    pair sits at the same level gives one."""
    if count <= 1:
        return [list(range(count))]
    levels = [level(i, j) for i in range(count) for j in range(i + 1, count)]
    top = max(levels)
    if min(levels) == top:
        return [list(range(count))]
    parent = list(range(count))

    def find(x: int) -> int:
        while parent[x] != x:
            parent[x] = parent[parent[x]]
            x = parent[x]
        return x

    for i in range(count):
        for j in range(i + 1, count):
            if level(i, j) < top:
                parent[find(j)] = find(i)
    groups: dict[int, list[int]] = {}
    for i in range(count):
        groups.setdefault(find(i), []).append(i)
    return sorted(groups.values())


def spread_devices(local_world: int, groups: list[list[int]]) -> list[int]:
    """GPU ordinal of each local rank: round-robin over the host-link groups, lowest ordinal first,
    so that N ranks on a box with more GPUs than ranks put equal load on each host attachment.
    With as many ranks as GPUs every GPU is used and rank r keeps GPU r."""
    count = sum(len(g) for g in groups)
    if local_world >= count or len(groups) <= 1:
        return list(range(local_world))
    order, queues = [], [list(g) for g in groups]
    while len(order) < local_world:
        for q in queues:
            if q and len(order) < local_world:
                order.append(q.pop(0))
    return order


def nvml_levels(count: int, nvml=None) -> Callable[[int, int], int] | None:
    """NVML topology level between the CUDA devices ``i`` and ``j`` of this process (matched by PCI
    bus id), or None when NVML or the device properties cannot tell."""
    try:
        if nvml is None:
            import pynvml as nvml
        nvml.nvmlInit()
        handles = []
        for i in range(count):
            p = torch.cuda.get_device_properties(i)
            bus = f"{p.pci_domain_id:08x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
            handles.append(nvml.nvmlDeviceGetHandleByPciBusId(bus))
        cache = {}
        for i in range(count):
            for j in range(i + 1, count):
                cache[(i, j)] = int(nvml.nvmlDeviceGetTopologyCommonAncestor(handles[i], handles[j]))
    except Exception:
        return None
    return lambda i, j: cache[(min(i, j), max(i, j))]


def placed_device(local_rank: int, local_world: int) -> tuple[int, list[list[int]]]:
    """CUDA device of ``local_rank`` among ``local_world`` ranks on this host, and the host-link
    groups it was chosen from (one group: identity placement)."""
    count = torch.cuda.device_count()
    if local_world >= count:
        return local_rank, [list(range(count))]
    level = nvml_levels(count)
    groups = host_link_groups(count, level) if level is not None else [list(range(count))]
    return spread_devices(local_world, groups)[local_rank], groups
