"""Request sharding and end-of-run statistics for multi-GPU runs (one process per GPU).

Requests are independent (each owns its tables, slot pool and host rows), so a job of
``total`` requests is split into contiguous ranges, one per rank, with no collective on the
data path.  The only collectives are the end-of-run reductions below (NCCL on GPUs, gloo in
the CPU tests).
"""

from __future__ import annotations

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
