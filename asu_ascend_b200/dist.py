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


def placement_candidates(count: int, n: int, groups: list[list[int]] | None = None) -> list[list[int]]:
    """Device orders worth measuring for ``n`` ranks on ``count`` GPUs: the identity, the GPUs'
    two halves interleaved (0, count/2, 1, count/2 + 1, ...), and the round-robin over the
    host-link ``groups`` when NVML shows more than one; first ``n`` entries of each, no repeats."""
    half = count // 2
    inter = [d for pair in zip(range(half), range(half, count)) for d in pair] + list(range(2 * half, count))
    cands = [list(range(n)), inter[:n]]
    if groups is not None and len(groups) > 1:
        cands.append(spread_devices(n, groups))
    out: list[list[int]] = []
    for c in cands:
        if c not in out:
            out.append(c)
    return out


def choose_placement(cands: list[list[int]], rates: list[dict[int, float]], margin: float = 0.05) -> int:
    """Index of the candidate whose slowest GPU copies fastest with all of them copying at once
    (``rates[i]``: GB/s per device of candidate i); another candidate replaces the first (the
    identity) only when its slowest GPU is ``margin`` faster."""
    slowest = [min(r.values()) if r else 0.0 for r in rates]
    best = 0
    for i in range(1, len(cands)):
        if slowest[i] > slowest[best] * (1.0 + margin):
            best = i
    return best


def concurrent_h2d_gbs(devices: list[int], nbytes: int = 256 << 20, reps: int = 3) -> dict[int, float]:
    """Pinned host -> device copy bandwidth of each of ``devices`` with all of them copying at once
    (one process, one stream per device; median of ``reps``)."""
    import statistics

    src = {d: torch.empty(nbytes, dtype=torch.uint8).pin_memory() for d in devices}
    dst = {d: torch.empty(nbytes, dtype=torch.uint8, device=f"cuda:{d}") for d in devices}
    streams = {d: torch.cuda.Stream(device=d) for d in devices}
    rates: dict[int, list[float]] = {d: [] for d in devices}
    for _ in range(reps + 1):  # the first round warms up
        ev = {}
        for d in devices:
            torch.cuda.synchronize(d)
        for d in devices:
            with torch.cuda.device(d), torch.cuda.stream(streams[d]):
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record()
                dst[d].copy_(src[d], non_blocking=True)
                b.record()
                ev[d] = (a, b)
        for d in devices:
            torch.cuda.synchronize(d)
        for d in devices:
            rates[d].append(nbytes / (ev[d][0].elapsed_time(ev[d][1]) * 1e-3) / 1e9)
    return {d: statistics.median(v[1:]) for d, v in rates.items()}


def measure_placement(n: int) -> dict:
    """Run in a process of its own (it opens a context on every visible GPU): measure each
    candidate order's concurrent H2D rates and pick one (``choose_placement``)."""
    count = torch.cuda.device_count()
    level = nvml_levels(count)
    groups = host_link_groups(count, level) if level is not None else None
    cands = placement_candidates(count, n, groups)
    rates = [concurrent_h2d_gbs(c) for c in cands]
    best = choose_placement(cands, rates)
    return {"devices": cands[best], "candidates": cands,
            "slowest_gbs": [round(min(r.values()), 1) for r in rates], "host_link_groups": groups}


def placed_device(local_rank: int, local_world: int, store=None, key: str = "asu_b200/placement",
                  timeout_s: float = 180.0) -> tuple[int, dict]:
    """CUDA device of ``local_rank`` among ``local_world`` ranks on this host, and how it was chosen.

    With as many ranks as visible GPUs, rank r takes GPU r.  With fewer, GPUs can share a host
    attachment unevenly (on the 8-GPU B200 boxes measured here GPUs 0-3 share ~116 GB/s of host
    -> device bandwidth while GPUs 4-7 get ~54 GB/s each, and NVML reports every pair at the same
    topology level), so local rank 0 measures the candidate orders in a child process and puts the
    choice in ``store`` (a c10d store shared by the host's ranks); the other ranks read it there."""
    import json
    import subprocess
    import sys

    count = torch.cuda.device_count()
    if local_world >= count or store is None:
        return local_rank, {"rule": "GPU = local rank"}
    if local_rank == 0:
        try:
            res = subprocess.run([sys.executable, "-m", "asu_ascend_b200.dist", "--measure-placement",
                                  str(local_world)], capture_output=True, text=True, timeout=timeout_s)
            info = json.loads(res.stdout.strip().splitlines()[-1]) if res.returncode == 0 else None
        except (subprocess.TimeoutExpired, ValueError, IndexError):
            info = None
        if info is None:
            info = {"devices": list(range(local_world)), "error": "placement measurement failed"}
        info["rule"] = "measured: the candidate order whose slowest GPU copies fastest"
        store.set(key, json.dumps(info))
    info = json.loads(store.get(key))
    return int(info["devices"][local_rank]), info


if __name__ == "__main__":
    import json
    import sys

    if len(sys.argv) == 3 and sys.argv[1] == "--measure-placement":
        print(json.dumps(measure_placement(int(sys.argv[2]))))
    else:
        raise SystemExit("usage: python -m asu_ascend_b200.dist --measure-placement N")
