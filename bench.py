#!/usr/bin/env python
"""Benchmark of the KV-resolver hot path on B200: one step = one decode-layer resolve for a
batch of requests -- exact-LRU maintain + lookup (one kernel) followed by the swap-in
gather of every missed 656-byte KV row from pinned, mapped host memory into the HBM slot
pool (one kernel).

    python bench.py [--gpus N --steps K --warmup W] [--impl b200|reference]

Workload (per GPU; requests are sharded, so N GPUs run N x 128 independent requests, weak
scaling, no collective on the data path): 128 requests, 128K-token context, top-k 2048
per step with reuse + Zipf locality (70% of the previous step's ids kept, 30% Zipf(1.1)
draws), 8192 HBM slots per request, LRU free target 2048, KV rows of 656 B (512 fp8 +
64 bf16 + 16 B scales, random bytes) in a 2^20-row pinned host pool.  Inputs are
synthetic and seeded.  The pools are first filled by `--prefill` untimed steps so the
timed steps run at the steady-state miss rate (~13%).

Prints one JSON line (rank 0).  `value` is resolved KV indices/s for the whole job with
inputs resident in HBM; `e2e` is the same through the public API with the step's top-k
copied from pinned host memory and the slot ids + hit mask copied back inside the timed
region.  `--impl reference` times the CPU restatement of the reference algorithm on all
host cores (the reference's own implementation is Python / AscendC and cannot run here).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from datetime import timedelta
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

R, K, S, Q, TARGET, ROW = 128, 131072, 8192, 2048, 2048, 656
POOL_ROWS = 1 << 20
# From the ncu captures summarised in profiles/ (first timed step of this workload):
SWAPIN_PCIE_READ_BYTES_PER_LAUNCH = 52.49e9 * 714.4e-6   # pcie__read_bytes.sum.per_second x duration
SWAPIN_NCU_INSTALLS = 31.0e6 / ROW                        # rows swapped in by that launch (~31 MB)
LRU_DRAM_BYTES_PER_LAUNCH = 22.05e6 + 0.055e6             # dram__bytes_read.sum + dram__bytes_write.sum
METRIC = "resolved KV indices/sec (lookup + LRU maintain + swap-in gather)"
UNIT = "indices/s"


def parse_args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--prefill", type=int, default=8)
    p.add_argument("--impl", choices=("b200", "reference"), default="b200")
    p.add_argument("--seed", type=int, default=2026)
    p.add_argument("--cpu-sample-s", type=float, default=12.0)
    p.add_argument("--no-cpu-baseline", action="store_true")
    return p.parse_args()


def load_peaks():
    try:
        return json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
    except Exception:
        return {}


def config_dict(world: int) -> dict:
    return {"workload": f"resolver: {R} req/GPU x top-k {Q}, 128K context, {S} slots/req, LRU target {TARGET}, "
                        f"{ROW} B rows from a pinned host pool ({POOL_ROWS} rows)",
            "requests_per_gpu": R, "global_batch": R * world, "topk": Q, "context": K, "slots_per_request": S,
            "free_target": TARGET, "row_bytes": ROW, "locality": "70% reuse + 30% zipf(1.1)",
            "l2": "flushed before every timed step (256 MiB write, then 256 MiB read so no dirty lines remain)", "parallelism": f"request-sharded x{world}"}


# ------------------------------------------------------------------ clocks

class ClockSampler:
    """nvidia-smi samples every 200 ms while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu_index = gpu_index
        self.lines: list[str] = []
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader",
                                          "-lms", "200", "-i", str(self.gpu_index)],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
        except Exception:
            self.proc = None

    def _read(self):
        for ln in self.proc.stdout:
            self.lines.append(ln.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1].split()[0]))
                mx.append(float(parts[2].split()[0]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------------ CPU side

def make_trace(seed: int, n_steps: int) -> np.ndarray:
    from asu_ascend_b200.workloads import LocalityTrace

    tr = LocalityTrace(R, K, topk=Q, reuse=0.7, zipf_s=1.1, seed=seed)
    return np.stack([tr.step() for _ in range(n_steps)])


def cpu_port_run(trace: np.ndarray, prefill: int, timed: int, time_cap_s: float, threads: int):
    """The C restatement of LRUManagedCache + the row copy on `threads` host cores."""
    from asu_ascend_b200.workloads import record_addresses
    from oracle import c_oracle

    rng = np.random.Generator(np.random.PCG64(7))
    host = rng.integers(0, 256, (POOL_ROWS, ROW), dtype=np.uint8)
    rec = record_addresses(R, K, POOL_ROWS)
    slot_pool = np.zeros((R, S, ROW), np.uint8)
    pools = c_oracle.LruPools(R, K, S, TARGET)
    for i in range(prefill):
        pools.step_all(trace[i], threads=threads, want_outputs=False, host_pool=host, record=rec,
                       slot_pool=slot_pool)
    # The timed top-k sets are replayed in a cycle until about time_cap_s of CPU work has
    # been done (one pass takes milliseconds on a many-core host).
    done, t_total = 0, 0.0
    while t_total < time_cap_s and done < 200000:
        i = prefill + done % timed
        t0 = time.perf_counter()
        pools.step_all(trace[i], threads=threads, want_outputs=True, host_pool=host, record=rec,
                       slot_pool=slot_pool)
        t_total += time.perf_counter() - t0
        done += 1
    pools.close()
    return done * R * Q / t_total, done, t_total


def run_reference(args, world: int, rank: int):
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    trace = make_trace(args.seed, args.prefill + args.warmup + args.steps)
    value, done, secs = cpu_port_run(trace, args.prefill + args.warmup, args.steps, args.cpu_sample_s, threads)
    line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": done, "warmup": args.warmup,
            "ms_per_step": secs / done * 1e3, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "int32", "data": "synthetic", "config": config_dict(1), "impl": "reference",
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                             "sample": f"{done} steps x {R} requests x top-k {Q} ({secs:.1f} s, cycling the "
                                       f"{args.steps} timed top-k sets after {args.prefill + args.warmup} untimed "
                                       "steps), C restatement of LRUManagedCache + row memcpy, all host threads"},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ GPU side

def h2d_peak_gbs(torch, dev) -> float:
    n = 256 << 20
    src = torch.empty(n, dtype=torch.uint8, pin_memory=True)
    dst = torch.empty(n, dtype=torch.uint8, device=dev)
    best = 0.0
    for _ in range(10):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        dst.copy_(src, non_blocking=True)
        b.record()
        b.synchronize()
        best = max(best, n / (a.elapsed_time(b) * 1e-3) / 1e9)
    return best


def run_b200(args, world: int, rank: int, local_rank: int):
    import torch
    import torch.distributed as dist

    import asu_ascend_b200

    asu_ascend_b200.load()
    from asu_ascend_b200.dist import max_over_ranks, reduce_stats
    from asu_ascend_b200.host_pool import HostRowPool, check_status
    from asu_ascend_b200.lru import LruSlotPools
    from asu_ascend_b200.workloads import record_addresses

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    K_steps, W = args.steps, args.warmup
    n_steps = args.prefill + W + 2 * K_steps
    trace = make_trace(args.seed + 1000 * rank, n_steps)
    q_dev = torch.from_numpy(trace).to(dev)
    q_host = torch.from_numpy(trace).pin_memory()

    host = HostRowPool(POOL_ROWS, ROW)
    host.fill_random(11 + rank)
    rec = torch.from_numpy(record_addresses(R, K, POOL_ROWS)).to(dev)
    slot_pool = torch.zeros((R, S, ROW), dtype=torch.uint8, device=dev)
    pools = LruSlotPools(R, K, S, TARGET, Q, device=dev)
    outs = [pools.new_output(), pools.new_output()]
    status = torch.zeros(R, dtype=torch.int32, device=dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    flush_read = torch.ones(64 << 20, dtype=torch.int32, device=dev)  # 256 MiB

    def flush_l2():
        # Write 256 MiB (evicts everything), then read another 256 MiB so the write-back of the
        # dirty lines happens here, outside the timed region: the step starts on a cold, clean L2.
        flush.zero_()
        flush_read.sum()
    h2d_peak = h2d_peak_gbs(torch, dev)

    def step(i, o):
        pools.step(q_dev[i], out=o)
        host.swapin(rec, q_dev[i], o.slot, o.install, slot_pool, status=status)

    for i in range(args.prefill + W):  # untimed: fill the pools, then warm up
        step(i, outs[i % 2])
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()

    base = args.prefill + W
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(K_steps)]
    free_before = torch.empty(K_steps, dtype=torch.int64, device=dev)
    free_after = torch.empty(K_steps, dtype=torch.int64, device=dev)
    stats0 = pools.stats.sum(0).clone()
    gpu_index = int(os.environ.get("CUDA_VISIBLE_DEVICES", str(local_rank)).split(",")[local_rank]) \
        if os.environ.get("CUDA_VISIBLE_DEVICES") else local_rank
    clocks = ClockSampler(gpu_index)
    clocks.start()
    torch.cuda.synchronize()
    for k in range(K_steps):
        o = outs[k % 2]
        flush_l2()
        free_before[k] = pools.free_count.sum()
        torch.cuda._sleep(100_000)  # keep the GPU busy while the host queues the step
        ev[k][0].record()
        pools.step(q_dev[base + k], out=o)
        ev[k][1].record()
        host.swapin(rec, q_dev[base + k], o.slot, o.install, slot_pool, status=status)
        ev[k][2].record()
        free_after[k] = pools.free_count.sum()
    torch.cuda.synchronize()
    clk = clocks.stop()
    resolve_ms = [e[0].elapsed_time(e[1]) for e in ev]
    swapin_ms = [e[1].elapsed_time(e[2]) for e in ev]
    step_ms = [e[0].elapsed_time(e[2]) for e in ev]
    d_stats = (pools.stats.sum(0) - stats0).cpu().tolist()
    installs, evictions = int(d_stats[2]), int(d_stats[4])
    res0 = (R * S * K_steps - int(free_before.sum().item()))
    res2 = (R * S * K_steps - int(free_after.sum().item()))

    # e2e through the public API: host top-k in, slot ids + hit mask out, copies timed
    base2 = base + K_steps
    slot_host = torch.empty((R, Q), dtype=torch.int32, pin_memory=True)
    hit_host = torch.empty((R, Q), dtype=torch.bool, pin_memory=True)
    q_in = torch.empty((R, Q), dtype=torch.int32, device=dev)
    ev2 = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(K_steps)]
    for k in range(K_steps):
        o = outs[k % 2]
        flush_l2()
        torch.cuda._sleep(100_000)
        ev2[k][0].record()
        q_in.copy_(q_host[base2 + k], non_blocking=True)
        pools.step(q_in, out=o)
        host.swapin(rec, q_in, o.slot, o.install, slot_pool, status=status)
        slot_host.copy_(o.slot, non_blocking=True)
        hit_host.copy_(o.hit, non_blocking=True)
        ev2[k][1].record()
    torch.cuda.synchronize()
    e2e_ms = [e[0].elapsed_time(e[1]) for e in ev2]
    pools.check_status()
    check_status(status, "swapin")

    max_ms, max_e2e_ms = max_over_ranks([sum(step_ms), sum(e2e_ms)], dev)  # slowest rank
    job_stats = reduce_stats(pools.stats).cpu().tolist()  # end-of-run statistics (NCCL all-reduce)

    if rank == 0:
        peaks = load_peaks()
        hbm_peak = float(peaks.get("hbm_gbs", 6650.0))
        alg_bytes = K_steps * R * Q * 14 + 4 * (res0 + res2) + 12 * installs + 20 * evictions
        resolve_s = sum(resolve_ms) * 1e-3
        achieved = alg_bytes / K_steps / (resolve_s / K_steps) / 1e9
        swap_bytes = installs * ROW
        swap_gbs = swap_bytes / (sum(swapin_ms) * 1e-3) / 1e9
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            threads = os.cpu_count() or 1
            v, done, secs = cpu_port_run(trace, base, K_steps, args.cpu_sample_s, threads)
            cpu = {"value": v, "unit": UNIT, "cores": threads, "kind": "port",
                   "sample": f"{done} steps x {R} requests x top-k {Q} ({secs:.1f} s, cycling the {K_steps} timed "
                             "top-k sets of this workload), C restatement of LRUManagedCache + row memcpy, all host "
                             "threads"}
        line = {
            "metric": METRIC, "value": world * R * Q * K_steps / (max_ms * 1e-3), "unit": UNIT, "n_gpus": world,
            "steps": K_steps, "warmup": W, "ms_per_step": max_ms / K_steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int32", "data": "synthetic",
            "config": config_dict(world),
            "p50_resolve_us": statistics.median(resolve_ms) * 1e3,
            "p50_swapin_us": statistics.median(swapin_ms) * 1e3,
            "miss_rate": installs / (K_steps * R * Q),
            "swapin_gbs": swap_gbs,
            # dominant kernel by time (ncu launch list: ~93% of the step) -- bound by the host link
            "roofline": {"bound": "host_link", "kernel": "swapin_kernel", "achieved": swap_gbs, "peak": h2d_peak,
                         "unit": "GB/s", "frac": swap_gbs / h2d_peak,
                         "traffic": SWAPIN_PCIE_READ_BYTES_PER_LAUNCH * installs / K_steps / SWAPIN_NCU_INSTALLS,
                         "traffic_kind": "PCIe read bytes per launch (ncu pcie__read_bytes, scaled to this run's "
                                         "installs per step)",
                         "peak_source": "pinned cudaMemcpyAsync H2D 256 MiB, best of 10, this run"},
            "roofline_lru": {"bound": "hbm", "kernel": "lru_step_kernel", "achieved": achieved, "peak": hbm_peak,
                             "unit": "GB/s", "frac": achieved / hbm_peak,
                             "traffic": LRU_DRAM_BYTES_PER_LAUNCH,
                             "traffic_kind": "dram__bytes_read.sum + dram__bytes_write.sum of one launch (ncu)",
                             "algorithmic_bytes_per_launch": alg_bytes / K_steps,
                             "peak_source": "measured HBM copy bandwidth (MEASURED_PEAKS.json hbm_gbs)"},
            "e2e": {"value": world * R * Q * K_steps / (max_e2e_ms * 1e-3), "unit": UNIT,
                    "h2d_bytes_per_step": R * Q * 4, "d2h_bytes_per_step": R * Q * 5},
            "gpu_launches": 2 * K_steps,
            "job_stats": dict(zip(LruSlotPools.STAT_NAMES, job_stats)),
            "cpu_baseline": cpu,
            "clocks": clk,
        }
        print(json.dumps(line), flush=True)
    host.close()


def main():
    args = parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, world, rank)
        return
    if world > 1:
        import torch
        import torch.distributed as dist

        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local_rank))
    try:
        run_b200(args, world, rank, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
