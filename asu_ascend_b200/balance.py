"""Swap-in balancing across the ranks of one box (request-sharded multi-GPU runs).

Requests are sharded over the GPUs with no collective on the data path (``dist.py``), and each rank
swaps in its own requests' rows through its own host link.  When every GPU of a box reads host
memory at once, the host serves them unevenly: on the 8-GPU B200 boxes measured here, pinned H2D
copies with all eight ranks copying reach ~22 GB/s per GPU on GPUs 0-3 and ~36 GB/s on GPUs 4-7.
The slowest ranks then set the job's step time while the others idle.

The balancer pairs ranks, slowest with fastest, and lets the helper (fast link) swap in the rows of
the last ``m`` requests of its owner (slow link).  Per step and layer:

* owner: LRU step -> NCCL send of those requests' query / slot / install rows to the helper ->
  swap-in of its first ``R - m`` requests -> wait for the helper's 4-byte done message;
* helper: NCCL receive -> ``asu_swapin_gather_to_peer`` on a side stream, which reads the owner's
  host pool (a shared-memory file the owner handed over, mapped and registered in this process)
  through this GPU's host link and stores the rows into the owner's slot pool (a CUDA IPC mapping)
  over NVLink -> NCCL send of the done message.  Its own swap-in runs meanwhile on the main stream.

Every cross-GPU wait is a NCCL message; no kernel waits on another GPU.  The split is chosen by a
calibration (``calibrate``): a few steps with every rank swapping in its own rows, all ranks at
once, give each rank's rate; ranks are paired and ``m`` solves
``(R_o - m) / rate_o = (R_h + m) / rate_h``; two more rounds with the pairs balancing refine ``m``.

The reference has nothing like it: its swap-in is a per-request MicroKV socket fetch on one NPU
(docs/v0.1/kv-cache-offload-v0.1-real-ops-design.md:293-312), and it runs no multi-NPU job.
"""

from __future__ import annotations

import ctypes
import json
import os
import socket
import statistics
import struct
import time
from dataclasses import dataclass, field
from typing import Callable, Sequence

import torch

from ._lib import check, lib, raise_on_status

# ------------------------------------------------------------------ planning (pure)


def balanced_share(req_owner: int, req_helper: int, rate_owner: float, rate_helper: float) -> int:
    """Requests ``m`` of the owner that the helper takes so that both finish together:
    ``(req_owner - m) / rate_owner == (req_helper + m) / rate_helper`` (rates in requests per
    second), rounded, and clamped to [0, req_owner - 1]."""
    if rate_owner <= 0 or rate_helper <= 0 or req_owner <= 1:
        return 0
    m = (req_owner * rate_helper - req_helper * rate_owner) / (rate_owner + rate_helper)
    return max(0, min(req_owner - 1, int(round(m))))


def plan_pairs(rates: Sequence[float], req: Sequence[int], min_share: float = 0.02) -> list[tuple[int, int, int]]:
    """Pair ranks for balancing: the i-th slowest with the i-th fastest.

    ``rates[r]``: requests per second rank r swapped in with every rank swapping in at once;
    ``req[r]``: its requests.  Returns ``[(owner, helper, m)]`` for the pairs worth balancing
    (``m >= 1`` and at least ``min_share`` of the owner's requests); each rank is in at most one
    pair, and every rank computes the same plan from the same inputs."""
    n = len(rates)
    if len(req) != n:
        raise ValueError("rates and req must have one entry per rank")
    order = sorted(range(n), key=lambda r: (rates[r], r))
    pairs = []
    for i in range(n // 2):
        o, h = order[i], order[n - 1 - i]
        m = balanced_share(req[o], req[h], rates[o], rates[h])
        if m >= 1 and m >= min_share * req[o]:
            pairs.append((o, h, m))
    return pairs


def best_plan(measured: Sequence[tuple[float, list[tuple[int, int, int]]]], unbalanced_ms: float | None = None,
              margin: float = 0.02) -> list[tuple[int, int, int]]:
    """The measured plan whose slowest rank finished first: ``measured`` holds (slowest rank's
    swap-in ms, plan) per calibration round (the earlier round wins a tie).  With the unbalanced
    round's figure, a plan is kept only if it beats it by ``margin``; otherwise every share is 0."""
    if not measured:
        return []
    ms, plan = min(measured, key=lambda x: x[0])
    if unbalanced_ms is not None and not ms < (1.0 - margin) * unbalanced_ms:
        return [(o, h, 0) for o, h, _ in plan]
    return list(plan)


def refine_share(req_owner: int, req_helper: int, m: int, owner_ms: float, helper_ms: float) -> int:
    """New share from a round run with share ``m``: the owner swapped in ``req_owner - m`` requests
    in ``owner_ms``, the helper ``req_helper + m`` in ``helper_ms``."""
    if owner_ms <= 0 or helper_ms <= 0:
        return m
    return balanced_share(req_owner, req_helper, (req_owner - m) / owner_ms, (req_helper + m) / helper_ms)


# ------------------------------------------------------------------ fd hand-over (Unix socket)


def socket_name(token: str, rank: int) -> str:
    """Abstract-namespace Unix socket of ``rank`` (no file to clean up)."""
    return f"\0asu-balance-{token}-{rank}"


class FdServer:
    """Owner side: hands one file descriptor plus a payload to the helper that connects."""

    def __init__(self, name: str):
        self.sock = socket.socket(socket.AF_UNIX, socket.SOCK_STREAM)
        self.sock.bind(name)
        self.sock.listen(1)

    def serve(self, fd: int, payload: bytes, timeout_s: float = 120.0) -> None:
        self.sock.settimeout(timeout_s)
        conn, _ = self.sock.accept()
        with conn:
            socket.send_fds(conn, [struct.pack("<Q", len(payload)) + payload], [fd])

    def close(self) -> None:
        self.sock.close()


def fetch_fd(name: str, timeout_s: float = 120.0) -> tuple[int, bytes]:
    """Helper side: connect to ``name`` and receive (fd, payload).  The caller owns the fd."""
    deadline = time.monotonic() + timeout_s
    while True:
        s = socket.socket(socket.AF_UNIX, socket.SOCK_STREAM)
        try:
            s.settimeout(max(1.0, deadline - time.monotonic()))
            s.connect(name)
            break
        except (ConnectionRefusedError, FileNotFoundError):
            s.close()
            if time.monotonic() > deadline:
                raise TimeoutError(f"no fd server at {name[1:]!r}")
            time.sleep(0.05)
    with s:
        msg, fds, _, _ = socket.recv_fds(s, 1 << 16, 1)
        if len(fds) != 1 or len(msg) < 8:
            for f in fds:
                os.close(f)
            raise RuntimeError("fd hand-over: malformed message")
        (n,) = struct.unpack("<Q", msg[:8])
        data = bytearray(msg[8:])
        while len(data) < n:
            chunk = s.recv(n - len(data))
            if not chunk:
                os.close(fds[0])
                raise RuntimeError("fd hand-over: connection closed early")
            data += chunk
    return fds[0], bytes(data)


# ------------------------------------------------------------------ IPC of device allocations


def ipc_export(t: torch.Tensor) -> tuple[str, int]:
    """(hex handle, offset) of the CUDA allocation holding ``t``'s first byte."""
    h = (ctypes.c_uint8 * 64)()
    off = ctypes.c_uint64()
    with torch.cuda.device(t.device):
        check(lib.asu_ipc_export(t.data_ptr(), h, ctypes.byref(off)), "asu_ipc_export")
    return bytes(h).hex(), off.value


def ipc_open(handle_hex: str, device: torch.device) -> int:
    """Map an exported allocation into this process on ``device``; returns the mapping's base."""
    raw = bytes.fromhex(handle_hex)
    h = (ctypes.c_uint8 * 64).from_buffer_copy(raw)
    base = ctypes.c_void_p()
    with torch.cuda.device(device):
        check(lib.asu_ipc_open(h, ctypes.byref(base)), "asu_ipc_open")
    return base.value


# ------------------------------------------------------------------ the balancer


@dataclass
class _HelperSide:
    owner: int
    req: int                     # the owner's requests
    pool: object                 # HostRowPool attached to the owner's shared pool
    peer_bases: list[int]        # IPC mapping bases, one per layer
    peer_pools: list[int]        # owner's slot pool addresses in this process, one per layer
    slot_count: int
    row_bytes: int
    recs: list[torch.Tensor]     # copies of the owner's record tables, one per layer
    q: torch.Tensor              # receive buffers [req, Q]
    slot: torch.Tensor
    install: torch.Tensor
    status: torch.Tensor         # [req] device status of the rows swapped in for the owner


@dataclass
class _Window:
    events: list = field(default_factory=list)


class SwapinBalancer:
    """Drop-in for ``HostRowPool.swapin`` in a request-sharded multi-rank loop (see module doc).

    ``host``: this rank's pool, created with ``shared=True``; ``recs[layer]``: [R, K] record tables;
    ``slot_pools[layer]``: [R, S, row] slot pools; ``status``: [R] swap-in status; ``query_count``:
    the top-k per request and step.  Until ``calibrate``
    sets a plan every call is a plain local swap-in."""

    def __init__(self, host, recs: list[torch.Tensor], slot_pools: list[torch.Tensor], status: torch.Tensor,
                 query_count: int, min_share: float = 0.02):
        import torch.distributed as dist

        if host.shared is None:
            raise RuntimeError("the balancer needs a host pool created with shared=True")
        self.dist = dist
        self.rank, self.world = dist.get_rank(), dist.get_world_size()
        self.host, self.recs, self.pools, self.status = host, recs, slot_pools, status
        self.device = slot_pools[0].device
        self.R = recs[0].shape[0]
        self.query_count = query_count
        self.min_share = min_share
        self.pairs: list[tuple[int, int, int]] = []
        self.role: str | None = None
        self.peer = -1
        self.m = 0
        self.helper: _HelperSide | None = None
        self.side = torch.cuda.Stream(self.device)
        self.done_tx = torch.ones(1, dtype=torch.int32, device=self.device)
        self.done_rx = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.window: _Window | None = None
        self.history: list[dict] = []

    # ---- per step ----
    def swapin(self, layer: int, query: torch.Tensor, out) -> None:
        """Swap in the rows of ``out.install`` for ``query`` (this rank's [R, Q] top-k) on the current
        stream; with a plan, part of them is done by (or for) the paired rank."""
        main = torch.cuda.current_stream(self.device)
        ev = None
        if self.window is not None:
            ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
            ev[0].record(main)
        dist, R, m = self.dist, self.R, self.m
        if self.role == "owner" and m > 0:
            k = R - m
            # The done message is a separate operation: NCCL runs the operations of one group to
            # the same peer as paired work items in order, so a receive grouped with these sends
            # would hold the later sends back until the helper's done message, which needs them.
            works = dist.batch_isend_irecv([
                dist.P2POp(dist.isend, query[k:], self.peer), dist.P2POp(dist.isend, out.slot[k:], self.peer),
                dist.P2POp(dist.isend, out.install[k:], self.peer)])
            works.append(dist.irecv(self.done_rx, self.peer))
            self.host.swapin(self.recs[layer][:k], query[:k], out.slot[:k], out.install[:k], self.pools[layer][:k],
                             status=self.status[:k])
            if ev:
                ev[1].record(main)
            for w in works:
                w.wait()  # the stream waits for the helper's done message (rows landed)
        elif self.role == "helper" and m > 0:
            hs = self.helper
            k = hs.req - m
            works = dist.batch_isend_irecv([
                dist.P2POp(dist.irecv, hs.q[:m], self.peer), dist.P2POp(dist.irecv, hs.slot[:m], self.peer),
                dist.P2POp(dist.irecv, hs.install[:m], self.peer)])
            with torch.cuda.stream(self.side):
                for w in works:
                    w.wait()
                hs.pool.swapin_to_peer(hs.recs[layer][k:], hs.q[:m], hs.slot[:m], hs.install[:m],
                                       hs.peer_pools[layer] + k * hs.slot_count * hs.row_bytes, hs.slot_count,
                                       status=hs.status[k:], stream=self.side)
                dist.isend(self.done_tx, self.peer).wait()
            self.host.swapin(self.recs[layer], query, out.slot, out.install, self.pools[layer], status=self.status)
            if ev:
                ev[1].record(main)
            main.wait_stream(self.side)
        else:
            self.host.swapin(self.recs[layer], query, out.slot, out.install, self.pools[layer], status=self.status)
            if ev:
                ev[1].record(main)
        if ev:
            ev[2].record(main)
            self.window.events.append(ev)

    # ---- calibration ----
    def _gather(self, values: list[float]) -> torch.Tensor:
        t = torch.zeros((self.world, len(values)), dtype=torch.float64, device=self.device)
        t[self.rank] = torch.tensor(values, dtype=torch.float64)
        self.dist.all_reduce(t)
        return t.cpu()

    def _measure(self, run_steps: Callable[[int], None], steps: int) -> tuple[float, float]:
        self.window = _Window()
        run_steps(steps)
        torch.cuda.synchronize(self.device)
        ev, self.window = self.window.events, None
        own = statistics.median(a.elapsed_time(b) for a, b, _ in ev)
        total = statistics.median(a.elapsed_time(c) for a, _, c in ev)
        return own, total

    def calibrate(self, run_steps: Callable[[int], None], steps: int = 3, rounds: int = 2,
                  initial_pairs: list[tuple[int, int, int]] | None = None) -> dict:
        """Choose the pairs and shares.  ``run_steps(n)`` runs n steps of the caller's loop (which
        swaps in through ``self.swapin``); every rank must call this with the same arguments.
        ``initial_pairs`` skips the first round (the unbalanced measurement) and starts the
        refinement from that plan.  Every plan tried is measured, and the one whose slowest rank
        finished first is kept; without ``initial_pairs`` it must also beat the unbalanced round by
        2%, else every share goes to 0.  (Shares refined from one round's rates can overshoot: a
        host link shared by several GPUs serves each faster when the others read less, so the
        refined plan is not always better than the one it came from.)  Runs at most
        ``steps * (rounds + 2)`` steps."""
        req = [int(x) for x in self._gather([float(self.R)])[:, 0].tolist()]
        unbalanced = None
        if initial_pairs is None:
            own, total = self._measure(run_steps, steps)
            g = self._gather([total])
            rates = [req[r] / g[r, 0].item() if g[r, 0] > 0 else 0.0 for r in range(self.world)]
            unbalanced = max(g[:, 0].tolist())
            self.history.append({"round": 0, "ms": g[:, 0].tolist()})
            self.set_plan(plan_pairs(rates, req, self.min_share))
        else:
            self.set_plan(initial_pairs)
        measured: list[tuple[float, list[tuple[int, int, int]]]] = []
        for i in range(rounds + (1 if initial_pairs is None else 0)):
            if not any(m > 0 for _, _, m in self.pairs):
                break
            own, total = self._measure(run_steps, steps)
            g = self._gather([own, total])
            measured.append((max(g[:, 1].tolist()), list(self.pairs)))
            self.history.append({"round": i + 1, "own_ms": g[:, 0].tolist(), "ms": g[:, 1].tolist(),
                                 "pairs": [list(p) for p in self.pairs]})
            if i == rounds:  # the last plan is measured, not refined
                break
            # a share refined to 0 leaves the pair in place but swaps in locally (no messages)
            self.pairs = [(o, h, refine_share(req[o], req[h], m, g[o, 0].item(), g[h, 1].item()))
                          for o, h, m in self.pairs]
            self._apply_share()
        if self.pairs:
            self.pairs = best_plan(measured, unbalanced) if measured else [(o, h, 0) for o, h, _ in self.pairs]
            self._apply_share()
            self.history.append({"round": "kept", "pairs": [list(p) for p in self.pairs],
                                 "slowest_ms": min((x[0] for x in measured), default=None),
                                 "unbalanced_ms": unbalanced})
        return {"pairs": [list(p) for p in self.pairs], "history": self.history}

    def _apply_share(self) -> None:
        self.m = 0
        for o, h, m in self.pairs:
            if self.rank in (o, h):
                self.m = m

    # ---- set-up of a plan (collective) ----
    def set_plan(self, pairs: list[tuple[int, int, int]]) -> None:
        dist = self.dist
        if self.pairs:
            raise RuntimeError("the plan is set once")
        self.pairs = list(pairs)
        for o, h, m in self.pairs:
            if self.rank == o:
                self.role, self.peer = "owner", h
            elif self.rank == h:
                self.role, self.peer = "helper", o
        self._apply_share()
        if not self.pairs:
            return
        token = [os.urandom(8).hex() if self.rank == 0 else None]
        dist.broadcast_object_list(token, src=0)
        server = FdServer(socket_name(token[0], self.rank)) if self.role == "owner" else None
        dist.barrier()
        try:
            if server is not None:
                layers = [ipc_export(p) for p in self.pools]
                payload = json.dumps({"rows": self.host.rows, "row_bytes": self.host.row_bytes,
                                      "pitch": self.host.pitch, "req": self.R, "slots": self.pools[0].shape[1],
                                      "keys": self.recs[0].shape[1], "layers": layers}).encode()
                server.serve(self.host.shared.fd, payload)
            elif self.role == "helper":
                fd, payload = fetch_fd(socket_name(token[0], self.peer))
                self._attach(fd, json.loads(payload))
        finally:
            if server is not None:
                server.close()
        # the owner's record tables, once (NCCL, also opens the pair's communicator)
        if self.role == "owner":
            for r in self.recs:
                dist.send(r, self.peer)
        elif self.role == "helper":
            for r in self.helper.recs:
                dist.recv(r, self.peer)
        torch.cuda.synchronize(self.device)
        dist.barrier()

    def _attach(self, fd: int, info: dict) -> None:
        from .host_pool import HostRowPool

        dev = self.device
        with torch.cuda.device(dev):
            pool = HostRowPool.attach(fd, info["rows"], info["row_bytes"], info["pitch"])
        bases = [ipc_open(hx, dev) for hx, _ in info["layers"]]
        req, Q = info["req"], self.query_count
        self.helper = _HelperSide(
            owner=self.peer, req=req, pool=pool, peer_bases=bases,
            peer_pools=[b + off for b, (_, off) in zip(bases, info["layers"])],
            slot_count=info["slots"], row_bytes=info["row_bytes"],
            recs=[torch.empty((req, info["keys"]), dtype=torch.int32, device=dev) for _ in info["layers"]],
            q=torch.empty((req, Q), dtype=torch.int32, device=dev),
            slot=torch.empty((req, Q), dtype=torch.int32, device=dev),
            install=torch.empty((req, Q), dtype=torch.bool, device=dev),
            status=torch.zeros(req, dtype=torch.int32, device=dev))

    # ---- end ----
    def check_status(self) -> None:
        raise_on_status(self.status, "swapin")
        if self.helper is not None:
            raise_on_status(self.helper.status, f"swapin for rank {self.helper.owner}")

    def close(self) -> None:
        torch.cuda.synchronize(self.device)
        hs, self.helper = self.helper, None
        if hs is not None:
            for b in hs.peer_bases:
                with torch.cuda.device(self.device):
                    check(lib.asu_ipc_close(b), "asu_ipc_close")
            hs.pool.close()
