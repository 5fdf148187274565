"""Pinned, GPU-mapped host row pool and the swap-in gather into the HBM slot pool.

The pool replaces the MicroKV backing store of the reference's v0/v0.1 designs
(MicroKV/src/kv_store.h:14-37 keyed by (request, layer, token, type);
MicroKV/python/microkv/client.py:43-63): records are fixed-size rows in page-locked,
mapped host memory, and ``record_addr[r, key]`` gives the row of request r's key (a
dense index instead of a hash map).  ``swapin`` copies the rows of every installing
position into ``slot_pool[r, slot]`` with one kernel that reads host memory directly.
"""

from __future__ import annotations

import ctypes
import mmap
import os

import numpy as np
import torch

from ._lib import check, lib, raise_on_status


class SharedRows:
    """Rows in an anonymous shared-memory file (memfd): the backing of a host pool that other
    processes of the box map too.  ``fd`` can be handed to another process (over a Unix socket,
    see ``balance.py``), which maps the same pages with ``SharedRows(nbytes, fd=received_fd)``.
    No CUDA here: page-locking and GPU mapping are the pool's job."""

    def __init__(self, nbytes: int, fd: int | None = None):
        if nbytes <= 0:
            raise ValueError("nbytes must be positive")
        if fd is None:
            fd = os.memfd_create("asu-host-pool", os.MFD_CLOEXEC)
            os.ftruncate(fd, nbytes)
        elif os.fstat(fd).st_size < nbytes:
            os.close(fd)
            raise ValueError("the shared file is smaller than the pool")
        self.fd, self.nbytes = fd, nbytes
        self.mm = mmap.mmap(fd, nbytes, mmap.MAP_SHARED, mmap.PROT_READ | mmap.PROT_WRITE)
        self.flat = np.frombuffer(self.mm, dtype=np.uint8)
        self.address = self.flat.ctypes.data

    def close(self) -> None:
        if self.mm is None:
            return
        self.flat = None
        try:
            self.mm.close()
        except BufferError:  # a view is still referenced elsewhere: the pages go at process exit
            pass
        os.close(self.fd)
        self.mm = None


class HostRowPool:
    """``rows`` records of ``row_bytes`` bytes in page-locked, GPU-mapped host memory.

    Consecutive rows start ``pitch`` bytes apart.  The default pads rows of up to 1 KiB to a
    multiple of 128 bytes (656 -> 768) and packs larger rows: the swap-in copies small rows with
    one TMA bulk copy each, and a row that starts on a 128-byte boundary is read from host
    memory in whole 128-byte lines (measured on B200 with 656-byte rows: ~48 GB/s at a 768-byte
    pitch, ~41 GB/s packed).  ``array`` is a [rows, row_bytes] view of the records.

    ``shared=True`` backs the pool with a shared-memory file (``SharedRows``) registered for this
    process's GPU, so another rank of the box can map the same rows (``HostRowPool.attach``) and
    swap them in through its own host link.  The default is a plain cudaHostAlloc allocation.
    """

    def __init__(self, rows: int, row_bytes: int, pitch: int | None = None, shared: bool = False,
                 _fd: int | None = None):
        if rows <= 0 or row_bytes <= 0 or row_bytes % 16:
            raise ValueError("rows must be positive and row_bytes a positive multiple of 16")
        if pitch is None:
            pitch = (row_bytes + 127) // 128 * 128 if row_bytes <= 1024 else row_bytes
        if pitch < row_bytes or pitch % 16:
            raise ValueError("pitch must be a multiple of 16 and at least row_bytes")
        self.rows, self.row_bytes, self.pitch = rows, row_bytes, pitch
        self.nbytes = rows * pitch
        self.shared = None
        host = ctypes.c_void_p()
        dev = ctypes.c_void_p()
        if shared or _fd is not None:
            self.shared = SharedRows(self.nbytes, _fd)
            rc = lib.asu_host_register(self.shared.address, self.nbytes, ctypes.byref(dev))
            if rc != 0:
                self.shared.close()
                check(rc, "asu_host_register")
            self._host = self.shared.address
            buf = self.shared.flat
        else:
            check(lib.asu_host_pool_alloc(self.nbytes, ctypes.byref(host), ctypes.byref(dev)), "asu_host_pool_alloc")
            self._host = host.value
            buf = np.frombuffer((ctypes.c_uint8 * self.nbytes).from_address(self._host), dtype=np.uint8)
        self.device_ptr = dev.value
        self.array = buf.reshape(rows, pitch)[:, :row_bytes]
        self.tensor = torch.from_numpy(self.array)  # CPU view of the same pinned bytes

    @classmethod
    def attach(cls, fd: int, rows: int, row_bytes: int, pitch: int) -> "HostRowPool":
        """Map another process's shared pool (its ``shared.fd``, received by this process) and
        register it for this process's GPU.  The pool takes ownership of ``fd``."""
        return cls(rows, row_bytes, pitch, _fd=fd)

    def fill_random(self, seed: int) -> None:
        rng = np.random.Generator(np.random.PCG64(seed))
        step = max(1, (64 << 20) // self.row_bytes)
        for i in range(0, self.rows, step):
            j = min(self.rows, i + step)
            self.array[i:j] = rng.integers(0, 256, (j - i, self.row_bytes), dtype=np.uint8)

    def close(self) -> None:
        if getattr(self, "_host", None):
            self.array = None
            self.tensor = None
            if self.shared is not None:
                check(lib.asu_host_unregister(self._host), "asu_host_unregister")
                self.shared.close()
            else:
                check(lib.asu_host_pool_free(self._host), "asu_host_pool_free")
            self._host = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def swapin(self, record_addr: torch.Tensor, query: torch.Tensor, slot: torch.Tensor, install: torch.Tensor,
               slot_pool: torch.Tensor, status: torch.Tensor | None = None,
               stream: torch.cuda.Stream | None = None) -> None:
        """slot_pool[r, slot[r,p]] = pool[record_addr[r, query[r,p]]] for every p with install[r,p]."""
        dev = slot_pool.device
        R, Q = query.shape
        for name, t in (("record_addr", record_addr), ("query", query), ("slot", slot)):
            if t.dtype != torch.int32 or t.device != dev or not t.is_contiguous():
                raise RuntimeError(f"{name} must be a contiguous int32 CUDA tensor on {dev}")
        if install.dtype not in (torch.bool, torch.uint8) or install.shape != query.shape:
            raise RuntimeError("install must be a bool/uint8 tensor shaped like query")
        if slot_pool.dim() < 2 or not slot_pool.is_contiguous() or slot_pool.shape[0] != R:
            raise RuntimeError("slot_pool must be a contiguous [R, slots, row] tensor")
        row = slot_pool[0, 0].numel() * slot_pool.element_size()
        if row != self.row_bytes:
            raise RuntimeError(f"slot_pool rows are {row} bytes, the host pool's are {self.row_bytes}")
        if record_addr.dim() != 2 or record_addr.shape[0] != R:
            raise RuntimeError("record_addr must be [R, key_space]")
        s = (stream or torch.cuda.current_stream(dev)).cuda_stream
        with torch.cuda.device(dev):
            check(lib.asu_swapin_gather(
                s, self.device_ptr, self.rows, self.row_bytes, self.pitch, record_addr.data_ptr(), record_addr.shape[1],
                query.data_ptr(), slot.data_ptr(), install.data_ptr(), Q, slot_pool.data_ptr(), slot_pool.shape[1],
                R, None if status is None else status.data_ptr()), "asu_swapin_gather")


    def swapin_to_peer(self, record_addr: torch.Tensor, query: torch.Tensor, slot: torch.Tensor,
                       install: torch.Tensor, peer_slot_pool: int, slot_count: int,
                       status: torch.Tensor | None = None, stream: torch.cuda.Stream | None = None) -> None:
        """``swapin`` into another GPU's slot pool: ``peer_slot_pool`` is the device address (in this
        process) of a CUDA IPC mapping of a [R, slot_count, row_bytes] pool on a peer GPU.  The
        index tensors live on this process's GPU.  The rows land in the peer's memory before the
        launch completes (system-scope fence), so work ordered after it on ``stream`` may signal
        the peer."""
        dev = query.device
        R, Q = query.shape
        for name, t in (("record_addr", record_addr), ("query", query), ("slot", slot)):
            if t.dtype != torch.int32 or t.device != dev or not t.is_contiguous():
                raise RuntimeError(f"{name} must be a contiguous int32 CUDA tensor on {dev}")
        if install.dtype not in (torch.bool, torch.uint8) or install.shape != query.shape or not install.is_contiguous():
            raise RuntimeError("install must be a contiguous bool/uint8 tensor shaped like query")
        if record_addr.dim() != 2 or record_addr.shape[0] != R:
            raise RuntimeError("record_addr must be [R, key_space]")
        if not peer_slot_pool:
            raise RuntimeError("peer_slot_pool must be a mapped peer address")
        s = (stream or torch.cuda.current_stream(dev)).cuda_stream
        with torch.cuda.device(dev):
            check(lib.asu_swapin_gather_to_peer(
                s, self.device_ptr, self.rows, self.row_bytes, self.pitch, record_addr.data_ptr(), record_addr.shape[1],
                query.data_ptr(), slot.data_ptr(), install.data_ptr(), Q, peer_slot_pool, slot_count, R,
                None if status is None else status.data_ptr()), "asu_swapin_gather_to_peer")

    def writeback(self, src: torch.Tensor, dst_rows: torch.Tensor, src_index: torch.Tensor | None = None,
                  status: torch.Tensor | None = None, stream: torch.cuda.Stream | None = None) -> None:
        """pool[dst_rows[i]] = src[src_index[i] if given else i] (the producer side of ``swapin``).

        ``src`` is a CUDA tensor of rows of ``row_bytes`` bytes (any dtype, rows contiguous);
        negative ``dst_rows`` entries are skipped.  Asynchronous: synchronize ``stream`` before
        reading the rows on the host."""
        dev = src.device
        if src.device.type != "cuda" or src.dim() < 2 or not src.is_contiguous():
            raise RuntimeError("src must be a contiguous [n, ...] CUDA tensor")
        row = src[0].numel() * src.element_size()
        if row != self.row_bytes:
            raise RuntimeError(f"src rows are {row} bytes, the host pool's are {self.row_bytes}")
        for name, t in (("dst_rows", dst_rows), ("src_index", src_index)):
            if t is not None and (t.dtype != torch.int32 or t.device != dev or not t.is_contiguous()):
                raise RuntimeError(f"{name} must be a contiguous int32 CUDA tensor on {dev}")
        n = dst_rows.numel()
        if src_index is None and n > src.shape[0]:
            raise RuntimeError("dst_rows has more entries than src has rows")
        if src_index is not None and src_index.numel() != n:
            raise RuntimeError("src_index and dst_rows must have the same length")
        s = (stream or torch.cuda.current_stream(dev)).cuda_stream
        with torch.cuda.device(dev):
            check(lib.asu_host_pool_writeback(
                s, self.device_ptr, self.rows, self.row_bytes, self.pitch, src.data_ptr(), src.shape[0], row,
                None if src_index is None else src_index.data_ptr(), dst_rows.data_ptr(), n,
                None if status is None else status.data_ptr()), "asu_host_pool_writeback")


    def writeback_range(self, src: torch.Tensor, first_row: int, status: torch.Tensor | None = None,
                        stream: torch.cuda.Stream | None = None) -> None:
        """pool[first_row + i] = src[i] for every row of ``src``: a contiguous range of host rows,
        with no row-index tensor."""
        dev = src.device
        if src.device.type != "cuda" or src.dim() < 2 or not src.is_contiguous():
            raise RuntimeError("src must be a contiguous [n, ...] CUDA tensor")
        row = src[0].numel() * src.element_size()
        if row != self.row_bytes:
            raise RuntimeError(f"src rows are {row} bytes, the host pool's are {self.row_bytes}")
        n = src.shape[0]
        if first_row < 0 or first_row + n > self.rows:
            raise RuntimeError("row range exceeds the pool")
        s = (stream or torch.cuda.current_stream(dev)).cuda_stream
        with torch.cuda.device(dev):
            check(lib.asu_host_pool_writeback(
                s, self.device_ptr + first_row * self.pitch, n, self.row_bytes, self.pitch, src.data_ptr(), n, row,
                None, None, n, None if status is None else status.data_ptr()), "asu_host_pool_writeback")


def check_status(status: torch.Tensor, what: str, ignore: int = 0) -> None:
    raise_on_status(status, what, ignore)


def _device_address(t: torch.Tensor, dev: torch.device, name: str) -> int:
    if not t.is_contiguous():
        raise RuntimeError(f"{name} must be contiguous")
    if t.device.type == "cuda":
        if t.device != dev:
            raise RuntimeError(f"{name} must be on {dev}")
        return t.data_ptr()
    if not t.is_pinned():
        raise RuntimeError(f"{name} must be a CUDA tensor or pinned host memory")
    d = ctypes.c_void_p()
    check(lib.asu_host_device_pointer(t.data_ptr(), ctypes.byref(d)), f"{name}: device address of pinned memory")
    return d.value


def mapped_copy_(dst: torch.Tensor, src: torch.Tensor, stream: torch.cuda.Stream | None = None) -> torch.Tensor:
    """``dst.copy_(src)`` of equal-size contiguous tensors, one in HBM and the other in pinned host
    memory (or both in HBM), done by the SMs through the host mapping instead of a copy engine
    (``asu_mapped_copy``): for per-step uploads and read-backs on a box whose copy engines share
    the host unevenly.  Bytes are copied as they are (no dtype conversion).  Asynchronous on
    ``stream`` (default: the current stream of the CUDA side); synchronise before reading a host
    result."""
    if dst.numel() * dst.element_size() != src.numel() * src.element_size():
        raise RuntimeError("mapped_copy_: dst and src must have the same size in bytes")
    cuda_side = dst if dst.device.type == "cuda" else src
    if cuda_side.device.type != "cuda":
        raise RuntimeError("mapped_copy_: one of dst and src must be a CUDA tensor")
    dev = cuda_side.device
    d = _device_address(dst, dev, "dst")
    s = _device_address(src, dev, "src")
    st = (stream or torch.cuda.current_stream(dev)).cuda_stream
    with torch.cuda.device(dev):
        check(lib.asu_mapped_copy(st, d, s, dst.numel() * dst.element_size()), "asu_mapped_copy")
    return dst
