"""Host-pool producer: MicroKV-compatible keys over the pinned row pool.

The reference's offload designs keep every prefilled token record in MicroKV, a C++ process
that maps ``(cache_type, 32-byte key)`` to opaque bytes behind a Unix socket
(MicroKV/src/kv_store.h:14-37, MicroKV/python/microkv/client.py:43-63).  Here the values live
in the rows of the pinned, GPU-mapped host pool that the swap-in kernel reads, and keys keep
MicroKV's layout so tools written against its client keep working:

    | req_index 16 B | layer_id u32 | token_pos u32 | cache_type u8 | 7 reserved |   (little endian)

A string request id becomes the first 16 bytes of its SHA-256, an integer one its u64
followed by 8 zero bytes (client.py:43-63).

Rows are handed out in extents: the first key of a (cache_type, request, layer) reserves
``tokens_per_extent`` consecutive rows, and token ``pos`` of that triple is row ``base + pos``.
That makes the dense ``record_addr`` table the swap-in kernel needs a plain ``base + arange``
and lets the GPU write a prefilled range of tokens straight into its rows
(``write_back``, one ``asu_host_pool_writeback`` launch).  The dict-style API
(``put``/``get``/``exists``/``batch_*``/``clear``/``size``) follows MicroKV's client, with one
difference: a value is stored in one row, so values longer than the row size are refused
(``put`` returns False) where MicroKV grows its heap.
"""

from __future__ import annotations

import hashlib
import struct
from typing import Iterable

import numpy as np

KEY_LENGTH = 32
KV_ATTENTION_K = 0
KV_MLA_TOKEN = KV_ATTENTION_K
KV_ATTENTION_V = 1
DSA_INDEX = 2
DSA_INDEX_SCALE = 3

_U32 = 0xFFFFFFFF


def _request_bytes(req_index: int | str) -> bytes:
    if isinstance(req_index, bool) or not isinstance(req_index, (int, str)):
        raise TypeError("req_index must be int or str")
    if isinstance(req_index, str):
        return hashlib.sha256(req_index.encode()).digest()[:16]
    if not 0 <= req_index <= 0xFFFFFFFFFFFFFFFF:
        raise ValueError("integer req_index must fit uint64")
    return req_index.to_bytes(8, "little") + bytes(8)


def _check_u32(name: str, v: int) -> None:
    if not isinstance(v, int):
        raise TypeError(f"{name} must be int")
    if not 0 <= v <= _U32:
        raise ValueError(f"{name} must fit uint32")


def _check_type(cache_type: int) -> None:
    if not isinstance(cache_type, int):
        raise TypeError("cache_type must be int")
    if not 0 <= cache_type <= 0xFF:
        raise ValueError("cache_type must fit uint8")


def _check_key(key: bytes) -> None:
    if not isinstance(key, bytes):
        raise TypeError("key must be bytes")
    if len(key) != KEY_LENGTH:
        raise ValueError(f"key must be {KEY_LENGTH} bytes, got {len(key)}")


def make_key(req_index: int | str, layer_id: int, token_pos: int, cache_type: int = KV_ATTENTION_K) -> bytes:
    """The 32-byte MicroKV key of one token record."""
    req = _request_bytes(req_index)
    _check_u32("layer_id", layer_id)
    _check_u32("token_pos", token_pos)
    _check_type(cache_type)
    return req + struct.pack("<IIB", layer_id, token_pos, cache_type) + bytes(7)


def parse_key(key: bytes) -> tuple[bytes, int, int, int]:
    """(request bytes, layer_id, token_pos, cache_type byte) of a 32-byte key."""
    _check_key(key)
    layer, pos, ctype = struct.unpack_from("<IIB", key, 16)
    return key[:16], layer, pos, ctype


class HostKVStore:
    """(cache_type, key) -> bytes over ``rows`` ([n_rows, row_bytes] uint8, e.g. a HostRowPool's
    ``array``).  ``pool`` (a HostRowPool over the same rows) enables the GPU write-back."""

    def __init__(self, rows: np.ndarray, tokens_per_extent: int, pool=None):
        if rows.ndim != 2 or rows.dtype != np.uint8:
            raise ValueError("rows must be a [n_rows, row_bytes] uint8 array")
        if tokens_per_extent <= 0 or tokens_per_extent > rows.shape[0]:
            raise ValueError("tokens_per_extent must be in 1..n_rows")
        self.rows = rows
        self.row_bytes = rows.shape[1]
        self.tokens_per_extent = tokens_per_extent
        self.pool = pool
        n_ext = rows.shape[0] // tokens_per_extent
        self._free = list(range((n_ext - 1) * tokens_per_extent, -1, -tokens_per_extent))  # lowest base on top
        self._extents: dict[tuple[int, bytes, int], int] = {}
        self._present = np.zeros(rows.shape[0], bool)
        self._length = np.zeros(rows.shape[0], np.uint32)
        self._count: dict[int, int] = {}

    # ------------------------------------------------------------ extents
    def _extent(self, cache_type: int, req: bytes, layer: int, create: bool) -> int | None:
        k = (cache_type, req, layer)
        base = self._extents.get(k)
        if base is None and create and self._free:
            base = self._free.pop()
            self._extents[k] = base
            self._present[base:base + self.tokens_per_extent] = False
        return base

    def _row(self, cache_type: int, key: bytes, create: bool) -> int | None:
        req, layer, pos, _ = parse_key(key)
        if pos >= self.tokens_per_extent:
            return None
        base = self._extent(cache_type, req, layer, create)
        return None if base is None else base + pos

    def extent_base(self, cache_type: int, req_index: int | str, layer_id: int) -> int:
        """First row of the (cache_type, request, layer) extent, reserving it if new."""
        _check_type(cache_type)
        _check_u32("layer_id", layer_id)
        base = self._extent(cache_type, _request_bytes(req_index), layer_id, True)
        if base is None:
            raise MemoryError("host pool has no free extent")
        return base

    def record_rows(self, cache_type: int, req_index: int | str, layer_id: int, tokens: int) -> np.ndarray:
        """Host rows of tokens 0..tokens-1: a row of the swap-in's record_addr table."""
        if not 0 <= tokens <= self.tokens_per_extent:
            raise ValueError("tokens exceeds the extent")
        return (self.extent_base(cache_type, req_index, layer_id) + np.arange(tokens)).astype(np.int32)

    def _mark(self, lo: int, hi: int, cache_type: int, length: int) -> None:
        new = int(hi - lo - self._present[lo:hi].sum())
        self._present[lo:hi] = True
        self._length[lo:hi] = length
        self._count[cache_type] = self._count.get(cache_type, 0) + new

    # ------------------------------------------------------------ MicroKV client API
    def put(self, cache_type: int, key: bytes, value: bytes) -> bool:
        _check_type(cache_type)
        _check_key(key)
        value = bytes(value)
        if len(value) > self.row_bytes:
            return False
        row = self._row(cache_type, key, True)
        if row is None:
            return False
        self.rows[row, :len(value)] = np.frombuffer(value, np.uint8)
        self._mark(row, row + 1, cache_type, len(value))
        return True

    def get(self, cache_type: int, key: bytes) -> bytes | None:
        _check_type(cache_type)
        row = self._row(cache_type, key, False)
        if row is None or not self._present[row]:
            return None
        return self.rows[row, :self._length[row]].tobytes()

    def exists(self, cache_type: int, key: bytes) -> bool:
        _check_type(cache_type)
        row = self._row(cache_type, key, False)
        return row is not None and bool(self._present[row])

    def batch_put(self, cache_type: int, keys: list[bytes], values: list[bytes]) -> bool:
        if len(keys) != len(values):
            raise ValueError("keys and values must have the same length")
        ok = True
        for k, v in zip(keys, values):
            ok &= self.put(cache_type, k, v)
        return ok

    def batch_get(self, cache_type: int, keys: Iterable[bytes]) -> list[bytes | None]:
        return [self.get(cache_type, k) for k in keys]

    def batch_exists(self, cache_type: int, keys: Iterable[bytes]) -> list[bool]:
        return [self.exists(cache_type, k) for k in keys]

    def clear(self, cache_type: int) -> None:
        _check_type(cache_type)
        for k in [k for k in self._extents if k[0] == cache_type]:
            base = self._extents.pop(k)
            self._present[base:base + self.tokens_per_extent] = False
            self._free.append(base)
        self._count[cache_type] = 0

    def size(self, cache_type: int) -> int:
        _check_type(cache_type)
        return self._count.get(cache_type, 0)

    # ------------------------------------------------------------ GPU producer
    def write_back(self, cache_type: int, req_index: int | str, layer_id: int, start: int, src, stream=None) -> None:
        """Store tokens start..start+n-1 of (request, layer) from HBM rows ``src`` ([n, row_bytes]
        CUDA tensor, any dtype) with one GPU launch.  Asynchronous on ``stream``: synchronize it
        before reading these rows on the host."""
        if self.pool is None:
            raise RuntimeError("write_back needs the HostRowPool that owns the rows")
        n = src.shape[0]
        if start < 0 or start + n > self.tokens_per_extent:
            raise ValueError("token range exceeds the extent")
        if src.dim() < 2 or src[0].numel() * src.element_size() != self.row_bytes:
            raise ValueError(f"src rows must be {self.row_bytes} bytes")
        base = self.extent_base(cache_type, req_index, layer_id)
        self.pool.writeback_range(src.reshape(n, -1) if src.dim() > 2 else src, base + start, stream=stream)
        self._mark(base + start, base + start + n, cache_type, self.row_bytes)
