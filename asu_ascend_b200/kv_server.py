"""MicroKV's Unix-socket protocol in front of a HostKVStore (tooling parity).

Tools written for MicroKV -- its Python client, the Phase-1 compare path of the offload
designs -- talk to a `kv_stored` process over a Unix socket (MicroKV/src/server.cpp:120-320,
MicroKV/python/microkv/client.py).  This server speaks the same protocol, so those tools can
read and write the rows of the pinned host pool that the swap-in kernel uses:

    request  | command u8 | cache_type u8 | reserved u16 | key_len u16 | val_len u32 | body
    response | status u8 | payload_len u32 | payload                              (little endian)

Commands PUT / GET / EXISTS / BATCH_PUT / BATCH_GET / BATCH_EXISTS / CLEAR / SIZE keep the
reference's payload layouts and status codes; a malformed request gets BAD_REQUEST and the
connection is closed, as the reference server does.  The one difference is the store
underneath: a value lives in one pool row, so a value longer than the row, or a key whose
extent cannot be allocated, is answered with INTERNAL_ERROR (the client's put returns False)
where MicroKV would grow its heap.

    python -m asu_ascend_b200.kv_server --socket /tmp/microkv.sock --rows 1048576 --row-bytes 656
"""

from __future__ import annotations

import argparse
import os
import socketserver
import struct
import threading

import numpy as np

from .kv_store import KEY_LENGTH, HostKVStore

CMD_PUT, CMD_GET, CMD_EXISTS = 0x01, 0x02, 0x03
CMD_BATCH_PUT, CMD_BATCH_GET, CMD_BATCH_EXISTS = 0x04, 0x05, 0x06
CMD_CLEAR, CMD_SIZE = 0x11, 0x12
STATUS_OK, STATUS_NOT_FOUND, STATUS_BAD_REQUEST, STATUS_INTERNAL_ERROR = 0, 1, 2, 3
MAX_BATCH_COUNT = 1_000_000  # the reference server's limit (MicroKV/src/server.cpp:18)

_REQ = struct.Struct("<BBHHI")
_RESP = struct.Struct("<BI")
_U32 = struct.Struct("<I")


class _BadRequest(Exception):
    pass


class _Closed(Exception):
    pass


def _read(rfile, n: int) -> bytes:
    data = rfile.read(n) if n else b""
    if len(data) != n:
        raise _Closed()
    return data


class _Handler(socketserver.StreamRequestHandler):
    def handle(self) -> None:
        while True:
            try:
                head = _read(self.rfile, _REQ.size)
            except _Closed:
                return
            try:
                status, payload = self.server.dispatch(self.rfile, *_REQ.unpack(head))
            except _BadRequest:
                self._reply(STATUS_BAD_REQUEST, b"")
                return  # the reference server drops the connection after a bad request
            except _Closed:
                return
            self._reply(status, payload)

    def _reply(self, status: int, payload: bytes) -> None:
        self.wfile.write(_RESP.pack(status, len(payload)) + payload)
        self.wfile.flush()


class MicroKVServer(socketserver.ThreadingMixIn, socketserver.UnixStreamServer):
    """Serve ``store`` on the Unix socket ``path``; ``start()`` runs it on a daemon thread."""

    daemon_threads = True

    def __init__(self, store: HostKVStore, path: str):
        if os.path.exists(path):
            os.unlink(path)
        self.store = store
        self.lock = threading.Lock()  # HostKVStore is not thread-safe
        self.path = path
        self._thread: threading.Thread | None = None
        super().__init__(path, _Handler)

    # -------------------------------------------------------------- protocol
    def dispatch(self, rfile, cmd: int, ctype: int, _reserved: int, key_len: int, val_len: int):
        s = self.store
        if cmd in (CMD_PUT, CMD_GET, CMD_EXISTS):
            if key_len != KEY_LENGTH or (cmd != CMD_PUT and val_len != 0):
                raise _BadRequest()
            key = _read(rfile, KEY_LENGTH)
            if cmd == CMD_PUT:
                value = _read(rfile, val_len)
                with self.lock:
                    ok = s.put(ctype, key, value)
                return (STATUS_OK if ok else STATUS_INTERNAL_ERROR), b""
            with self.lock:
                if cmd == CMD_GET:
                    value = s.get(ctype, key)
                    return (STATUS_NOT_FOUND, b"") if value is None else (STATUS_OK, value)
                return STATUS_OK, bytes([1 if s.exists(ctype, key) else 0])
        if cmd in (CMD_BATCH_PUT, CMD_BATCH_GET, CMD_BATCH_EXISTS):
            if key_len != KEY_LENGTH or val_len != 0:
                raise _BadRequest()
            (count,) = _U32.unpack(_read(rfile, _U32.size))
            if count > MAX_BATCH_COUNT:
                raise _BadRequest()
            if cmd == CMD_BATCH_PUT:
                ok = True
                for _ in range(count):
                    key = _read(rfile, KEY_LENGTH)
                    (n,) = _U32.unpack(_read(rfile, _U32.size))
                    value = _read(rfile, n)
                    with self.lock:
                        ok &= s.put(ctype, key, value)
                return (STATUS_OK if ok else STATUS_INTERNAL_ERROR), b""
            keys = [_read(rfile, KEY_LENGTH) for _ in range(count)]
            out = bytearray(_U32.pack(count))
            with self.lock:
                for key in keys:
                    if cmd == CMD_BATCH_EXISTS:
                        out.append(1 if s.exists(ctype, key) else 0)
                        continue
                    value = s.get(ctype, key)
                    out.append(0 if value is None else 1)
                    out += _U32.pack(0 if value is None else len(value))
                    if value is not None:
                        out += value
            return STATUS_OK, bytes(out)
        if cmd in (CMD_CLEAR, CMD_SIZE):
            if key_len != 0 or val_len != 0:
                raise _BadRequest()
            with self.lock:
                if cmd == CMD_CLEAR:
                    s.clear(ctype)
                    return STATUS_OK, b""
                return STATUS_OK, struct.pack("<Q", s.size(ctype))
        raise _BadRequest()

    # -------------------------------------------------------------- lifecycle
    def start(self) -> "MicroKVServer":
        self._thread = threading.Thread(target=self.serve_forever, name="microkv-server", daemon=True)
        self._thread.start()
        return self

    def close(self) -> None:
        if self._thread is not None:  # shutdown() waits for a running serve_forever()
            self.shutdown()
            self._thread.join()
            self._thread = None
        self.server_close()
        if os.path.exists(self.path):
            os.unlink(self.path)


def main(argv: list[str] | None = None) -> None:
    p = argparse.ArgumentParser(description="MicroKV protocol server over a host row pool")
    p.add_argument("--socket", default="/tmp/microkv.sock")
    p.add_argument("--rows", type=int, default=1 << 20)
    p.add_argument("--row-bytes", type=int, default=656)
    p.add_argument("--tokens-per-extent", type=int, default=131072)
    p.add_argument("--pinned", action="store_true",
                   help="rows in pinned, GPU-mapped memory (needs CUDA); default: ordinary host memory")
    a = p.parse_args(argv)
    pool = None
    if a.pinned:
        from .host_pool import HostRowPool

        pool = HostRowPool(a.rows, a.row_bytes)
        rows = pool.array
    else:
        rows = np.zeros((a.rows, a.row_bytes), np.uint8)
    server = MicroKVServer(HostKVStore(rows, a.tokens_per_extent, pool=pool), a.socket)
    try:
        server.serve_forever()
    except KeyboardInterrupt:
        pass
    finally:
        server.server_close()
        if os.path.exists(a.socket):
            os.unlink(a.socket)


if __name__ == "__main__":
    main()
