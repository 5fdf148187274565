"""The MicroKV socket front-end on CPU: a client that frames requests exactly as MicroKV's
Python client does (MicroKV/python/microkv/client.py) drives the server over a Unix socket;
the behaviours of MicroKV/tests/test_microkv_e2e.py are restated against it."""

import os
import socket
import struct
import tempfile

import numpy as np
import pytest

from asu_ascend_b200 import kv_server as S
from asu_ascend_b200 import kv_store as KV


class Client:
    def __init__(self, path):
        self.sock = socket.socket(socket.AF_UNIX, socket.SOCK_STREAM)
        self.sock.connect(path)

    def close(self):
        self.sock.close()

    def _recv(self, n):
        buf = b""
        while len(buf) < n:
            chunk = self.sock.recv(n - len(buf))
            if not chunk:
                raise ConnectionError("closed")
            buf += chunk
        return buf

    def request(self, cmd, ctype, key_len, val_len, body):
        self.sock.sendall(struct.pack("<BBHHI", cmd, ctype, 0, key_len, val_len) + body)
        status, n = struct.unpack("<BI", self._recv(5))
        return status, self._recv(n)

    def put(self, t, key, value):
        return self.request(S.CMD_PUT, t, len(key), len(value), key + value)[0] == S.STATUS_OK

    def get(self, t, key):
        st, p = self.request(S.CMD_GET, t, len(key), 0, key)
        return None if st == S.STATUS_NOT_FOUND else p

    def exists(self, t, key):
        return self.request(S.CMD_EXISTS, t, len(key), 0, key)[1] == b"\x01"

    def batch_put(self, t, keys, values):
        body = struct.pack("<I", len(keys)) + b"".join(k + struct.pack("<I", len(v)) + v for k, v in zip(keys, values))
        return self.request(S.CMD_BATCH_PUT, t, KV.KEY_LENGTH, 0, body)[0] == S.STATUS_OK

    def batch_get(self, t, keys):
        st, p = self.request(S.CMD_BATCH_GET, t, KV.KEY_LENGTH, 0, struct.pack("<I", len(keys)) + b"".join(keys))
        (count,), off, out = struct.unpack_from("<I", p), 4, []
        for _ in range(count):
            present, n = p[off], struct.unpack_from("<I", p, off + 1)[0]
            off += 5
            out.append(p[off:off + n] if present else None)
            off += n
        assert off == len(p)
        return out

    def batch_exists(self, t, keys):
        st, p = self.request(S.CMD_BATCH_EXISTS, t, KV.KEY_LENGTH, 0, struct.pack("<I", len(keys)) + b"".join(keys))
        return [b != 0 for b in p[4:]]

    def clear(self, t):
        return self.request(S.CMD_CLEAR, t, 0, 0, b"")[0]

    def size(self, t):
        return struct.unpack("<Q", self.request(S.CMD_SIZE, t, 0, 0, b"")[1])[0]


@pytest.fixture()
def server():
    d = tempfile.mkdtemp()
    path = os.path.join(d, "kv.sock")
    store = KV.HostKVStore(np.zeros((64, 48), np.uint8), tokens_per_extent=8)
    srv = S.MicroKVServer(store, path).start()
    yield srv
    srv.close()
    os.rmdir(d)


def test_batch_reads_and_namespaces_over_the_socket(server):
    c = Client(server.path)
    keys = [KV.make_key("req-phase1", 2, t) for t in range(4)]
    assert c.batch_put(KV.KV_ATTENTION_K, [keys[0], keys[1], keys[3]], [b"k0", b"k1", b"k3"])
    assert c.batch_exists(KV.KV_ATTENTION_K, keys) == [True, True, False, True]
    assert c.batch_get(KV.KV_ATTENTION_K, [keys[3], keys[2], keys[0]]) == [b"k3", None, b"k0"]
    assert c.put(KV.KV_ATTENTION_V, keys[0], b"v0") and c.get(KV.KV_ATTENTION_V, keys[0]) == b"v0"
    assert c.get(KV.DSA_INDEX, keys[0]) is None and not c.exists(KV.DSA_INDEX, keys[0])
    assert (c.size(KV.KV_ATTENTION_K), c.size(KV.KV_ATTENTION_V)) == (3, 1)
    assert c.clear(KV.KV_ATTENTION_K) == S.STATUS_OK and c.size(KV.KV_ATTENTION_K) == 0
    c.close()


def test_state_is_shared_between_clients_and_visible_in_the_rows(server):
    a, b = Client(server.path), Client(server.path)
    key = KV.make_key("shared-server", 0, 0)
    assert a.put(KV.KV_ATTENTION_K, key, b"written-by-first-client")
    assert b.get(KV.KV_ATTENTION_K, key) == b"written-by-first-client" and b.exists(KV.KV_ATTENTION_K, key)
    # the bytes are in the pool row the swap-in would read
    row = server.store.record_rows(KV.KV_ATTENTION_K, "shared-server", 0, 1)[0]
    assert server.store.rows[row, :22].tobytes() == b"written-by-first-client"[:22]
    assert a.put(KV.KV_ATTENTION_K, key, b"") and b.get(KV.KV_ATTENTION_K, key) == b""
    assert not a.put(KV.KV_ATTENTION_K, key, bytes(49))  # longer than a 48-byte row
    a.close()
    b.close()


def test_bad_request_closes_the_connection(server):
    c = Client(server.path)
    st, _ = c.request(S.CMD_GET, 0, 16, 0, bytes(16))  # wrong key length
    assert st == S.STATUS_BAD_REQUEST
    with pytest.raises((ConnectionError, OSError)):
        c.size(0)
    c.close()
    c2 = Client(server.path)  # the server itself keeps serving
    assert c2.size(0) == 0
    c2.close()
