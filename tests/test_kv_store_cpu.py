"""Host-pool producer on CPU: MicroKV key layout against keys made by the reference's own
client, and the MicroKV client behaviours (MicroKV/tests/test_microkv_e2e.py) restated on the
row store."""

import struct

import numpy as np
import pytest

from asu_ascend_b200 import kv_store as KV


def test_make_key_matches_reference_client(golden):
    g = golden("microkv_keys")
    for i in range(len(g["keys"])):
        req = str(g["req_str"][i]) if g["is_str"][i] else int(g["req_int"][i])
        layer, pos, t = (int(v) for v in g["fields"][i])
        key = KV.make_key(req, layer, pos, t)
        assert key == g["keys"][i].tobytes(), (req, layer, pos, t)
        r16, l2, p2, t2 = KV.parse_key(key)
        assert (l2, p2, t2) == (layer, pos, t) and r16 == key[:16]


def test_make_key_argument_errors():
    with pytest.raises(TypeError):
        KV.make_key(1.5, 0, 0)
    with pytest.raises(ValueError):
        KV.make_key(-1, 0, 0)
    with pytest.raises(ValueError):
        KV.make_key(1 << 64, 0, 0)
    with pytest.raises(ValueError):
        KV.make_key("r", 1 << 32, 0)
    with pytest.raises(ValueError):
        KV.make_key("r", 0, 0, 256)
    with pytest.raises(ValueError):
        KV.parse_key(b"short")


def _store(rows=64, row_bytes=32, tokens=8):
    return KV.HostKVStore(np.zeros((rows, row_bytes), np.uint8), tokens_per_extent=tokens)


def test_batch_read_keeps_slot_semantics_in_caller():
    """test_microkv_e2e.py:25-48 restated: the caller packs its slot id into the value."""
    s = _store()
    keys = {t: KV.make_key("req-phase1", layer_id=2, token_pos=t, cache_type=KV.KV_ATTENTION_K) for t in range(4)}
    for t, slot in ((0, 100), (1, 101), (3, 130)):
        assert s.put(KV.KV_ATTENTION_K, keys[t], struct.pack("<I", slot) + f"k-token-{t}".encode())
    order = [keys[3], keys[2], keys[1], keys[0]]
    assert s.batch_exists(KV.KV_ATTENTION_K, [keys[0], keys[1], keys[2], keys[3]]) == [True, True, False, True]
    vals = s.batch_get(KV.KV_ATTENTION_K, order)
    parsed = [None if v is None else (struct.unpack("<I", v[:4])[0], v[4:]) for v in vals]
    assert parsed == [(130, b"k-token-3"), None, (101, b"k-token-1"), (100, b"k-token-0")]


def test_overwrite_zero_length_and_row_sized_payload():
    """test_microkv_e2e.py:70-88 restated; values are bounded by the row size here."""
    s = _store(row_bytes=48)
    key = KV.make_key("opaque-bytes", layer_id=4, token_pos=5)
    assert s.put(KV.KV_ATTENTION_K, key, b"first")
    assert s.size(KV.KV_ATTENTION_K) == 1
    assert s.put(KV.KV_ATTENTION_K, key, b"")
    assert s.get(KV.KV_ATTENTION_K, key) == b"" and s.exists(KV.KV_ATTENTION_K, key)
    assert s.size(KV.KV_ATTENTION_K) == 1
    big = bytes(range(48))
    assert s.put(KV.KV_ATTENTION_K, key, big)
    assert s.get(KV.KV_ATTENTION_K, key) == big and s.size(KV.KV_ATTENTION_K) == 1
    assert not s.put(KV.KV_ATTENTION_K, key, bytes(49))  # longer than a row: refused
    assert s.get(KV.KV_ATTENTION_K, key) == big


def test_cache_type_namespaces_and_clear():
    """test_microkv_e2e.py:104-117 restated, plus clear/size."""
    s = _store()
    a = KV.make_key("type-space", layer_id=1, token_pos=0)
    b = KV.make_key("type-space", layer_id=1, token_pos=1)
    assert s.batch_put(KV.KV_ATTENTION_K, [a, b], [b"k-a", b"k-b"])
    assert s.batch_put(KV.KV_ATTENTION_V, [a, b], [b"v-a", b"v-b"])
    assert s.put(KV.DSA_INDEX, a, struct.pack("<I", 77))
    assert s.batch_get(KV.KV_ATTENTION_K, [a, b]) == [b"k-a", b"k-b"]
    assert s.batch_get(KV.KV_ATTENTION_V, [a, b]) == [b"v-a", b"v-b"]
    assert s.batch_get(KV.DSA_INDEX, [a, b]) == [struct.pack("<I", 77), None]
    assert (s.size(KV.KV_ATTENTION_K), s.size(KV.KV_ATTENTION_V), s.size(KV.DSA_INDEX)) == (2, 2, 1)
    s.clear(KV.KV_ATTENTION_K)
    assert s.size(KV.KV_ATTENTION_K) == 0 and s.get(KV.KV_ATTENTION_K, a) is None
    assert s.get(KV.KV_ATTENTION_V, a) == b"v-a"


def test_extents_and_record_rows():
    s = _store(rows=32, tokens=8)  # 4 extents
    r0 = s.record_rows(KV.KV_MLA_TOKEN, "req-a", 0, 8)
    r1 = s.record_rows(KV.KV_MLA_TOKEN, "req-a", 1, 5)
    assert r0.tolist() == list(range(8)) and r1.tolist() == list(range(8, 13))
    assert s.record_rows(KV.KV_MLA_TOKEN, "req-a", 0, 3).tolist() == [0, 1, 2]  # same extent again
    key = KV.make_key("req-a", 1, 4)
    assert s.put(KV.KV_MLA_TOKEN, key, b"x") and s.rows[12, 0] == ord("x")
    assert not s.put(KV.KV_MLA_TOKEN, KV.make_key("req-a", 1, 8), b"y")  # beyond the extent
    s.extent_base(KV.KV_MLA_TOKEN, "req-b", 0)
    s.extent_base(KV.KV_MLA_TOKEN, "req-c", 0)
    with pytest.raises(MemoryError):
        s.extent_base(KV.KV_MLA_TOKEN, "req-d", 0)
    assert not s.put(KV.KV_MLA_TOKEN, KV.make_key("req-d", 0, 0), b"z")  # pool full
    s.clear(KV.KV_MLA_TOKEN)
    assert s.extent_base(KV.KV_MLA_TOKEN, "req-d", 0) in (0, 8, 16, 24)
    assert s.get(KV.KV_MLA_TOKEN, key) is None


def test_write_back_needs_the_pool():
    s = _store()
    with pytest.raises(RuntimeError):
        s.write_back(KV.KV_MLA_TOKEN, "r", 0, 0, np.zeros((2, 32), np.uint8))
