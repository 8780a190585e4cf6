"""KV snapshots (soso_b200/kvsnap.py) against the reference's own kvsnap tests
(crates/soso-llm-core/src/kvsnap.rs:127-190), restated byte for byte, plus a round trip of a
multi-layer snapshot.  CPU only."""
import hashlib
import struct

import numpy as np
import pytest

from soso_b200 import kvsnap
from soso_b200.kvsnap import KvSnapError, Snapshot


def example() -> bytes:
    """ejemplo (kvsnap.rs:131-135): tokens [1, 2], hidden [0.5], one layer of width 2 with
    K = 1.0 and V = 2.0 everywhere, profile [9; 32]."""
    s = Snapshot(np.array([1, 2]), np.array([0.5], np.float32),
                 [(np.full(4, 0x3C00, np.uint16), np.full(4, 0x4000, np.uint16))])
    return kvsnap.encode(s, bytes([9] * 32), [2], 1024)


def read(b, profile, dims, max_bytes):
    return kvsnap.decode(b, profile, dims, 10, 100, 1, max_bytes)


def kind(fn):
    with pytest.raises(KvSnapError) as e:
        fn()
    return e.value.kind


def recalc(b: bytearray) -> bytes:
    n = len(b) - kvsnap.DIGEST
    b[n:] = hashlib.sha256(bytes(b[:n])).digest()
    return bytes(b)


def test_layout_of_the_example():
    b = example()
    assert len(b) == kvsnap.bytes_needed(2, 1, [2]) == 52 + 4 + 8 + 4 + 16 + 32
    assert b[:8] == b"SOSOKV01" and b[8:40] == bytes([9] * 32)
    assert struct.unpack_from("<4I", b, 40) == (2, 1, 1, 2)      # n, layers, hidden, width
    assert struct.unpack_from("<2If", b, 56) == (1, 2, 0.5)     # tokens, hidden
    assert struct.unpack_from("<8H", b, 68) == (0x3C00,) * 4 + (0x4000,) * 4
    assert b[-32:] == hashlib.sha256(b[:-32]).digest()
    s = read(b, bytes([9] * 32), [2], 1024)
    assert s.tokens.tolist() == [1, 2] and s.hidden.tolist() == [0.5]


def test_rejects_changes_and_lengths():
    """rechaza_cambios_y_longitudes_sin_reservas_excesivas (kvsnap.rs:143-159)."""
    b = example()
    assert kind(lambda: read(b, bytes([8] * 32), [2], 1024)) == "incompatible"
    assert kind(lambda: read(b, bytes([9] * 32), [3], 1024)) == "length"
    assert kind(lambda: read(b, bytes([9] * 32), [2], len(b) - 1)) == "length"
    for cut in range(len(b)):
        with pytest.raises(KvSnapError):
            read(b[:cut], bytes([9] * 32), [2], 1024)
    bad = bytearray(b)
    bad[56] ^= 1
    assert kind(lambda: read(bytes(bad), bytes([9] * 32), [2], 1024)) == "integrity"
    bad[40:44] = struct.pack("<I", 0xFFFFFFFF)
    assert kind(lambda: read(bytes(bad), bytes([9] * 32), [2], 1024)) == "length"


def test_rejects_invalid_values_with_a_correct_digest():
    """rechaza_valores_invalidos_incluso_con_checksum_correcto (kvsnap.rs:161-176): a token
    beyond the vocabulary, a NaN hidden value, an infinite K value."""
    b = bytearray(example())
    b[56:60] = struct.pack("<I", 100)
    assert kind(lambda: read(recalc(b), bytes([9] * 32), [2], 1024)) == "incompatible"
    b = bytearray(example())
    b[64:68] = struct.pack("<f", float("nan"))
    assert kind(lambda: read(recalc(b), bytes([9] * 32), [2], 1024)) == "non_finite"
    b = bytearray(example())
    b[68:70] = struct.pack("<H", 0x7C00)
    assert kind(lambda: read(recalc(b), bytes([9] * 32), [2], 1024)) == "non_finite"


def test_rejects_other_geometry_of_the_same_size():
    """rechaza_geometria_distinta_aunque_tenga_el_mismo_tamano (kvsnap.rs:178-188)."""
    z = lambda n: np.zeros(n, np.uint16)
    s = Snapshot(np.array([1]), np.array([0.0], np.float32), [(z(1), z(1)), (z(3), z(3))])
    b = kvsnap.encode(s, bytes([4] * 32), [1, 3], 1024)
    assert kind(lambda: kvsnap.decode(b, bytes([4] * 32), [2, 2], 10, 100, 1, 1024)) == "incompatible"


def test_encode_refuses_what_decode_would():
    z = lambda n: np.zeros(n, np.uint16)
    p = bytes(32)
    assert kind(lambda: kvsnap.encode(Snapshot(np.array([], np.uint32), np.ones(1, np.float32), [(z(0), z(0))]), p,
                                      [2], 1 << 20)) == "length"
    assert kind(lambda: kvsnap.encode(Snapshot(np.array([1]), np.array([np.inf], np.float32), [(z(2), z(2))]), p,
                                      [2], 1 << 20)) == "non_finite"
    assert kind(lambda: kvsnap.encode(Snapshot(np.array([1]), np.ones(1, np.float32), [(z(3), z(2))]), p, [2],
                                      1 << 20)) == "length"
    inf = np.full(2, 0xFC00, np.uint16)  # -inf
    assert kind(lambda: kvsnap.encode(Snapshot(np.array([1]), np.ones(1, np.float32), [(z(2), inf)]), p, [2],
                                      1 << 20)) == "non_finite"


def test_round_trip_of_a_decode_prefix():
    """A prefix of a GQA model's caches (36 layers of 2 kv heads x 128, 200 positions): the
    rows come back bit for bit."""
    g = np.random.default_rng(3)
    n, dims, hidden = 200, [256] * 36, 2048
    layers = [(g.standard_normal(n * d).astype(np.float16).view(np.uint16),
               g.standard_normal(n * d).astype(np.float16).view(np.uint16)) for d in dims]
    s = Snapshot(g.integers(0, 151936, n), g.standard_normal(hidden).astype(np.float32), layers)
    prof = hashlib.sha256(b"model fingerprint").digest()
    b = kvsnap.encode(s, prof, dims, 1 << 30)
    assert len(b) == kvsnap.bytes_needed(n, hidden, dims)
    r = kvsnap.decode(b, prof, dims, 4096, 151936, hidden, 1 << 30)
    assert np.array_equal(r.tokens, s.tokens) and np.array_equal(r.hidden, s.hidden)
    for (k, v), (k2, v2) in zip(layers, r.layers):
        assert np.array_equal(k, k2) and np.array_equal(v, v2)


def test_profile_of_a_model_directory(tmp_path):
    """identidad_kv::calcular: the fields in order, each length-prefixed; any byte of any
    file it covers changes the profile; paths leaving shards/ are refused."""
    import os
    import oracle
    gold = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "som_tiny")
    from soso_b200 import som
    idx = open(os.path.join(gold, "index.som"), "rb").read()
    man = open(os.path.join(gold, "manifest.som"), "rb").read()
    (tmp_path / "index.som").write_bytes(idx)
    (tmp_path / "manifest.som").write_bytes(man)
    (tmp_path / "tokenizer.som").write_bytes(b"tokenizer bytes")
    (tmp_path / "shards").mkdir()
    entries = som.parse_index(idx)
    for sh in sorted({e.shard for e in entries}):
        (tmp_path / "shards" / sh).write_bytes(oracle.pack_shard(sh.encode() * 3))
    got = kvsnap.profile(str(tmp_path), b"engine v1, f16 KV")

    def field(b):
        return len(b).to_bytes(8, "little") + b
    want = field(b"soso-kv-perfil-v1") + field(b"engine v1, f16 KV")
    for name in ("manifest.som", "index.som", "tokenizer.som"):
        want += field(name.encode()) + field(hashlib.sha256((tmp_path / name).read_bytes()).digest())
    for sh in sorted({e.shard for e in entries}):
        want += field(sh.encode()) + field(hashlib.sha256((tmp_path / "shards" / sh).read_bytes()).digest())
    assert got == hashlib.sha256(want).digest()
    assert kvsnap.profile(str(tmp_path), b"engine v2, f16 KV") != got
    victim = tmp_path / "shards" / entries[5].shard
    victim.write_bytes(victim.read_bytes()[:-1] + b"\x01")
    assert kvsnap.profile(str(tmp_path), b"engine v1, f16 KV") != got
    with pytest.raises(ValueError):
        kvsnap.profile(str(tmp_path), b"")
    (tmp_path / "index.som").write_bytes(oracle.serialize_index([(0, "w", "../manifest.som", 0, 4, (1,), 1, 0)]))
    with pytest.raises(ValueError):
        kvsnap.profile(str(tmp_path), b"engine v1")
