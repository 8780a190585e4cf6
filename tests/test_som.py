"""The .som reader (soso_b200/som.py + sb_crc32c / sb_som_payload in the library), CPU only.

Pinned against: the CRC-32C check value of the published algorithm ("123456789" ->
0xE3069283; the `crc` crate's CRC_32_ISCSI, crc-catalog 2.5.0, which
crates/sosomodel/src/lib.rs:30-34 uses) and a bitwise restatement; the reference's own
tiny model headers (tests/golden/som_tiny, copied by make_som_fixture.py from
rootfs/models/tiny); the reference's shard / index / truncation tests
(crates/sosomodel/tests/roundtrip.rs:137-242), restated.
"""
import json
import os

import numpy as np
import pytest

import oracle
from soso_b200 import som

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "som_tiny")


def test_crc32c_check_value_and_bitwise():
    assert som.crc32c(b"123456789") == 0xE3069283
    assert som.crc32c(b"") == 0
    g = np.random.default_rng(5)
    buf = g.integers(0, 256, 300, dtype=np.uint8).tobytes()
    for start in range(0, 9):  # every alignment of the eight-byte steps
        for n in (0, 1, 7, 8, 9, 15, 16, 17, 63, 64, 65, 200):
            piece = buf[start:start + n]
            assert som.crc32c(piece) == oracle.crc32c_bitwise(piece), (start, n)


def test_reference_tiny_model_headers():
    """The index and manifest the reference wrote: headers and CRCs agree, every entry is an
    f32 tensor whose byte length is its shape's, and every shard it names is a file of the
    model that holds those bytes."""
    with open(os.path.join(GOLD, "index.som"), "rb") as f:
        entries = som.parse_index(f.read())
    with open(os.path.join(GOLD, "manifest.som"), "rb") as f:
        version, body = som.payload(f.read())
    assert version >= 1 and body.size > 0
    shards = json.load(open(os.path.join(GOLD, "shards.json")))
    assert len(entries) == 22 and len({e.name for e in entries}) == 22
    assert sorted(e.id for e in entries) == list(range(22))
    e0 = entries[0]
    assert (e0.name, e0.shard, e0.offset, e0.byte_len, e0.shape, e0.dtype, e0.quant) == (
        "L00.attn_q", "L00.attn_q.tensor", 0, 65536, (128, 128), 1, 0)
    for e in entries:
        assert e.dtype == 1 and e.quant == 0 and e.byte_len == 4 * int(np.prod(e.shape)), e
        assert e.shard in shards and e.offset + e.byte_len <= shards[e.shard], e


def test_shard_cases_of_the_reference():
    """roundtrip.rs:137-151, :172-207: pack -> verify returns the payload; a flipped magic
    byte is rejected; 600 payloads of 37 bytes verify whatever their CRC; the v2 payload
    sits at byte 64 and the file is a multiple of 4096; trailing zeros are kept."""
    p = oracle.pack_shard(bytes([1, 2, 3, 4]))
    assert som.payload(p, shard=True)[1].tobytes() == bytes([1, 2, 3, 4])
    bad = bytearray(p)
    bad[0] ^= 0xFF
    with pytest.raises(som.SomError):
        som.payload(bytes(bad), shard=True)
    for seed in range(600):
        data = bytes(((seed * 31 + i) % (1 << 32)) % 251 for i in range(37))
        assert som.payload(oracle.pack_shard(data), shard=True)[1].tobytes() == data, seed
    data = bytes(range(100))
    p = np.frombuffer(oracle.pack_shard(data), dtype=np.uint8)
    v, body = som.payload(p, shard=True)
    assert v == 2 and body.ctypes.data - p.ctypes.data == 64 and p.size % 4096 == 0 and body.tobytes() == data
    assert som.payload(oracle.pack_shard(bytes([1, 2, 3, 0, 0, 0])), shard=True)[1].tobytes() == bytes([1, 2, 3, 0,
                                                                                                        0, 0])
    flip = bytearray(oracle.pack_shard(data))
    flip[64 + 50] ^= 1  # a payload bit: the CRC no longer matches
    with pytest.raises(som.SomError):
        som.payload(bytes(flip), shard=True)


def test_truncated_and_corrupt_headers_raise():
    """roundtrip.rs:220-242: no truncation of an index or manifest is accepted, and a huge
    payload length is rejected."""
    idx = open(os.path.join(GOLD, "index.som"), "rb").read()
    man = open(os.path.join(GOLD, "manifest.som"), "rb").read()
    for data in (idx, man):
        for cut in range(len(data)):
            try:
                som.payload(data[:cut])
            except som.SomError:
                continue
            # a cut inside the zero padding after the payload is still a whole file
            assert cut >= 24 + int.from_bytes(data[16:24], "little"), cut
    evil = bytearray(man)
    evil[16:24] = (2 ** 64 - 1).to_bytes(8, "little")
    with pytest.raises(som.SomError):
        som.payload(bytes(evil))
    with pytest.raises(som.SomError):
        som.payload(b"NOTSOM01" + man[8:])


def test_model_directory_views(tmp_path):
    """A model directory with the reference's tiny index and manifest and shards written by
    the reference's pack_shard: every tensor comes back as the bytes written, as a view of
    its mapped shard; a corrupted shard is refused on first use."""
    for f in ("index.som", "manifest.som"):
        (tmp_path / f).write_bytes(open(os.path.join(GOLD, f), "rb").read())
    with open(os.path.join(GOLD, "index.som"), "rb") as f:
        entries = som.parse_index(f.read())
    (tmp_path / "shards").mkdir()
    want = {}
    g = np.random.default_rng(11)
    for shard in sorted({e.shard for e in entries}):  # tensors may share a shard
        mine = [e for e in entries if e.shard == shard]
        raw = g.integers(0, 256, max(e.offset + e.byte_len for e in mine), dtype=np.uint8).tobytes()
        for e in mine:
            want[e.name] = raw[e.offset:e.offset + e.byte_len]
        (tmp_path / "shards" / shard).write_bytes(oracle.pack_shard(raw))
    m = som.SomModel(str(tmp_path))
    try:
        assert m.manifest.name == "tiny" and m.manifest.n_layers == 4
        assert set(m.names()) == set(want)
        for name, raw in want.items():
            t = m.tensor(name)
            assert t.dtype == np.uint8 and t.tobytes() == raw
        with pytest.raises(KeyError):
            m.tensor("no.such.tensor")
    finally:
        m.close()
    victim = entries[3].shard
    b = bytearray((tmp_path / "shards" / victim).read_bytes())
    b[64 + 7] ^= 0x40
    (tmp_path / "shards" / victim).write_bytes(bytes(b))
    m = som.SomModel(str(tmp_path))
    try:
        with pytest.raises(som.SomError):
            m.tensor(entries[3].name)
        m2 = som.SomModel(str(tmp_path), verify=False)  # header-only checks load it
        assert m2.tensor(entries[3].name).size == entries[3].byte_len
        m2.close()
    finally:
        m.close()


def test_index_roundtrip_of_the_reference_writer(tmp_path):
    """index_roundtrip (roundtrip.rs:153-160) with the reference's serializer restated, and a
    shard name that would leave the shards directory refused."""
    data = oracle.serialize_index([(0, "w", "s.tensor", 0, 64, (4, 4), 1, 0),
                                   (1, "blk.0.attn_q.weight", "s.tensor", 64, 144, (1, 256), 3, 2)])
    es = som.parse_index(data)
    assert [(e.id, e.name, e.shard, e.offset, e.byte_len, e.shape, e.dtype, e.quant) for e in es] == [
        (0, "w", "s.tensor", 0, 64, (4, 4), 1, 0), (1, "blk.0.attn_q.weight", "s.tensor", 64, 144, (1, 256), 3, 2)]
    (tmp_path / "index.som").write_bytes(oracle.serialize_index([(0, "w", "../index.som", 0, 4, (1,), 1, 0)]))
    (tmp_path / "manifest.som").write_bytes(open(os.path.join(GOLD, "manifest.som"), "rb").read())
    m = som.SomModel(str(tmp_path))
    with pytest.raises(som.SomError):
        m.tensor("w")
    m.close()


def test_manifest_core_of_the_reference_tiny_model():
    """Manifest::tiny (manifest.rs), the model rootfs/models/tiny was written from: vocab 256,
    hidden 128, 4 layers of 4 heads, ffn 256, 128 positions; a version-1 manifest takes the
    v1 defaults (kv heads = heads, theta 1e4, eps 1e-5, no experts)."""
    mc = som.parse_manifest_core(open(os.path.join(GOLD, "manifest.som"), "rb").read())
    assert (mc.vocab, mc.hidden, mc.n_layers, mc.heads, mc.ffn, mc.max_seq) == (256, 128, 4, 4, 256, 128)
    assert (mc.kv_heads, mc.rope_theta, mc.n_experts, mc.experts_per_tok, mc.moe_ffn) == (4, 10000.0, 0, 0, 0)
    assert mc.version == 1 and abs(mc.rms_eps - 1e-5) < 1e-12
    # the reference's own index agrees with it: 4 layers of q/k/v at hidden x hidden, ffn_up at ffn x hidden
    es = {e.name: e for e in som.parse_index(open(os.path.join(GOLD, "index.som"), "rb").read())}
    for l in range(mc.n_layers):
        assert es[f"L{l:02d}.attn_q"].shape == (mc.hidden, mc.hidden)
        assert es[f"L{l:02d}.ffn_up"].shape in ((mc.ffn, mc.hidden), (mc.hidden, mc.ffn))
    assert es["embed"].shape in ((mc.vocab, mc.hidden), (mc.hidden, mc.vocab))


def test_manifest_prefetch_of_the_reference_tiny_model():
    """The whole version-1 payload the reference wrote parses: the leading fields, then the
    per-layer prefetch lists (layers 0-3, the five shard files each layer's tensors live in),
    with no byte left over."""
    m = som.parse_manifest(open(os.path.join(GOLD, "manifest.som"), "rb").read())
    shards = json.load(open(os.path.join(GOLD, "shards.json")))
    assert m.layers == () and m.chat_template == "" and m.rest == b""
    assert [l for l, _ in m.prefetch] == [0, 1, 2, 3]
    for l, names in m.prefetch:
        assert names == tuple(f"L{l:02d}.{t}.tensor" for t in ("attn_q", "attn_k", "attn_v", "ffn_up", "ffn_down"))
        assert all(n in shards for n in names)


def test_manifest_layer_specs_round_trip():
    """A version-5 manifest of a DeepSeek-V2-Lite-like model (an MLA layer with a dense FFN,
    then MLA + MoE layers) written by the reference's serializer restated: the layer specs,
    prefetch lists and chat template come back; unknown kinds and a spec count that differs
    from the layer count are refused."""
    import oracle
    core = ("dsv2lite", 102400, 2048, 3, 16, 10944, 2048, 16, 1e4, 1e-6, 64, 6, 1408)
    mla_dense = (1, 0, 16, 16, 10944, 512, 0, 64, 128, 128, 0, 0, 0, 0, 0)
    mla_moe = (1, 1, 16, 16, 10944, 512, 0, 64, 128, 128, 64, 6, 1408, 2, 0)
    pf = [(0, ["a.tensor", "b.tensor"]), (1, []), (2, ["c.tensor"])]
    m = som.parse_manifest(oracle.serialize_manifest_prefix(5, core, [mla_dense, mla_moe, mla_moe], pf, "{{x}}"))
    assert m.core.version == 5 and m.core.n_experts == 64 and abs(m.core.rms_eps - 1e-6) < 1e-12
    assert [(l.attn, l.ffn) for l in m.layers] == [("mla", "dense"), ("mla", "moe"), ("mla", "moe")]
    l1 = m.layers[1]
    assert (l1.kv_rank, l1.qk_rope, l1.qk_nope, l1.v_dim, l1.n_experts, l1.experts_per_tok, l1.moe_ffn,
            l1.n_shared) == (512, 64, 128, 128, 64, 6, 1408, 2)
    assert m.prefetch == ((0, ("a.tensor", "b.tensor")), (1, ()), (2, ("c.tensor",)))
    assert m.chat_template == "{{x}}" and m.rest == b""
    with pytest.raises(som.SomError):
        som.parse_manifest(oracle.serialize_manifest_prefix(5, core, [mla_dense, mla_moe, (9,) + mla_moe[1:]], pf))
    with pytest.raises(som.SomError):
        som.parse_manifest(oracle.serialize_manifest_prefix(5, core, [mla_dense, mla_moe], pf))


def test_manifest_versions_6_to_9_round_trip():
    """The fields after the chat template (manifest.rs:1082-1150), written by the reference's
    serializer restated: model and norm kinds with the audio spec (v6), the extensions (v7),
    YaRN (v8) and the pointer head (v9) come back, with no byte left; more windows than
    layers and an unknown model kind are refused."""
    import oracle
    core = ("m", 1024, 512, 2, 4, 1024, 160, 2, 1e4, 1e-6, 0, 0, 0)
    specs = [(0, 0, 4, 2, 1024, 0, 0, 0, 0, 0, 0, 0, 0, 0, 8)] * 2
    ext = (1.5, 30.0, 0.25, True, (0, 4096), (1e6, 0.0), (16.0, 8192, 32.0, 1.0))
    m = som.parse_manifest(oracle.serialize_manifest(9, core, specs, [], "t", model_kind=2, norm_kind=1,
                                                     audio=tuple(range(1, 10)), ext=ext, kev=(0.5, 256)))
    assert (m.model_kind, m.norm_kind, m.audio) == ("decision", "layer", tuple(range(1, 10)))
    assert m.ext.embed_scale == 1.5 and m.ext.logit_softcap == 30.0 and m.ext.attn_scale == 0.25
    assert m.ext.tied_lm_head and m.ext.window == (0, 4096) and m.ext.rope_theta == (1e6, 0.0)
    assert m.ext.yarn == (16.0, 8192, 32.0, 1.0) and m.ext.yarn_active()
    assert m.kev == (0.5, 256) and m.rest == b""
    m7 = som.parse_manifest(oracle.serialize_manifest(7, core, specs, [], ext=ext))
    assert m7.ext.yarn == (0.0, 0, 0.0, 0.0) and not m7.ext.yarn_active() and m7.kev is None and m7.rest == b""
    with pytest.raises(som.SomError):
        som.parse_manifest(oracle.serialize_manifest(7, core, specs, [], ext=ext[:4] + ((0, 0, 0),) + ext[5:]))
    with pytest.raises(som.SomError):
        som.parse_manifest(oracle.serialize_manifest(6, core, specs, [], model_kind=3))
