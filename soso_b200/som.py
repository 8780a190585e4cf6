"""Reader of the reference's model directories: ``manifest.som``, ``index.som`` and
``shards/*`` (crates/sosomodel/src/layout.rs:3-6).

Every .som file is a 24-byte header (magic ``SOMODL01``, CRC-32C of the payload, version,
payload length) and the payload (lib.rs:70-104); a shard of version >= 2 puts its payload
at byte 64 so that mmap'd weights are 64-byte aligned (index.rs:93-139).  The header
checks and the CRC run in the library (``sb_som_payload``, ``sb_crc32c``).  The index is
the tensor table (TensorIndex::parse, index.rs:61-91); a tensor's bytes are a slice of its
shard's payload, handed to the decode plan (``SbMat`` views) without a copy.  The
manifest (manifest.rs) is read whole by ``parse_manifest`` (versions 1 to 9: the leading
fields, per-layer specs, prefetch lists, chat template, model kind and audio spec, the
extensions with YaRN, the pointer head); ``parse_manifest_core`` reads only the leading
fields every version shares (sizes, heads, RoPE theta, RMS eps, expert counts).
"""
from __future__ import annotations

import ctypes
import mmap
import os
from dataclasses import dataclass

import numpy as np

from ._lib import c_size, lib

MANIFEST_FILE, INDEX_FILE, SHARDS_DIR = "manifest.som", "index.som", "shards"


class SomError(ValueError):
    """A .som file whose header, length, CRC or table does not hold together."""


def payload(buf, shard: bool = False) -> tuple[int, np.ndarray]:
    """(version, payload bytes as a uint8 view of `buf`) -- parse_som (lib.rs:88-104), or
    verify_shard (index.rs:118-139) when `shard`; raises SomError like their Err(())."""
    arr = np.frombuffer(buf, dtype=np.uint8)
    p, n, v = ctypes.c_void_p(), c_size(), ctypes.c_uint32()
    base = arr.ctypes.data if arr.size else None
    if lib().sb_som_payload(base, arr.size, int(shard), ctypes.byref(p), ctypes.byref(n), ctypes.byref(v)) != 1:
        raise SomError("not a .som file, or its length / CRC-32C does not match")
    off = p.value - arr.ctypes.data
    return int(v.value), arr[off:off + n.value]


def crc32c(buf) -> int:
    """CRC-32C of `buf` (sosomodel::crc32c, lib.rs:32-34)."""
    arr = np.frombuffer(buf, dtype=np.uint8)
    return int(lib().sb_crc32c(arr.ctypes.data if arr.size else None, arr.size))


@dataclass(frozen=True)
class TensorEntry:
    """One row of index.som (TensorEntry, index.rs:14-24)."""
    id: int
    name: str
    shard: str
    offset: int
    byte_len: int
    shape: tuple
    dtype: int
    quant: int


class _Cursor:
    """Bounds-checked little-endian reads (Reader, lib.rs:106-147)."""

    def __init__(self, b: bytes):
        self.b, self.off = b, 0

    def take(self, n: int) -> bytes:
        if n < 0 or self.off + n > len(self.b):
            raise SomError("truncated .som payload")
        s = self.b[self.off:self.off + n]
        self.off += n
        return s

    def u8(self) -> int:
        return self.take(1)[0]

    def u32(self) -> int:
        return int.from_bytes(self.take(4), "little")

    def u64(self) -> int:
        return int.from_bytes(self.take(8), "little")

    def f32(self) -> float:
        return float(np.frombuffer(self.take(4), "<f4")[0])

    def cstr(self) -> str:
        j = self.b.find(b"\0", self.off)
        if j < 0:
            raise SomError("unterminated string in .som payload")
        try:
            s = self.b[self.off:j].decode("utf-8")
        except UnicodeDecodeError as e:
            raise SomError("string in .som payload is not UTF-8") from e
        self.off = j + 1
        return s


def parse_index(buf) -> list[TensorEntry]:
    """TensorIndex::parse (index.rs:61-91): u32 count; per tensor u32 id, name NUL, shard NUL,
    u64 offset, u64 byte_len, u32 ndim, ndim x u32, u8 dtype, u8 quant, 2 padding bytes."""
    _, body = payload(buf)
    r = _Cursor(body.tobytes())
    out = []
    for _ in range(r.u32()):
        tid, name, shard = r.u32(), r.cstr(), r.cstr()
        offset, byte_len = r.u64(), r.u64()
        shape = tuple(r.u32() for _ in range(r.u32()))
        dtype, quant = r.u8(), r.u8()
        r.take(2)
        out.append(TensorEntry(tid, name, shard, offset, byte_len, shape, dtype, quant))
    return out


@dataclass(frozen=True)
class ManifestCore:
    """The fields every manifest version starts with (Manifest::parse, manifest.rs:1021-1050):
    v1 name .. max_seq; v2 adds kv_heads, rope_theta, rms_eps (v1: heads, 1e4, 1e-5);
    v3 adds the expert counts (earlier: 0).  Later versions continue with per-layer specs
    and extensions, which are not read here."""
    version: int
    name: str
    vocab: int
    hidden: int
    n_layers: int
    heads: int
    ffn: int
    max_seq: int
    kv_heads: int
    rope_theta: float
    rms_eps: float
    n_experts: int
    experts_per_tok: int
    moe_ffn: int


def parse_manifest_core(buf) -> ManifestCore:
    """The manifest's leading fields, with the reference's checks on them: heads and kv heads
    non-zero and, before version 4, hidden % heads == 0 and heads % kv_heads == 0."""
    version, body = payload(buf)
    return _read_core(version, _Cursor(body.tobytes()))


def _read_core(version: int, r: _Cursor) -> ManifestCore:
    name = r.cstr()
    vocab, hidden, n_layers, heads, ffn, max_seq = (r.u32() for _ in range(6))
    if version >= 2:
        kv_heads = r.u32()
        theta = float(np.frombuffer(r.take(4), "<f4")[0])
        eps = float(np.frombuffer(r.take(4), "<f4")[0])
    else:
        kv_heads, theta, eps = heads, 10000.0, float(np.float32(1e-5))
    n_exp, per_tok, moe_ffn = (r.u32(), r.u32(), r.u32()) if version >= 3 else (0, 0, 0)
    if heads == 0 or kv_heads == 0:
        raise SomError("manifest: zero heads")
    if version < 4 and (hidden % heads or heads % kv_heads):
        raise SomError("manifest: heads do not divide the hidden size / kv heads")
    return ManifestCore(version, name, vocab, hidden, n_layers, heads, ffn, max_seq, kv_heads, theta, eps, n_exp,
                        per_tok, moe_ffn)


ATTN_KINDS = ("gqa", "mla", "kda", "gated", "gdn", "bidirectional", "cross")  # AttnKind, manifest.rs:10-35
FFN_KINDS = ("dense", "moe", "latent_moe", "gelu_mlp")                          # FfnKind, manifest.rs:41-58


@dataclass(frozen=True)
class LayerSpec:
    """One layer of a version >= 4 manifest (LayerSpec::parse, manifest.rs:346-368): the
    attention and FFN kinds, then 13 u32 -- heads, kv heads, ffn width, the MLA ranks and
    head widths, the expert counts and widths, flags."""
    attn: str
    ffn: str
    heads: int
    kv_heads: int
    ffn_dim: int
    kv_rank: int
    q_rank: int
    qk_rope: int
    qk_nope: int
    v_dim: int
    n_experts: int
    experts_per_tok: int
    moe_ffn: int
    n_shared: int
    flags: int


MODEL_KINDS = ("decoder", "asr_encoder_decoder", "decision")  # ModelKind, manifest.rs:80-95
NORM_KINDS = ("rms", "layer")                                   # NormKind, manifest.rs:63-76


@dataclass(frozen=True)
class ManifestExt:
    """Version 7 / 8 extensions (ManifestExt and YarnSpec, manifest.rs:111-161), every field
    "no effect" by default: embedding scale (0 = none), logit soft cap (0 = none), attention
    scale (0 = 1/sqrt(head_dim)), tied output matrix, per-layer window (0 = full) and RoPE base
    (0 = the global one), and YaRN (factor, original context, beta_fast, beta_slow; active
    when factor > 1 and the context > 0, YarnSpec::activa, manifest.rs:131-135)."""
    embed_scale: float = 0.0
    logit_softcap: float = 0.0
    attn_scale: float = 0.0
    tied_lm_head: bool = False
    window: tuple = ()
    rope_theta: tuple = ()
    yarn: tuple = (0.0, 0, 0.0, 0.0)

    def yarn_active(self) -> bool:
        return self.yarn[0] > 1.0 and self.yarn[1] > 0


@dataclass(frozen=True)
class ManifestPlan:
    """The whole manifest (Manifest::parse, manifest.rs:1021-1176): the leading fields, the
    per-layer specs (version >= 4; before that the globals describe every layer), the
    per-layer prefetch lists of shard names, the chat template (version >= 5), the model and
    norm kinds and the audio spec (version >= 6), the extensions (versions 7 and 8) and the
    pointer head (version 9: temperature, pointer width).  ``rest`` holds any bytes after
    the last field the version defines (the reference ignores them)."""
    core: ManifestCore
    layers: tuple
    prefetch: tuple
    chat_template: str
    rest: bytes
    model_kind: str = "decoder"
    norm_kind: str = "rms"
    audio: tuple = (0,) * 9
    ext: ManifestExt = ManifestExt()
    kev: tuple | None = None


def parse_manifest(buf) -> ManifestPlan:
    version, body = payload(buf)
    r = _Cursor(body.tobytes())
    core = _read_core(version, r)
    layers = ()
    if version >= 4:
        n = r.u32()
        if n != core.n_layers:
            raise SomError("manifest: layer specs do not match the layer count")
        specs = []
        for _ in range(n):
            a, f = r.u8(), r.u8()
            r.take(2)
            if a >= len(ATTN_KINDS) or f >= len(FFN_KINDS):
                raise SomError("manifest: unknown attention or FFN kind")
            specs.append(LayerSpec(ATTN_KINDS[a], FFN_KINDS[f], *(r.u32() for _ in range(13))))
        layers = tuple(specs)
    prefetch = []
    for _ in range(r.u32()):
        layer = r.u32()
        prefetch.append((layer, tuple(r.cstr() for _ in range(r.u32()))))
    template = r.cstr() if version >= 5 else ""
    kinds = {}
    if version >= 6:  # model kind, norm kind, u16 pad, AudioSpec (manifest.rs:1082-1100)
        mk, nk = r.u8(), r.u8()
        r.take(2)
        if mk >= len(MODEL_KINDS) or nk >= len(NORM_KINDS):
            raise SomError("manifest: unknown model or norm kind")
        kinds = dict(model_kind=MODEL_KINDS[mk], norm_kind=NORM_KINDS[nk], audio=tuple(r.u32() for _ in range(9)))
    if version >= 7:  # ManifestExt (manifest.rs:1101-1130): window / theta lists <= n_layers
        es, cap, sc = r.f32(), r.f32(), r.f32()
        tied = r.u32() != 0
        n_w = r.u32()
        if n_w > core.n_layers:
            raise SomError("manifest: more windows than layers")
        window = tuple(r.u32() for _ in range(n_w))
        n_t = r.u32()
        if n_t > core.n_layers:
            raise SomError("manifest: more RoPE bases than layers")
        thetas = tuple(r.f32() for _ in range(n_t))
        yarn = (r.f32(), r.u32(), r.f32(), r.f32()) if version >= 8 else (0.0, 0, 0.0, 0.0)
        kinds["ext"] = ManifestExt(es, cap, sc, tied, window, thetas, yarn)
    if version >= 9:  # KevSpec (manifest.rs:1143-1150)
        kinds["kev"] = (r.f32(), r.u32())
    return ManifestPlan(core, layers, tuple(prefetch), template, r.b[r.off:], **kinds)


class SomModel:
    """A model directory: the index, the manifest payload, and each shard mapped once
    (read-only) with its CRC checked on first use (``verify=False`` skips the check)."""

    def __init__(self, path: str, verify: bool = True):
        self.path, self.verify = path, verify
        with open(os.path.join(path, MANIFEST_FILE), "rb") as f:
            raw = f.read()
        self.manifest_version, mp = payload(raw)
        self.manifest_payload = mp.tobytes()
        self.manifest = parse_manifest_core(raw)
        with open(os.path.join(path, INDEX_FILE), "rb") as f:
            self.entries = {e.name: e for e in parse_index(f.read())}
        self._shards: dict[str, tuple] = {}

    def names(self) -> list[str]:
        return list(self.entries)

    def _shard(self, shard: str) -> np.ndarray:
        if shard not in self._shards:
            if os.path.basename(shard) != shard or shard in ("", ".", ".."):
                raise SomError(f"shard name {shard!r} leaves the shards directory")
            with open(os.path.join(self.path, SHARDS_DIR, shard), "rb") as f:
                try:
                    mm = mmap.mmap(f.fileno(), 0, access=mmap.ACCESS_READ)
                except ValueError as e:  # an empty file
                    raise SomError(f"shard {shard}: empty file") from e
            raw = np.frombuffer(mm, dtype=np.uint8)
            if self.verify:
                _, body = payload(raw, shard=True)
            else:  # header fields only
                ver = int.from_bytes(raw[12:16].tobytes(), "little")
                plen = int.from_bytes(raw[16:24].tobytes(), "little")
                off = 64 if ver >= 2 else 24
                if raw[:8].tobytes() != b"SOMODL01" or off + plen > raw.size:
                    raise SomError(f"shard {shard}: bad header")
                body = raw[off:off + plen]
            self._shards[shard] = (mm, body)
        return self._shards[shard][1]

    def tensor(self, name: str) -> np.ndarray:
        """The tensor's bytes (uint8 view into its mapped shard, no copy)."""
        e = self.entries.get(name)
        if e is None:
            raise KeyError(name)
        body = self._shard(e.shard)
        if e.offset + e.byte_len > body.size:
            raise SomError(f"{name}: bytes {e.offset}..{e.offset + e.byte_len} beyond its shard's payload")
        return body[e.offset:e.offset + e.byte_len]

    def close(self):
        for mm, _ in self._shards.values():
            try:
                mm.close()
            except BufferError:  # views still alive: the map goes with them
                pass
        self._shards.clear()
