"""KV snapshots in the reference's portable format (crates/soso-llm-core/src/kvsnap.rs), so a
prefix decoded here can be resumed by the reference and the other way round.

Layout (little-endian): magic ``SOSOKV01``; a 32-byte profile (the fingerprint of weights,
tokenizer and inference settings the snapshot belongs to); u32 token count n, u32 layer
count, u32 hidden size; one u32 row width per layer; n u32 tokens; the f32 hidden vector;
per layer the f16 K rows then the f16 V rows (n x width each, positions from 0); SHA-256 of
everything before it.  ``decode`` makes the reference's checks in its order: length and
identity first (nothing is allocated from an unchecked count), then the digest, then the
row widths, token ids and finiteness.
"""
from __future__ import annotations

import hashlib
import os
from dataclasses import dataclass

import numpy as np

MAGIC = b"SOSOKV01"
HEADER = 8 + 32 + 4 + 4 + 4
DIGEST = 32


class KvSnapError(ValueError):
    """kvsnap::Error: kind is "incompatible", "length", "integrity" or "non_finite"."""

    def __init__(self, kind: str):
        super().__init__(kind)
        self.kind = kind


@dataclass
class Snapshot:
    """Snapshot (kvsnap.rs:27-31): tokens, the hidden vector, per layer (K, V) f16 bits,
    each n x width."""
    tokens: np.ndarray
    hidden: np.ndarray
    layers: list


def bytes_needed(tokens: int, hidden: int, dims) -> int:
    """bytes_necesarios (kvsnap.rs:33-39)."""
    return HEADER + 4 * tokens + 4 * len(dims) + 4 * hidden + 4 * tokens * int(sum(dims)) + DIGEST


def _finite_f16(bits: np.ndarray) -> bool:
    return not np.any((bits & 0x7C00) == 0x7C00)


def encode(s: Snapshot, profile: bytes, dims, max_bytes: int) -> bytes:
    """codificar (kvsnap.rs:43-72)."""
    dims = [int(d) for d in dims]
    tokens = np.asarray(s.tokens, dtype=np.uint32)
    hidden = np.asarray(s.hidden, dtype=np.float32)
    n = tokens.size
    if len(profile) != 32:
        raise KvSnapError("incompatible")
    nbytes = bytes_needed(n, hidden.size, dims)
    if n == 0 or n > 0xFFFFFFFF or hidden.size == 0 or not dims or len(s.layers) != len(dims) or nbytes > max_bytes:
        raise KvSnapError("length")
    if not np.all(np.isfinite(hidden)):
        raise KvSnapError("non_finite")
    rows = []
    for (k, v), d in zip(s.layers, dims):
        k = np.asarray(k, dtype=np.uint16).ravel()
        v = np.asarray(v, dtype=np.uint16).ravel()
        if d == 0 or d > 0xFFFFFFFF or k.size != n * d or v.size != n * d:
            raise KvSnapError("length")
        if not (_finite_f16(k) and _finite_f16(v)):
            raise KvSnapError("non_finite")
        rows += [k, v]
    head = MAGIC + bytes(profile) + np.array([n, len(dims), hidden.size], "<u4").tobytes()
    body = head + np.array(dims, "<u4").tobytes() + tokens.astype("<u4").tobytes() + hidden.astype("<f4").tobytes()
    body += b"".join(r.astype("<u2").tobytes() for r in rows)
    return body + hashlib.sha256(body).digest()


def decode(data: bytes, profile: bytes, dims, max_tokens: int, vocab: int, hidden_dim: int,
           max_bytes: int) -> Snapshot:
    """decodificar (kvsnap.rs:76-125)."""
    dims = [int(d) for d in dims]
    b = bytes(data)
    if len(b) < HEADER + DIGEST or len(b) > max_bytes:
        raise KvSnapError("length")
    if b[:8] != MAGIC or b[8:40] != bytes(profile):
        raise KvSnapError("incompatible")
    n, layers, hid = (int(x) for x in np.frombuffer(b, "<u4", 3, 40))
    if (n == 0 or n > max_tokens or hidden_dim == 0 or not dims or layers != len(dims) or any(d == 0 for d in dims)
            or hid != hidden_dim or bytes_needed(n, hidden_dim, dims) != len(b)):
        raise KvSnapError("length")
    end = len(b) - DIGEST
    if hashlib.sha256(b[:end]).digest() != b[end:]:
        raise KvSnapError("integrity")
    off = HEADER
    stored = np.frombuffer(b, "<u4", len(dims), off)
    if [int(x) for x in stored] != dims:
        raise KvSnapError("incompatible")
    off += 4 * len(dims)
    tokens = np.frombuffer(b, "<u4", n, off).astype(np.uint32)
    if np.any(tokens >= vocab):
        raise KvSnapError("incompatible")
    off += 4 * n
    hidden = np.frombuffer(b, "<f4", hidden_dim, off).astype(np.float32)
    if not np.all(np.isfinite(hidden)):
        raise KvSnapError("non_finite")
    off += 4 * hidden_dim
    out = []
    for d in dims:
        k = np.frombuffer(b, "<u2", n * d, off).astype(np.uint16)
        v = np.frombuffer(b, "<u2", n * d, off + 2 * n * d).astype(np.uint16)
        if not (_finite_f16(k) and _finite_f16(v)):
            raise KvSnapError("non_finite")
        out.append((k, v))
        off += 4 * n * d
    return Snapshot(tokens, hidden, out)


def _field(h, b: bytes) -> None:
    h.update(len(b).to_bytes(8, "little"))
    h.update(b)


def _file_sha256(path: str) -> bytes:
    """hash_fichero (identidad_kv.rs:16-36): SHA-256 of a regular file that must not change
    while it is read."""
    st0 = os.stat(path)
    if not os.path.isfile(path):
        raise OSError(f"{path}: not a regular file")
    h, total = hashlib.sha256(), 0
    with open(path, "rb") as f:
        while True:
            chunk = f.read(1 << 20)
            if not chunk:
                break
            total += len(chunk)
            h.update(chunk)
    st1 = os.stat(path)
    if total != st0.st_size or st0.st_size != st1.st_size or st0.st_mtime_ns != st1.st_mtime_ns:
        raise OSError(f"{path}: changed while its identity was computed")
    return h.digest()


def profile(model_dir: str, execution: bytes) -> bytes:
    """The 32-byte snapshot profile of a model directory (identidad_kv::calcular,
    crates/soso-llm-api/src/identidad_kv.rs:38-80): SHA-256 over length-prefixed fields --
    the tag "soso-kv-perfil-v1", the execution identity (every option that changes the KV
    values, and the engine version), then name and SHA-256 of manifest.som, index.som and
    tokenizer.som, then name and SHA-256 of every shard the index names, in sorted order.
    Shard paths that leave the shards directory are refused."""
    from .som import parse_index
    if not execution:
        raise ValueError("missing execution identity")
    h = hashlib.sha256()
    _field(h, b"soso-kv-perfil-v1")
    _field(h, bytes(execution))
    with open(os.path.join(model_dir, "index.som"), "rb") as f:
        index_bytes = f.read()
    entries = parse_index(index_bytes)
    for name in ("manifest.som", "index.som", "tokenizer.som"):
        _field(h, name.encode())
        digest = _file_sha256(os.path.join(model_dir, name))
        if name == "index.som" and digest != hashlib.sha256(index_bytes).digest():
            raise OSError("index.som changed while the identity was computed")
        _field(h, digest)
    shards = set()
    for e in entries:
        parts = e.shard.split("/")
        if not e.shard or any(p in ("", ".", "..") for p in parts) or os.path.isabs(e.shard):
            raise ValueError(f"invalid shard path {e.shard!r}")
        shards.add(e.shard)
    if not shards:
        raise ValueError("index without shards")
    root = os.path.realpath(os.path.join(model_dir, "shards"))
    for name in sorted(shards, key=lambda n: n.encode()):
        path = os.path.realpath(os.path.join(root, name))
        if os.path.commonpath([root, path]) != root:
            raise ValueError(f"shard {name!r} outside the shards directory")
        _field(h, name.encode())
        _field(h, _file_sha256(path))
    return h.digest()


def dims_of(cfg) -> list:
    """The per-layer row widths a snapshot of this configuration carries (dimensiones_snapshot,
    crates/soso-llm-core/src/runtime.rs:527-541): kv_heads x head_dim of every GQA layer.
    The reference refuses MLA latent caches (and MoE models run with a planner), so do we."""
    if getattr(cfg, "mla", False):
        raise KvSnapError("incompatible")
    return [cfg.kv_dim] * cfg.n_layers


def export_session(session, tokens, profile: bytes, max_bytes: int) -> bytes:
    """Runtime::exportar_kv (runtime.rs:544-556) over a decode session on the device: the
    cached tokens are `tokens` (one per decoded position, from 0); the rows of those
    positions of every layer and the hidden vector the last step left come down from the
    device (sb_decode_download_state) and are encoded."""
    tokens = np.asarray(tokens, dtype=np.uint32)
    cfg = session.cfg
    if tokens.size == 0 or tokens.size > cfg.ctx:
        raise KvSnapError("incompatible")
    layers, hidden = session.download_state(int(tokens.size))
    return encode(Snapshot(tokens, hidden, [(k, v) for k, v in layers]), profile, dims_of(cfg), max_bytes)


def import_session(session, image: bytes, profile: bytes, max_bytes: int) -> Snapshot:
    """Runtime::importar_kv (runtime.rs:558-580) into a decode session on the device: every
    check of `decode` first (a refused image changes nothing), then the rows go up
    (sb_decode_upload_state at position len(tokens)); returns the snapshot, whose tokens and
    hidden vector the caller keeps as the runtime does."""
    cfg = session.cfg
    snap = decode(image, profile, dims_of(cfg), cfg.ctx, cfg.vocab, cfg.hidden, max_bytes)
    n = int(snap.tokens.size)
    session.upload_state([(k.reshape(n, -1), v.reshape(n, -1)) for k, v in snap.layers], n)
    return snap
