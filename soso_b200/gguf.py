"""GGUF checkpoints into the decode session, by the reference's GGUF -> .som conversion
rules (crates/gguf2som/src/lib.rs): the same weight bytes the reference's converter writes,
mapped to the ``DenseConfig`` and tensor dict ``decode.DecodeSession`` takes.

* The container (``parse_gguf``, lib.rs:1450-1505): magic ``GGUF``, version >= 2, tensor
  and metadata counts, typed metadata values (lib.rs:1665-1735), tensor infos (name, GGML
  dims fastest first, GGML type, offset), data at the next multiple of
  ``general.alignment`` (32 when absent or not a power of two).
* Per tensor (``read_tensor``, lib.rs:1507-1624): F32 as it is; F16 widened to F32; GGML
  Q8_0 (f16 scale + 32 i8, 34 bytes) repacked as .som Q8_0 (f32 scale, 36 bytes); Q4_0,
  Q4_K, MXFP4 and the other K- / i-quants passed through; Q5_0 and Q6_K dequantised and
  quantised again to Q8_0 (``quantize_q8_0``, crates/soso-llm-core/src/quant.rs:8-25).
  ``keep_q6k=True`` keeps Q6_K blocks as they are instead (this backend runs Q6_K matrices
  natively: fewer bytes than the Q8_0 copy, no requantisation).
* Per layer (lib.rs:300-690): the GGUF names ``blk.{l}.{part}.weight`` of the llama / qwen2 /
  qwen3 / qwen3moe layouts, ``attn_{q,k,v}.bias`` (qwen2), a layer's experts stored as one
  3-D tensor ``ffn_{gate,up,down}_exps`` sliced per expert (``emit_moe_experts``,
  lib.rs:1160-1199; or the older 2-D ``ffn_gate.{e}``), a shared expert
  ``ffn_*_shexp`` with its gate row ``ffn_gate_inp_shexp``; ``token_embd``, ``output``
  (the embedding when absent), ``output_norm``.
* The model's widths from the metadata of ``general.architecture`` (lib.rs:221-300), NeoX
  RoPE for qwen2 / qwen3 layouts and QK-norm and the head width from
  ``attention.key_length`` for qwen3 (lib.rs:784-809).

DeepSeek-V2 (MLA) GGUFs are not mapped here: convert them with the reference's gguf2som
and open the model directory with ``som_load``.
"""
from __future__ import annotations

import mmap
import struct

import numpy as np

from .decode import DenseConfig
from .formats import DTYPE_F32, DTYPE_Q4_K, DTYPE_Q6_K, DTYPE_Q8_0

# GGML tensor types (ggml.h) and the .som dtype codes (crates/sosomodel/src/layout.rs:8-46)
GGML_F32, GGML_F16, GGML_Q4_0, GGML_Q5_0, GGML_Q8_0 = 0, 1, 2, 6, 8
GGML_Q3_K, GGML_Q4_K, GGML_Q5_K, GGML_Q6_K = 11, 12, 13, 14
GGML_IQ3_XXS, GGML_IQ3_S, GGML_IQ2_S, GGML_IQ4_XS, GGML_IQ2_XS = 18, 21, 22, 23, 17
GGML_MXFP4 = 39
DTYPE_MXFP4, DTYPE_Q4_0 = 4, 5
# passthrough blocks: GGML type -> (.som dtype, elements, bytes per block)
_PASS = {GGML_Q4_0: (DTYPE_Q4_0, 32, 18), GGML_Q4_K: (DTYPE_Q4_K, 256, 144), GGML_MXFP4: (DTYPE_MXFP4, 32, 17),
         GGML_Q3_K: (6, 256, 110), GGML_Q5_K: (7, 256, 176), GGML_IQ2_XS: (8, 256, 74), GGML_IQ2_S: (9, 256, 82),
         GGML_IQ3_XXS: (10, 256, 98), GGML_IQ3_S: (11, 256, 110), GGML_IQ4_XS: (12, 256, 136)}


class GgufError(ValueError):
    pass


class GgufFile:
    """A GGUF file mapped read-only: ``meta`` (key -> int / float / str / list) and
    ``tensors`` (name -> (dims fastest first, GGML type, byte offset in the data))."""

    def __init__(self, path: str):
        self._f = open(path, "rb")
        try:
            self.buf = mmap.mmap(self._f.fileno(), 0, access=mmap.ACCESS_READ)
        except ValueError as e:  # an empty file
            self._f.close()
            raise GgufError(f"{path}: {e}") from e
        self._pos = 0
        try:
            self._parse()
        except (struct.error, IndexError, UnicodeDecodeError) as e:
            self.close()
            raise GgufError(f"{path}: truncated or malformed GGUF ({e})") from e

    def close(self):
        if self.buf is not None:
            self.buf.close()
            self.buf = None
            self._f.close()

    def _take(self, n: int) -> bytes:
        if self._pos + n > len(self.buf):
            raise GgufError("truncated GGUF")
        b = self.buf[self._pos:self._pos + n]
        self._pos += n
        return b

    def _u(self, n: int) -> int:
        return int.from_bytes(self._take(n), "little")

    def _str(self) -> str:
        return self._take(self._u(8)).decode("utf-8")

    def _value(self, vtype: int):
        # 0 u8, 1 i8, 2 u16, 3 i16, 4 u32, 5 i32, 6 f32, 7 bool, 8 string, 9 array,
        # 10 u64, 11 i64, 12 f64 (lib.rs:1665-1709: integers read as unsigned little-endian)
        if vtype in (0, 1, 7):
            return self._u(1)
        if vtype in (2, 3):
            return self._u(2)
        if vtype in (4, 5):
            return self._u(4)
        if vtype in (10, 11):
            return self._u(8)
        if vtype == 6:
            return struct.unpack("<f", self._take(4))[0]
        if vtype == 12:
            return float(np.float32(struct.unpack("<d", self._take(8))[0]))
        if vtype == 8:
            return self._str()
        if vtype == 9:
            et, count = self._u(4), self._u(8)
            return [self._value(et) for _ in range(count)]
        raise GgufError(f"unknown metadata type {vtype}")

    def _parse(self):
        if self._take(4) != b"GGUF":
            raise GgufError("bad GGUF magic")
        version = self._u(4)
        if version < 2:
            raise GgufError(f"GGUF version {version} not supported")
        n_tensors, n_kv = self._u(8), self._u(8)
        self.meta = {}
        for _ in range(n_kv):
            key = self._str()
            self.meta[key] = self._value(self._u(4))
        self.tensors = {}
        for _ in range(n_tensors):
            name = self._str()
            dims = [self._u(8) for _ in range(self._u(4))]
            self.tensors[name] = (dims, self._u(4), self._u(8))
        a = self.meta.get("general.alignment")
        align = a if isinstance(a, int) and a > 0 and (a & (a - 1)) == 0 else 32
        self.data_offset = (self._pos + align - 1) // align * align

    def raw(self, name: str, nbytes: int) -> np.ndarray:
        dims, _, off = self.tensors[name]
        start = self.data_offset + off
        if start + nbytes > len(self.buf):
            raise GgufError(f"{name}: data beyond the end of the file")
        return np.frombuffer(self.buf, dtype=np.uint8, count=nbytes, offset=start)


def _f16_to_f32(b: np.ndarray) -> np.ndarray:
    """f16.rs:40-60 (IEEE half -> single, exact, subnormals / inf / NaN included)."""
    return b.view(np.float16).astype(np.float32)


def dequant_q6_k(raw: np.ndarray, nblocks: int) -> np.ndarray:
    """dequant_q6_k_block (lib.rs:1639-1661) over nblocks 210-byte blocks: per half n,
    y[l + 32k] = (d * sc[is + 2k]) * q, q = 6-bit code - 32, in f32 in that order."""
    b = raw.reshape(nblocks, 210)
    ql, qh = b[:, :128].reshape(nblocks, 2, 64), b[:, 128:192].reshape(nblocks, 2, 32)
    sc = b[:, 192:208].view(np.int8).astype(np.float32).reshape(nblocks, 2, 8)
    d = _f16_to_f32(np.ascontiguousarray(b[:, 208:210])).reshape(nblocks, 1, 1)
    lo, hi = ql[:, :, :32], ql[:, :, 32:]
    q = np.stack([(lo & 15) | ((qh & 3) << 4), (hi & 15) | (((qh >> 2) & 3) << 4),
                  (lo >> 4) | (((qh >> 4) & 3) << 4), (hi >> 4) | (((qh >> 6) & 3) << 4)], axis=2)
    q = q.astype(np.int32) - 32  # [block, half, k, l]
    is_ = (np.arange(32) // 16)[None, None, None, :] + 2 * np.arange(4)[None, None, :, None]
    s = np.take_along_axis(sc[:, :, None, :].repeat(4, axis=2), np.broadcast_to(is_, (nblocks, 2, 4, 32)), axis=3)
    y = (d[..., None] * s).astype(np.float32) * q.astype(np.float32)
    return y.astype(np.float32).reshape(nblocks * 256)


def dequant_q5_0(raw: np.ndarray, nblocks: int) -> np.ndarray:
    """dequant_q5_0_block (lib.rs:1624-1637): (q - 16) * d, q = nibble + bit j (+16) of qh."""
    b = raw.reshape(nblocks, 22)
    d = _f16_to_f32(np.ascontiguousarray(b[:, 0:2])).reshape(nblocks, 1)
    qh = b[:, 2:6].copy().view("<u4").reshape(nblocks, 1).astype(np.uint32)
    qs = b[:, 6:22].astype(np.int32)
    j = np.arange(16, dtype=np.uint32)
    x0 = (qs & 15) | (((qh >> j) & 1).astype(np.int32) << 4)
    x1 = (qs >> 4) | (((qh >> (j + 16)) & 1).astype(np.int32) << 4)
    out = np.concatenate([(x0 - 16).astype(np.float32) * d, (x1 - 16).astype(np.float32) * d], axis=1)
    return out.astype(np.float32).reshape(nblocks * 32)


def quantize_q8_0(src: np.ndarray) -> np.ndarray:
    """quantize_q8_0 (crates/soso-llm-core/src/quant.rs:8-25): blocks of 32 (the last padded
    with zeros), scale = max|v| / 127 (1 for an all-zero block) in f32, codes
    roundf(v / scale) (half away from zero) clamped to [-127, 127]; .som Q8_0 blocks."""
    src = np.asarray(src, np.float32).ravel()
    nb = (src.size + 31) // 32
    v = np.zeros(nb * 32, np.float32)
    v[:src.size] = src
    v = v.reshape(nb, 32)
    mx = np.abs(v).max(axis=1)
    scale = np.where(mx > 0, (mx / np.float32(127.0)).astype(np.float32), np.float32(1.0)).astype(np.float32)
    r = (v / scale[:, None]).astype(np.float32).astype(np.float64)
    q = np.clip(np.sign(r) * np.floor(np.abs(r) + 0.5), -127, 127).astype(np.int8)
    out = np.empty((nb, 36), np.uint8)
    out[:, :4] = scale.view(np.uint8).reshape(nb, 4)
    out[:, 4:] = q.view(np.uint8)
    return out.reshape(-1)


def convert_tensor(gtype: int, raw: np.ndarray, elems: int, keep_q6k: bool = False) -> tuple[np.ndarray, int]:
    """read_tensor (lib.rs:1507-1624): the .som payload and dtype of a GGUF tensor's bytes."""
    if gtype == GGML_F32:
        return np.asarray(raw[:elems * 4]).copy(), DTYPE_F32
    if gtype == GGML_F16:
        return _f16_to_f32(np.ascontiguousarray(raw[:elems * 2])).view(np.uint8).copy(), DTYPE_F32
    if gtype == GGML_Q8_0:
        if elems % 32:
            raise GgufError(f"Q8_0 tensor of {elems} elements (not a multiple of 32)")
        nb = elems // 32
        b = np.asarray(raw[:nb * 34]).reshape(nb, 34)
        out = np.empty((nb, 36), np.uint8)
        out[:, :4] = _f16_to_f32(np.ascontiguousarray(b[:, :2])).view(np.uint8).reshape(nb, 4)
        out[:, 4:] = b[:, 2:]
        return out.reshape(-1), DTYPE_Q8_0
    if gtype == GGML_Q5_0:
        if elems % 32:
            raise GgufError(f"Q5_0 tensor of {elems} elements (not a multiple of 32)")
        return quantize_q8_0(dequant_q5_0(np.asarray(raw[:elems // 32 * 22]), elems // 32)), DTYPE_Q8_0
    if gtype == GGML_Q6_K:
        if elems % 256:
            raise GgufError(f"Q6_K tensor of {elems} elements (not a multiple of 256)")
        blocks = np.asarray(raw[:elems // 256 * 210])
        if keep_q6k:
            return blocks.copy(), DTYPE_Q6_K
        return quantize_q8_0(dequant_q6_k(blocks, elems // 256)), DTYPE_Q8_0
    if gtype in _PASS:
        dt, be, bb = _PASS[gtype]
        if elems % be:
            raise GgufError(f"GGML type {gtype} tensor of {elems} elements (not a multiple of {be})")
        return np.asarray(raw[:elems // be * bb]).copy(), dt
    raise GgufError(f"GGML type {gtype} not supported")


def _bytes_of(gtype: int, elems: int) -> int:
    if gtype == GGML_F32:
        return elems * 4
    if gtype == GGML_F16:
        return elems * 2
    per = {GGML_Q8_0: (32, 34), GGML_Q5_0: (32, 22), GGML_Q6_K: (256, 210)}
    per.update({k: (be, bb) for k, (_, be, bb) in _PASS.items()})
    if gtype not in per:
        raise GgufError(f"GGML type {gtype} not supported")
    be, bb = per[gtype]
    return (elems + be - 1) // be * bb


def read_tensor(g: GgufFile, name: str, keep_q6k: bool = False) -> tuple[np.ndarray, int, list]:
    """(payload, .som dtype, shape slowest first) of one GGUF tensor."""
    dims, gtype, _ = g.tensors[name]
    elems = int(np.prod(dims)) if dims else 1
    data, dt = convert_tensor(gtype, g.raw(name, _bytes_of(gtype, elems)), elems, keep_q6k)
    return data, dt, list(reversed(dims))


def _expert_slices(data: np.ndarray, n_exp: int) -> list:
    """slice_expert_3d (lib.rs:1285-1400): expert e's rows are the e-th n_exp-th of the payload."""
    if data.size % n_exp:
        raise GgufError("expert tensor not divisible by its expert count")
    per = data.size // n_exp
    return [data[e * per:(e + 1) * per] for e in range(n_exp)]


def load_gguf_model(path: str, ctx: int | None = None, keep_q6k: bool = False):
    """(DenseConfig, tensors, GgufFile) of a llama / qwen2 / qwen3 / qwen3moe GGUF: the
    tensors are the converted payloads (passthrough blocks copied out of the mapping)."""
    g = GgufFile(path)
    try:
        return _load(g, ctx, keep_q6k) + (g,)
    except BaseException:
        g.close()
        raise


def _load(g: GgufFile, ctx, keep_q6k):
    m = g.meta
    arch = m.get("general.architecture", "llama")
    if arch == "deepseek2":
        raise GgufError("MLA (deepseek2) GGUFs are not mapped here: convert with gguf2som and load the .som")
    if arch not in ("llama", "qwen2", "qwen3", "qwen3moe"):
        raise GgufError(f"architecture {arch} not taken (llama | qwen2 | qwen3 | qwen3moe)")
    qwen3 = arch in ("qwen3", "qwen3moe")
    pre = arch if arch != "llama" else "llama"

    def u32(key, default=None):
        v = m.get(f"{pre}.{key}")
        if isinstance(v, int):
            return v
        if default is None:
            raise GgufError(f"missing metadata {pre}.{key}")
        return default

    def f32(key, default):
        v = m.get(f"{pre}.{key}")
        return float(np.float32(v)) if isinstance(v, (int, float)) else default

    hidden, n_layers = u32("embedding_length"), u32("block_count")
    ffn = m.get(f"{pre}.feed_forward_length")
    ffn = ffn if isinstance(ffn, int) else u32("expert_feed_forward_length")
    heads = u32("attention.head_count")
    kv_heads = u32("attention.head_count_kv", heads)
    theta, eps = f32("rope.freq_base", 10000.0), f32("attention.layer_norm_rms_epsilon", 1e-5)
    tokens = m.get("tokenizer.ggml.tokens")
    vocab = m.get(f"{pre}.vocab_size") if isinstance(m.get(f"{pre}.vocab_size"), int) else \
        (len(tokens) if isinstance(tokens, list) else 256)
    max_seq = u32("context_length", 2048)
    n_exp = u32("expert_count", 0)
    top_k = u32("expert_used_count", 2 if n_exp else 0)
    moe_ffn = u32("expert_feed_forward_length", ffn) if n_exp else 0

    t, dtypes = {}, {}

    def put(dst, src, kind, keep=keep_q6k):
        data, dt, shape = read_tensor(g, src, keep)
        if kind is not None and dtypes.setdefault(kind, dt) != dt:
            raise GgufError(f"{src}: dtype {dt}, other {kind} tensors {dtypes[kind]}")
        t[dst] = data  # matrices as their bytes, whatever the dtype (f32 routers included)
        return shape

    def vec(dst, src):
        data, dt, _ = read_tensor(g, src)
        if dt != DTYPE_F32:
            raise GgufError(f"{src}: a vector stored as dtype {dt}")
        t[dst] = data.view(np.float32)

    q_shape = g.tensors.get("blk.0.attn_q.weight")
    if q_shape is None:
        raise GgufError("missing blk.0.attn_q.weight")
    head_dim = (u32("attention.key_length", 0) if qwen3 else 0) or q_shape[0][1] // heads
    moe_layers = [l for l in range(n_layers) if f"blk.{l}.ffn_gate_inp.weight" in g.tensors]
    first_moe = moe_layers[0] if moe_layers else 0
    if moe_layers and moe_layers != list(range(first_moe, n_layers)):
        raise GgufError("dense FFN layers after MoE layers")
    shared_ffn = 0
    for l in range(n_layers):
        p = f"blk.{l}."
        for n in ("attn_q", "attn_k", "attn_v", "attn_output"):
            put(p + n, p + n + ".weight", n)
        vec(p + "attn_norm", p + "attn_norm.weight")
        vec(p + "ffn_norm", p + "ffn_norm.weight")
        if arch == "qwen2" and p + "attn_q.bias" in g.tensors:
            parts = []
            for n in ("attn_q", "attn_k", "attn_v"):
                vec("_b", p + n + ".bias")
                parts.append(t.pop("_b"))
            t[p + "qkv_bias"] = np.concatenate(parts)
        if p + "attn_q_norm.weight" in g.tensors:
            vec(p + "attn_q_norm", p + "attn_q_norm.weight")
            vec(p + "attn_k_norm", p + "attn_k_norm.weight")
        if l not in moe_layers:
            for n in ("ffn_gate", "ffn_up", "ffn_down"):
                put(p + n, p + n + ".weight", n)
            continue
        data, dt, _ = read_tensor(g, p + "ffn_gate_inp.weight", keep_q6k)
        if dtypes.setdefault("ffn_gate_inp", dt) != dt:
            raise GgufError(f"{p}ffn_gate_inp: dtype {dt}")
        t[p + "ffn_gate_inp"] = data
        for n in ("ffn_gate", "ffn_up", "ffn_down"):
            fused = p + n + "_exps.weight"
            if fused in g.tensors:
                data, dt, shape = read_tensor(g, fused, keep_q6k)
                if len(shape) != 3 or shape[0] != n_exp:
                    raise GgufError(f"{fused}: shape {shape}, want {n_exp} experts")
                pieces = _expert_slices(data, n_exp)
            else:  # the older layout: one 2-D tensor per expert
                pieces, dt = [], None
                for e in range(n_exp):
                    d_, dt_, _ = read_tensor(g, f"{p}{n}.{e}.weight", keep_q6k)
                    pieces.append(d_)
                    if dt is not None and dt_ != dt:
                        raise GgufError(f"{p}{n}.{e}: dtype {dt_}")
                    dt = dt_
            if dtypes.setdefault(n, dt) != dt:
                raise GgufError(f"{p}{n} experts: dtype {dt}, other {n} tensors {dtypes[n]}")
            for e, piece in enumerate(pieces):
                t[f"{p}E{e:03d}.{n}"] = piece
        if p + "ffn_gate_shexp.weight" in g.tensors:
            for n in ("ffn_gate", "ffn_up", "ffn_down"):
                shape = put(f"{p}S00.{n}", f"{p}{n}_shexp.weight", n)
                if n == "ffn_gate":
                    shared_ffn = shape[0]
            if p + "ffn_gate_inp_shexp.weight" in g.tensors:
                vec(p + "ffn_gate_inp_shexp", p + "ffn_gate_inp_shexp.weight")
    vec("output_norm", "output_norm.weight")
    put("token_embd", "token_embd.weight", "token_embd")
    put("output", "output.weight" if "output.weight" in g.tensors else "token_embd.weight", "output")
    kw = dict(n_layers=n_layers, hidden=hidden, heads=heads, kv_heads=kv_heads, head_dim=head_dim,
              ffn=ffn if len(moe_layers) < n_layers else 0, vocab=vocab, ctx=ctx or max_seq, theta=theta, eps=eps,
              neox=arch != "llama", qkv_bias=any(k.endswith("qkv_bias") for k in t),
              qk_norm=any(k.endswith("attn_q_norm") for k in t), dtypes=dtypes)
    if moe_layers:
        kw.update(n_exp=n_exp, top_k=top_k, moe_ffn=moe_ffn, first_moe=first_moe, shared_ffn=shared_ffn,
                  shared_gate=any(k.endswith("ffn_gate_inp_shexp") for k in t))
    return DenseConfig(**kw), t


__all__ = ["GgufFile", "GgufError", "convert_tensor", "quantize_q8_0", "dequant_q6_k", "dequant_q5_0",
           "read_tensor", "load_gguf_model"]
