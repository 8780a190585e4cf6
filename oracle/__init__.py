"""CPU oracle for the quantized decode hot path -- TEST INFRASTRUCTURE ONLY.

This package is the checker, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / ``--impl reference``
legs import it.  ``soso_b200`` (the product) never imports it and has no CPU
fallback.

The C restatement lives in ``oracle.c`` (block decoders, scalar matvecs in the
reference's operation order, quantizers) and ``cpu_baseline.c`` (the
reference's AVX2 kernels, threaded with ``row_strip``); ``ops.py`` restates the
float ops (RMSNorm, RoPE, softmax/top-k, SwiGLU, attention, MoE, MLA, layer
forward).  Each function cites the reference file:line it follows.

Parity pins: ``tests/test_oracle_golden.py`` checks this oracle against the
reference's golden vectors (crates/sosomodel/tests/dequant_golden.rs,
crates/gguf2som/src/lib.rs:1866-1889) and against the reference's own C decoder
``lxdde/ports/nouveau/q4k_decode.h`` compiled into ``oracle/_ref/``.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")
REF_PATH = os.path.join(HERE, "_ref", "libq4kref.so")

F32, Q8_0, Q4_K, Q6_K = 1, 2, 3, 13
BLOCK = {Q8_0: (32, 36), Q4_K: (256, 144), Q6_K: (256, 210)}

_lib = None
_ref = None

_u8p = ctypes.POINTER(ctypes.c_uint8)
_f32p = ctypes.POINTER(ctypes.c_float)
_f64p = ctypes.POINTER(ctypes.c_double)


def build(force: bool = False) -> None:
    """Compile liboracle.so (and _ref/ when the reference checkout exists)."""
    if force or not os.path.exists(LIB_PATH):
        subprocess.run(["make", "-s", "-C", HERE], check=True)


def lib():
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(LIB_PATH)
        L.or_f16_to_f32.restype = ctypes.c_float
        L.or_f16_to_f32.argtypes = [ctypes.c_uint16]
        L.or_f32_to_f16.restype = ctypes.c_uint16
        L.or_f32_to_f16.argtypes = [ctypes.c_float]
        L.or_row_bytes.restype = ctypes.c_size_t
        L.or_row_bytes.argtypes = [ctypes.c_uint8, ctypes.c_size_t]
        L.or_q4k_scale_min.argtypes = [_u8p, ctypes.c_int, _u8p, _u8p]
        L.or_q4k_dot_sub.restype = ctypes.c_float
        L.or_q4k_dot_sub.argtypes = [_u8p, ctypes.c_int, _f32p]
        L.or_q4k_dot_ref.restype = ctypes.c_float
        L.or_q4k_dot_ref.argtypes = [_u8p, _f32p]
        for n in ("or_dequant_q8_0", "or_dequant_q4_k", "or_dequant_q6_k"):
            f = getattr(L, n)
            f.restype = ctypes.c_int
            f.argtypes = [_u8p, ctypes.c_size_t, _f32p, ctypes.c_size_t]
        L.or_dequant.restype = ctypes.c_int
        L.or_dequant.argtypes = [ctypes.c_uint8, _u8p, ctypes.c_size_t, _f32p, ctypes.c_size_t]
        L.or_matvec.restype = ctypes.c_int
        L.or_matvec.argtypes = [ctypes.c_uint8, _u8p, ctypes.c_size_t, ctypes.c_size_t, _f32p, _f32p]
        L.or_matvec_f64.restype = ctypes.c_int
        L.or_matvec_f64.argtypes = [ctypes.c_uint8, _u8p, ctypes.c_size_t, ctypes.c_size_t, _f32p,
                                    ctypes.c_size_t, _f64p]
        L.or_cpu_matvec.restype = ctypes.c_int
        L.or_cpu_matvec.argtypes = [ctypes.c_uint8, _u8p, ctypes.c_size_t, ctypes.c_size_t, _f32p, _f32p,
                                    ctypes.c_int]
        for n in ("or_quantize_q8_0", "or_quantize_q4_k", "or_quantize_q6_k"):
            f = getattr(L, n)
            f.restype = None
            f.argtypes = [_f32p, ctypes.c_size_t, _u8p]
        L.or_dequant_q6_k_block.argtypes = [_u8p, _f32p]
        L.or_row_strip.argtypes = [ctypes.c_size_t] * 3 + [ctypes.POINTER(ctypes.c_size_t)] * 2
        _lib = L
    return _lib


def ref_lib():
    """The reference's own q4k_decode.h, compiled from source; None if absent."""
    global _ref
    if _ref is None and os.path.exists(REF_PATH):
        R = ctypes.CDLL(REF_PATH)
        R.ref_q4k_f16.restype = ctypes.c_float
        R.ref_q4k_f16.argtypes = [ctypes.c_ushort]
        R.ref_q4k_scale_min.argtypes = [_u8p, ctypes.c_int, _u8p, _u8p]
        R.ref_q4k_dot_sub.restype = ctypes.c_float
        R.ref_q4k_dot_sub.argtypes = [_u8p, ctypes.c_int, _f32p]
        R.ref_q4k_dot_block.restype = ctypes.c_float
        R.ref_q4k_dot_block.argtypes = [_u8p, _f32p]
        R.ref_q80_dot_block.restype = ctypes.c_float
        R.ref_q80_dot_block.argtypes = [_u8p, _f32p]
        _ref = R
    return _ref


def _u8(a: np.ndarray):
    a = np.ascontiguousarray(a, dtype=np.uint8)
    return a, a.ctypes.data_as(_u8p)


def _f32(a: np.ndarray):
    a = np.ascontiguousarray(a, dtype=np.float32)
    return a, a.ctypes.data_as(_f32p)


def f16_to_f32(bits: int) -> float:
    return lib().or_f16_to_f32(bits)


def f32_to_f16(v: float) -> int:
    return lib().or_f32_to_f16(v)


def row_bytes(dtype: int, cols: int) -> int | None:
    rb = lib().or_row_bytes(dtype, cols)
    return rb or None


def q4k_scale_min(scales: bytes, j: int) -> tuple[int, int]:
    s, p = _u8(np.frombuffer(bytes(scales), dtype=np.uint8))
    sc, m = ctypes.c_uint8(), ctypes.c_uint8()
    lib().or_q4k_scale_min(p, j, ctypes.byref(sc), ctypes.byref(m))
    return sc.value, m.value


def q4k_dot_ref(blk: np.ndarray, x: np.ndarray) -> float:
    b, bp = _u8(blk)
    xx, xp = _f32(x)
    return lib().or_q4k_dot_ref(bp, xp)


def dequant(dtype: int, w: np.ndarray, n: int) -> np.ndarray:
    b, bp = _u8(w)
    out = np.empty(n, dtype=np.float32)
    rc = lib().or_dequant(dtype, bp, b.size, out.ctypes.data_as(_f32p), n)
    if rc:
        raise ValueError(f"dequant rc={rc}")
    return out


def matvec(dtype: int, w: np.ndarray, rows: int, cols: int, x: np.ndarray) -> np.ndarray:
    """Reference-order f32 matvec (gemm.rs scalar kernels)."""
    b, bp = _u8(w)
    xx, xp = _f32(x)
    out = np.empty(rows, dtype=np.float32)
    rc = lib().or_matvec(dtype, bp, rows, cols, xp, out.ctypes.data_as(_f32p))
    if rc:
        raise ValueError(f"matvec rc={rc}")
    return out


def matvec_f64(dtype: int, w: np.ndarray, rows: int, cols: int, x: np.ndarray, n: int = 1) -> np.ndarray:
    """Exact-dequant, f64-accumulated truth; x is n vectors of cols, out n x rows."""
    b, bp = _u8(w)
    xx, xp = _f32(x)
    out = np.empty(n * rows, dtype=np.float64)
    rc = lib().or_matvec_f64(dtype, bp, rows, cols, xp, n, out.ctypes.data_as(_f64p))
    if rc:
        raise ValueError(f"matvec_f64 rc={rc}")
    return out


def cpu_matvec(dtype: int, w: np.ndarray, rows: int, cols: int, x: np.ndarray, threads: int = 1,
               out: np.ndarray | None = None) -> np.ndarray:
    """The reference's AVX2 kernels (gemm.rs:806-894), row_strip-threaded."""
    b, bp = _u8(w)
    xx, xp = _f32(x)
    if out is None:
        out = np.empty(rows, dtype=np.float32)
    rc = lib().or_cpu_matvec(dtype, bp, rows, cols, xp, out.ctypes.data_as(_f32p), threads)
    if rc:
        raise ValueError(f"cpu_matvec rc={rc}")
    return out


def quantize(dtype: int, v: np.ndarray) -> np.ndarray:
    v, vp = _f32(v)
    be, bb = BLOCK[dtype]
    nb = (v.size + be - 1) // be
    out = np.zeros(nb * bb, dtype=np.uint8)
    fn = {Q8_0: lib().or_quantize_q8_0, Q4_K: lib().or_quantize_q4_k, Q6_K: lib().or_quantize_q6_k}[dtype]
    fn(vp, v.size, out.ctypes.data_as(_u8p))
    return out


def row_strip(rows: int, i: int, n: int) -> tuple[int, int]:
    s, e = ctypes.c_size_t(), ctypes.c_size_t()
    lib().or_row_strip(rows, i, n, ctypes.byref(s), ctypes.byref(e))
    return s.value, e.value


# ---------------------------------------------------------------- float ops
def _ops_lib():
    L = lib()
    if not getattr(L, "_ops_ready", False):
        L.or_rmsnorm.argtypes = [_f32p, ctypes.c_size_t, ctypes.c_size_t, ctypes.c_float]
        L.or_rmsnorm.argtypes = [_f32p, _f32p, ctypes.c_size_t, ctypes.c_float]
        L.or_rope_heads.argtypes = [_f32p, ctypes.c_size_t, ctypes.c_size_t, ctypes.c_size_t, ctypes.c_float,
                                    ctypes.c_int]
        L.or_rope_llama_n.argtypes = [_f32p, ctypes.c_size_t, ctypes.c_float, ctypes.c_size_t]
        L.or_topk_softmax.argtypes = [_f32p, ctypes.c_size_t, ctypes.c_size_t, ctypes.POINTER(ctypes.c_int32), _f32p]
        L.or_swiglu.argtypes = [_f32p, _f32p, ctypes.c_size_t]
        _u16p = ctypes.POINTER(ctypes.c_uint16)
        L.or_attention_decode_f16.argtypes = [_f32p, _u16p, _u16p, ctypes.c_size_t, ctypes.c_size_t,
                                              ctypes.c_size_t, ctypes.c_size_t, _f32p]
        L.or_argmax.restype = ctypes.c_int32
        L.or_argmax.argtypes = [_f32p, ctypes.c_size_t]
        L._ops_ready = True
    return L


def rmsnorm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    """gemm.rs:93-100; returns a new array."""
    y = np.array(x, dtype=np.float32, copy=True)
    ww, wp = _f32(w)
    _ops_lib().or_rmsnorm(y.ctypes.data_as(_f32p), wp, y.size, eps)
    return y


def rope_heads(x: np.ndarray, n_heads: int, hd: int, pos: int, theta: float, neox: bool) -> np.ndarray:
    """gemm.rs:1452-1491 (rope_cabezas)."""
    y = np.array(x, dtype=np.float32, copy=True)
    _ops_lib().or_rope_heads(y.ctypes.data_as(_f32p), n_heads, hd, pos, theta, 1 if neox else 0)
    return y


def rope_llama_n(x: np.ndarray, pos: int, theta: float, n_rot: int) -> np.ndarray:
    y = np.array(x, dtype=np.float32, copy=True)
    _ops_lib().or_rope_llama_n(y.ctypes.data_as(_f32p), pos, theta, n_rot)
    return y


# ---- YaRN RoPE (f32 throughout, as the reference).  Parity unpinned: the reference's
# tests hold no YaRN values; the two forms below are checked against each other, which is
# the reference's own claim (yarn_factores "reproduces rope_neox_yarn", gemm.rs:1412-1413).
_F = np.float32


def _yarn_corr_dims(n_dims: int, orig_ctx: int, theta: float, beta_fast: float, beta_slow: float):
    """yarn_corr_dims (crates/soso-llm-core/src/gemm.rs:1430-1441)."""
    def dim(n_rot):
        return _F(n_dims) * np.log(_F(orig_ctx) / (_F(n_rot) * _F(2.0) * _F(np.pi))) / (_F(2.0) * np.log(_F(theta)))
    start = max(np.floor(dim(beta_fast)), _F(0.0))
    end = min(np.ceil(dim(beta_slow)), _F(n_dims - 1))
    return _F(start), _F(end)


def _yarn_ramp(low, high, pair: int):
    """yarn_ramp (gemm.rs:1443-1446)."""
    y = (_F(pair) - low) / max(high - low, _F(0.001))
    return _F(1.0) - _F(min(max(y, _F(0.0)), _F(1.0)))


def yarn_factors(head_dim: int, theta: float, factor: float, orig_ctx: int, beta_fast: float,
                 beta_slow: float) -> tuple[np.ndarray, np.float32]:
    """yarn_factores (gemm.rs:1413-1428): per pair i the divisor of its RoPE frequency,
    1 / (freq_scale (1 - ramp_i) + ramp_i) with freq_scale = 1 / factor, and the magnitude
    mscale = 1 + 0.1 ln(factor) that multiplies cos and sin -- what the reference passes to
    its GPU rope (gm_rope, lxdde/ports/nouveau/gemma_capa.cu:99-125; moe_gpu.rs:182)."""
    low, high = _yarn_corr_dims(head_dim, orig_ctx, theta, beta_fast, beta_slow)
    fs = _F(1.0) / _F(factor)
    f = np.array([_F(1.0) / (fs * (_F(1.0) - _yarn_ramp(low, high, i)) + _yarn_ramp(low, high, i))
                  for i in range(head_dim // 2)], dtype=np.float32)
    return f, _F(_F(1.0) + _F(0.1) * np.log(_F(factor)))


def rope_neox_yarn(x: np.ndarray, n_heads: int, hd: int, pos: int, theta: float, factor: float, orig_ctx: int,
                   beta_fast: float, beta_slow: float) -> np.ndarray:
    """rope_neox_yarn (gemm.rs:1372-1410), the reference's CPU YaRN: per pair the angle
    blends interpolation (pos theta^(-2i/d) / factor) and extrapolation by the ramp, the
    angle advancing by repeated multiplication; cos and sin scaled by mscale; NeoX pairs
    (i, i + d/2) of every head.  Does nothing when YaRN is inactive (factor <= 1)."""
    y = np.array(x, dtype=np.float32, copy=True)
    if hd < 2 or n_heads == 0 or not (factor > 1.0 and orig_ctx > 0):
        return y
    half = hd // 2
    fs = _F(1.0) / _F(factor)
    low, high = _yarn_corr_dims(hd, orig_ctx, theta, beta_fast, beta_slow)
    theta_scale = np.power(_F(theta), _F(-2.0) / _F(hd))
    mscale = _F(_F(1.0) + _F(0.1) * np.log(_F(factor)))
    cs, sn = np.empty(half, np.float32), np.empty(half, np.float32)
    ang = _F(pos)
    for i in range(half):
        mix = _yarn_ramp(low, high, i)
        ext = ang
        a = (fs * ext) * (_F(1.0) - mix) + ext * mix
        cs[i], sn[i] = np.cos(_F(a)) * mscale, np.sin(_F(a)) * mscale
        ang = _F(ang * theta_scale)
    for h in range(n_heads):
        v = y[h * hd:(h + 1) * hd]
        a0, b0 = v[:half].copy(), v[half:].copy()
        v[:half] = a0 * cs - b0 * sn
        v[half:] = a0 * sn + b0 * cs
    return y


def rope_heads_div(x: np.ndarray, n_heads: int, hd: int, pos: int, theta: float, neox: bool,
                   factors: np.ndarray | None, mscale: float) -> np.ndarray:
    """The reference's GPU rope with per-frequency divisors (gm_rope,
    lxdde/ports/nouveau/gemma_capa.cu:99-125): freq_i = exp(-ln(theta) 2i / d) / factors[i],
    angle pos freq_i, cos and sin times mscale; NeoX pairs (i, i + d/2) or llama pairs
    (2i, 2i + 1)."""
    y = np.array(x, dtype=np.float32, copy=True)
    half = hd // 2
    i = np.arange(half, dtype=np.float32)
    freq = np.exp(-np.log(_F(theta)) * (_F(2.0) * i) / _F(hd)).astype(np.float32)
    if factors is not None:
        freq = (freq / np.asarray(factors, np.float32)).astype(np.float32)
    ang = (_F(pos) * freq).astype(np.float32)
    c, s = (np.cos(ang) * _F(mscale)).astype(np.float32), (np.sin(ang) * _F(mscale)).astype(np.float32)
    e0 = np.arange(half) if neox else 2 * np.arange(half)
    e1 = e0 + half if neox else e0 + 1
    for h in range(n_heads):
        v = y[h * hd:(h + 1) * hd]
        a0, b0 = v[e0].copy(), v[e1].copy()
        v[e0] = a0 * c - b0 * s
        v[e1] = a0 * s + b0 * c
    return y


def topk_softmax(logits: np.ndarray, k: int) -> tuple[np.ndarray, np.ndarray]:
    """gemm.rs:62-91; returns (idx int32[k], weights f32[k]) in rank order."""
    lg = np.array(logits, dtype=np.float32, copy=True)
    idx = np.zeros(k, dtype=np.int32)
    w = np.zeros(k, dtype=np.float32)
    _ops_lib().or_topk_softmax(lg.ctypes.data_as(_f32p), lg.size, k, idx.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)),
                               w.ctypes.data_as(_f32p))
    return idx, w


def swiglu(up: np.ndarray, gate: np.ndarray) -> np.ndarray:
    """gemm.rs:210-226: silu(gate) * up."""
    u = np.array(up, dtype=np.float32, copy=True)
    g, gp = _f32(gate)
    _ops_lib().or_swiglu(u.ctypes.data_as(_f32p), gp, u.size)
    return u


def attention_decode_f16(q: np.ndarray, k16: np.ndarray, v16: np.ndarray, hd: int, kv_dim: int, kv_head: int,
                         n_tokens: int) -> np.ndarray:
    """attn.rs:73-140 over f16 rows [token][kv_dim] (uint16 bit arrays)."""
    qq, qp = _f32(q)
    k = np.ascontiguousarray(k16, dtype=np.uint16)
    v = np.ascontiguousarray(v16, dtype=np.uint16)
    out = np.zeros(hd, dtype=np.float32)
    _u16p = ctypes.POINTER(ctypes.c_uint16)
    _ops_lib().or_attention_decode_f16(qp, k.ctypes.data_as(_u16p), v.ctypes.data_as(_u16p), hd, kv_dim, kv_head,
                                       n_tokens, out.ctypes.data_as(_f32p))
    return out


def argmax(v: np.ndarray) -> int:
    """runtime.rs:2021-2028 (ties -> last index)."""
    vv, vp = _f32(v)
    return int(_ops_lib().or_argmax(vp, vv.size))


def f32_to_f16_array(v: np.ndarray) -> np.ndarray:
    """f16.rs:10-37 elementwise (the reference KV-cache rounding)."""
    L = lib()
    return np.array([L.or_f32_to_f16(float(a)) for a in np.asarray(v, dtype=np.float32).ravel()], dtype=np.uint16)


# ---- .som container writers (test infrastructure: the reference's writers restated, to build
# files the product's reader must accept or reject)
def crc32c_bitwise(data: bytes) -> int:
    """CRC-32C one bit at a time: the published definition of the `crc` crate's CRC_32_ISCSI
    (crc-catalog 2.5.0: reflected poly 0x1EDC6F41, init / xorout 0xFFFFFFFF), which
    sosomodel::crc32c uses (crates/sosomodel/src/lib.rs:30-34)."""
    crc = 0xFFFFFFFF
    for b in bytes(data):
        crc ^= b
        for _ in range(8):
            crc = (crc >> 1) ^ (0x82F63B78 if crc & 1 else 0)
    return crc ^ 0xFFFFFFFF


def pack_som(body: bytes, version: int, align: int) -> bytes:
    """pack_som (lib.rs:72-85): magic, CRC-32C of body, version, u64 length, body, zeros to align."""
    out = b"SOMODL01" + crc32c_bitwise(body).to_bytes(4, "little") + version.to_bytes(4, "little") + \
        len(body).to_bytes(8, "little") + bytes(body)
    return out + bytes(-len(out) % align)


def pack_shard(data: bytes) -> bytes:
    """pack_shard (index.rs:97-115): version-2 header, payload at byte 64, zeros to 4096."""
    head = b"SOMODL01" + crc32c_bitwise(data).to_bytes(4, "little") + (2).to_bytes(4, "little") + \
        len(data).to_bytes(8, "little")
    out = head + bytes(64 - len(head)) + bytes(data)
    return out + bytes(-len(out) % 4096)


def serialize_index(entries) -> bytes:
    """TensorIndex::serialize (index.rs:37-58); entries: (id, name, shard, offset, byte_len,
    shape, dtype, quant) tuples."""
    body = len(entries).to_bytes(4, "little")
    for tid, name, shard, offset, byte_len, shape, dtype, quant in entries:
        body += tid.to_bytes(4, "little") + name.encode() + b"\0" + shard.encode() + b"\0"
        body += offset.to_bytes(8, "little") + byte_len.to_bytes(8, "little") + len(shape).to_bytes(4, "little")
        body += b"".join(int(d).to_bytes(4, "little") for d in shape) + bytes([dtype, quant, 0, 0])
    return pack_som(body, 1, 64)


def serialize_manifest_prefix(version: int, core: tuple, layers, prefetch, chat_template: str = "") -> bytes:
    """Manifest::serialize up to the chat template (the mirror of Manifest::parse,
    crates/sosomodel/src/manifest.rs:1021-1080), as a version-`version` .som file (4 <= version
    <= 5): core = (name, vocab, hidden, n_layers, heads, ffn, max_seq, kv_heads, theta, eps,
    n_experts, experts_per_tok, moe_ffn); layers = (attn kind, ffn kind, 13 u32) tuples;
    prefetch = (layer, [shard names]) pairs."""
    import struct
    name, vocab, hidden, n_layers, heads, ffn, max_seq, kvh, theta, eps, ne, ept, mf = core
    body = name.encode() + b"\0" + struct.pack("<6I", vocab, hidden, n_layers, heads, ffn, max_seq)
    body += struct.pack("<Iff", kvh, theta, eps) + struct.pack("<3I", ne, ept, mf)
    body += struct.pack("<I", len(layers))
    for a, f, *vals in layers:
        body += bytes([a, f, 0, 0]) + struct.pack("<13I", *vals)
    body += struct.pack("<I", len(prefetch))
    for layer, shards in prefetch:
        body += struct.pack("<II", layer, len(shards)) + b"".join(n.encode() + b"\0" for n in shards)
    if version >= 5:
        body += chat_template.encode() + b"\0"
    return pack_som(body, version, 64)


def serialize_manifest(version: int, core: tuple, layers, prefetch, chat_template: str = "", model_kind: int = 0,
                       norm_kind: int = 0, audio=(0,) * 9, ext=None, kev=None) -> bytes:
    """Manifest::serialize to its end (crates/sosomodel/src/manifest.rs:940-1019), as a
    version-`version` .som file (5 <= version <= 9): the fields of serialize_manifest_prefix,
    then the version-6 block (model kind u8, norm kind u8, u16 pad, nine u32 of AudioSpec),
    the version-7 trailer ext = (embed_scale, logit_softcap, attn_scale, tied, [windows],
    [rope thetas], yarn) with YaRN (factor f32, orig_ctx u32, beta_fast f32, beta_slow f32)
    only from version 8, and the version-9 pointer head kev = (temperature f32, width u32)."""
    import struct
    out = serialize_manifest_prefix(min(version, 5), core, layers, prefetch, chat_template)
    body = bytearray(out[24:24 + int.from_bytes(out[16:24], "little")])
    if version >= 6:
        body += bytes([model_kind, norm_kind, 0, 0]) + struct.pack("<9I", *audio)
    if version >= 7:
        es, cap, sc, tied, window, thetas, yarn = ext or (0.0, 0.0, 0.0, False, (), (), (0.0, 0, 0.0, 0.0))
        body += struct.pack("<fffI", es, cap, sc, int(tied)) + struct.pack("<I", len(window))
        body += b"".join(struct.pack("<I", w) for w in window) + struct.pack("<I", len(thetas))
        body += b"".join(struct.pack("<f", t) for t in thetas)
        if version >= 8:
            body += struct.pack("<fIff", *yarn)
    if version >= 9:
        body += struct.pack("<fI", *kev)
    return pack_som(bytes(body), version, 64)
