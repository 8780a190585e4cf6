"""A GGUF writer for tests (GGUF v3, as the reference's converter tests build theirs:
crates/gguf2som/src/lib.rs tests, gguf_string / gguf_kv_*): metadata, tensor infos with
GGML dims fastest first, data aligned to 32 bytes."""
import struct

import numpy as np

from soso_b200 import gguf
from soso_b200.formats import DTYPE_F32, DTYPE_Q4_K, DTYPE_Q6_K, DTYPE_Q8_0


def _s(b: bytearray, s: str):
    e = s.encode()
    b += struct.pack("<Q", len(e)) + e


def _kv(b: bytearray, key: str, v):
    _s(b, key)
    if isinstance(v, bool):
        b += struct.pack("<IB", 7, int(v))
    elif isinstance(v, int):
        b += struct.pack("<II", 4, v)
    elif isinstance(v, float):
        b += struct.pack("<If", 6, v)
    elif isinstance(v, str):
        b += struct.pack("<I", 8)
        _s(b, v)
    elif isinstance(v, list) and all(isinstance(x, str) for x in v):
        b += struct.pack("<IIQ", 9, 8, len(v))
        for x in v:
            _s(b, x)
    else:
        raise TypeError(key)


def write_gguf(path, meta: dict, tensors: list):
    """tensors: (name, ggml type, dims fastest first, payload bytes)."""
    b = bytearray(b"GGUF") + struct.pack("<IQQ", 3, len(tensors), len(meta))
    for k, v in meta.items():
        _kv(b, k, v)
    off, blobs = 0, []
    for name, gt, dims, data in tensors:
        _s(b, name)
        b += struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims)
        b += struct.pack("<IQ", gt, off)
        data = bytes(data)
        blobs.append(data + b"\0" * ((-len(data)) % 32))
        off += len(blobs[-1])
    b += b"\0" * ((-len(b)) % 32)
    with open(path, "wb") as f:
        f.write(bytes(b) + b"".join(blobs))


def _ggml(dt: int, data: np.ndarray):
    """A .som payload of the synthetic model as the GGML tensor gguf2som reads it back from."""
    data = np.ascontiguousarray(data).view(np.uint8).reshape(-1)
    if dt == DTYPE_F32:
        return gguf.GGML_F32, data
    if dt == DTYPE_Q4_K:
        return gguf.GGML_Q4_K, data
    if dt == DTYPE_Q6_K:
        return gguf.GGML_Q6_K, data
    if dt == DTYPE_Q8_0:  # f32 scales (f16-exact in the synthetic models) -> f16
        b = data.reshape(-1, 36)
        out = np.empty((b.shape[0], 34), np.uint8)
        out[:, :2] = b[:, :4].copy().view(np.float32).astype(np.float16).view(np.uint8).reshape(-1, 2)
        out[:, 2:] = b[:, 4:]
        return gguf.GGML_Q8_0, out.reshape(-1)
    raise ValueError(dt)


def model_to_gguf(path, cfg, model, arch: str):
    """The synthetic decode model (decode.synth_model) as a GGUF of `arch`: experts stacked
    into ffn_*_exps, the q|k|v bias split into attn_*.bias."""
    pre = arch
    meta = {"general.architecture": arch, f"{pre}.embedding_length": cfg.hidden,
            f"{pre}.block_count": cfg.n_layers, f"{pre}.attention.head_count": cfg.heads,
            f"{pre}.attention.head_count_kv": cfg.kv_heads, f"{pre}.rope.freq_base": float(cfg.theta),
            f"{pre}.attention.layer_norm_rms_epsilon": float(cfg.eps), f"{pre}.context_length": cfg.ctx,
            f"{pre}.vocab_size": cfg.vocab}
    if cfg.ffn:
        meta[f"{pre}.feed_forward_length"] = cfg.ffn
    if arch in ("qwen3", "qwen3moe"):
        meta[f"{pre}.attention.key_length"] = cfg.head_dim
    if cfg.n_exp:
        meta.update({f"{pre}.expert_count": cfg.n_exp, f"{pre}.expert_used_count": cfg.top_k,
                     f"{pre}.expert_feed_forward_length": cfg.moe_ffn})
        if not cfg.ffn:
            meta[f"{pre}.feed_forward_length"] = cfg.moe_ffn
    H = cfg.hidden
    ts = []

    def mat(name, key, rows, cols, kind):
        gt, data = _ggml(cfg.dtypes[kind], model[key])
        ts.append((name + ".weight", gt, [cols, rows], data))

    def vec(name, arr):
        a = np.asarray(arr, np.float32)
        ts.append((name, gguf.GGML_F32, [a.size], a.view(np.uint8)))

    for l in range(cfg.n_layers):
        p = f"blk.{l}."
        mat(p + "attn_q", p + "attn_q", cfg.q_dim, H, "attn_q")
        mat(p + "attn_k", p + "attn_k", cfg.kv_dim, H, "attn_k")
        mat(p + "attn_v", p + "attn_v", cfg.kv_dim, H, "attn_v")
        mat(p + "attn_output", p + "attn_output", H, cfg.q_dim, "attn_output")
        vec(p + "attn_norm.weight", model[p + "attn_norm"])
        vec(p + "ffn_norm.weight", model[p + "ffn_norm"])
        if p + "qkv_bias" in model:
            b = np.asarray(model[p + "qkv_bias"], np.float32)
            vec(p + "attn_q.bias", b[:cfg.q_dim])
            vec(p + "attn_k.bias", b[cfg.q_dim:cfg.q_dim + cfg.kv_dim])
            vec(p + "attn_v.bias", b[cfg.q_dim + cfg.kv_dim:])
        if p + "attn_q_norm" in model:
            vec(p + "attn_q_norm.weight", model[p + "attn_q_norm"])
            vec(p + "attn_k_norm.weight", model[p + "attn_k_norm"])
        if not cfg.is_moe(l):
            mat(p + "ffn_gate", p + "ffn_gate", cfg.ffn, H, "ffn_gate")
            mat(p + "ffn_up", p + "ffn_up", cfg.ffn, H, "ffn_up")
            mat(p + "ffn_down", p + "ffn_down", H, cfg.ffn, "ffn_down")
            continue
        mat(p + "ffn_gate_inp", p + "ffn_gate_inp", cfg.n_exp, H, "ffn_gate_inp")
        for kind, rows, cols in (("ffn_gate", cfg.moe_ffn, H), ("ffn_up", cfg.moe_ffn, H), ("ffn_down", H, cfg.moe_ffn)):
            parts = [_ggml(cfg.dtypes[kind], model[f"{p}E{e:03d}.{kind}"]) for e in range(cfg.n_exp)]
            ts.append((f"{p}{kind}_exps.weight", parts[0][0], [cols, rows, cfg.n_exp],
                       np.concatenate([d for _, d in parts])))
    vec("output_norm.weight", model["output_norm"])
    mat("token_embd", "token_embd", cfg.vocab, H, "token_embd")
    mat("output", "output", cfg.vocab, H, "output")
    write_gguf(path, meta, ts)
