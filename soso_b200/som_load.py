"""A decode model from one of the reference's model directories: the ``DenseConfig`` and the
tensor dict that ``decode.DecodeSession`` takes, the matrices as zero-copy views of the
mapped shards.

Names follow the reference's layer code (crates/soso-llm-core/src/layer.rs:973-982,
:1096-1173, :1307, :1510-1518, :1752-1781, :1959-2061): ``L{ll}.attn_q`` .. ``ffn_down``,
``L{ll}.attn_q.bias``, ``attn_q_norm`` / ``attn_k_norm``, ``ffn_gate_inp`` (router),
``E{ee}.ffn_*`` (routed experts), ``S{ss}.ffn_*`` and ``ffn_gate_inp_shexp`` (shared
expert), the MLA projections ``attn_q_down`` .. ``attn_v_up``; ``embed``, ``lm_head``,
``output_norm``.  The layer kinds, widths and flags come from the manifest (version >= 4:
per layer; earlier: the globals).  Taken: GQA or MLA attention on every layer, dense FFN
layers then MoE layers, at most one shared expert; anything else raises SomError.
"""
from __future__ import annotations

import numpy as np

from .decode import DenseConfig
from .formats import DTYPE_F32
from .som import ATTN_KINDS, FFN_KINDS, LayerSpec, SomError, SomModel, parse_manifest

FLAG_ROPE_NEOX, FLAG_QK_NORM = 1 << 3, 1 << 4  # manifest.rs:220-222


def _f32(m: SomModel, name: str) -> np.ndarray:
    e = m.entries[name]
    if e.dtype != DTYPE_F32:
        raise SomError(f"{name}: a vector stored as dtype {e.dtype}, not f32")
    return m.tensor(name).view(np.float32)


def load_decode_model(path: str, ctx: int | None = None, verify: bool = True):
    """(DenseConfig, tensors, SomModel): keep the SomModel open while the tensors are in use
    (they are views of its mapped shards)."""
    m = SomModel(path, verify=verify)
    try:
        return _load(m, path, ctx)
    except BaseException:
        m.close()
        raise


def _load(m: SomModel, path: str, ctx: int | None):
    with open(f"{path}/manifest.som", "rb") as f:
        plan = parse_manifest(f.read())
    c = plan.core
    specs = plan.layers or tuple(LayerSpec("gqa", "moe" if c.n_experts else "dense", *([0] * 13))
                                 for _ in range(c.n_layers))
    kinds = {s.attn for s in specs}
    if len(kinds) != 1 or kinds - {"gqa", "mla"}:
        raise SomError(f"attention kinds {sorted(kinds)}: one of gqa / mla on every layer is taken")
    mla = kinds == {"mla"}
    ffns = [s.ffn for s in specs]
    if set(ffns) - {"dense", "moe"}:
        raise SomError(f"FFN kinds {sorted(set(ffns))}: dense and moe are taken")
    first_moe = ffns.index("moe") if "moe" in ffns else 0
    if "moe" in ffns and "dense" in ffns[first_moe:]:
        raise SomError("dense FFN layers after MoE layers")
    s0 = specs[-1]
    heads = s0.heads or c.heads
    kv_heads = s0.kv_heads or c.kv_heads
    if any((s.heads or c.heads, s.kv_heads or c.kv_heads, s.flags) != (heads, kv_heads, s0.flags) for s in specs):
        raise SomError("layers with different head counts or flags")
    # Manifest::effective_head_dim (manifest.rs:453-465): the layer's v_head_dim when set
    # (Qwen3-style GQA layers, MLA), else hidden / heads
    head_dims = {(s.v_dim or c.hidden // heads) for s in specs}
    if len(head_dims) != 1:
        raise SomError(f"layers with different head widths {sorted(head_dims)}")
    moe = "moe" in ffns
    dense_ffn = {(s.ffn_dim or c.ffn) for s, f in zip(specs, ffns) if f == "dense"}
    if len(dense_ffn) > 1:
        raise SomError(f"dense layers with different FFN widths {sorted(dense_ffn)}")
    moe_specs = [s for s, f in zip(specs, ffns) if f == "moe"]
    widths = {(s.n_experts or c.n_experts, s.experts_per_tok or c.experts_per_tok, s.moe_ffn or c.moe_ffn,
               s.n_shared) for s in moe_specs}
    if len(widths) > 1:
        raise SomError("MoE layers with different expert counts or widths")
    if mla and len({(s.q_rank, s.kv_rank, s.qk_nope, s.qk_rope, s.v_dim) for s in specs}) != 1:
        raise SomError("MLA layers with different ranks or head widths")
    ext = plan.ext
    if ext.embed_scale not in (0.0, 1.0) or ext.logit_softcap != 0.0 or ext.attn_scale != 0.0:
        raise SomError("manifest extensions (embedding scale, logit soft cap, attention scale) are not taken")
    if any(ext.window) or any(t not in (0.0, c.rope_theta) for t in ext.rope_theta):
        raise SomError("per-layer attention windows or RoPE bases are not taken")
    if plan.model_kind != "decoder" or plan.norm_kind != "rms" or plan.kev is not None:
        raise SomError(f"model kind {plan.model_kind} / norm {plan.norm_kind}: a decoder with RMSNorm is taken")
    if ext.yarn_active() and mla:
        raise SomError("YaRN on MLA layers is not taken")
    n_exp = (s0.n_experts or c.n_experts) if moe else 0
    n_shared = s0.n_shared if moe else 0
    if n_shared > 1:
        raise SomError(f"{n_shared} shared experts: one is taken")
    names = set(m.entries)
    L = lambda l, n: f"L{l:02d}.{n}"  # noqa: E731
    shared_ffn = m.entries[L(first_moe, "S00.ffn_gate")].shape[0] if moe and L(first_moe, "S00.ffn_gate") in names \
        else 0

    t, dtypes = {}, {}

    def mat(dst: str, src: str, kind: str):
        e = m.entries.get(src)
        if e is None:
            raise SomError(f"missing tensor {src}")
        if dtypes.setdefault(kind, e.dtype) != e.dtype:
            raise SomError(f"{src}: dtype {e.dtype}, other {kind} tensors {dtypes[kind]}")
        t[dst] = m.tensor(src)

    attn = ("attn_q_down", "attn_q_up", "attn_kv_down", "attn_k_up", "attn_v_up") if mla else \
        ("attn_q", "attn_k", "attn_v")
    for l in range(c.n_layers):
        for n in attn + ("attn_output",):
            mat(f"blk.{l}.{n}", L(l, n), n)
        if ffns[l] == "dense":
            for n in ("ffn_gate", "ffn_up", "ffn_down"):
                mat(f"blk.{l}.{n}", L(l, n), n)
        else:
            mat(f"blk.{l}.ffn_gate_inp", L(l, "ffn_gate_inp"), "ffn_gate_inp")
            for e in range(n_exp):
                for n in ("ffn_gate", "ffn_up", "ffn_down"):
                    mat(f"blk.{l}.E{e:03d}.{n}", L(l, f"E{e:02d}.{n}"), n)
            if shared_ffn:
                for n in ("ffn_gate", "ffn_up", "ffn_down"):
                    mat(f"blk.{l}.S00.{n}", L(l, f"S00.{n}"), n)
                if L(l, "ffn_gate_inp_shexp") in names:
                    t[f"blk.{l}.ffn_gate_inp_shexp"] = _f32(m, L(l, "ffn_gate_inp_shexp"))
        t[f"blk.{l}.attn_norm"] = _f32(m, L(l, "attn_norm"))
        t[f"blk.{l}.ffn_norm"] = _f32(m, L(l, "ffn_norm"))
        if not mla and L(l, "attn_q.bias") in names:
            t[f"blk.{l}.qkv_bias"] = np.concatenate([_f32(m, L(l, f"{n}.bias")) for n in ("attn_q", "attn_k", "attn_v")])
        if L(l, "attn_q_norm") in names:
            t[f"blk.{l}.attn_q_norm"] = _f32(m, L(l, "attn_q_norm"))
            t[f"blk.{l}.attn_k_norm"] = _f32(m, L(l, "attn_k_norm"))
    t["output_norm"] = _f32(m, "output_norm")
    mat("token_embd", "embed", "token_embd")
    mat("output", "lm_head" if "lm_head" in names and not ext.tied_lm_head else "embed", "output")

    head_dim = head_dims.pop()
    kw = dict(n_layers=c.n_layers, hidden=c.hidden, heads=heads, kv_heads=kv_heads, head_dim=head_dim,
              ffn=dense_ffn.pop() if dense_ffn else 0, vocab=c.vocab, ctx=ctx or c.max_seq,
              theta=c.rope_theta, eps=c.rms_eps, neox=bool(s0.flags & FLAG_ROPE_NEOX),
              qkv_bias=any(k.endswith("qkv_bias") for k in t), qk_norm=bool(s0.flags & FLAG_QK_NORM) or any(k.endswith("attn_q_norm") for k in t),
              dtypes=dtypes)
    if mla:
        kw.update(mla=True, q_rank=s0.q_rank, kv_rank=s0.kv_rank, qk_nope=s0.qk_nope, qk_rope=s0.qk_rope,
                  v_dim=s0.v_dim)
    if moe:
        kw.update(n_exp=n_exp, top_k=s0.experts_per_tok or c.experts_per_tok, moe_ffn=s0.moe_ffn or c.moe_ffn,
                  first_moe=first_moe, shared_ffn=shared_ffn,
                  shared_gate=any(k.endswith("ffn_gate_inp_shexp") for k in t))
    if ext.yarn_active():  # YaRN of every full-attention layer (manifest v8, YarnSpec)
        kw.update(yarn=(float(ext.yarn[0]), int(ext.yarn[1]), float(ext.yarn[2]), float(ext.yarn[3])))
    return DenseConfig(**kw), t, m


__all__ = ["load_decode_model", "ATTN_KINDS", "FFN_KINDS"]
