"""Whole-token decode through the C ABI (GpuDispatch::decode_preparar / decode_token,
crates/soso-llm-core/src/gpu.rs:654-684): model configurations, seeded synthetic
models in the reference's block layouts, and a session object that owns the plan.

The model of a config is a dict of numpy arrays keyed like the reference's
tensors (`blk.{l}.attn_q`, ..., `output`, `token_embd`); weights are bytes in
the reference layout, norms and biases f32.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, field

import numpy as np

from . import synth
from ._lib import (SbDecodePlan, SbLayerPlan, SbLayerRows, SbLayerState, SbMat, SbMlaPlan, SbMoePlan, SbView,
                   SbError, c_f32p, c_u8p, last_error, lib)
from .formats import DTYPE_Q4_K, DTYPE_Q6_K, DTYPE_Q8_0


@dataclass(frozen=True)
class DenseConfig:
    """A dense GQA decoder (Qwen2-style: q/k/v bias, NeoX RoPE, SwiGLU)."""
    n_layers: int
    hidden: int
    heads: int
    kv_heads: int
    head_dim: int
    ffn: int
    vocab: int
    ctx: int
    theta: float = 1e6
    eps: float = 1e-6
    neox: bool = True
    qkv_bias: bool = True
    qk_norm: bool = False
    # MoE FFN on layers >= first_moe when n_exp > 0 (forward_moe_ffn, layer.rs:1938-2109):
    # n_exp routed experts of width moe_ffn, top_k chosen per token, and an optional shared
    # expert of width shared_ffn (gated by sigmoid(ffn_gate_inp_shexp . x) when shared_gate)
    # MLA attention (arch.rs:51-202) on every layer when mla: q_down / q_up (q-LoRA),
    # kv_down to a kv_rank latent, k_up / v_up; q and k rows per head nope then rope
    mla: bool = False
    q_rank: int = 0
    kv_rank: int = 0
    qk_nope: int = 0
    qk_rope: int = 0
    v_dim: int = 0
    n_exp: int = 0
    top_k: int = 0
    moe_ffn: int = 0
    first_moe: int = 0
    shared_ffn: int = 0
    shared_gate: bool = False
    # YaRN RoPE on every layer (manifest v8 YarnSpec: factor, orig_ctx, beta_fast, beta_slow);
    # empty = plain RoPE
    yarn: tuple = ()
    # Q4_K_M mix: Q4_K everywhere, Q6_K for ffn_down and the output matrix
    dtypes: dict = field(default_factory=lambda: {"attn_q": DTYPE_Q4_K, "attn_k": DTYPE_Q4_K, "attn_v": DTYPE_Q4_K,
                                                  "attn_output": DTYPE_Q4_K, "ffn_gate": DTYPE_Q4_K,
                                                  "ffn_up": DTYPE_Q4_K, "ffn_down": DTYPE_Q6_K,
                                                  "output": DTYPE_Q6_K, "token_embd": DTYPE_Q4_K})

    @property
    def q_dim(self) -> int:
        """width of the attention output (heads * v_dim for MLA)"""
        return self.heads * (self.v_dim if self.mla else self.head_dim)

    @property
    def kv_dim(self) -> int:
        """width of one layer's cache row (the latent row for MLA)"""
        return self.kv_rank if self.mla else self.kv_heads * self.head_dim

    def is_moe(self, layer: int) -> bool:
        return self.n_exp > 0 and layer >= self.first_moe


# Qwen2.5-3B-style dense decoder, fp16 KV at 4096 context
QWEN25_3B = DenseConfig(n_layers=36, hidden=2048, heads=16, kv_heads=2, head_dim=128, ffn=11008, vocab=151936,
                        ctx=4096)
# a small model of the same structure, for parity tests against the CPU oracle
TINY = DenseConfig(n_layers=2, hidden=512, heads=4, kv_heads=2, head_dim=128, ffn=1024, vocab=1024, ctx=160)
# the same with YaRN (factor 16 over a 64-position original context: pairs 0-10 ramp, the
# rest are divided by 16)
TINY_YARN = DenseConfig(n_layers=2, hidden=512, heads=4, kv_heads=2, head_dim=128, ffn=1024, vocab=1024, ctx=160,
                        theta=1e4, yarn=(16.0, 64, 32.0, 1.0))

_ALL_Q4K = {k: DTYPE_Q4_K for k in ("attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate", "ffn_up", "ffn_down",
                                    "output", "token_embd", "ffn_gate_inp", "attn_q_down", "attn_q_up",
                                    "attn_kv_down", "attn_k_up", "attn_v_up")}
# Qwen3-30B-A3B-style MoE decoder, all Q4_K, QK-norm, fp16 KV at 2048
QWEN3_30B_A3B = DenseConfig(n_layers=48, hidden=2048, heads=32, kv_heads=4, head_dim=128, ffn=0, vocab=151936,
                            ctx=2048, qkv_bias=False, qk_norm=True, n_exp=128, top_k=8, moe_ffn=768,
                            dtypes=dict(_ALL_Q4K))
# small MoE models of the same structure for parity tests: one dense layer first, then MoE
# layers with a gated shared expert (TINY_MOE) or none (TINY_MOE_NS)
TINY_MOE = DenseConfig(n_layers=3, hidden=512, heads=4, kv_heads=2, head_dim=128, ffn=1024, vocab=1024, ctx=96,
                       qkv_bias=False, qk_norm=True, n_exp=16, top_k=4, moe_ffn=256, first_moe=1, shared_ffn=512,
                       shared_gate=True, dtypes=dict(_ALL_Q4K, ffn_down=DTYPE_Q6_K, output=DTYPE_Q6_K))
# a small MLA + MoE model (configs[4]'s structure): MLA on every layer, a dense FFN first,
# then MoE layers with an ungated shared expert
# (down projections Q8_0 like configs[4]'s, the experts' 160 wide: rows padded on upload)
TINY_MLA = DenseConfig(n_layers=3, hidden=512, heads=4, kv_heads=4, head_dim=128, ffn=1024, vocab=1024, ctx=96,
                       theta=1e4, neox=False, qkv_bias=False, mla=True, q_rank=256, kv_rank=512, qk_nope=64,
                       qk_rope=32, v_dim=128, n_exp=8, top_k=2, moe_ffn=160, first_moe=1, shared_ffn=512,
                       dtypes=dict(_ALL_Q4K, ffn_down=DTYPE_Q8_0))
# DeepSeek-V2-Lite-style MLA + MoE (q-LoRA rank 512 synthesized, as the
# reference's MLA requires it), layer 0 dense FFN 10944, then 64 routed experts (top-6, 1408)
# plus the 2 shared experts (held as one expert of 2816, ungated); down projections Q8_0
# (1408 / 10944 are not whole Q4_K blocks), all else Q4_K; RoPE theta 1e4, llama pairs
DEEPSEEK_V2_LITE = DenseConfig(n_layers=27, hidden=2048, heads=16, kv_heads=16, head_dim=128, ffn=10944,
                               vocab=102400, ctx=2048, theta=1e4, neox=False, qkv_bias=False, mla=True, q_rank=512,
                               kv_rank=512, qk_nope=128, qk_rope=64, v_dim=128, n_exp=64, top_k=6, moe_ffn=1408,
                               first_moe=1, shared_ffn=2816, dtypes=dict(_ALL_Q4K, ffn_down=DTYPE_Q8_0))
TINY_MOE_NS = DenseConfig(n_layers=2, hidden=512, heads=8, kv_heads=2, head_dim=128, ffn=0, vocab=1024, ctx=96,
                          qkv_bias=False, qk_norm=True, n_exp=32, top_k=8, moe_ffn=256, dtypes=dict(_ALL_Q4K))


def shapes(cfg: DenseConfig) -> dict:
    """tensor name suffix -> (rows, cols)"""
    H = cfg.hidden
    if cfg.mla:
        qk = cfg.qk_nope + cfg.qk_rope
        return {"attn_q_down": (cfg.q_rank, H), "attn_q_up": (cfg.heads * qk, cfg.q_rank),
                "attn_kv_down": (cfg.kv_rank, H), "attn_k_up": (cfg.kv_heads * qk, cfg.kv_rank),
                "attn_v_up": (cfg.kv_heads * cfg.v_dim, cfg.kv_rank), "attn_output": (H, cfg.q_dim),
                "ffn_gate": (cfg.ffn, H), "ffn_up": (cfg.ffn, H), "ffn_down": (H, cfg.ffn)}
    return {"attn_q": (cfg.q_dim, H), "attn_k": (cfg.kv_dim, H), "attn_v": (cfg.kv_dim, H),
            "attn_output": (H, cfg.q_dim), "ffn_gate": (cfg.ffn, H), "ffn_up": (cfg.ffn, H),
            "ffn_down": (H, cfg.ffn)}


def synth_model(cfg: DenseConfig, seed: str = "model", held=None) -> dict:
    """Seeded random-init weights of the config's architecture (synth.model_weights).
    held = (rank, world): leave out the experts that rank does not hold under expert
    parallelism (soso_b200.tp: routed experts by ID range, shared experts by layer); every
    tensor that is made has the same bytes either way."""
    m = {}
    H = cfg.hidden
    ex_lo, ex_hi = 0, cfg.n_exp
    if held is not None and cfg.n_exp:
        from .tp import row_strip
        ex_lo, ex_hi = row_strip(cfg.n_exp, held[0], held[1])
    for l in range(cfg.n_layers):
        for name, (rows, cols) in shapes(cfg).items():
            if cfg.is_moe(l) and name.startswith("ffn_"):
                continue
            m[f"blk.{l}.{name}"] = synth.model_weights(cfg.dtypes[name], rows, cols, synth.rng(seed, l, name))
        if cfg.is_moe(l):
            # router rows scaled so the logits are about N(0, 1)
            m[f"blk.{l}.ffn_gate_inp"] = synth.model_weights(cfg.dtypes["ffn_gate_inp"], cfg.n_exp, H,
                                                              synth.rng(seed, l, "router"), std=1.0 / np.sqrt(H))
            for e in range(ex_lo, ex_hi):
                for name, (rows, cols) in (("ffn_gate", (cfg.moe_ffn, H)), ("ffn_up", (cfg.moe_ffn, H)),
                                           ("ffn_down", (H, cfg.moe_ffn))):
                    m[f"blk.{l}.E{e:03d}.{name}"] = synth.model_weights(cfg.dtypes[name], rows, cols,
                                                                         synth.rng(seed, l, e, name))
            if cfg.shared_ffn:
                for name, (rows, cols) in (("ffn_gate", (cfg.shared_ffn, H)), ("ffn_up", (cfg.shared_ffn, H)),
                                           ("ffn_down", (H, cfg.shared_ffn))):
                    if held is not None and l % held[1] != held[0]:
                        continue
                    m[f"blk.{l}.S00.{name}"] = synth.model_weights(cfg.dtypes[name], rows, cols,
                                                                    synth.rng(seed, l, "shared", name))
                if cfg.shared_gate:
                    m[f"blk.{l}.ffn_gate_inp_shexp"] = (synth.rng(seed, l, "sg").standard_normal(H) /
                                                        np.sqrt(H)).astype(np.float32)
        g = synth.rng(seed, l, "vec")
        m[f"blk.{l}.attn_norm"] = (1.0 + 0.1 * g.standard_normal(H)).astype(np.float32)
        m[f"blk.{l}.ffn_norm"] = (1.0 + 0.1 * g.standard_normal(H)).astype(np.float32)
        if cfg.qkv_bias:
            m[f"blk.{l}.qkv_bias"] = (0.1 * g.standard_normal(cfg.q_dim + 2 * cfg.kv_dim)).astype(np.float32)
        if cfg.qk_norm:
            m[f"blk.{l}.attn_q_norm"] = (1.0 + 0.1 * g.standard_normal(cfg.head_dim)).astype(np.float32)
            m[f"blk.{l}.attn_k_norm"] = (1.0 + 0.1 * g.standard_normal(cfg.head_dim)).astype(np.float32)
    g = synth.rng(seed, "out")
    m["output_norm"] = (1.0 + 0.1 * g.standard_normal(H)).astype(np.float32)
    m["output"] = synth.model_weights(cfg.dtypes["output"], cfg.vocab, H, synth.rng(seed, "output"))
    m["token_embd"] = synth.model_weights(cfg.dtypes["token_embd"], cfg.vocab, H, synth.rng(seed, "embd"), std=1.0)
    return m


def _f32(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(c_f32p)


def yarn_divisors(head_dim: int, theta: float, factor: float, orig_ctx: int, beta_fast: float,
                  beta_slow: float) -> tuple[np.ndarray, float]:
    """The per-pair frequency divisors and the cos/sin magnitude the reference hands its GPU
    rope for a YaRN layer (yarn_factores with yarn_corr_dims and yarn_ramp,
    crates/soso-llm-core/src/gemm.rs:1413-1446), in f32 as there: the ramp runs between the
    corrected dims of beta_fast and beta_slow; divisor_i = 1 / (ramp_i + (1 - ramp_i) / factor);
    mscale = 1 + 0.1 ln(factor)."""
    f = np.float32

    def dim(n_rot):
        return f(head_dim) * np.log(f(orig_ctx) / (f(n_rot) * f(2.0) * f(np.pi))) / (f(2.0) * np.log(f(theta)))

    low = f(max(np.floor(dim(beta_fast)), f(0.0)))
    high = f(min(np.ceil(dim(beta_slow)), f(head_dim - 1)))
    scale = f(1.0) / f(factor)
    out = np.empty(head_dim // 2, np.float32)
    for i in range(head_dim // 2):
        ramp = f(1.0) - f(min(max((f(i) - low) / max(high - low, f(0.001)), f(0.0)), f(1.0)))
        out[i] = f(1.0) / (scale * (f(1.0) - ramp) + ramp)
    return out, float(f(f(1.0) + f(0.1) * np.log(f(factor))))


class DecodeSession:
    """A prepared whole-token decode on one device (sb_decode_prepare)."""

    def __init__(self, cfg: DenseConfig, model: dict, device: int = 0, ctx_handle=None, group=None):
        """group = (rank, world, all_gather): decode across `world` processes, sharded as
        soso_b200.tp describes; all_gather(bytes) -> every rank's bytes, and it doubles as
        the host barrier before the first (exchanging) warm-up token.  Under expert
        parallelism `model` may leave out the experts this rank does not hold
        (synth_model(..., held=(rank, world)))."""
        self.cfg = cfg
        self.model = model
        L = lib()
        self._own = ctx_handle is None
        if ctx_handle is None:
            h = ctypes.c_void_p()
            if L.sb_create(device, ctypes.byref(h)) != 0:
                raise SbError(last_error())
            ctx_handle = h
        self.ctx = ctx_handle
        if group is not None and group[1] > 1:
            from . import tp
            tp.open_group(self.ctx, group[0], group[1], group[2])
        self._keep = []
        H = cfg.hidden
        layers = (SbLayerPlan * cfg.n_layers)()
        for l in range(cfg.n_layers):
            lp = layers[l]
            lp.heads, lp.kv_heads, lp.head_dim = cfg.heads, cfg.kv_heads, cfg.head_dim
            lp.theta, lp.neox = cfg.theta, int(cfg.neox)
            if cfg.yarn and not cfg.mla:
                yf, lp.rope_mscale = yarn_divisors(cfg.head_dim, cfg.theta, *cfg.yarn)
                self._keep.append(yf)
                lp.rope_factors = _f32(yf)
            lp.q_norm = _f32(model.get(f"blk.{l}.attn_q_norm"))
            lp.k_norm = _f32(model.get(f"blk.{l}.attn_k_norm"))
            lp.qkv_bias = _f32(model.get(f"blk.{l}.qkv_bias"))
            lp.norm_attn = _f32(model[f"blk.{l}.attn_norm"])
            lp.norm_ffn = _f32(model[f"blk.{l}.ffn_norm"])
            for fld, name in (("q", "attn_q"), ("k", "attn_k"), ("v", "attn_v"), ("o", "attn_output"),
                              ("gate", "ffn_gate"), ("up", "ffn_up"), ("down", "ffn_down")):
                if (cfg.is_moe(l) and name.startswith("ffn_")) or (cfg.mla and name in ("attn_q", "attn_k", "attn_v")):
                    continue
                rows, cols = shapes(cfg)[name]
                setattr(lp, fld, self._mat(f"blk.{l}.{name}", cfg.dtypes[name], rows, cols))
            if cfg.is_moe(l):
                lp.moe = ctypes.pointer(self._moe_plan(l))
            if cfg.mla:
                mp = SbMlaPlan()
                mp.q_rank, mp.kv_rank, mp.qk_nope, mp.qk_rope, mp.v_dim = (cfg.q_rank, cfg.kv_rank, cfg.qk_nope,
                                                                          cfg.qk_rope, cfg.v_dim)
                for fld in ("q_down", "q_up", "kv_down", "k_up", "v_up"):
                    name = "attn_" + fld
                    rows, cols = shapes(cfg)[name]
                    setattr(mp, fld, self._mat(f"blk.{l}.{name}", cfg.dtypes[name], rows, cols))
                self._keep.append(mp)
                lp.mla = ctypes.pointer(mp)
        plan = SbDecodePlan()
        plan.layers = layers
        plan.n_layers = cfg.n_layers
        plan.hidden, plan.vocab, plan.ctx, plan.eps = H, cfg.vocab, cfg.ctx, cfg.eps
        plan.final_norm = _f32(model["output_norm"])
        plan.lm_head = self._mat("output", cfg.dtypes["output"], cfg.vocab, H)
        plan.embed = self._mat("token_embd", cfg.dtypes["token_embd"], cfg.vocab, H)
        self._keep += [layers, plan]
        rc = L.sb_decode_prepare(self.ctx, ctypes.byref(plan))
        if rc != 1:
            raise SbError(f"sb_decode_prepare returned {rc}: {last_error()}")
        if group is not None and group[1] > 1:
            group[2](b"prepared")  # every rank has its shards resident: the warm-up may exchange
            rc = L.sb_decode_finish(self.ctx)
            if rc != 1:
                raise SbError(f"sb_decode_finish returned {rc}: {last_error()}")

    def _moe_plan(self, l: int) -> SbMoePlan:
        """MoeDec (gpu.rs:130-137) of layer l: router, experts [gate, up, down] each, shared expert."""
        cfg, H = self.cfg, self.cfg.hidden
        mp = SbMoePlan()
        mp.n_exp, mp.top_k, mp.ffn = cfg.n_exp, cfg.top_k, cfg.moe_ffn
        mp.router = self._mat(f"blk.{l}.ffn_gate_inp", cfg.dtypes["ffn_gate_inp"], cfg.n_exp, H)
        ex = (SbMat * (3 * cfg.n_exp))()
        for e in range(cfg.n_exp):
            for k, (name, rows, cols) in enumerate((("ffn_gate", cfg.moe_ffn, H), ("ffn_up", cfg.moe_ffn, H),
                                                     ("ffn_down", H, cfg.moe_ffn))):
                ex[3 * e + k] = self._mat(f"blk.{l}.E{e:03d}.{name}", cfg.dtypes[name], rows, cols)
        mp.experts = ex
        if cfg.shared_ffn:
            sh = (SbMat * 3)()
            for k, (name, rows, cols) in enumerate((("ffn_gate", cfg.shared_ffn, H), ("ffn_up", cfg.shared_ffn, H),
                                                     ("ffn_down", H, cfg.shared_ffn))):
                sh[k] = self._mat(f"blk.{l}.S00.{name}", cfg.dtypes[name], rows, cols)
            mp.shared = sh
            self._keep.append(sh)
            if cfg.shared_gate:
                mp.shared_gate = _f32(self.model[f"blk.{l}.ffn_gate_inp_shexp"])
        self._keep += [ex, mp]
        return mp

    def _mat(self, key: str, dtype: int, rows: int, cols: int) -> SbMat:
        w = self.model.get(key)
        if w is None:  # not held by this rank (expert parallelism): the library does not read it
            return SbMat(None, SbView(None, 0, dtype, rows * cols), rows, cols)
        k = key.encode()
        self._keep.append(k)
        return SbMat(k, SbView(w.ctypes.data_as(c_u8p), w.size, dtype, rows * cols), rows, cols)

    def token(self, embed: np.ndarray, pos: int, kv_rows: bool = False):
        """decode_token: logits of the token whose embedding row is `embed`, at `pos`."""
        cfg = self.cfg
        e = np.ascontiguousarray(embed, dtype=np.float32)
        logits = np.empty(cfg.vocab, np.float32)
        kv = np.empty(cfg.n_layers * 2 * cfg.kv_dim, np.uint16) if kv_rows else None
        rc = lib().sb_decode_token(self.ctx, e.ctypes.data_as(c_f32p), pos, logits.ctypes.data_as(c_f32p),
                                   kv.ctypes.data_as(ctypes.POINTER(ctypes.c_uint16)) if kv is not None else None)
        if rc != 1:
            raise SbError(f"sb_decode_token returned {rc}: {last_error()}")
        return (logits, kv) if kv_rows else logits

    def greedy(self, prompt, n: int, pos: int = 0) -> np.ndarray:
        """n device-side steps from `pos`: prompt tokens fed first, then the argmax chain;
        returns the argmax of every step."""
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.empty(n, np.int32)
        rc = lib().sb_decode_greedy(self.ctx, p.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), p.size, pos, n,
                                    out.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)))
        if rc != 1:
            raise SbError(f"sb_decode_greedy returned {rc}: {last_error()}")
        return out

    def download_state(self, rows: int, hidden: bool = True):
        """sb_decode_download_state: per layer (K, V) f16 bits [rows][kv_dim] (an MLA layer's
        latent rows and None), and the hidden vector the last step left (before the output
        norm)."""
        cfg = self.cfg
        out = [(np.empty((rows, cfg.kv_dim), np.uint16), None if cfg.mla else np.empty((rows, cfg.kv_dim), np.uint16))
               for _ in range(cfg.n_layers)]
        arr = (SbLayerRows * cfg.n_layers)()
        for l, (k, v) in enumerate(out):
            arr[l].k = k.ctypes.data
            arr[l].v = v.ctypes.data if v is not None else None
        h = np.empty(cfg.hidden, np.float32) if hidden else None
        rc = lib().sb_decode_download_state(self.ctx, arr, cfg.n_layers, rows, _f32(h))
        if rc != 1:
            raise SbError(f"sb_decode_download_state returned {rc}: {last_error()}")
        return out, h

    def upload_state(self, layers, pos: int, valid=None) -> list:
        """sb_decode_upload_state: layers = per layer (K, V) f16 bits with at least pos rows
        (V None for MLA); valid = rows the device already holds per layer (default 0).
        Returns the new valid-row counts (pos each)."""
        cfg = self.cfg
        arr = (SbLayerState * cfg.n_layers)()
        counts = (ctypes.c_size_t * cfg.n_layers)(*(valid or [0] * cfg.n_layers))
        keep = []
        for l, (k, v) in enumerate(layers):
            k = np.ascontiguousarray(k, dtype=np.uint16)
            keep.append(k)
            arr[l].k = k.ctypes.data
            if v is not None:
                v = np.ascontiguousarray(v, dtype=np.uint16)
                keep.append(v)
                arr[l].v = v.ctypes.data
            arr[l].valid_rows = ctypes.cast(ctypes.addressof(counts) + l * ctypes.sizeof(ctypes.c_size_t),
                                            ctypes.POINTER(ctypes.c_size_t))
        rc = lib().sb_decode_upload_state(self.ctx, arr, cfg.n_layers, pos)
        if rc != 1:
            raise SbError(f"sb_decode_upload_state returned {rc}: {last_error()}")
        return list(counts)

    def prefill(self, tokens, pos: int = 0, logits: bool = True):
        """sb_decode_prefill: the block of tokens at positions pos.., all layers at once on
        the tensor cores; returns (logits of the last token or None, its argmax)."""
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        lg = np.empty(self.cfg.vocab, np.float32) if logits else None
        nxt = ctypes.c_int32(-1)
        rc = lib().sb_decode_prefill(self.ctx, t.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), t.size, pos,
                                     _f32(lg), ctypes.byref(nxt))
        if rc != 1:
            raise SbError(f"sb_decode_prefill returned {rc}: {last_error()}")
        return lg, int(nxt.value)

    def routes(self) -> dict:
        """sb_decode_routes: layer -> the experts its router chose at the last step (rank order)."""
        cfg = self.cfg
        moe = [l for l in range(cfg.n_layers) if cfg.is_moe(l)]
        out = np.empty(max(1, len(moe) * cfg.top_k), np.int32)
        rc = lib().sb_decode_routes(self.ctx, out.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), out.size)
        if rc != 1:
            raise SbError(f"sb_decode_routes returned {rc}: {last_error()}")
        return {l: out[i * cfg.top_k:(i + 1) * cfg.top_k].copy() for i, l in enumerate(moe)}

    def route_trace(self, pos: int) -> tuple[dict, dict]:
        """sb_decode_route_trace: for the decode step at position pos, layer -> the experts
        its router chose (rank order), and layer -> the router-logit gap between the k-th
        choice and the best expert not chosen."""
        cfg = self.cfg
        moe = [l for l in range(cfg.n_layers) if cfg.is_moe(l)]
        out = np.empty(max(1, len(moe) * cfg.top_k), np.int32)
        gaps = np.empty(max(1, len(moe)), np.float32)
        rc = lib().sb_decode_route_trace(self.ctx, pos, out.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), out.size,
                                          gaps.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), gaps.size)
        if rc != 1:
            raise SbError(f"sb_decode_route_trace returned {rc}: {last_error()}")
        return ({l: out[i * cfg.top_k:(i + 1) * cfg.top_k].copy() for i, l in enumerate(moe)},
                {l: float(gaps[i]) for i, l in enumerate(moe)})

    def close(self):
        if self._own and self.ctx:
            lib().sb_destroy(self.ctx)
            self.ctx = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
