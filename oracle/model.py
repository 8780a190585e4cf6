"""CPU restatement of the reference's dense decode step -- TEST INFRASTRUCTURE ONLY.

The checker for soso_b200's whole-token decode engine: one token of a dense GQA
decoder, op by op, with the oracle's restated kernels (oracle.c), in the order
of crates/soso-llm-core/src/layer.rs:947-1398 and runtime.rs:787-802,
1976-2028.  Only tests import this module.

The model is the dict of soso_b200.decode.synth_model (reference block layouts,
keyed like the reference's tensors); cfg is a DenseConfig.
"""
from __future__ import annotations

import numpy as np

import oracle


class DenseOracle:
    """threads > 0: the matvecs run the reference's AVX2 kernels (gemm.rs:806-894, restated in
    cpu_baseline.c) on that many row strips (parallel.rs:22-31) -- the path the reference
    takes on an AVX2 host -- instead of the scalar kernels; for models of full size."""

    def __init__(self, cfg, model: dict, threads: int = 0):
        self.cfg = cfg
        self.m = model
        self.threads = threads
        self.k = [np.zeros((cfg.ctx, cfg.kv_dim), np.uint16) for _ in range(cfg.n_layers)]
        self.v = [np.zeros((cfg.ctx, cfg.kv_dim), np.uint16) for _ in range(cfg.n_layers)]
        self._embd = None
        self._mla_kv = [dict() for _ in range(cfg.n_layers)]  # (layer) expanded K / V rows of the latent rows

    def _mv(self, name: str, x: np.ndarray, rows: int, cols: int) -> np.ndarray:
        dt = self.cfg.dtypes[name.split(".")[-1]]  # by tensor kind (experts share their kind's dtype)
        if self.threads and dt != 1:  # (the AVX2 restatement has no f32 kernel: f32 matrices run scalar)
            return oracle.cpu_matvec(dt, self.m[name], rows, cols, x, threads=self.threads)
        return oracle.matvec(dt, self.m[name], rows, cols, x)

    def embed(self, token: int) -> np.ndarray:
        """Runtime::embed_token (runtime.rs:787-802): the dequantised row."""
        cfg = self.cfg
        from soso_b200.formats import row_bytes
        rb = row_bytes(cfg.dtypes["token_embd"], cfg.hidden)
        row = self.m["token_embd"][token * rb:(token + 1) * rb]
        return oracle.dequant(cfg.dtypes["token_embd"], row, cfg.hidden).astype(np.float32)

    def step(self, h: np.ndarray, pos: int, routes: dict | None = None) -> np.ndarray:
        """One token from its embedding row at `pos`; returns the logits (and keeps K/V).
        routes: layer -> the experts another run chose there (rank order); where they differ
        from this run's top-k the step follows them and records (layer, router logit gap)
        in route_ties, so a comparison can tell a near-tie from a wrong choice."""
        cfg, m = self.cfg, self.m
        self.force_routes = routes
        self.route_ties = []
        H, qd, kvd, hd = cfg.hidden, cfg.q_dim, cfg.kv_dim, cfg.head_dim
        group = cfg.heads // cfg.kv_heads
        h = np.array(h, np.float32, copy=True)
        self.route_gaps = []  # per MoE layer of this step
        for l in range(cfg.n_layers):
            p = f"blk.{l}."
            if getattr(cfg, "mla", False):
                h = (h + self._mla(p, oracle.rmsnorm(h, m[p + "attn_norm"], cfg.eps), l, pos)).astype(np.float32)
            else:
                h = self._gqa(p, h, l, pos)
            xn = oracle.rmsnorm(h, m[p + "ffn_norm"], cfg.eps)
            if getattr(cfg, "n_exp", 0) and l >= cfg.first_moe:
                h = (self._moe(p, xn, l) + h).astype(np.float32)  # hidden = moe_acc; += residual (:1389)
                continue
            # dense FFN (layer.rs:1300-1389)
            gate = self._mv(p + "ffn_gate", xn, cfg.ffn, H)
            up = self._mv(p + "ffn_up", xn, cfg.ffn, H)
            act = oracle.swiglu(up, gate)
            down = self._mv(p + "ffn_down", act, H, cfg.ffn)
            h = (h + down).astype(np.float32)  # add_assign_f32 (layer.rs:1391)
        # logits (runtime.rs:1976-2019)
        hn = oracle.rmsnorm(h, m["output_norm"], cfg.eps)
        return self._mv("output", hn, cfg.vocab, H)

    def _gqa(self, p: str, h: np.ndarray, l: int, pos: int) -> np.ndarray:
        """GQA attention block (layer.rs:1088-1296): returns h + attention output."""
        cfg, m = self.cfg, self.m
        H, qd, kvd, hd = cfg.hidden, cfg.q_dim, cfg.kv_dim, cfg.head_dim
        group = cfg.heads // cfg.kv_heads
        if True:
            # attention block (layer.rs:1088-1283)
            xn = oracle.rmsnorm(h, m[p + "attn_norm"], cfg.eps)
            q = self._mv(p + "attn_q", xn, qd, H)
            k = self._mv(p + "attn_k", xn, kvd, H)
            v = self._mv(p + "attn_v", xn, kvd, H)
            if p + "qkv_bias" in m:  # add_optional_bias (layer.rs:1146-1163)
                b = m[p + "qkv_bias"]
                q = (q + b[:qd]).astype(np.float32)
                k = (k + b[qd:qd + kvd]).astype(np.float32)
                v = (v + b[qd + kvd:]).astype(np.float32)
            if p + "attn_q_norm" in m:  # FLAG_QK_NORM (layer.rs:1164-1181)
                q = np.concatenate([oracle.rmsnorm(q[i * hd:(i + 1) * hd], m[p + "attn_q_norm"], cfg.eps)
                                    for i in range(cfg.heads)])
                k = np.concatenate([oracle.rmsnorm(k[i * hd:(i + 1) * hd], m[p + "attn_k_norm"], cfg.eps)
                                    for i in range(cfg.kv_heads)])
            if cfg.yarn:  # rope_neox_yarn on full-attention layers (layer.rs:1184-1189)
                q = oracle.rope_neox_yarn(q, cfg.heads, hd, pos, cfg.theta, *cfg.yarn)
                k = oracle.rope_neox_yarn(k, cfg.kv_heads, hd, pos, cfg.theta, *cfg.yarn)
            else:
                q = oracle.rope_heads(q, cfg.heads, hd, pos, cfg.theta, cfg.neox)  # rope_cabezas (layer.rs:1190-1193)
                k = oracle.rope_heads(k, cfg.kv_heads, hd, pos, cfg.theta, cfg.neox)
            self.k[l][pos] = oracle.f32_to_f16_array(k)  # LayerKv::append_f16 (kv.rs:258-275)
            self.v[l][pos] = oracle.f32_to_f16_array(v)
            att = np.concatenate([
                oracle.attention_decode_f16(q[i * hd:(i + 1) * hd], self.k[l][:pos + 1], self.v[l][:pos + 1], hd,
                                            kvd, i // group, pos + 1)
                for i in range(cfg.heads)])
            o = self._mv(p + "attn_output", att, H, qd)
            return (h + o).astype(np.float32)  # add_f32 (layer.rs:1296)

    def _mla(self, p: str, xn: np.ndarray, l: int, pos: int) -> np.ndarray:
        """forward_mla_attn (arch.rs:51-202) with attention_decode_mla_latent (attn.rs:306-404),
        restated with q and k rows per head of qk_nope + qk_rope (nope first): the latent row
        c = kv_down . xn is cached as f16; every cached row is re-expanded k = k_up . c_t (RoPE,
        llama pairs, on each head's rope slice at position t) and v = v_up . c_t; softmax in the
        reference's order; returns the attention output projected by attn_output."""
        cfg, m, H = self.cfg, self.m, self.cfg.hidden
        qk = cfg.qk_nope + cfg.qk_rope
        group = cfg.heads // cfg.kv_heads
        cq = self._mv(p + "attn_q_down", xn, cfg.q_rank, H)
        q = self._mv(p + "attn_q_up", cq, cfg.heads * qk, cfg.q_rank)
        c = self._mv(p + "attn_kv_down", xn, cfg.kv_rank, H)
        for hh in range(cfg.heads):
            s0 = hh * qk + cfg.qk_nope
            q[s0:s0 + cfg.qk_rope] = oracle.rope_llama_n(q[s0:s0 + cfg.qk_rope], pos, cfg.theta, cfg.qk_rope)
        self.k[l][pos] = oracle.f32_to_f16_array(c)  # append_mla_latent (kv.rs:293-315)
        cache = self._mla_kv[l]
        if not cache:  # expanded rows of every cached position: K [ctx][kv_heads][qk], V [ctx][kv_heads][v_dim]
            cache["k"] = np.zeros((cfg.ctx, cfg.kv_heads, qk), np.float32)
            cache["v"] = np.zeros((cfg.ctx, cfg.kv_heads, cfg.v_dim), np.float32)
            cache["n"] = 0
        for t in range(cache["n"], pos + 1):
            ct = self.k[l][t].view(np.float16).astype(np.float32)
            kf = self._mv(p + "attn_k_up", ct, cfg.kv_heads * qk, cfg.kv_rank)
            for g in range(cfg.kv_heads):
                s0 = g * qk + cfg.qk_nope
                kf[s0:s0 + cfg.qk_rope] = oracle.rope_llama_n(kf[s0:s0 + cfg.qk_rope], t, cfg.theta, cfg.qk_rope)
            cache["k"][t] = kf.reshape(cfg.kv_heads, qk)
            cache["v"][t] = self._mv(p + "attn_v_up", ct, cfg.kv_heads * cfg.v_dim, cfg.kv_rank).reshape(
                cfg.kv_heads, cfg.v_dim)
        cache["n"] = pos + 1
        # softmax(q . k_t / sqrt(qk)) . v_t per head over t = 0..pos (attention_decode_mla_latent,
        # attn.rs:306-404), f32 throughout
        inv = np.float32(1.0 / np.sqrt(np.float32(qk)))
        att = np.zeros(cfg.heads * cfg.v_dim, np.float32)
        for hh in range(cfg.heads):
            g = hh // group
            qh = q[hh * qk:(hh + 1) * qk]
            lg = (cache["k"][:pos + 1, g, :] @ qh).astype(np.float32) * inv
            lg = np.exp(lg - lg.max()).astype(np.float32)
            lg = (lg / lg.sum()).astype(np.float32)
            att[hh * cfg.v_dim:(hh + 1) * cfg.v_dim] = (lg @ cache["v"][:pos + 1, g, :]).astype(np.float32)
        return self._mv(p + "attn_output", att, H, cfg.q_dim)

    def _moe(self, p: str, xn: np.ndarray, l: int) -> np.ndarray:
        """forward_moe_ffn / moe_expertos_agrupados (layer.rs:1938-1972, :1862-1935): router
        logits, topk_softmax (gemm.rs:62-91), per chosen expert down(swiglu(up, gate)) summed
        in rank order with its weight, then the shared expert weighted by
        sigmoid(ffn_gate_inp_shexp . xn) (or 1)."""
        cfg, m, H = self.cfg, self.m, self.cfg.hidden
        logits = self._mv(p + "ffn_gate_inp", xn, cfg.n_exp, H)
        self.last_route = oracle.topk_softmax(logits, cfg.top_k)
        # the routing margin: router logit gap between the k-th and (k+1)-th expert (a gap
        # near the two sides' rounding difference lets either pick the other expert)
        srt = np.sort(logits.astype(np.float64))
        self.route_gaps.append(float(srt[-cfg.top_k] - srt[-cfg.top_k - 1]) if cfg.top_k < cfg.n_exp else np.inf)
        idx, wts = self.last_route
        forced = self.force_routes.get(l) if self.force_routes else None
        if forced is not None and set(int(e) for e in forced) != set(int(e) for e in idx):
            # the other side chose differently: record how far its choice is from this side's
            # k-th expert (router logit gap; a near-tie lets rounding pick either), and follow
            # it, with this side's probabilities renormalised over the chosen set
            lg = logits.astype(np.float64)
            kth = float(min(lg[int(e)] for e in idx))
            gap = max(kth - float(lg[int(e)]) for e in forced if int(e) not in set(int(i) for i in idx))
            self.route_ties.append((l, gap))
            m_ = np.float32(logits.max())
            ex = np.exp((logits - m_).astype(np.float32)).astype(np.float32)
            prob = (ex / np.float32(ex.sum(dtype=np.float32))).astype(np.float32)
            idx = np.asarray(forced, np.int32)
            w = prob[idx]
            wts = (w / np.float32(w.sum(dtype=np.float32))).astype(np.float32)
            self.last_route = (idx, wts)
        acc = np.zeros(H, np.float32)
        for e, w in zip(idx, wts):
            q = f"{p}E{int(e):03d}."
            gate = self._mv(q + "ffn_gate", xn, cfg.moe_ffn, H)
            up = self._mv(q + "ffn_up", xn, cfg.moe_ffn, H)
            down = self._mv(q + "ffn_down", oracle.swiglu(up, gate), H, cfg.moe_ffn)
            acc = (acc + down * np.float32(w)).astype(np.float32)
        if cfg.shared_ffn:
            q = f"{p}S00."
            gate = self._mv(q + "ffn_gate", xn, cfg.shared_ffn, H)
            up = self._mv(q + "ffn_up", xn, cfg.shared_ffn, H)
            down = self._mv(q + "ffn_down", oracle.swiglu(up, gate), H, cfg.shared_ffn)
            pg = np.float32(1.0)
            if cfg.shared_gate:
                d = np.float32(np.dot(m[p + "ffn_gate_inp_shexp"].astype(np.float64), xn.astype(np.float64)))
                pg = np.float32(1.0 / (1.0 + np.exp(-np.float64(d))))
            acc = (acc + down * pg).astype(np.float32)
        return acc

    def greedy(self, prompt, n: int) -> tuple[np.ndarray, list]:
        """n steps from position 0: prompt tokens first, then argmax (runtime.rs:2021-2028)."""
        toks, logits_all = [], []
        tok = int(prompt[0])
        for i in range(n):
            lg = self.step(self.embed(tok), i)
            logits_all.append(lg)
            a = oracle.argmax(lg)
            toks.append(a)
            tok = int(prompt[i + 1]) if i + 1 < len(prompt) else a
        return np.array(toks, np.int32), logits_all
