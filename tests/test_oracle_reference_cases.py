"""The reference's own tests of the decode ops, restated against the CPU oracle (CPU only),
so that the oracle the GPU tests trust is pinned to what the reference asserts:

* attention (crates/soso-llm-core/tests/attn_grupo.rs:29-128): against an f64 softmax over
  the f16-rounded rows (error < 2e-5, hd 64 / 128, 1..257 tokens), a query's result
  independent of the others, a prefix of a longer cache equal to the shorter cache, large
  scores finite and within 1e-3;
* RoPE (crates/soso-llm-core/src/gemm.rs:1513-1590): rope_cabezas equal bit for bit to RoPE
  head by head, NeoX at position 0 the identity, NeoX different from llama pairs, and the
  YaRN golden vector the reference computed from ggml's rope_yarn (1e-4) with the pure
  magnitude factor at position 0 (1e-5);
* MoE (crates/soso-llm-core/tests/moe.rs:145-273): topk_softmax renormalises to 1 and ranks
  the largest first; the scalar MoE FFN of moe_ffn_referencia_escalar through the oracle's
  MoE step equals the test's own f32 steps;
* MLA (crates/soso-llm-core/tests/arch_ext.rs:156-330, :531-592): on the reference's
  consistent dims (qk_nope + qk_rope = hidden / heads) and its f32 weights, the oracle's MLA
  attention equals mla_oracle_attn_out restated here, within the reference's 1e-4, over
  positions 0..2 with the latent history read back from the f16 cache.
"""
import dataclasses

import numpy as np

import oracle
from oracle.model import DenseOracle
from soso_b200 import decode

F = np.float32


class Lcg:
    """The reference tests' lcg (attn_grupo.rs:9-12; rope_tests' closure): (s >> 33) as f32
    / 2^31, then scaled and shifted in f32."""

    def __init__(self, s: int):
        self.s = s

    def unit(self) -> np.float32:
        self.s = (self.s * 6364136223846793005 + 1442695040888963407) & 0xFFFFFFFFFFFFFFFF
        return F(self.s >> 33) / F(1 << 31)

    def sym(self, scale=2.0, shift=1.0) -> np.float32:
        return F(self.unit() * F(scale) - F(shift))


def _caso(tokens, kv_heads, hd, r: Lcg):
    """caso (attn_grupo.rs:20-26): K = f16(lcg * 3), V = f16(lcg), token-major."""
    kvd = kv_heads * hd
    k = np.array([oracle.f32_to_f16(float(F(r.sym() * F(3.0)))) for _ in range(tokens * kvd)], np.uint16)
    v = np.array([oracle.f32_to_f16(float(r.sym())) for _ in range(tokens * kvd)], np.uint16)
    return k.reshape(tokens, kvd), v.reshape(tokens, kvd), kvd


def _ref64(q, k, v, hd, kv_head, n):
    """referencia (attn_grupo.rs:29-49): f64 softmax(q.k / sqrt(d)) . v over the f16 values."""
    kk = k[:n, kv_head * hd:(kv_head + 1) * hd].view(np.float16).astype(np.float64)
    vv = v[:n, kv_head * hd:(kv_head + 1) * hd].view(np.float16).astype(np.float64)
    s = kk @ np.asarray(q, np.float64) / np.sqrt(hd)
    e = np.exp(s - s.max())
    return (e / e.sum()) @ vv


def test_attention_against_f64():
    r = Lcg(7)
    for hd in (64, 128):
        for n in (1, 2, 7, 8, 9, 31, 32, 33, 64, 100, 257):
            k, v, kvd = _caso(n, 2, hd, r)
            qs = [np.array([r.sym() * F(2.0) for _ in range(hd)], np.float32) for _ in range(5)]
            for j, q in enumerate(qs):
                out = oracle.attention_decode_f16(q, k, v, hd, kvd, 1, n)
                err = float(np.max(np.abs(out.astype(np.float64) - _ref64(q, k, v, hd, 1, n))))
                assert err < 2e-5, (hd, n, j, err)


def test_attention_query_independent_and_prefix():
    r = Lcg(99)
    hd = 64
    k, v, kvd = _caso(130, 4, hd, r)
    qs = [np.array([r.sym() * F(2.0) for _ in range(hd)], np.float32) for _ in range(7)]
    alone = [oracle.attention_decode_f16(q, k, v, hd, kvd, 2, 130) for q in qs]
    again = [oracle.attention_decode_f16(q, k, v, hd, kvd, 2, 130) for q in reversed(qs)][::-1]
    assert all(np.array_equal(a, b) for a, b in zip(alone, again))
    # un_prefijo_da_lo_mismo_que_una_secuencia_mas_corta (attn_grupo.rs:96-113)
    r = Lcg(5)
    hd = 128
    kl, vl, kvd = _caso(200, 2, hd, r)
    n = 77
    for _ in range(3):
        q = np.array([r.sym() for _ in range(hd)], np.float32)
        a = oracle.attention_decode_f16(q, kl, vl, hd, kvd, 0, n)
        b = oracle.attention_decode_f16(q, kl[:n].copy(), vl[:n].copy(), hd, kvd, 0, n)
        assert np.array_equal(a, b)


def test_attention_large_scores():
    """puntuaciones_grandes_no_desbordan (attn_grupo.rs:115-127)."""
    r = Lcg(3)
    hd = 128
    k, v, kvd = _caso(64, 1, hd, r)
    q = np.array([r.sym() * F(40.0) for _ in range(hd)], np.float32)
    out = oracle.attention_decode_f16(q, k, v, hd, kvd, 0, 64)
    assert np.all(np.isfinite(out))
    assert float(np.max(np.abs(out.astype(np.float64) - _ref64(q, k, v, hd, 0, 64)))) < 1e-3


def test_rope_heads_equals_rope_per_head():
    """rope_cabezas_es_identico_a_rope_por_cabeza (gemm.rs:1517-1545)."""
    r = Lcg(17)
    for hd, nh in ((64, 3), (128, 5), (256, 2), (320, 2)):
        for pos in (0, 1, 7, 1000, 31999):
            for theta in (10000.0, 1e6):
                orig = np.array([r.sym(4.0, 2.0) for _ in range(hd * nh)], np.float32)
                for neox in (False, True):
                    each = np.concatenate([oracle.rope_heads(orig[h * hd:(h + 1) * hd], 1, hd, pos, theta, neox)
                                           for h in range(nh)])
                    both = oracle.rope_heads(orig, nh, hd, pos, theta, neox)
                    assert np.array_equal(each.view(np.uint32), both.view(np.uint32)), (hd, pos, theta, neox)


def test_rope_neox_identity_and_not_llama():
    """neox_pos0_es_identidad, neox_no_es_llama (gemm.rs:1547-1562)."""
    x = np.array([1.0, 2.0, 3.0, 4.0], np.float32)
    assert np.array_equal(oracle.rope_heads(x, 1, 4, 0, 10000.0, True), x)
    assert not np.array_equal(oracle.rope_heads(x, 1, 4, 3, 10000.0, False), oracle.rope_heads(x, 1, 4, 3, 10000.0, True))


def test_yarn_golden_vector():
    """yarn_neox_coincide_con_ggml (gemm.rs:1564-1589): the values the reference computed with
    ggml's rope_yarn formula, and the magnitude factor alone at position 0."""
    x = np.arange(1, 9, dtype=np.float32)
    got = oracle.rope_neox_yarn(x, 1, 8, 1, 10000.0, 4.0, 32, 32.0, 1.0)
    want = np.array([-4.17541405, 2.10577064, 3.39595164, 4.55224034, 4.03414418, 6.88656734, 7.97892086,
                     9.11017383], np.float32)
    assert float(np.max(np.abs(got - want))) < 1e-4
    m = F(1.0) + F(0.1) * np.log(F(16.0))
    z = np.array([3.0, -1.0, 0.5, 2.0], np.float32)
    got = oracle.rope_neox_yarn(z, 1, 4, 0, 500000.0, 16.0, 8192, 32.0, 1.0)
    assert float(np.max(np.abs(got - z * m))) < 1e-5
    # the divisor form the GPU rope takes (gm_rope with yarn_factores) gives the same values
    f, ms = oracle.yarn_factors(8, 10000.0, 4.0, 32, 32.0, 1.0)
    assert float(np.max(np.abs(oracle.rope_heads_div(x, 1, 8, 1, 10000.0, True, f, ms) - want))) < 1e-4


def test_topk_softmax_renormalises():
    """topk_softmax_renormaliza (moe.rs:145-153)."""
    idx, w = oracle.topk_softmax(np.array([1.0, 2.0, 3.0, 0.5], np.float32), 2)
    assert abs(float(w.sum()) - 1.0) < 1e-5 and idx[0] == 2 and idx.size == 2


def test_scalar_moe_ffn():
    """moe_ffn_referencia_escalar (moe.rs:240-272): h 4, ffn 8, two experts, top-1, constant
    f32 gate / up / down matrices; the oracle's MoE step against the test's own f32 steps."""
    h, ffn = 4, 8
    hidden = np.array([0.5, -0.25, 0.1, 0.0], np.float32)
    router = np.zeros((2, h), np.float32)
    router[0, 0], router[1, 1] = 1.0, 2.0
    gate = np.full((ffn, h), 0.01, np.float32)
    up = np.full((ffn, h), 0.02, np.float32)
    down = np.full((h, ffn), 0.03, np.float32)
    f32 = {k: 1 for k in ("ffn_gate_inp", "ffn_gate", "ffn_up", "ffn_down")}
    cfg = dataclasses.replace(decode.TINY_MOE_NS, n_layers=1, hidden=h, n_exp=2, top_k=1, moe_ffn=ffn,
                              dtypes=dict(decode.TINY_MOE_NS.dtypes, **f32))
    model = {"blk.0.ffn_gate_inp": router.view(np.uint8).ravel()}
    for e in range(2):
        model[f"blk.0.E{e:03d}.ffn_gate"] = gate.view(np.uint8).ravel()
        model[f"blk.0.E{e:03d}.ffn_up"] = up.view(np.uint8).ravel()
        model[f"blk.0.E{e:03d}.ffn_down"] = down.view(np.uint8).ravel()
    orc = DenseOracle(cfg, model)
    orc.route_gaps, orc.force_routes = [], None
    got = orc._moe("blk.0.", hidden, 0)
    # the reference test's steps
    lg = np.array([np.dot(router[i].astype(np.float32), hidden) for i in range(2)], np.float32)
    (e,), (w,) = oracle.topk_softmax(lg, 1)
    g = (gate @ hidden).astype(np.float32)
    u = (up @ hidden).astype(np.float32)
    act = (g / (F(1.0) + np.exp(-g)) * u).astype(np.float32)
    want = ((down @ act).astype(np.float32) * w).astype(np.float32)
    assert np.all(np.isfinite(got)) and float(np.max(np.abs(got - want))) < 1e-6


def _fill(shape, fill):
    """add_tensor (arch_ext.rs:19-41): fill + i * 1e-7, f32."""
    n = int(np.prod(shape))
    return (F(fill) + np.arange(n, dtype=np.float32) * F(1e-7)).astype(np.float32)


def test_mla_against_the_reference_mla_oracle():
    """mla_latent_rope_golden_parity (arch_ext.rs:531-592) with build_tiny_mla_parity's model
    (hidden 64, 2 heads, 1 kv head, head_dim 32 = qk_nope 16 + qk_rope 16, q / kv ranks 16,
    f32 weights, attn_output the identity): the oracle's MLA attention against
    mla_oracle_attn_out (arch_ext.rs:233-359) restated in f32, within 1e-4."""
    h, heads, kvh, hd, nope, rope, qr, kr = 64, 2, 1, 32, 16, 16, 16, 16
    eps, theta = 1e-5, 10000.0
    W = {"attn_q_down": _fill((qr, h), 0.1), "attn_q_up": _fill((h, qr), 0.1), "attn_kv_down": _fill((kr, h), 0.1),
         "attn_k_up": _fill((kvh * (nope + rope), kr), 0.1), "attn_v_up": _fill((kvh * hd, kr), 0.1),
         "attn_output": np.eye(h, dtype=np.float32).ravel(), "attn_norm": _fill((h,), 1.0)}
    cfg = decode.DenseConfig(n_layers=1, hidden=h, heads=heads, kv_heads=kvh, head_dim=hd, ffn=0, vocab=8, ctx=8,
                             theta=theta, eps=eps, neox=False, qkv_bias=False, mla=True, q_rank=qr, kv_rank=kr,
                             qk_nope=nope, qk_rope=rope, v_dim=hd, dtypes={k: 1 for k in W})
    model = {f"blk.0.{k}": (v.view(np.uint8).ravel() if k != "attn_norm" else v) for k, v in W.items()}
    orc = DenseOracle(cfg, model)

    def mv(name, rows, cols, x):
        return oracle.matvec(1, W[name].view(np.uint8), rows, cols, x)

    hidden = (F(0.01) * (np.arange(h, dtype=np.float32) + F(1.0))).astype(np.float32)
    for pos in range(3):
        hidden = (hidden + F(pos) * F(0.001)).astype(np.float32)
        xn = oracle.rmsnorm(hidden, W["attn_norm"], eps)
        got = orc._mla("blk.0.", xn, 0, pos)
        if pos == 0:
            continue
        # mla_oracle_attn_out, step by step
        q = mv("attn_q_up", h, qr, mv("attn_q_down", qr, h, xn))
        for hh in range(heads):
            b = hh * hd + nope
            q[b:b + rope] = oracle.rope_llama_n(q[b:b + rope], pos, theta, rope)
        inv = F(1.0) / np.sqrt(F(nope + rope))
        hist = [orc.k[0][t].view(np.float16).astype(np.float32) for t in range(pos + 1)]
        want = np.zeros(h, np.float32)
        for hh in range(heads):
            g, qh = hh // (heads // kvh), q[hh * hd:(hh + 1) * hd]
            lg = np.zeros(pos + 1, np.float32)
            for t in range(pos + 1):
                kf = mv("attn_k_up", kvh * (nope + rope), kr, hist[t])
                o = g * (nope + rope)
                kf[o + nope:o + nope + rope] = oracle.rope_llama_n(kf[o + nope:o + nope + rope], t, theta, rope)
                acc = F(0.0)
                for d in range(nope + rope):
                    acc = F(acc + qh[d] * kf[o + d])
                lg[t] = F(acc * inv)
            lg = np.exp(lg - lg.max()).astype(np.float32)
            lg = (lg / lg.sum(dtype=np.float32)).astype(np.float32)
            out = np.zeros(hd, np.float32)
            for t in range(pos + 1):
                vf = mv("attn_v_up", kvh * hd, kr, hist[t])
                out = (out + lg[t] * vf[g * hd:(g + 1) * hd]).astype(np.float32)
            want[hh * hd:(hh + 1) * hd] = out
        assert float(np.max(np.abs(got - want))) < 1e-4, pos
