"""`moe_capa` (crates/soso-llm-core/src/gpu.rs:424-429, MoeCapa :294-335) through the C ABI
(sb_moe_layer): whole Qwen3-MoE-style layers of a block on the device -- attention with
QK-norm and NeoX RoPE over the layer's KV cache held on the device, f32 router, top-k, the
experts' SwiGLU -- against the CPU restatement of the reference's layer (oracle/model.py:
the GQA block, layer.rs:1088-1296, and forward_moe_ffn, :1938-2109) run one token at a
time over the same rows.

Bars: the layer's output rows against the oracle's, every element within 2e-2 of the rms of
the layer's contribution (output - input) and the rms relative error of that contribution
under 5e-3 (the block path takes f16 operands, the reference's prefill precision).  A
token whose top-k is a router near-tie (the oracle's k-th / (k+1)-th logit gap below 1e-2)
may route either way and is left out of the comparison; in a single layer that changes only
its own row.

Also: a second block continues from the KV rows the first one left on the device; a
rewind to position 0 gives the first block's rows again, bit for bit; two layers chained
on the device (encadenar / continuar) equal the two run one after the other; moe_volcar
brings a pending output down; a sliding-window layer is declined and not tried again.
"""
import dataclasses

import numpy as np
import pytest

import oracle
from oracle.model import DenseOracle
from soso_b200 import decode, synth
from soso_b200.dispatch import CudaGpu, MoeCapa, MoeNormas, TensorView
from soso_b200.formats import DTYPE_F32, row_bytes

pytestmark = pytest.mark.gpu
CFG = dataclasses.replace(decode.TINY_MOE_NS, n_layers=2, ctx=128,
                          dtypes=dict(decode.TINY_MOE_NS.dtypes, ffn_gate_inp=DTYPE_F32))
ROUTE_TIE = 1e-2


@pytest.fixture(scope="module")
def setup():
    cfg = CFG
    model = decode.synth_model(cfg, "moe_capa")
    gpu = CudaGpu.nueva()
    H, qd, kvd = cfg.hidden, cfg.q_dim, cfg.kv_dim

    def up(key, src, rows, cols, kind):
        dt = cfg.dtypes[kind]
        arr = np.ascontiguousarray(model[src]).view(np.uint8).reshape(-1)
        assert arr.size == rows * row_bytes(dt, cols)
        assert gpu.gemma_subir(key, TensorView(arr, dt, rows * cols), rows, cols)

    for l in range(cfg.n_layers):
        p, k = f"blk.{l}.", f"L{l:02d}."
        up(k + "attn_q", p + "attn_q", qd, H, "attn_q")
        up(k + "attn_k", p + "attn_k", kvd, H, "attn_k")
        up(k + "attn_v", p + "attn_v", kvd, H, "attn_v")
        up(k + "attn_output", p + "attn_output", H, qd, "attn_output")
        for e in range(cfg.n_exp):
            for kind, rows, cols in (("ffn_gate", cfg.moe_ffn, H), ("ffn_up", cfg.moe_ffn, H),
                                     ("ffn_down", H, cfg.moe_ffn)):
                up(f"{k}E{e:02d}.{kind}", f"{p}E{e:03d}.{kind}", rows, cols, kind)
    yield cfg, model, gpu
    gpu.close()


def _f32(a):
    a = np.ascontiguousarray(a)
    return a.view(np.float32) if a.dtype == np.uint8 else a.astype(np.float32)


def _capa(cfg, model, layer, pos0, hidden, normas=True, src=None, **kw):
    p = f"blk.{layer if src is None else src}."
    nm = MoeNormas(model[p + "attn_norm"], model[p + "attn_q_norm"], model[p + "attn_k_norm"], model[p + "ffn_norm"],
                   _f32(model[p + "ffn_gate_inp"])) if normas else None
    args = dict(layer=layer, pos0=pos0, n=hidden.shape[0], hidden=hidden, h=cfg.hidden, heads=cfg.heads,
                kv_heads=cfg.kv_heads, head_dim=cfg.head_dim, ffn=cfg.moe_ffn, n_exp=cfg.n_exp, top_k=cfg.top_k,
                ventana=0, ctx_max=cfg.ctx, eps=cfg.eps, theta=cfg.theta,
                escala=float(np.float32(1.0) / np.sqrt(np.float32(cfg.head_dim))), qk_norm=True, rope_mscale=1.0,
                continuar=False, encadenar=False, clave_q=f"L{layer:02d}.attn_q", clave_k=f"L{layer:02d}.attn_k",
                clave_v=f"L{layer:02d}.attn_v", clave_o=f"L{layer:02d}.attn_output", prefijo=f"L{layer:02d}",
                normas=nm, flujo=None)
    args.update(kw)
    return MoeCapa(**args)


class _Ref:
    """The oracle's layer l over rows at consecutive positions (its own KV cache)."""

    def __init__(self, cfg, model):
        self.cfg, self.m = cfg, model
        self.orc = DenseOracle(cfg, model)

    def layer(self, l, rows, pos0):
        o, cfg, p = self.orc, self.cfg, f"blk.{l}."
        out, gaps = np.empty_like(rows), []
        for t in range(rows.shape[0]):
            h = o._gqa(p, rows[t].astype(np.float32), l, pos0 + t)
            xn = oracle.rmsnorm(h, self.m[p + "ffn_norm"], cfg.eps)
            o.force_routes, o.route_gaps = None, []
            out[t] = (h + o._moe(p, xn, l)).astype(np.float32)
            gaps.append(o.route_gaps[-1])
        return out, np.asarray(gaps)


def _check(got, want, inp, gaps):
    keep = gaps >= ROUTE_TIE
    assert keep.sum() >= 0.8 * len(gaps)
    d_want = (want - inp).astype(np.float64)[keep]
    d_got = (got - inp).astype(np.float64)[keep]
    rms = np.sqrt(np.mean(d_want ** 2, axis=1, keepdims=True))
    assert float((np.abs(d_got - d_want) / rms).max()) <= 2e-2
    assert float(np.sqrt(np.sum((d_got - d_want) ** 2) / np.sum(d_want ** 2))) < 5e-3


def test_moe_capa_two_blocks_and_rewind(setup):
    cfg, model, gpu = setup
    g = synth.rng("moe_capa", "rows")
    a = g.standard_normal((40, cfg.hidden)).astype(np.float32)
    b = g.standard_normal((24, cfg.hidden)).astype(np.float32)
    ref = _Ref(cfg, model)
    want_a, gaps_a = ref.layer(0, a, 0)
    want_b, gaps_b = ref.layer(0, b, 40)
    ha = a.copy()
    assert gpu.moe_capa(_capa(cfg, model, 0, 0, ha))
    assert gpu.moe_lista(0)
    hb = b.copy()
    capa = _capa(cfg, model, 0, 40, hb, normas=False)
    assert gpu.moe_capa(capa) and capa.expulsadas == 0
    _check(ha, want_a, a, gaps_a)
    _check(hb, want_b, b, gaps_b)
    # back to position 0: the first block again, the same rows
    ha2 = a.copy()
    assert gpu.moe_capa(_capa(cfg, model, 0, 0, ha2, normas=False))
    assert np.array_equal(ha2, ha)


def test_moe_capa_chained_layers(setup):
    cfg, model, gpu = setup
    g = synth.rng("moe_capa", "chain")
    x = g.standard_normal((33, cfg.hidden)).astype(np.float32)
    # one after the other, through the host
    h0 = x.copy()
    assert gpu.moe_capa(_capa(cfg, model, 0, 0, h0))
    h1 = h0.copy()
    assert gpu.moe_capa(_capa(cfg, model, 1, 0, h1))
    # chained: layer 0's output stays on the device, layer 1 continues from it
    hc = x.copy()
    assert gpu.moe_capa(_capa(cfg, model, 0, 0, hc, encadenar=True))
    assert np.array_equal(hc, x)  # not written
    assert gpu.moe_pendiente(0, 0, 33) and not gpu.moe_pendiente(0, 0, 32)
    assert gpu.moe_capa(_capa(cfg, model, 1, 0, hc, normas=False, continuar=True))
    assert not gpu.moe_pendiente(1, 0, 33)
    assert np.array_equal(hc, h1)
    # a chained output brought down by moe_volcar
    hv = x.copy()
    assert gpu.moe_capa(_capa(cfg, model, 0, 0, hv, normas=False, encadenar=True))
    out = np.zeros_like(x)
    gpu.moe_volcar(out)
    assert np.array_equal(out, h0)
    assert not gpu.moe_pendiente(0, 0, 33)
    # against the oracle: layer 0 on x, layer 1 on the device's layer-0 rows
    ref = _Ref(cfg, model)
    w0, g0 = ref.layer(0, x, 0)
    w1, g1 = ref.layer(1, h0, 0)
    _check(h0, w0, x, g0)
    _check(h1, w1, h0, g1)


def test_moe_capa_declines_sliding_window(setup):
    cfg, model, gpu = setup
    h = np.zeros((4, cfg.hidden), np.float32)
    capa = _capa(cfg, model, 7, 0, h, src=0, ventana=64, clave_q="L00.attn_q", clave_k="L00.attn_k", clave_v="L00.attn_v",
                 clave_o="L00.attn_output", prefijo="L00")
    assert gpu.moe_puede(7)
    assert not gpu.moe_capa(capa)
    assert not gpu.moe_puede(7)
    assert not gpu.moe_capa(capa)


@pytest.mark.parametrize("n", [1, 3, 100])
def test_moe_capa_block_sizes(setup, n):
    """One token, a few, and most of the context in a block, then one more token after it."""
    cfg, model, gpu = setup
    g = synth.rng("moe_capa", "n", n)
    a = g.standard_normal((n, cfg.hidden)).astype(np.float32)
    b = g.standard_normal((1, cfg.hidden)).astype(np.float32)
    ref = _Ref(cfg, model)
    want_a, gaps_a = ref.layer(1, a, 0)
    want_b, gaps_b = ref.layer(1, b, n)
    ha, hb = a.copy(), b.copy()
    assert gpu.moe_capa(_capa(cfg, model, 1, 0, ha))
    assert gpu.moe_capa(_capa(cfg, model, 1, n, hb, normas=False))
    if (gaps_a >= ROUTE_TIE).any():
        _check(ha[gaps_a >= ROUTE_TIE], want_a[gaps_a >= ROUTE_TIE], a[gaps_a >= ROUTE_TIE], gaps_a[gaps_a >= ROUTE_TIE])
    if gaps_b[0] >= ROUTE_TIE:
        _check(hb, want_b, b, gaps_b)
