"""Block prefill on the tensor cores (sb_decode_prefill): a prompt through every layer at
once -- the reference's forward_layer_block path (crates/soso-llm-core/src/layer.rs:1433)
with its GPU offload (gpu.rs:443-530) -- against the CPU restatement of the reference's
decode run over the same tokens one at a time (oracle/model.py).

Bars: the last token's logits within 1e-2 relative (per logit
|gpu - cpu| <= 1e-2 x max(|cpu|, rms)); the K / V (or MLA latent) rows the block wrote
within 1e-2 of the rows' largest magnitude (the GEMMs take f16 operands, the reference's
prefill precision, so a row may differ from the decode step's by a few f16 steps); the
greedy continuation from the block's last position equal to the oracle's, except at a
top-1 / top-2 tie (gap below 1e-3 x rms).  Tiny models of the configs' structures: dense
GQA (Q4_K downs; Q6_K downs through the matvec fallback), MoE with and without a shared
expert (routed experts grouped by the device), MLA + MoE with Q8_0 downs.
"""
import dataclasses

import numpy as np
import pytest

import oracle
from oracle.model import DenseOracle
from soso_b200 import decode, synth
from soso_b200.formats import DTYPE_Q4_K, DTYPE_Q8_0

pytestmark = pytest.mark.gpu
LOGIT_REL, ROW_REL, TIE = 1e-2, 1e-2, 1e-3

_Q4 = {k: DTYPE_Q4_K for k in decode.TINY.dtypes}
CONFIGS = {
    "dense_q4k": dataclasses.replace(decode.TINY, dtypes=dict(_Q4), ctx=192),
    "dense_q6k_down": dataclasses.replace(decode.TINY, ctx=192),
    "moe_shared": dataclasses.replace(decode.TINY_MOE, dtypes=dict(decode.TINY_MOE_NS.dtypes), ctx=192),
    "moe": dataclasses.replace(decode.TINY_MOE_NS, ctx=192),
    "moe_f32_router": dataclasses.replace(decode.TINY_MOE_NS, ctx=192,
                                          dtypes=dict(decode.TINY_MOE_NS.dtypes, ffn_gate_inp=1)),
    "mla_moe": dataclasses.replace(decode.TINY_MLA, moe_ffn=256, ctx=192),
}


def _rel(g, t):
    t = np.asarray(t, np.float64)
    rms = float(np.sqrt(np.mean(t ** 2)))
    return float((np.abs(np.asarray(g, np.float64) - t) / np.maximum(np.abs(t), rms)).max())


def _gap(lg):
    top = np.partition(lg.astype(np.float64), -2)[-2:]
    return float(top[1] - top[0]) / float(np.sqrt(np.mean(lg.astype(np.float64) ** 2)))


@pytest.mark.parametrize("which", sorted(CONFIGS))
def test_prefill_matches_oracle(which):
    cfg = CONFIGS[which]
    model = decode.synth_model(cfg, "pf_" + which)
    prompt = synth.rng("pf_prompt", which).integers(0, cfg.vocab, 70).astype(np.int32)
    sess = decode.DecodeSession(cfg, model)
    try:
        lg, nxt = sess.prefill(prompt)
        orc = DenseOracle(cfg, model)
        for i, t in enumerate(prompt):
            want = orc.step(orc.embed(int(t)), i)
        assert _rel(lg, want) <= LOGIT_REL, which
        assert nxt == oracle.argmax(want) or _gap(want) < TIE
        # the cache rows the block wrote
        layers, _ = sess.download_state(len(prompt))
        for l, (k, v) in enumerate(layers):
            for got, ref in ((k, orc.k[l][:len(prompt)]), (v, None if v is None else orc.v[l][:len(prompt)])):
                if got is None:
                    continue
                g = got.view(np.float16).astype(np.float32)
                w = ref.view(np.float16).astype(np.float32)
                assert np.max(np.abs(g - w)) <= ROW_REL * max(1.0, float(np.abs(w).max())), (which, l)
        # greedy continuation from the block's last position
        m = 12
        got = sess.greedy(np.array([nxt], np.int32), m, pos=len(prompt))
        tok, gaps, toks = nxt, [], []
        for j in range(m):
            o = orc.step(orc.embed(int(tok)), len(prompt) + j)
            tok = oracle.argmax(o)
            toks.append(tok)
            gaps.append(_gap(o))
        diff = next((j for j in range(m) if got[j] != toks[j]), None)
        assert diff is None or gaps[diff] < TIE, (which, diff, gaps[diff] if diff is not None else None)
    finally:
        sess.close()


def test_prefill_after_decoded_tokens():
    """A block at pos0 > 0 (a prompt continued after decoded tokens): its queries attend the
    rows the decode steps wrote before it; its logits against the oracle run over all tokens."""
    cfg = CONFIGS["moe"]
    model = decode.synth_model(cfg, "pf_pos0")
    head = synth.rng("pf_pos0", "head").integers(0, cfg.vocab, 9).astype(np.int32)
    block = synth.rng("pf_pos0", "block").integers(0, cfg.vocab, 33).astype(np.int32)
    sess = decode.DecodeSession(cfg, model)
    try:
        sess.greedy(head, len(head))  # positions 0..8 through the decode step (argmaxes unused)
        lg, _ = sess.prefill(block, pos=len(head))
    finally:
        sess.close()
    orc = DenseOracle(cfg, model)
    for i, t in enumerate(np.concatenate([head, block])):
        want = orc.step(orc.embed(int(t)), i)
    assert _rel(lg, want) <= LOGIT_REL


def test_prefill_declines_what_it_does_not_take():
    """A plan whose expert downs are Q6_K (no GEMM form): declined, nothing launched."""
    cfg = dataclasses.replace(decode.TINY_MOE, ctx=96)  # ffn_down Q6_K
    sess = decode.DecodeSession(cfg, decode.synth_model(cfg, "pf_decline"))
    try:
        with pytest.raises(decode.SbError, match="returned 0"):
            sess.prefill(np.arange(8, dtype=np.int32))
    finally:
        sess.close()


@pytest.mark.parametrize("which,n", [("moe", 1), ("moe", 2), ("moe", 64), ("moe", 65), ("dense_q6k_down", 1),
                                     ("dense_q6k_down", 129), ("mla_moe", 1), ("mla_moe", 150), ("moe_shared", 191)])
def test_prefill_block_sizes(which, n):
    """Blocks of 1 token, of a tile width and one past it, and up to the context: the last
    token's logits against the oracle run over the same tokens one at a time."""
    cfg = CONFIGS[which]
    model = decode.synth_model(cfg, f"pf_n_{which}")
    prompt = synth.rng("pf_n", which, n).integers(0, cfg.vocab, n).astype(np.int32)
    sess = decode.DecodeSession(cfg, model)
    try:
        lg, nxt = sess.prefill(prompt)
    finally:
        sess.close()
    orc = DenseOracle(cfg, model)
    for i, t in enumerate(prompt):
        want = orc.step(orc.embed(int(t)), i)
    assert _rel(lg, want) <= LOGIT_REL, (which, n)
    assert nxt == oracle.argmax(want) or _gap(want) < TIE
