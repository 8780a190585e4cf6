"""Whole-token decode engine (sb_decode_prepare / sb_decode_token / sb_decode_greedy)
against the CPU restatement of the reference's dense decode step (oracle/model.py).

Bars: identical greedy top-1 tokens over 64 decode
steps; logits within 1e-2 relative, here per logit |gpu - cpu| <= 1e-2 *
max(|cpu|, rms(cpu logits)).
"""
import numpy as np
import pytest

from oracle.model import DenseOracle
from soso_b200 import decode, synth

pytestmark = pytest.mark.gpu

LOGIT_REL = 1e-2


def logits_close(g, t):
    rms = float(np.sqrt(np.mean(t.astype(np.float64) ** 2)))
    err = np.abs(g.astype(np.float64) - t) / np.maximum(np.abs(t), rms)
    return float(err.max())


@pytest.fixture(scope="module")
def tiny():
    cfg = decode.TINY
    return cfg, decode.synth_model(cfg, "tiny")


def test_greedy_64_steps_match_oracle(gpu, tiny):
    cfg, model = tiny
    prompt = synth.rng("prompt", "tiny").integers(0, cfg.vocab, 16).astype(np.int32)
    sess = decode.DecodeSession(cfg, model)
    got = sess.greedy(prompt, 64)
    want, logits = DenseOracle(cfg, model).greedy(prompt, 64)
    gaps = [float(np.sort(lg)[-1] - np.sort(lg)[-2]) for lg in logits]
    assert np.array_equal(got, want), (np.nonzero(got != want)[0][:5], min(gaps))


def test_decode_token_logits_and_kv_rows(gpu, tiny):
    cfg, model = tiny
    sess = decode.DecodeSession(cfg, model)
    orc = DenseOracle(cfg, model)
    toks = synth.rng("toks", "tiny").integers(0, cfg.vocab, 12)
    for pos, t in enumerate(toks):
        e = orc.embed(int(t))
        lg, kv = sess.token(e, pos, kv_rows=True)
        want = orc.step(e, pos)
        assert logits_close(lg, want) <= LOGIT_REL
        # new K/V rows, layer order, [k | v] per layer (f16 bits), against the oracle's cache rows
        kvd = cfg.kv_dim
        for l in range(cfg.n_layers):
            k = kv[l * 2 * kvd:l * 2 * kvd + kvd].view(np.float16).astype(np.float32)
            v = kv[l * 2 * kvd + kvd:(l + 1) * 2 * kvd].view(np.float16).astype(np.float32)
            kt = orc.k[l][pos].view(np.float16).astype(np.float32)
            vt = orc.v[l][pos].view(np.float16).astype(np.float32)
            assert np.max(np.abs(k - kt)) <= 2e-3 * max(1.0, float(np.abs(kt).max()))
            assert np.max(np.abs(v - vt)) <= 2e-3 * max(1.0, float(np.abs(vt).max()))


@pytest.fixture(scope="module")
def tiny_yarn():
    cfg = decode.TINY_YARN
    return cfg, decode.synth_model(cfg, "tiny_yarn")


def test_yarn_greedy_and_logits_match_oracle(gpu, tiny_yarn):
    """YaRN layers: the engine applies the reference's GPU form (gm_rope with yarn_factores
    divisors), the oracle the reference's CPU form (rope_neox_yarn, layer.rs:1184-1189); the
    two agree to f32 rounding of the angles at these positions."""
    cfg, model = tiny_yarn
    # a prompt whose greedy chain has no near-tie (top-2 logit gaps >= 0.046 at logit rms 1.1):
    # the two RoPE forms differ by ~1e-5 relative, which a gap of ~1e-4 would not survive
    prompt = synth.rng("prompt", "tiny_yarn2").integers(0, cfg.vocab, 16).astype(np.int32)
    sess = decode.DecodeSession(cfg, model)
    try:
        got = sess.greedy(prompt, 40)
        want, logits = DenseOracle(cfg, model).greedy(prompt, 40)
        gaps = [float(np.sort(lg)[-1] - np.sort(lg)[-2]) for lg in logits]
        assert np.array_equal(got, want), (np.nonzero(got != want)[0][:5], min(gaps))
        orc = DenseOracle(cfg, model)
        for pos, t in enumerate(synth.rng("toks", "tiny_yarn").integers(0, cfg.vocab, 8)):
            e = orc.embed(int(t))
            assert logits_close(sess.token(e, pos), orc.step(e, pos)) <= LOGIT_REL, pos
    finally:
        sess.close()


def test_prepare_declines_unsupported_head_dim(gpu):
    cfg = decode.DenseConfig(n_layers=1, hidden=256, heads=4, kv_heads=2, head_dim=64, ffn=256, vocab=256, ctx=16)
    model = decode.synth_model(cfg, "hd64")
    with pytest.raises(decode.SbError, match="returned 0"):
        decode.DecodeSession(cfg, model)
