"""MoE decode on the whole-token engine (router matvec, on-device top-k routing, expert
gate/up and down launches over device-side batches, weighted combine folded into the
next norm) against the CPU restatement of forward_moe_ffn (oracle/model.py,
crates/soso-llm-core/src/layer.rs:1862-2109).

Bars: identical greedy top-1 tokens over 64 decode steps;
logits within 1e-2 relative (per logit, |gpu - cpu| <= 1e-2 * max(|cpu|, rms)).
"""
import numpy as np
import pytest

from oracle.model import DenseOracle
from soso_b200 import decode, synth

pytestmark = pytest.mark.gpu
LOGIT_REL = 1e-2


def logits_close(g, t):
    rms = float(np.sqrt(np.mean(t.astype(np.float64) ** 2)))
    return float((np.abs(g.astype(np.float64) - t) / np.maximum(np.abs(t), rms)).max())


@pytest.fixture(scope="module", params=["TINY_MOE", "TINY_MOE_NS", "TINY_MOE_F32_ROUTER"])
def moe_model(request):
    if request.param == "TINY_MOE_F32_ROUTER":
        # the router in f32, as the reference keeps ffn_gate_inp (its router matvec runs in f32)
        import dataclasses
        from soso_b200.formats import DTYPE_F32
        cfg = dataclasses.replace(decode.TINY_MOE, dtypes=dict(decode.TINY_MOE.dtypes, ffn_gate_inp=DTYPE_F32))
    else:
        cfg = getattr(decode, request.param)
    return cfg, decode.synth_model(cfg, request.param.lower())


def test_moe_greedy_64_steps_match_oracle(gpu, moe_model):
    cfg, model = moe_model
    prompt = synth.rng("prompt", "moe").integers(0, cfg.vocab, 12).astype(np.int32)
    sess = decode.DecodeSession(cfg, model)
    try:
        got = sess.greedy(prompt, 64)
    finally:
        sess.close()
    want, logits = DenseOracle(cfg, model).greedy(prompt, 64)
    gaps = [float(np.sort(lg)[-1] - np.sort(lg)[-2]) for lg in logits]
    assert np.array_equal(got, want), (np.nonzero(got != want)[0][:5], min(gaps))


def test_moe_decode_token_logits(gpu, moe_model):
    cfg, model = moe_model
    sess = decode.DecodeSession(cfg, model)
    orc = DenseOracle(cfg, model)
    try:
        for pos, t in enumerate(synth.rng("toks", "moe").integers(0, cfg.vocab, 10)):
            e = orc.embed(int(t))
            lg = sess.token(e, pos)
            assert logits_close(lg, orc.step(e, pos)) <= LOGIT_REL, pos
    finally:
        sess.close()


def test_route_trace_per_position(gpu, moe_model):
    """sb_decode_route_trace: the experts each MoE layer chose at every decode position, and the
    router-logit gap between the k-th choice and the next expert, against the oracle's router
    (topk_softmax, gemm.rs:62-91) teacher forced on the same tokens: the same experts wherever
    the oracle's gap is not a near-tie, gaps within 1e-3; the last position's trace equals
    sb_decode_routes."""
    cfg, model = moe_model
    sess = decode.DecodeSession(cfg, model)
    orc = DenseOracle(cfg, model)
    toks = synth.rng("toks", "moe_trace").integers(0, cfg.vocab, 12)
    try:
        want = []
        for pos, t in enumerate(toks):
            e = orc.embed(int(t))
            sess.token(e, pos)
            orc.step(e, pos)
            want.append(list(orc.route_gaps))
        last = sess.routes()
        for pos in range(len(toks)):
            ids, gaps = sess.route_trace(pos)
            moe = sorted(ids)
            assert len(moe) == len(want[pos])
            for i, l in enumerate(moe):
                assert abs(gaps[l] - want[pos][i]) <= 1e-3, (pos, l, gaps[l], want[pos][i])
                assert gaps[l] >= 0.0
            if pos == len(toks) - 1:
                for l in moe:
                    assert np.array_equal(ids[l], last[l])
    finally:
        sess.close()
