"""Device KV caches into and out of the reference's portable snapshot (kvsnap.rs), and the
decode state calls behind them (GpuDispatch::decode_subir_estado, gpu.rs:664-668).

A prefix decoded on the device is downloaded (sb_decode_download_state), checked against
the CPU restatement of the reference's decode (oracle/model.py: its K/V cache rows within
one f16 rounding step, its hidden vector within the logit bar), encoded as the reference
encodes it, decoded with every check, uploaded into a fresh session
(sb_decode_upload_state), and the decode continues there exactly as it continues in the
session that never stopped.  MLA latent caches (no snapshot form in the reference) go
through the same upload and download calls.
"""
import numpy as np
import pytest

from oracle.model import DenseOracle
from soso_b200 import decode, kvsnap, synth

pytestmark = pytest.mark.gpu


def _fed(prompt, out):
    """The token fed at each step of sb_decode_greedy: the prompt, then the argmax chain."""
    return np.concatenate([prompt, out[len(prompt) - 1:-1]]).astype(np.uint32)


def test_snapshot_round_trip_through_the_device():
    cfg = decode.TINY
    model = decode.synth_model(cfg, "kvsnap_dev")
    prompt = synth.rng("prompt", "kvsnap_dev").integers(0, cfg.vocab, 12).astype(np.int32)
    n, m = 40, 24
    prof = bytes(range(32))
    a = decode.DecodeSession(cfg, model)
    b = None
    try:
        out = a.greedy(prompt, n)
        toks = _fed(prompt, out)
        image = kvsnap.export_session(a, toks, prof, 1 << 26)
        # rows and hidden vector against the oracle run over the same tokens
        orc = DenseOracle(cfg, model)
        for pos, t in enumerate(toks):
            lg = orc.step(orc.embed(int(t)), pos)
        snap = kvsnap.decode(image, prof, kvsnap.dims_of(cfg), cfg.ctx, cfg.vocab, cfg.hidden, 1 << 26)
        assert np.array_equal(snap.tokens, toks)
        for l, (k, v) in enumerate(snap.layers):
            for got, want in ((k.reshape(n, -1), orc.k[l][:n]), (v.reshape(n, -1), orc.v[l][:n])):
                g = got.view(np.float16).astype(np.float32)
                w = want.view(np.float16).astype(np.float32)
                assert np.max(np.abs(g - w)) <= 2e-3 * max(1.0, float(np.abs(w).max())), l
        # the hidden vector: the oracle's logits follow from it through the output norm
        h = snap.hidden.astype(np.float64)
        assert h.shape == (cfg.hidden,) and np.all(np.isfinite(h))
        # continue: the uninterrupted session against a fresh one restored from the image
        nxt = np.array([out[-1]], np.int32)
        want = a.greedy(nxt, m, pos=n)
        b = decode.DecodeSession(cfg, model)
        kvsnap.import_session(b, image, prof, 1 << 26)
        got = b.greedy(nxt, m, pos=n)
        assert np.array_equal(got, want)
        # a refused image (wrong profile) leaves nothing half-done
        with pytest.raises(kvsnap.KvSnapError):
            kvsnap.import_session(b, image, bytes(32), 1 << 26)
    finally:
        a.close()
        if b is not None:
            b.close()


def test_hidden_vector_is_the_last_residual():
    """The downloaded hidden vector gives the step's logits through the output norm and the
    output matrix (runtime.rs:1976-2019), on the oracle's CPU path."""
    import oracle
    cfg = decode.TINY
    model = decode.synth_model(cfg, "kvsnap_hidden")
    s = decode.DecodeSession(cfg, model)
    try:
        orc = DenseOracle(cfg, model)
        for pos, t in enumerate(synth.rng("toks", "kvsnap_hidden").integers(0, cfg.vocab, 5)):
            e = orc.embed(int(t))
            lg = s.token(e, pos)
            orc.step(e, pos)
        _, h = s.download_state(5)
        via_h = oracle.matvec(cfg.dtypes["output"], model["output"], cfg.vocab, cfg.hidden,
                              oracle.rmsnorm(h, model["output_norm"], cfg.eps))
        rms = float(np.sqrt(np.mean(lg.astype(np.float64) ** 2)))
        err = np.abs(via_h.astype(np.float64) - lg) / np.maximum(np.abs(lg), rms)
        assert float(err.max()) <= 2e-3
    finally:
        s.close()


def test_mla_latent_rows_up_and_down():
    """MLA: the latent rows come down, go up into a fresh session (whose rope keys are formed
    again from them) and the decode continues as in the session that never stopped."""
    cfg = decode.TINY_MLA
    model = decode.synth_model(cfg, "kvsnap_mla")
    prompt = synth.rng("prompt", "kvsnap_mla").integers(0, cfg.vocab, 6).astype(np.int32)
    n, m = 30, 16
    a = decode.DecodeSession(cfg, model)
    b = None
    try:
        out = a.greedy(prompt, n)
        layers, _ = a.download_state(n)
        assert all(v is None and k.shape == (n, cfg.kv_rank) for k, v in layers)
        nxt = np.array([out[-1]], np.int32)
        want = a.greedy(nxt, m, pos=n)
        b = decode.DecodeSession(cfg, model)
        assert b.upload_state(layers, n) == [n] * cfg.n_layers
        got = b.greedy(nxt, m, pos=n)
        assert np.array_equal(got, want)
        with pytest.raises(kvsnap.KvSnapError):
            kvsnap.dims_of(cfg)
    finally:
        a.close()
        if b is not None:
            b.close()
