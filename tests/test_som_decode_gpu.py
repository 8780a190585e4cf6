"""Decoding a model directory in the reference's layout on the GPU: the directory is written
with the reference's writers restated (manifest, index, shards; tests/test_som_load.py),
read back by soso_b200.som_load (zero-copy views of the mapped shards), and decoded by the
whole-token engine (a 24-token prompt, then the greedy chain, all on the device) against the
CPU restatement of the reference's decode run over the same loaded tensors.

Bars: identical greedy tokens except at a top-1 / top-2 tie (gap below 1e-3 x rms), logits
within 1e-2 relative."""
import dataclasses

import numpy as np
import pytest

import oracle
from oracle.model import DenseOracle
from soso_b200 import decode, synth
from soso_b200.som_load import load_decode_model
from tests.test_som_load import write_model

pytestmark = pytest.mark.gpu


def _gap(lg):
    top = np.partition(lg.astype(np.float64), -2)[-2:]
    return float(top[1] - top[0]) / float(np.sqrt(np.mean(lg.astype(np.float64) ** 2)))


@pytest.mark.parametrize("which", ["TINY", "TINY_MOE_NS", "TINY_MLA"])
def test_decode_a_model_directory(tmp_path, which):
    cfg0 = getattr(decode, which)
    if cfg0.mla:
        cfg0 = dataclasses.replace(cfg0, head_dim=cfg0.hidden // cfg0.heads)
    # a head width other than hidden / heads travels in the layer spec's v_dim, as gguf2som
    # writes it for such models (crates/gguf2som/src/lib.rs:804-808)
    vd = cfg0.head_dim if not cfg0.mla and cfg0.head_dim != cfg0.hidden // cfg0.heads else None
    write_model(tmp_path, cfg0, decode.synth_model(cfg0, "somdec_" + which), n_shared=1 if cfg0.shared_ffn else 0,
                v_dim=vd)
    cfg, tensors, m = load_decode_model(str(tmp_path))
    try:
        prompt = synth.rng("somdec", which).integers(0, cfg.vocab, 24).astype(np.int32)
        sess = decode.DecodeSession(cfg, tensors)
        try:
            got = sess.greedy(prompt, 48)
        finally:
            sess.close()
        want, logits = DenseOracle(cfg, tensors).greedy(prompt, 48)
        diff = next((i for i in range(48) if got[i] != want[i]), None)
        assert diff is None or _gap(logits[diff]) < 1e-3, (which, diff)
    finally:
        m.close()
