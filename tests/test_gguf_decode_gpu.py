"""A GGUF checkpoint decoded on the GPU: the synthetic tiny models written as GGUF (llama
layout with Q6_K downs and output, which the reference's conversion turns into Q8_0; and
kept as Q6_K, which this backend also runs; qwen3moe with its experts in 3-D tensors),
loaded by soso_b200.gguf and decoded by DecodeSession, against the oracle model on the same
converted tensors: 48 greedy tokens equal except at a top-1 / top-2 tie."""
import dataclasses

import numpy as np
import pytest

from oracle.model import DenseOracle
from soso_b200 import decode, gguf, synth
from tests._gguf import model_to_gguf

pytestmark = pytest.mark.gpu


def _gap(lg):
    top = np.partition(lg.astype(np.float64), -2)[-2:]
    return float(top[1] - top[0]) / float(np.sqrt(np.mean(lg.astype(np.float64) ** 2)))


@pytest.mark.parametrize("which,arch,keep", [("TINY", "llama", False), ("TINY", "llama", True),
                                            ("TINY_MOE_NS", "qwen3moe", False)])
def test_decode_a_gguf(tmp_path, which, arch, keep):
    cfg0 = dataclasses.replace(getattr(decode, which), neox=arch != "llama",
                               qkv_bias=False if arch == "llama" else getattr(decode, which).qkv_bias)
    path = str(tmp_path / "m.gguf")
    model_to_gguf(path, cfg0, decode.synth_model(cfg0, "ggufdec_" + which), arch)
    cfg, tensors, g = gguf.load_gguf_model(path, keep_q6k=keep)
    try:
        prompt = synth.rng("ggufdec", which).integers(0, cfg.vocab, 24).astype(np.int32)
        sess = decode.DecodeSession(cfg, tensors)
        try:
            got = sess.greedy(prompt, 48)
        finally:
            sess.close()
        want, logits = DenseOracle(cfg, tensors).greedy(prompt, 48)
        diff = next((i for i in range(48) if got[i] != want[i]), None)
        assert diff is None or _gap(logits[diff]) < 1e-3, (which, keep, diff)
    finally:
        g.close()
