"""GGUF checkpoints through the reference's GGUF -> .som conversion rules (soso_b200/gguf.py,
crates/gguf2som/src/lib.rs), on the CPU.

Pinned on the reference's own converter tests (lib.rs tests module): f16 conversions
(`f16_conversion`), a Q4_K superblock passed through byte for byte and an all-(-32) Q6_K
block with d = 1/32 arriving as Q8_0 values of -1.0 (`q4k_passthrough_y_q6k_a_q8`), Q4_0
passed through and refused when not a whole number of blocks (`q4_0_pasa_tal_cual`).
Then whole models: the synthetic dense (llama / qwen2 layouts), MoE (qwen3moe, experts in
one 3-D tensor) configurations written as GGUF come back as the same DenseConfig and the
same weight bytes; Q6_K matrices converted to Q8_0 as gguf2som converts them (within half
a Q8_0 step of the Q6_K values), or kept as Q6_K on request; GGML Q8_0 repacked to .som
Q8_0 exactly."""
import dataclasses
import struct

import numpy as np
import pytest

from soso_b200 import decode, gguf
from soso_b200.formats import DTYPE_F32, DTYPE_Q4_K, DTYPE_Q6_K, DTYPE_Q8_0
from tests._gguf import model_to_gguf, write_gguf

FIELDS = ("n_layers", "hidden", "heads", "kv_heads", "head_dim", "ffn", "vocab", "ctx", "neox", "qkv_bias",
          "qk_norm", "n_exp", "top_k", "moe_ffn", "first_moe")


def _deq_q80(b: np.ndarray) -> np.ndarray:
    b = b.reshape(-1, 36)
    return (b[:, 4:].view(np.int8).astype(np.float32) * b[:, :4].copy().view(np.float32)).reshape(-1)


def test_f16_conversion_reference_cases():
    f = lambda bits: gguf._f16_to_f32(np.array([bits], np.uint16).view(np.uint8))[0]  # noqa: E731
    assert f(0) == 0.0 and f(0x3C00) == 1.0 and f(0xBC00) == -1.0 and f(0x3800) == 0.5
    assert np.isinf(f(0x7C00)) and np.isnan(f(0x7E00))
    assert f(0x0001) == np.float32(2.0 ** -24)


def test_q4k_passthrough_and_q6k_to_q8_reference_case():
    q4 = np.array([(i * 13) % 251 for i in range(144)], np.uint8)
    out, dt = gguf.convert_tensor(gguf.GGML_Q4_K, q4, 256)
    assert dt == DTYPE_Q4_K and np.array_equal(out, q4)
    q6 = np.zeros(210, np.uint8)
    q6[192:208] = 1
    q6[208:210] = np.array([1.0 / 32.0], np.float16).view(np.uint8)
    out6, dt6 = gguf.convert_tensor(gguf.GGML_Q6_K, q6, 256)
    assert dt6 == DTYPE_Q8_0
    vals = _deq_q80(out6)
    assert vals.size == 256 and np.all(np.abs(vals + 1.0) < 0.02)
    kept, dtk = gguf.convert_tensor(gguf.GGML_Q6_K, q6, 256, keep_q6k=True)
    assert dtk == DTYPE_Q6_K and np.array_equal(kept, q6)


def test_q4_0_passthrough_reference_case():
    b = np.array([(i * 29) % 253 for i in range(3 * 18)], np.uint8)
    out, dt = gguf.convert_tensor(gguf.GGML_Q4_0, b, 96)
    assert dt == gguf.DTYPE_Q4_0 and np.array_equal(out, b)
    with pytest.raises(gguf.GgufError):
        gguf.convert_tensor(gguf.GGML_Q4_0, b, 33)


def test_q8_0_repack_f16_and_q5_0():
    g = np.random.default_rng(1)
    blk = np.empty((4, 34), np.uint8)
    blk[:, :2] = g.uniform(0.01, 0.1, 4).astype(np.float16).view(np.uint8).reshape(4, 2)
    blk[:, 2:] = g.integers(-127, 128, (4, 32)).astype(np.int8).view(np.uint8)
    out, dt = gguf.convert_tensor(gguf.GGML_Q8_0, blk.reshape(-1), 128)
    assert dt == DTYPE_Q8_0
    o = out.reshape(4, 36)
    assert np.array_equal(o[:, 4:], blk[:, 2:])
    assert np.array_equal(o[:, :4].copy().view(np.float32).ravel(), blk[:, :2].copy().view(np.float16).astype(np.float32).ravel())
    h = g.standard_normal(40).astype(np.float16)
    out, dt = gguf.convert_tensor(gguf.GGML_F16, h.view(np.uint8), 40)
    assert dt == DTYPE_F32 and np.array_equal(out.view(np.float32), h.astype(np.float32))
    # Q5_0: codes 0..31 with the fifth bit from qh; d * (q - 16), then Q8_0 again
    q5 = np.zeros(22, np.uint8)
    q5[0:2] = np.array([0.5], np.float16).view(np.uint8)
    q5[2:6] = np.array([0xFFFF0000], "<u4").view(np.uint8)  # the fifth bit on for elements 16..31
    q5[6:22] = np.arange(16, dtype=np.uint8) | (np.arange(16, dtype=np.uint8) << 4)
    f = gguf.dequant_q5_0(q5, 1)
    want = np.array([(j - 16) * 0.5 for j in range(16)] + [(j + 16 - 16) * 0.5 for j in range(16)], np.float32)
    assert np.array_equal(f, want)


def test_quantize_q8_0_rounds_half_away_from_zero():
    v = np.zeros(32, np.float32)
    v[0], v[1], v[2] = 127.0, 2.5, -2.5  # scale 1: 2.5 -> 3, -2.5 -> -3 (roundf, not round-half-even)
    q = gguf.quantize_q8_0(v).reshape(36)
    assert q[:4].copy().view(np.float32)[0] == 1.0
    assert q[4:].view(np.int8)[:3].tolist() == [127, 3, -3]
    z = gguf.quantize_q8_0(np.zeros(40, np.float32))  # last block padded; zero blocks scale 1
    assert z.size == 72 and z[:4].copy().view(np.float32)[0] == 1.0


@pytest.mark.parametrize("which,arch", [("TINY", "llama"), ("TINY_QWEN2", "qwen2"), ("TINY_MOE_NS", "qwen3moe")])
def test_model_round_trip(tmp_path, which, arch):
    if which == "TINY_QWEN2":
        cfg = dataclasses.replace(decode.TINY, qkv_bias=True)
    elif arch == "llama":  # gguf2som takes q / k / v biases from qwen2 files only (lib.rs:673-680)
        cfg = dataclasses.replace(decode.TINY, qkv_bias=False)
    else:
        cfg = getattr(decode, which)
    cfg = dataclasses.replace(cfg, neox=arch != "llama")
    model = decode.synth_model(cfg, "gguf_" + which)
    path = str(tmp_path / "m.gguf")
    model_to_gguf(path, cfg, model, arch)
    got, t, g = gguf.load_gguf_model(path, keep_q6k=True)
    try:
        for f in FIELDS:
            assert getattr(got, f) == getattr(cfg, f), f
        assert abs(got.theta - cfg.theta) <= 1e-6 * cfg.theta and abs(got.eps - cfg.eps) <= 1e-6 * cfg.eps
        assert set(t) == set(model)
        for k, v in model.items():
            assert np.array_equal(np.asarray(t[k]).view(np.uint8), np.asarray(v).view(np.uint8)), k
        for k, v in got.dtypes.items():
            assert cfg.dtypes[k] == v, k
    finally:
        g.close()


def test_q6k_matrices_converted_as_gguf2som_does(tmp_path):
    cfg = decode.TINY  # Q6_K ffn_down and output
    model = decode.synth_model(cfg, "gguf_q6")
    path = str(tmp_path / "m.gguf")
    model_to_gguf(path, cfg, model, "llama")
    got, t, g = gguf.load_gguf_model(path)
    try:
        assert got.dtypes["ffn_down"] == DTYPE_Q8_0 and got.dtypes["output"] == DTYPE_Q8_0
        src = np.asarray(model["blk.0.ffn_down"]).view(np.uint8)
        want = gguf.dequant_q6_k(src, src.size // 210)
        have = _deq_q80(t["blk.0.ffn_down"])
        scale = np.repeat(t["blk.0.ffn_down"].reshape(-1, 36)[:, :4].copy().view(np.float32).ravel(), 32)
        assert np.all(np.abs(have - want) <= (0.5 + 1e-5) * scale)  # half a step, f32 rounding of v / scale
    finally:
        g.close()


def test_malformed_files(tmp_path):
    p = tmp_path / "bad.gguf"
    p.write_bytes(b"GGUX" + b"\0" * 40)
    with pytest.raises(gguf.GgufError):
        gguf.GgufFile(str(p))
    p.write_bytes(b"GGUF" + struct.pack("<IQQ", 1, 0, 0))
    with pytest.raises(gguf.GgufError):
        gguf.GgufFile(str(p))
    p.write_bytes(b"GGUF" + struct.pack("<IQQ", 3, 1, 0))  # a tensor announced, none written
    with pytest.raises(gguf.GgufError):
        gguf.GgufFile(str(p))
    write_gguf(str(p), {"general.architecture": "deepseek2"}, [])
    with pytest.raises(gguf.GgufError, match="MLA"):
        gguf.load_gguf_model(str(p))
