"""The oracle's YaRN RoPE restatements against each other (CPU only).

The reference's tests hold no YaRN values, so YaRN parity is unpinned; what is checked is
the reference's own claim that the per-frequency divisors of yarn_factores
(crates/soso-llm-core/src/gemm.rs:1412-1428), applied the way its GPU rope applies them
(gm_rope, lxdde/ports/nouveau/gemma_capa.cu:99-125), reproduce its CPU YaRN
(rope_neox_yarn, gemm.rs:1372-1410).  The two compute the angle differently (a product
with a divided frequency vs repeated multiplication), so they agree to f32 rounding of
angles of up to pos radians: the check stays at positions below 64 (angle error ~1e-5).
"""
import numpy as np
import pytest

import oracle

# Mellum's YaRN (manifest v8: factor 16 over an 8192 original context) and a milder one
SPECS = [(16.0, 8192, 32.0, 1.0, 1e4), (4.0, 32768, 32.0, 1.0, 1e6)]


@pytest.mark.parametrize("factor,orig_ctx,beta_fast,beta_slow,theta", SPECS)
@pytest.mark.parametrize("pos", [0, 1, 7, 37, 63])
def test_divisor_form_reproduces_cpu_yarn(factor, orig_ctx, beta_fast, beta_slow, theta, pos):
    hd, heads = 128, 4
    x = np.random.default_rng(pos).standard_normal(heads * hd).astype(np.float32)
    want = oracle.rope_neox_yarn(x, heads, hd, pos, theta, factor, orig_ctx, beta_fast, beta_slow)
    f, ms = oracle.yarn_factors(hd, theta, factor, orig_ctx, beta_fast, beta_slow)
    got = oracle.rope_heads_div(x, heads, hd, pos, theta, True, f, ms)
    assert np.max(np.abs(got - want) / (1.0 + np.abs(want))) < 2e-4


@pytest.mark.parametrize("factor,orig_ctx,beta_fast,beta_slow,theta", SPECS)
def test_yarn_factors_shape(factor, orig_ctx, beta_fast, beta_slow, theta):
    """High-frequency pairs (ramp 1) keep their frequency, low-frequency ones (ramp 0) are
    divided by the factor, the divisors in between are monotone; mscale = 1 + 0.1 ln(factor)."""
    f, ms = oracle.yarn_factors(128, theta, factor, orig_ctx, beta_fast, beta_slow)
    assert f.dtype == np.float32 and f.shape == (64,)
    assert f[0] == 1.0 and abs(f[-1] - factor) <= 1e-5 * factor
    assert np.all(np.diff(f) >= 0)
    assert abs(float(ms) - (1.0 + 0.1 * np.log(factor))) < 1e-6


def test_inactive_yarn():
    """factor <= 1: rope_neox_yarn leaves x alone (the reference returns early); divisors
    of 1 and mscale 1 give the plain NeoX RoPE (rope_cabezas)."""
    hd, heads, pos, theta = 128, 2, 37, 1e6
    x = np.random.default_rng(0).standard_normal(heads * hd).astype(np.float32)
    assert np.array_equal(oracle.rope_neox_yarn(x, heads, hd, pos, theta, 1.0, 8192, 32.0, 1.0), x)
    got = oracle.rope_heads_div(x, heads, hd, pos, theta, True, np.ones(hd // 2, np.float32), 1.0)
    want = oracle.rope_heads(x, heads, hd, pos, theta, True)
    assert np.max(np.abs(got - want) / (1.0 + np.abs(want))) < 2e-5


@pytest.mark.parametrize("factor,orig_ctx,beta_fast,beta_slow,theta", SPECS + [(16.0, 64, 32.0, 1.0, 1e4)])
def test_product_divisors_equal_oracle(factor, orig_ctx, beta_fast, beta_slow, theta):
    """The divisors the decode session hands the engine (host code of the product) are the
    oracle's yarn_factores restatement, bit for bit."""
    from soso_b200 import decode
    a, ma = decode.yarn_divisors(128, theta, factor, orig_ctx, beta_fast, beta_slow)
    b, mb = oracle.yarn_factors(128, theta, factor, orig_ctx, beta_fast, beta_slow)
    assert np.array_equal(a, b) and ma == float(mb)
