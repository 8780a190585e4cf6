"""The two MLA decode kernels one at a time, at DeepSeek-V2-Lite dims and at
contexts far longer than the engine tests reach, against an f64 restatement of the absorbed
form of the reference's re-expansion (attention_decode_mla_latent,
crates/soso-llm-core/src/attn.rs:306-404; RoPE as rope_inplace, gemm.rs:1493-1509):
  qt_h = W_kn,h^T q_nope,h      kr_t = rope_t(W_kr c_t)      qr_h = rope_pos(q_rope,h)
  score_t = (qt_h . c_t + qr_h . kr_t) / sqrt(qk_nope + qk_rope)
  cbar_h = sum_t softmax(score)_t c_t        (c_t: the f16 latent rows)

Bars: the appended latent row bit-equal to the reference's f16 rounding; qt within 1e-4 of
its rms (f32 sums of qk_nope terms); the roped slices within 1e-4 (f32 angles, pos <= 300);
cbar within 2e-4 relative per output (|g - t| / max(|t|, rms)): qt and P enter the tensor
cores as f16 hi + lo pairs (~2^-22 relative each), sums in f32 over up to 2048 positions.
"""
import numpy as np
import pytest

import oracle
from soso_b200 import synth
from soso_b200._lib import lib
from soso_b200.formats import DTYPE_Q4_K

pytestmark = pytest.mark.gpu
THETA = 1e4


def cuda(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def stream():
    import torch
    return torch.cuda.current_stream().cuda_stream


def rel_err(g, t):
    t = np.asarray(t, np.float64)
    rms = float(np.sqrt(np.mean(t ** 2)))
    return float(np.max(np.abs(np.asarray(g, np.float64) - t) / np.maximum(np.abs(t), rms)))


def rope64(x, pos, n):
    """Llama pairs (2i, 2i + 1), freq_i = theta^(-2i / n), in f64."""
    x = np.asarray(x, np.float64).copy()
    i = np.arange(n // 2)
    ang = pos * THETA ** (-2.0 * i / n)
    x0, x1 = x[0::2].copy(), x[1::2].copy()
    x[0::2] = x0 * np.cos(ang) - x1 * np.sin(ang)
    x[1::2] = x0 * np.sin(ang) + x1 * np.cos(ang)
    return x


@pytest.mark.parametrize("heads,kv_heads,kv_rank,qk_nope,qk_rope,pos", [
    (16, 16, 512, 128, 64, 37), (16, 16, 512, 128, 64, 300), (4, 4, 512, 64, 32, 5), (8, 2, 512, 128, 64, 211),
    (4, 4, 1024, 256, 128, 90), (2, 1, 256, 32, 16, 0)])
def test_mla_absorb(heads, kv_heads, kv_rank, qk_nope, qk_rope, pos):
    import torch
    qk, ctx = qk_nope + qk_rope, 512
    g = synth.rng("mla_absorb", heads, kv_heads, kv_rank, qk_nope, qk_rope)
    w = synth.model_weights(DTYPE_Q4_K, kv_heads * qk, kv_rank, g)
    q = g.standard_normal(heads * qk).astype(np.float32)
    c = g.standard_normal(kv_rank).astype(np.float32)
    latent = torch.zeros(ctx * kv_rank, dtype=torch.int16, device="cuda")
    krope = torch.zeros(ctx * kv_heads * qk_rope, dtype=torch.float32, device="cuda")
    qt = torch.full((heads * kv_rank,), float("nan"), device="cuda")
    qr = torch.full((heads * qk_rope,), float("nan"), device="cuda")
    wd, qd, cd, posd = cuda(w), cuda(q), cuda(c), cuda(np.array([pos], np.int32))
    rc = lib().sbk_mla_absorb(qd.data_ptr(), cd.data_ptr(), wd.data_ptr(), DTYPE_Q4_K, latent.data_ptr(),
                              krope.data_ptr(), qt.data_ptr(), qr.data_ptr(), posd.data_ptr(), heads, kv_heads,
                              kv_rank, qk_nope, qk_rope, ctx, THETA, 0, stream())
    assert rc == 0, rc
    torch.cuda.synchronize()
    rb = kv_rank // 256 * 144
    W = np.stack([oracle.dequant(DTYPE_Q4_K, w[r * rb:(r + 1) * rb], kv_rank) for r in range(kv_heads * qk)])
    W = W.astype(np.float64)
    c16 = oracle.f32_to_f16_array(c)
    got_lat = latent.cpu().numpy().view(np.uint16)[pos * kv_rank:(pos + 1) * kv_rank]
    assert np.array_equal(got_lat, c16), "latent row"
    cf = c16.view(np.float16).astype(np.float64)
    group = heads // kv_heads
    want_qt = np.concatenate([W[(h // group) * qk:(h // group) * qk + qk_nope].T @ q[h * qk:h * qk + qk_nope]
                              for h in range(heads)])
    assert float(np.max(np.abs(qt.cpu().numpy() - want_qt))) <= 1e-4 * float(np.sqrt(np.mean(want_qt ** 2)))
    want_qr = np.concatenate([rope64(q[h * qk + qk_nope:(h + 1) * qk], pos, qk_rope) for h in range(heads)])
    assert rel_err(qr.cpu().numpy(), want_qr) <= 1e-4
    kr = krope.cpu().numpy().reshape(ctx, kv_heads, qk_rope)[pos]
    want_kr = np.stack([rope64(W[k * qk + qk_nope:(k + 1) * qk] @ cf, pos, qk_rope) for k in range(kv_heads)])
    assert rel_err(kr, want_kr) <= 1e-4
    others = np.delete(krope.cpu().numpy().reshape(ctx, -1), pos, axis=0)
    assert not others.any(), "rope keys written outside row pos"


@pytest.mark.parametrize("heads,kv_heads,qk_rope", [(16, 16, 64), (8, 2, 64), (4, 4, 32)])
def test_mla_attn_long_context(heads, kv_heads, qk_rope):
    """Positions from a single span (one sub-chunk) to the full 2048 context: spans of
    several 32-row sub-chunks, the prefetch of the next sub-chunk's rope keys, merges of
    up to 16 spans."""
    import torch
    kv_rank, qk_nope, ctx = 512, 128, 2048
    g = synth.rng("mla_attn", heads, kv_heads, qk_rope)
    lat16 = g.standard_normal((ctx, kv_rank)).astype(np.float16)
    kr = g.standard_normal((ctx, kv_heads, qk_rope)).astype(np.float32)
    qt = g.standard_normal((heads, kv_rank)).astype(np.float32)
    qr = g.standard_normal((heads, qk_rope)).astype(np.float32)
    lat_d, kr_d, qt_d, qr_d = cuda(lat16.view(np.int16)), cuda(kr), cuda(qt), cuda(qr)
    ws = torch.zeros(int(lib().sbk_mla_ws_bytes(heads, kv_rank)), dtype=torch.uint8, device="cuda")
    cbar = torch.empty(heads * kv_rank, device="cuda")
    scale = 1.0 / np.sqrt(qk_nope + qk_rope)
    group = heads // kv_heads
    C = lat16.astype(np.float64)
    for pos in (0, 15, 16, 31, 33, 100, 511, 512, 1000, 1500, 2047):
        posd = cuda(np.array([pos], np.int32))
        cbar.fill_(float("nan"))
        rc = lib().sbk_mla_attn(qt_d.data_ptr(), qr_d.data_ptr(), lat_d.data_ptr(), kr_d.data_ptr(), cbar.data_ptr(),
                                posd.data_ptr(), heads, kv_heads, kv_rank, qk_nope, qk_rope, ctx, ws.data_ptr(), 0,
                                stream())
        assert rc == 0, rc
        torch.cuda.synchronize()
        got = cbar.cpu().numpy().reshape(heads, kv_rank)
        for h in range(heads):
            s = (C[:pos + 1] @ qt[h].astype(np.float64) + kr[:pos + 1, h // group].astype(np.float64) @
                 qr[h].astype(np.float64)) * scale
            p = np.exp(s - s.max())
            want = (p / p.sum()) @ C[:pos + 1]
            assert rel_err(got[h], want) <= 2e-4, (pos, h, rel_err(got[h], want))
        assert not ws[:16].any(), "workspace counter left non-zero"
