"""Decode-step kernels (RoPE+KV append, split-K attention, router, argmax, embed)
against the CPU oracle's restatements of the reference ops."""
import numpy as np
import pytest

import oracle
from soso_b200 import synth
from soso_b200._lib import lib
from soso_b200.formats import DTYPE_F32, DTYPE_Q4_K, DTYPE_Q6_K, DTYPE_Q8_0

pytestmark = pytest.mark.gpu


def cuda(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def stream():
    import torch
    return torch.cuda.current_stream().cuda_stream


@pytest.mark.parametrize("heads,kv_heads,neox,qk_norm,bias", [(16, 2, 1, 0, 1), (32, 4, 1, 1, 0), (8, 8, 0, 0, 0)])
def test_rope_kv_append(heads, kv_heads, neox, qk_norm, bias):
    import torch
    hd, ctx, pos, theta, eps = 128, 64, 37, 1e6, 1e-6
    g = np.random.default_rng(heads)
    qd, kvd = heads * hd, kv_heads * hd
    qkv = g.standard_normal(qd + 2 * kvd).astype(np.float32)
    b = g.standard_normal(qd + 2 * kvd).astype(np.float32) if bias else None
    qn = g.standard_normal(hd).astype(np.float32) if qk_norm else None
    kn = g.standard_normal(hd).astype(np.float32) if qk_norm else None
    # reference order (layer.rs:1146-1193): bias, qk-norm per head, rope, f16 append
    ref = qkv + (b if bias else 0)
    q, k, v = ref[:qd].copy(), ref[qd:qd + kvd].copy(), ref[qd + kvd:].copy()
    if qk_norm:
        q = np.concatenate([oracle.rmsnorm(q[h * hd:(h + 1) * hd], qn, eps) for h in range(heads)])
        k = np.concatenate([oracle.rmsnorm(k[h * hd:(h + 1) * hd], kn, eps) for h in range(kv_heads)])
    q = oracle.rope_heads(q, heads, hd, pos, theta, bool(neox))
    k = oracle.rope_heads(k, kv_heads, hd, pos, theta, bool(neox))
    d_qkv = cuda(qkv)
    kc = torch.zeros(ctx * kvd, dtype=torch.int16, device="cuda")
    vc = torch.zeros(ctx * kvd, dtype=torch.int16, device="cuda")
    dpos = cuda(np.array([pos], dtype=np.int32))
    keep = [cuda(b) if bias else None, cuda(qn) if qk_norm else None, cuda(kn) if qk_norm else None]
    args = [d_qkv.data_ptr()] + [t.data_ptr() if t is not None else None for t in keep]
    rc = lib().sbk_rope_kv_append(*args, kc.data_ptr(), vc.data_ptr(), dpos.data_ptr(), heads, kv_heads, hd, ctx,
                                  theta, eps, neox, 0, stream())
    assert rc == 0
    torch.cuda.synchronize()
    gq = d_qkv.cpu().numpy()[:qd]
    assert np.max(np.abs(gq - q) / (1 + np.abs(q))) < 2e-5
    kr = kc.cpu().numpy().view(np.uint16).reshape(ctx, kvd)
    vr = vc.cpu().numpy().view(np.uint16).reshape(ctx, kvd)
    # K/V rows at pos: the reference's f32->f16 rounding; V is exact, K within a rounding step
    np.testing.assert_array_equal(vr[pos], oracle.f32_to_f16_array(v))
    kref = oracle.f32_to_f16_array(k)
    kf = np.array([oracle.f16_to_f32(int(u)) for u in kr[pos]], dtype=np.float32)
    kreff = np.array([oracle.f16_to_f32(int(u)) for u in kref], dtype=np.float32)
    assert np.max(np.abs(kf - kreff) / (1e-3 + np.abs(kreff))) < 2e-3
    assert (kr[:pos] == 0).all() and (kr[pos + 1:] == 0).all()


@pytest.mark.parametrize("heads,kv_heads,neox", [(16, 2, 1), (8, 8, 0)])
def test_rope_kv_append_yarn(heads, kv_heads, neox):
    """gm_rope's frequency factors (gemma_capa.cu:99-125) from yarn_factores (gemm.rs:1413-1428,
    Mellum's YaRN: factor 16 over 8192 positions) against the oracle's restatement of gm_rope;
    with no factors and mscale 1 the result is bit-equal to sbk_rope_kv_append."""
    import torch
    hd, ctx, pos, theta, eps = 128, 64, 37, 1e6, 1e-6
    g = np.random.default_rng(100 + heads)
    qd, kvd = heads * hd, kv_heads * hd
    qkv = g.standard_normal(qd + 2 * kvd).astype(np.float32)
    f, ms = oracle.yarn_factors(hd, theta, 16.0, 8192, 32.0, 1.0)
    q = oracle.rope_heads_div(qkv[:qd], heads, hd, pos, theta, bool(neox), f, ms)
    k = oracle.rope_heads_div(qkv[qd:qd + kvd], kv_heads, hd, pos, theta, bool(neox), f, ms)
    dpos, df = cuda(np.array([pos], dtype=np.int32)), cuda(f)

    def run(entry, *extra):
        d = cuda(qkv)
        kc = torch.zeros(ctx * kvd, dtype=torch.int16, device="cuda")
        vc = torch.zeros(ctx * kvd, dtype=torch.int16, device="cuda")
        rc = entry(d.data_ptr(), None, None, None, kc.data_ptr(), vc.data_ptr(), dpos.data_ptr(), heads, kv_heads, hd,
                   ctx, theta, eps, neox, *extra, 0, stream())
        assert rc == 0, rc
        torch.cuda.synchronize()
        return d.cpu().numpy(), kc.cpu().numpy().view(np.uint16).reshape(ctx, kvd)

    gq, kr = run(lib().sbk_rope_kv_append_yarn, df.data_ptr(), float(ms))
    assert np.max(np.abs(gq[:qd] - q) / (1 + np.abs(q))) < 5e-5
    kf = np.array([oracle.f16_to_f32(int(u)) for u in kr[pos]], dtype=np.float32)
    kreff = np.array([oracle.f16_to_f32(int(u)) for u in oracle.f32_to_f16_array(k)], dtype=np.float32)
    assert np.max(np.abs(kf - kreff) / (1e-3 + np.abs(kreff))) < 2e-3
    a = run(lib().sbk_rope_kv_append_yarn, None, 1.0)
    b = run(lib().sbk_rope_kv_append)
    assert np.array_equal(a[0].view(np.uint32), b[0].view(np.uint32)) and np.array_equal(a[1], b[1])
    assert lib().sbk_rope_kv_append_yarn(dpos.data_ptr(), None, None, None, dpos.data_ptr(), dpos.data_ptr(),
                                         dpos.data_ptr(), heads, kv_heads, hd, ctx, theta, eps, neox, None, 0.0, 0,
                                         stream()) == -1  # mscale must be positive


@pytest.mark.parametrize("heads,kv_heads,seq", [(16, 2, 1), (16, 2, 16), (16, 2, 17), (16, 2, 100), (16, 2, 513),
                                                (16, 2, 2049), (16, 2, 4096), (32, 4, 777), (8, 8, 65)])
def test_attention_decode(heads, kv_heads, seq):
    import torch
    hd, ctx = 128, 4096
    g = np.random.default_rng(seq)
    kvd = kv_heads * hd
    q = g.standard_normal(heads * hd).astype(np.float32)
    k = oracle.f32_to_f16_array(g.standard_normal(seq * kvd).astype(np.float32)).reshape(seq, kvd)
    v = oracle.f32_to_f16_array(g.standard_normal(seq * kvd).astype(np.float32)).reshape(seq, kvd)
    kc = np.zeros((ctx, kvd), np.uint16)
    vc = np.zeros((ctx, kvd), np.uint16)
    kc[:seq], vc[:seq] = k, v
    ws = torch.zeros(lib().sbk_attn_ws_bytes(heads, kv_heads, hd, ctx), dtype=torch.uint8, device="cuda")
    out = torch.zeros(heads * hd, device="cuda")
    dpos = cuda(np.array([seq - 1], dtype=np.int32))
    dk, dv, dq = cuda(kc.view(np.int16)), cuda(vc.view(np.int16)), cuda(q)
    for _ in range(2):  # twice: the workspace counters must come back to zero
        rc = lib().sbk_attn_decode(dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), out.data_ptr(), dpos.data_ptr(),
                                   heads, kv_heads, hd, ctx, ws.data_ptr(), 0, stream())
        assert rc == 0
        torch.cuda.synchronize()
        o = out.cpu().numpy()
        G = heads // kv_heads
        for h in range(heads):
            r = oracle.attention_decode_f16(q[h * hd:(h + 1) * hd], kc, vc, hd, kvd, h // G, seq)
            assert np.max(np.abs(o[h * hd:(h + 1) * hd] - r)) < 1e-4 * (1 + np.max(np.abs(r))), h


@pytest.mark.parametrize("n,k", [(128, 8), (64, 6), (8, 2), (256, 8)])
def test_router_topk(n, k):
    import torch
    g = np.random.default_rng(n)
    lg = g.standard_normal(n).astype(np.float32)
    lg[3] = lg[5]  # a tie: the lower index must rank first
    ri, rw = oracle.topk_softmax(lg, k)
    idx = torch.zeros(k, dtype=torch.int32, device="cuda")
    wts = torch.zeros(k, device="cuda")
    dlg = cuda(lg)
    assert lib().sbk_router_topk(dlg.data_ptr(), n, k, idx.data_ptr(), wts.data_ptr(), 0, stream()) == 0
    torch.cuda.synchronize()
    np.testing.assert_array_equal(idx.cpu().numpy(), ri)
    np.testing.assert_allclose(wts.cpu().numpy(), rw, rtol=1e-5)


def test_argmax_ties_last():
    import torch
    ws = torch.zeros(lib().sbk_argmax_ws_bytes(), dtype=torch.uint8, device="cuda")
    out = torch.zeros(1, dtype=torch.int32, device="cuda")
    g = np.random.default_rng(1)
    for n in (1, 7, 151936, 102400):
        v = g.standard_normal(n).astype(np.float32)
        if n > 10:
            v[[5, n // 2, n - 3]] = 10.0  # ties: the last one wins
        dv = cuda(v)
        assert lib().sbk_argmax(dv.data_ptr(), n, out.data_ptr(), ws.data_ptr(), 0, stream()) == 0
        torch.cuda.synchronize()
        assert int(out.item()) == oracle.argmax(v)


@pytest.mark.parametrize("dt", [DTYPE_F32, DTYPE_Q8_0, DTYPE_Q4_K, DTYPE_Q6_K])
def test_embed_row(dt):
    import torch
    vocab, h = 64, 2048
    g = np.random.default_rng(dt)
    if dt == DTYPE_F32:
        table = g.standard_normal(vocab * h).astype(np.float32).view(np.uint8)
    else:
        table = synth.random_weights(dt, vocab, h, g)
    out = torch.zeros(h, device="cuda")
    dtab = cuda(table)
    for tok in (0, 17, vocab - 1):
        dtok = cuda(np.array([tok], dtype=np.int32))
        assert lib().sbk_embed_row(dtab.data_ptr(), dt, vocab, h, dtok.data_ptr(), out.data_ptr(), 0,
                                   stream()) == 0
        torch.cuda.synchronize()
        rb = (h * 4) if dt == DTYPE_F32 else oracle.row_bytes(dt, h)
        ref = oracle.dequant(dt, table[tok * rb:(tok + 1) * rb], h)
        np.testing.assert_array_equal(out.cpu().numpy(), ref)
