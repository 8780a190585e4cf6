"""Fused decode steps: the matvec whose input is formed by its own preparation
(residual add + RMSNorm, SwiGLU; sbk_matvec_batch_x) and attention with the
RoPE/KV-append step folded in (sbk_attn_rope_decode), against the CPU oracle's
restatements of the reference ops (gemm.rs:93-100, :210-226, :265; layer.rs:1146-1193;
attn.rs:73-140)."""
import numpy as np
import pytest

import oracle
from soso_b200 import synth
from soso_b200._lib import SbkMvOp, SbkXSrc, lib
from soso_b200.formats import DTYPE_Q4_K, DTYPE_Q6_K
from tests._util import MATVEC_REL, matvec_rel_err

pytestmark = pytest.mark.gpu
Q6KP = 14


def cuda(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def stream():
    import torch
    return torch.cuda.current_stream().cuda_stream


def XSrc(res, w, h_out, eps, mode):
    return SbkXSrc(res, w, h_out, eps, mode)


def device_weights(dt, w, rows, cols):
    import torch
    src = cuda(w)
    if dt != DTYPE_Q6_K:
        return src, dt
    dst = torch.zeros(int(lib().sbk_row_bytes(Q6KP, cols)) * rows + 64, dtype=torch.uint8, device="cuda")
    assert lib().sbk_q6k_pack(src.data_ptr(), rows, cols, dst.data_ptr(), stream()) == 0
    return dst, Q6KP


def run_x(dt, shapes, a, xs, seed):
    import ctypes

    import torch
    ws_, ops_, host = [], [], []
    da = cuda(a)
    for i, (rows, cols) in enumerate(shapes):
        g = synth.rng("fusedx", seed, i)
        w = synth.random_weights(dt, rows, cols, g)
        wd, ddt = device_weights(dt, w, rows, cols)
        y = torch.full((rows,), float("nan"), device="cuda")
        ws_.append((wd, y))
        host.append((w, rows, cols))
        ops_.append(SbkMvOp(wd.data_ptr(), rows, cols, da.data_ptr(), y.data_ptr()))
    ops = (SbkMvOp * len(ops_))(*ops_)
    rc = lib().sbk_matvec_batch_x(ddt, ops, len(ops_), ctypes.byref(xs), 1, stream())
    torch.cuda.synchronize()
    return rc, [(w, r, c, y.cpu().numpy()) for (w, r, c), (_, y) in zip(host, ws_)], da


@pytest.mark.parametrize("dt,shapes", [
    (DTYPE_Q4_K, [(2048, 2048), (256, 2048), (256, 2048)]),   # q|k|v of configs[2]
    (DTYPE_Q4_K, [(11008, 2048), (11008, 2048)]),             # gate|up
    (DTYPE_Q6_K, [(151936, 2048)]),                           # output matrix after the final norm
    (DTYPE_Q4_K, [(768, 2048)] * 16),                         # a batch over several matrices
])
@pytest.mark.parametrize("with_res", [0, 1])
def test_norm_input(dt, shapes, with_res):
    import torch
    cols = shapes[0][1]
    g = np.random.default_rng(cols + with_res)
    a = g.standard_normal(cols).astype(np.float32)
    res = g.standard_normal(cols).astype(np.float32)
    nw = (1.0 + 0.1 * g.standard_normal(cols)).astype(np.float32)
    eps = 1e-6
    dres, dw = cuda(res), cuda(nw)
    hout = torch.full((cols,), float("nan"), device="cuda")
    xs = XSrc(dres.data_ptr() if with_res else None, dw.data_ptr(), hout.data_ptr() if with_res else None, eps, 1)
    rc, outs, _ = run_x(dt, shapes, a, xs, f"n{with_res}")
    assert rc == 0
    h = (a + res).astype(np.float32) if with_res else a
    x = oracle.rmsnorm(h, nw, eps)
    if with_res:
        np.testing.assert_array_equal(hout.cpu().numpy(), h)
    for w, rows, cols_, y in outs:
        t = oracle.matvec_f64(dt, w, rows, cols_, x)
        ref = matvec_rel_err(oracle.matvec(dt, w, rows, cols_, x), t)
        assert not np.isnan(y).any()
        # the norm's scale carries a few f32 roundings on top of the matvec's
        assert matvec_rel_err(y, t) <= max(MATVEC_REL, 1.5 * ref), (rows, cols_)


@pytest.mark.parametrize("dt,rows,cols", [(DTYPE_Q6_K, 2048, 11008), (DTYPE_Q4_K, 2048, 11008),
                                          (DTYPE_Q4_K, 2048, 768)])
def test_swiglu_input(dt, rows, cols):
    g = np.random.default_rng(rows + cols)
    gate = (2.0 * g.standard_normal(cols)).astype(np.float32)
    up = g.standard_normal(cols).astype(np.float32)
    dup = cuda(up)
    xs = XSrc(dup.data_ptr(), None, None, 0.0, 2)
    rc, outs, _ = run_x(dt, [(rows, cols)], gate, xs, "sw")
    assert rc == 0
    x = oracle.swiglu(up, gate)
    for w, r, c, y in outs:
        t = oracle.matvec_f64(dt, w, r, c, x)
        ref = matvec_rel_err(oracle.matvec(dt, w, r, c, x), t)
        assert matvec_rel_err(y, t) <= max(MATVEC_REL, 1.5 * ref)


def test_fused_input_rejections():
    import ctypes
    g = np.random.default_rng(3)
    a = g.standard_normal(2048).astype(np.float32)
    # XS_NORM without a weight vector; an unknown mode; two different inputs in one fused batch
    for xs in (XSrc(None, None, None, 1e-6, 1), XSrc(None, None, None, 0.0, 7)):
        rc, _, _ = run_x(DTYPE_Q4_K, [(256, 2048)], a, xs, "rej")
        assert rc == -1
    # a dtype without the fused forms (reference-layout Q6_K) is rejected before any launch
    ops = (SbkMvOp * 1)(SbkMvOp(16, 4, 256, 16, 16))
    xs = XSrc(None, 16, None, 1e-6, 1)
    assert lib().sbk_matvec_batch_x(13, ops, 1, ctypes.byref(xs), 0, None) == -5


@pytest.mark.parametrize("heads,kv_heads,neox,qk_norm,bias,pos", [
    (16, 2, 1, 0, 1, 0), (16, 2, 1, 0, 1, 63), (16, 2, 1, 0, 1, 64), (16, 2, 1, 0, 1, 300),
    (32, 4, 1, 1, 0, 777), (8, 8, 0, 0, 0, 129), (16, 2, 1, 1, 1, 4095)])
def test_attn_rope_decode(heads, kv_heads, neox, qk_norm, bias, pos):
    import torch
    hd, ctx, theta, eps = 128, 4096, 1e6, 1e-6
    g = np.random.default_rng(pos + heads)
    qd, kvd = heads * hd, kv_heads * hd
    qkv = g.standard_normal(qd + 2 * kvd).astype(np.float32)
    b = (0.3 * g.standard_normal(qd + 2 * kvd)).astype(np.float32) if bias else None
    qn = (1 + 0.1 * g.standard_normal(hd)).astype(np.float32) if qk_norm else None
    kn = (1 + 0.1 * g.standard_normal(hd)).astype(np.float32) if qk_norm else None
    # cache rows before pos (already f16), then this token's rows formed as the reference does
    kc = np.zeros((ctx, kvd), np.uint16)
    vc = np.zeros((ctx, kvd), np.uint16)
    kc[:pos] = oracle.f32_to_f16_array(g.standard_normal(pos * kvd).astype(np.float32)).reshape(pos, kvd)
    vc[:pos] = oracle.f32_to_f16_array(g.standard_normal(pos * kvd).astype(np.float32)).reshape(pos, kvd)
    ref = qkv + (b if bias else 0)
    q, k, v = ref[:qd].copy(), ref[qd:qd + kvd].copy(), ref[qd + kvd:].copy()
    if qk_norm:
        q = np.concatenate([oracle.rmsnorm(q[h * hd:(h + 1) * hd], qn, eps) for h in range(heads)])
        k = np.concatenate([oracle.rmsnorm(k[h * hd:(h + 1) * hd], kn, eps) for h in range(kv_heads)])
    q = oracle.rope_heads(q, heads, hd, pos, theta, bool(neox))
    k = oracle.rope_heads(k, kv_heads, hd, pos, theta, bool(neox))
    kref, vref = kc.copy(), vc.copy()
    kref[pos] = oracle.f32_to_f16_array(k)
    vref[pos] = oracle.f32_to_f16_array(v)
    dk, dv = cuda(kc.view(np.int16)), cuda(vc.view(np.int16))
    keep = [cuda(qkv), cuda(b) if bias else None, cuda(qn) if qk_norm else None, cuda(kn) if qk_norm else None]
    ws = torch.zeros(lib().sbk_attn_ws_bytes(heads, kv_heads, hd, ctx), dtype=torch.uint8, device="cuda")
    out = torch.zeros(qd, device="cuda")
    dpos = cuda(np.array([pos], dtype=np.int32))
    f = lib().sbk_attn_rope_decode
    for rep in range(2):  # twice: counters must return to zero, the appended rows are rewritten identically
        rc = f(*[t.data_ptr() if t is not None else None for t in keep], dk.data_ptr(), dv.data_ptr(),
               out.data_ptr(), dpos.data_ptr(), heads, kv_heads, hd, ctx, theta, eps, neox, ws.data_ptr(), 1,
               stream())
        assert rc == 0
        torch.cuda.synchronize()
        kr = dk.cpu().numpy().view(np.uint16).reshape(ctx, kvd)
        vr = dv.cpu().numpy().view(np.uint16).reshape(ctx, kvd)
        np.testing.assert_array_equal(vr, vref)  # V: exact (no transcendental on its path)
        np.testing.assert_array_equal(kr[:pos], kref[:pos])
        assert (kr[pos + 1:] == 0).all()
        kf = kr[pos].view(np.float16).astype(np.float32)
        kt = kref[pos].view(np.float16).astype(np.float32)
        assert np.max(np.abs(kf - kt) / (1e-3 + np.abs(kt))) < 2e-3
        o = out.cpu().numpy()
        G = heads // kv_heads
        for h in range(heads):
            # attention over the cache the GPU wrote (its own rounding of row pos)
            r = oracle.attention_decode_f16(q[h * hd:(h + 1) * hd], kr, vr, hd, kvd, h // G, pos + 1)
            assert np.max(np.abs(o[h * hd:(h + 1) * hd] - r)) < 2e-4 * (1 + np.max(np.abs(r))), h


@pytest.mark.parametrize("heads,kv_heads,neox,pos", [(16, 2, 1, 37), (16, 2, 1, 700), (8, 8, 0, 129)])
def test_attn_rope_decode_yarn(heads, kv_heads, neox, pos):
    """The fused RoPE with YaRN divisors (Mellum's: factor 16 over 8192 positions; gm_rope,
    gemma_capa.cu:99-125) against the oracle's gm_rope restatement and the f16 attention over
    the cache the kernel wrote."""
    import torch
    hd, ctx, theta, eps = 128, 1024, 1e4, 1e-6
    g = np.random.default_rng(7 * pos + heads)
    qd, kvd = heads * hd, kv_heads * hd
    qkv = g.standard_normal(qd + 2 * kvd).astype(np.float32)
    kc = np.zeros((ctx, kvd), np.uint16)
    vc = np.zeros((ctx, kvd), np.uint16)
    kc[:pos] = oracle.f32_to_f16_array(g.standard_normal(pos * kvd).astype(np.float32)).reshape(pos, kvd)
    vc[:pos] = oracle.f32_to_f16_array(g.standard_normal(pos * kvd).astype(np.float32)).reshape(pos, kvd)
    f, ms = oracle.yarn_factors(hd, theta, 16.0, 8192, 32.0, 1.0)
    q = oracle.rope_heads_div(qkv[:qd], heads, hd, pos, theta, bool(neox), f, ms)
    k = oracle.rope_heads_div(qkv[qd:qd + kvd], kv_heads, hd, pos, theta, bool(neox), f, ms)
    kt = oracle.f32_to_f16_array(k).view(np.float16).astype(np.float32)
    dk, dv, dq, df = cuda(kc.view(np.int16)), cuda(vc.view(np.int16)), cuda(qkv), cuda(f)
    ws = torch.zeros(lib().sbk_attn_ws_bytes(heads, kv_heads, hd, ctx), dtype=torch.uint8, device="cuda")
    out = torch.zeros(qd, device="cuda")
    dpos = cuda(np.array([pos], dtype=np.int32))
    rc = lib().sbk_attn_rope_decode_yarn(dq.data_ptr(), None, None, None, dk.data_ptr(), dv.data_ptr(), out.data_ptr(),
                                         dpos.data_ptr(), heads, kv_heads, hd, ctx, theta, eps, neox, df.data_ptr(),
                                         float(ms), ws.data_ptr(), 1, stream())
    assert rc == 0, rc
    torch.cuda.synchronize()
    kr = dk.cpu().numpy().view(np.uint16).reshape(ctx, kvd)
    vr = dv.cpu().numpy().view(np.uint16).reshape(ctx, kvd)
    kf = kr[pos].view(np.float16).astype(np.float32)
    # f32 angles of up to pos radians: the divided frequencies differ from the oracle's by an ulp
    tol = 2e-3 + 2e-7 * pos
    assert np.max(np.abs(kf - kt) / (1e-3 + np.abs(kt))) < tol
    o = out.cpu().numpy()
    G = heads // kv_heads
    for h in range(heads):
        r = oracle.attention_decode_f16(q[h * hd:(h + 1) * hd], kr, vr, hd, kvd, h // G, pos + 1)
        assert np.max(np.abs(o[h * hd:(h + 1) * hd] - r)) < (2e-4 + 2e-7 * pos) * (1 + np.max(np.abs(r))), h
