"""The block-level GpuDispatch methods on host buffers (crates/soso-llm-core/src/gpu.rs:
364-517) through the C ABI, against the CPU restatement of the reference:

* router_topk: router logits of a block against an f32 matrix, softmax, stable top-k,
  renormalisation (topk_softmax, gemm.rs:62-91): the same experts wherever the oracle's
  k-th / (k+1)-th logit gap is not a near-tie, weights within 1e-5;
* expertos_bloque: the experts of a block grouped by expert (one grouped GEMM for every
  gate and up, one for the downs, f16 operands): per token the weighted sum in rank order
  within 1e-2 of its rms (the f16 operands of the reference's own prefill path) against
  the oracle's per-token matvecs; an expert whose matrices are of a format the GEMM does
  not take is left to the caller (hecho stays false), the rest still run;
* atencion_prefill: causal attention of a block over a host-mirrored f16 KV cache, against
  attention_decode_f16 (attn.rs:73-140) per query row.  The kernel multiplies the softmax
  weights P in f16 (q is split into f16 hi + lo, so Q K^T is exact to f32 rounding): every
  output element within 2e-3 of the row's rms, and the rms relative error of the whole block
  under 1e-3 (the reference's own test of its f16 tensor-core attention,
  crates/soso-llm-api/tests/cuda_atencion_mma.rs:57-60, allows 1e-2 with Q and P in f16).
  Two blocks in a row, the second reusing the rows the first put on the device; the
  reference test's shapes (hd 256 group 8, hd 128 group 4, cuda_atencion_mma.rs:65-77) and
  widths / groups its scalar kernel takes (hd 80, 96, 64; groups 1, 3, 6, 16).
"""
import numpy as np
import pytest

import oracle
from soso_b200 import synth
from soso_b200.dispatch import CudaGpu, ExpertoBloque, TensorView
from soso_b200.formats import DTYPE_Q4_K, DTYPE_Q6_K, DTYPE_Q8_0

pytestmark = pytest.mark.gpu


def test_router_topk_block(gpu):
    n, h, n_exp, k = 37, 512, 64, 6
    g = synth.rng("blk_router")
    w = (g.standard_normal((n_exp, h)) / np.sqrt(h)).astype(np.float32)
    xs = g.standard_normal((n, h)).astype(np.float32)
    idx = np.zeros(n * k, np.int32)
    wts = np.zeros(n * k, np.float32)
    assert gpu.router_topk("blk.router", w.ravel(), xs.ravel(), n, h, n_exp, k, idx, wts)
    for t in range(n):
        lg = (w.astype(np.float64) @ xs[t].astype(np.float64)).astype(np.float32)
        oi, ow = oracle.topk_softmax(lg, k)
        s = np.sort(lg.astype(np.float64))
        if s[-k] - s[-k - 1] < 1e-4:  # a near-tie may go either way
            continue
        assert np.array_equal(idx[t * k:(t + 1) * k], oi), t
        assert np.max(np.abs(wts[t * k:(t + 1) * k] - ow)) <= 1e-5, t


def _swiglu_expert(mats, x, h, ffn):
    gw, uw, dw = mats
    gate = oracle.matvec_f64(gw[1], gw[0], ffn, h, x)
    up = oracle.matvec_f64(uw[1], uw[0], ffn, h, x)
    act = gate / (1.0 + np.exp(-gate)) * up
    return oracle.matvec_f64(dw[1], dw[0], h, ffn, act.astype(np.float32))


@pytest.mark.parametrize("down_dt", [DTYPE_Q4_K, DTYPE_Q8_0])
def test_expertos_bloque(gpu, down_dt):
    n, h, ffn, k, n_exp = 24, 512, 256, 3, 6
    g = synth.rng("blk_experts", down_dt)
    xs = g.standard_normal((n, h)).astype(np.float32)
    mats = []
    for e in range(n_exp + 1):  # the last: a shared expert
        mats.append([(synth.model_weights(DTYPE_Q4_K, ffn, h, synth.rng("be", down_dt, e, 0)), DTYPE_Q4_K),
                     (synth.model_weights(DTYPE_Q4_K, ffn, h, synth.rng("be", down_dt, e, 1)), DTYPE_Q4_K),
                     (synth.model_weights(down_dt, h, ffn, synth.rng("be", down_dt, e, 2)), down_dt)])
    # a routed expert in a format the GEMM does not take: the caller's
    mats[2][2] = (synth.model_weights(DTYPE_Q6_K, h, ffn, synth.rng("be", down_dt, 2, 9)), DTYPE_Q6_K)
    # routing: top-(k-1) routed experts per token + the shared one at rank k-1
    kr = k - 1
    choice = np.array([g.choice(n_exp, kr, replace=False) for _ in range(n)])
    pesos = g.uniform(0.1, 1.0, (n, k)).astype(np.float32)
    exps = []
    for e in range(n_exp + 1):
        if e < n_exp:
            toks, dest = np.nonzero(choice == e)
            dests = toks * k + dest
        else:
            toks = np.arange(n)
            dests = toks * k + kr
        views = [TensorView(m[0], m[1], (ffn * h)) for m in mats[e]]
        exps.append(ExpertoBloque([f"be{down_dt}.{e}.{s}" for s in ("ffn_gate", "ffn_up", "ffn_down")], views,
                                  toks.astype(np.uint32), e == n_exp, dests.astype(np.uint32)))
    suma = np.zeros(n * h, np.float32)
    hecho = [False] * len(exps)
    gpu.expertos_bloque(xs.ravel(), n, h, ffn, k, pesos.ravel(), exps, suma, hecho)
    assert hecho == [e != 2 for e in range(n_exp + 1)]
    got = suma.reshape(n, h)
    for t in range(n):
        want = np.zeros(h)
        for r in range(k):
            e = choice[t, r] if r < kr else n_exp
            if e != 2:
                want += pesos[t, r] * _swiglu_expert(mats[e], xs[t], h, ffn)
        rms = float(np.sqrt(np.mean(want ** 2)))
        assert float(np.max(np.abs(got[t] - want))) <= 1e-2 * rms, t


def _check_attention(q, out, k16, v16, n, seq_before, heads, kvh, hd, step=7):
    """Sampled rows against the oracle: per element 2e-3 of the row's rms, rms relative 1e-3."""
    kvd = kvh * hd
    rows = seq_before + n
    got = out.reshape(n, heads, hd)
    q = q.reshape(n, heads * hd)
    err2 = ref2 = 0.0
    for i in sorted(set(range(0, n, step)) | {n - 1}):
        for hh in range(heads):
            want = oracle.attention_decode_f16(q[i, hh * hd:(hh + 1) * hd], k16[:rows], v16[:rows], hd, kvd,
                                               hh // (heads // kvh), seq_before + i + 1)
            rms = float(np.sqrt(np.mean(want.astype(np.float64) ** 2)))
            d = got[i, hh].astype(np.float64) - want
            assert float(np.max(np.abs(d))) <= 2e-3 * max(rms, 1e-3), (seq_before, i, hh)
            err2 += float(np.sum(d * d))
            ref2 += float(np.sum(want.astype(np.float64) ** 2))
    assert np.sqrt(err2 / max(ref2, 1e-30)) < 1e-3


def test_atencion_prefill_two_blocks(gpu):
    heads, kvh, hd = 8, 2, 128
    kvd = kvh * hd
    g = synth.rng("blk_attn")
    total = 150
    k16 = g.standard_normal((total, kvd)).astype(np.float16).view(np.uint16)
    v16 = g.standard_normal((total, kvd)).astype(np.float16).view(np.uint16)
    valid = [0]
    for seq_before, n in ((0, 70), (70, 80)):
        q = g.standard_normal((n, heads * hd)).astype(np.float32)
        out = np.zeros(n * heads * hd, np.float32)
        rows = seq_before + n
        assert gpu.atencion_prefill(3, q.ravel(), out, n, seq_before, heads, kvh, hd, k16[:rows], v16[:rows], valid)
        assert valid == [rows]
        _check_attention(q, out, k16, v16, n, seq_before, heads, kvh, hd)


# (heads, kv_heads, hd, n, seq_before): the reference test's five cases (values of its
# magnitudes: q and k uniform in [-3, 3), v in [-1, 1)), then other widths and groups
@pytest.mark.parametrize("heads,kvh,hd,n,seq_before", [
    (16, 2, 256, 70, 45), (16, 2, 256, 1, 0), (16, 2, 256, 200, 0), (8, 2, 128, 70, 45), (8, 2, 128, 33, 100),
    (12, 4, 80, 41, 9), (6, 6, 96, 65, 0), (12, 2, 64, 30, 77), (16, 1, 128, 19, 3),
])
def test_atencion_prefill_shapes(gpu, heads, kvh, hd, n, seq_before):
    kvd = kvh * hd
    g = synth.rng(f"blk_attn_{heads}_{kvh}_{hd}_{n}_{seq_before}")
    total = seq_before + n
    q = (g.uniform(-3, 3, (n, heads * hd))).astype(np.float32)
    k16 = g.uniform(-3, 3, (total, kvd)).astype(np.float16).view(np.uint16)
    v16 = g.uniform(-1, 1, (total, kvd)).astype(np.float16).view(np.uint16)
    out = np.zeros(n * heads * hd, np.float32)
    valid = [0]
    assert gpu.atencion_prefill(5, q.ravel(), out, n, seq_before, heads, kvh, hd, k16, v16, valid)
    assert valid == [total]
    _check_attention(q, out, k16, v16, n, seq_before, heads, kvh, hd, step=11)
