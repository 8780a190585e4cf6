"""The reference's own CUDA kernels, built from its sources for sm_100a (oracle/Makefile
builds lxdde/ports/nouveau/matvec_iq.cu into oracle/_ref/matvec_iq.cubin when the reference
checkout is given), run beside this library's kernels on the same inputs on the same B200:
the kernels the drop-in replaces, checked for equal results and timed.

* decode matvec: `dec_matvec` with the Q4_K decoder (code 1002, matvec_iq.cu:1930-1975), as
  the reference's resident decode graph launches it, and `gm_matvec_q4k` (gemma_capa.cu:433,
  the whole-layer path's matvec; grid ceil(rows / 8), cuda.rs:817-840) (grid ceil(rows / 16), 256 threads,
  (cols + cols / 32 + 1) floats of shared memory: crates/soso-llm-api/src/cuda/decode.rs:
  729-741), one launch per matrix, against sbk_matvec (one launch per matrix, PDL chain)
  and sbk_matvec_batch (the matrices in one launch), on configs[1]'s shapes (11008x4096
  and 4096x4096, eight copies of each: 278 MB, more than L2).  Results within 1e-3 of the
  row vector's rms of each other (both decode to f32 and sum in f32).
* block prefill GEMM: `cvt_f16` then `iq_matmul_mma_h` (f16 mma.sync, matvec_iq.cu:966-980)
  with the Q4_K decoder, launched as the reference's matmul_blq does (grid (rows / 64,
  n / 64), 128 threads: cuda.rs:1136-1156), against sbk_matmul with f16 operands, on
  configs[4]'s dense gate shape (10944x2048) and a 512-token block.  Both round the decoded
  weights and x to f16 the same way and sum in f32: within 1e-3 of the rms of Y.

* decode attention: `mo_attn_split` + `mo_attn_combine` (gemma_capa.cu:765-926, launched
  as atencion_split_dev does: grid (ceil(positions / 256), kv heads), 256 threads, then
  (heads), 128 threads: cuda/capa.rs:787-845) against sbk_attn_decode, configs[2]'s 16 query
  / 2 kv heads x 128 over a 4096-row f16 cache, at positions 200, 1000 and 4000.  Results
  within 1e-3 of the output's largest magnitude (both f32 softmax over f16 K / V).

Each case prints one REFKERN line with both sides' times (CUDA events on the launching
stream, after warm-up; the best of three runs, against other work on a shared GPU).
Nothing here asserts on speed.
"""
import ctypes
import json
import os

import numpy as np
import pytest

from soso_b200 import synth
from soso_b200._lib import SbkMvOp, lib
from soso_b200.formats import DTYPE_Q4_K, row_bytes

pytestmark = pytest.mark.gpu
REF = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle", "_ref")
CUBIN = os.path.join(REF, "matvec_iq.cubin")
CUBIN_CAPA = os.path.join(REF, "gemma_capa.cubin")
Q4K_CODE = 1002  # the reference's decoder code for Q4_K (crates/soso-llm-api/src/cuda.rs:39-44)


class _Module:
    """The reference's cubin in the current (torch's primary) context, through the driver API."""

    def __init__(self, path):
        self.cu = ctypes.CDLL("libcuda.so.1")
        data = open(path, "rb").read()
        self.mod = ctypes.c_void_p()
        rc = self.cu.cuModuleLoadData(ctypes.byref(self.mod), ctypes.c_char_p(data))
        assert rc == 0, f"cuModuleLoadData {rc}"
        self.fns = {}

    def fn(self, name):
        if name not in self.fns:
            f = ctypes.c_void_p()
            rc = self.cu.cuModuleGetFunction(ctypes.byref(f), self.mod, name.encode())
            assert rc == 0, f"cuModuleGetFunction({name}) {rc}"
            self.fns[name] = f
        return self.fns[name]

    def launch(self, name, grid, block, smem, stream, args):
        vals = []
        for kind, v in args:
            vals.append({"p": ctypes.c_uint64, "i": ctypes.c_int32, "l": ctypes.c_int64, "f": ctypes.c_float}[kind](v))
        params = (ctypes.c_void_p * len(vals))(*[ctypes.cast(ctypes.pointer(v), ctypes.c_void_p) for v in vals])
        rc = self.cu.cuLaunchKernel(self.fn(name), ctypes.c_uint(grid[0]), ctypes.c_uint(grid[1]),
                                    ctypes.c_uint(grid[2] if len(grid) > 2 else 1),
                                    ctypes.c_uint(block), ctypes.c_uint(1), ctypes.c_uint(1), ctypes.c_uint(smem),
                                    ctypes.c_void_p(stream), params, None)
        assert rc == 0, f"cuLaunchKernel({name}) {rc}"

    def close(self):
        self.cu.cuModuleUnload(self.mod)


@pytest.fixture(scope="module")
def refmod():
    if not os.path.exists(CUBIN):
        pytest.skip("oracle/_ref/matvec_iq.cubin not built (needs the reference checkout at build time)")
    import torch
    torch.zeros(1, device="cuda")  # torch's primary context current on this thread
    m = _Module(CUBIN)
    yield m
    torch.cuda.synchronize()
    m.close()


@pytest.fixture(scope="module")
def capamod():
    if not os.path.exists(CUBIN_CAPA):
        pytest.skip("oracle/_ref/gemma_capa.cubin not built (needs the reference checkout at build time)")
    import torch
    torch.zeros(1, device="cuda")
    m = _Module(CUBIN_CAPA)
    yield m
    torch.cuda.synchronize()
    m.close()


def _time(fn, reps, warm=3, trials=3):
    """Seconds per call: the best of `trials` runs of `reps` calls, after `warm` calls."""
    import torch
    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    best = float("inf")
    for _ in range(trials):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(reps):
            fn()
        b.record()
        torch.cuda.synchronize()
        best = min(best, a.elapsed_time(b) / reps * 1e-3)
    return best


def test_decode_matvec_vs_reference(refmod, capamod):
    import torch
    s = torch.cuda.current_stream()
    g = synth.rng("refkern", "q4k")
    shapes = [(11008, 4096), (4096, 4096)]
    mats = []
    for rows, cols in shapes:
        w = torch.from_numpy(synth.random_weights(DTYPE_Q4_K, rows, cols, g)).cuda()
        mats += [(w if k == 0 else w.clone(), rows, cols) for k in range(8)]
    x = torch.from_numpy(synth.randn(4096, g)).cuda()
    ys_ref = [torch.empty(r, device="cuda") for _, r, _ in mats]
    ys_our = [torch.empty(r, device="cuda") for _, r, _ in mats]
    L = lib()

    def ref():
        for (w, rows, cols), y in zip(mats, ys_ref):
            refmod.launch("dec_matvec", ((rows + 15) // 16, 1), 256, (cols + cols // 32 + 1) * 4, s.cuda_stream,
                          [("p", w.data_ptr()), ("p", x.data_ptr()), ("p", y.data_ptr()), ("i", rows), ("i", cols),
                           ("i", Q4K_CODE), ("l", row_bytes(DTYPE_Q4_K, cols))])

    def ours_each():
        for (w, rows, cols), y in zip(mats, ys_our):
            assert L.sbk_matvec(DTYPE_Q4_K, w.data_ptr(), rows, cols, x.data_ptr(), y.data_ptr(), 1,
                                s.cuda_stream) == 0

    batch = (SbkMvOp * len(mats))()
    for i, ((w, rows, cols), y) in enumerate(zip(mats, ys_our)):
        batch[i] = SbkMvOp(w.data_ptr(), rows, cols, x.data_ptr(), y.data_ptr())

    def ours_batch():
        assert L.sbk_matvec_batch(DTYPE_Q4_K, batch, len(mats), 1, s.cuda_stream) == 0

    ys_gm = [torch.empty(r, device="cuda") for _, r, _ in mats]

    def ref_gm():  # the Gemma-layer path's Q4_K matvec (gemma_capa.cu:433; grid ceil(rows / 8), cuda.rs:817-840)
        for (w, rows, cols), y in zip(mats, ys_gm):
            capamod.launch("gm_matvec_q4k", ((rows + 7) // 8, 1), 256, 0, s.cuda_stream,
                           [("p", w.data_ptr()), ("p", x.data_ptr()), ("p", y.data_ptr()), ("i", rows), ("i", cols)])

    ref()
    ref_gm()
    ours_batch()
    torch.cuda.synchronize()
    for (w, rows, cols), yr, yo in zip(mats, ys_gm, ys_our):
        yr, yo = yr.cpu().numpy().astype(np.float64), yo.cpu().numpy().astype(np.float64)
        assert float(np.abs(yr - yo).max()) <= 1e-3 * float(np.sqrt(np.mean(yo ** 2))), (rows, cols)
    for (w, rows, cols), yr, yo in zip(mats, ys_ref, ys_our):
        yr, yo = yr.cpu().numpy().astype(np.float64), yo.cpu().numpy().astype(np.float64)
        rms = float(np.sqrt(np.mean(yo ** 2)))
        assert float(np.abs(yr - yo).max()) <= 1e-3 * rms, (rows, cols)
    nbytes = sum(w.numel() for w, _, _ in mats)
    t_ref, t_each, t_batch = _time(ref, 10), _time(ours_each, 10), _time(ours_batch, 10)
    t_gm = _time(ref_gm, 10)
    print("REFKERN " + json.dumps({
        "case": "Q4_K decode matvec, configs[1] shapes (8 x 11008x4096 + 8 x 4096x4096, x f32)",
        "bytes": nbytes,
        "reference_dec_matvec": {"us": round(t_ref * 1e6, 1), "GBps": round(nbytes / t_ref / 1e9, 1)},
        "reference_gm_matvec_q4k": {"us": round(t_gm * 1e6, 1), "GBps": round(nbytes / t_gm / 1e9, 1)},
        "sbk_matvec_per_matrix": {"us": round(t_each * 1e6, 1), "GBps": round(nbytes / t_each / 1e9, 1)},
        "sbk_matvec_batch": {"us": round(t_batch * 1e6, 1), "GBps": round(nbytes / t_batch / 1e9, 1)},
        "speedup_batch_vs_reference": round(t_ref / t_batch, 2)}))


def test_prefill_gemm_vs_reference(refmod):
    import torch
    s = torch.cuda.current_stream()
    g = synth.rng("refkern", "gemm")
    rows, cols, n = 10944, 2048, 512
    w = torch.from_numpy(synth.random_weights(DTYPE_Q4_K, rows, cols, g)).cuda()
    x = torch.from_numpy(g.standard_normal((n, cols)).astype(np.float32)).cuda()
    xh = torch.empty(n * cols, dtype=torch.float16, device="cuda")
    y_ref = torch.empty(n * rows, device="cuda")
    y_our = torch.empty(n * rows, device="cuda")
    L = lib()
    ws = torch.empty(int(L.sbk_matmul_ws_bytes(n, cols)), dtype=torch.uint8, device="cuda")

    def ref():
        refmod.launch("cvt_f16", ((n * cols // 2 + 255) // 256, 1), 256, 0, s.cuda_stream,
                      [("p", x.data_ptr()), ("p", xh.data_ptr()), ("l", n * cols)])
        refmod.launch("iq_matmul_mma_h", ((rows + 63) // 64, (n + 63) // 64), 128, 0, s.cuda_stream,
                      [("p", w.data_ptr()), ("p", xh.data_ptr()), ("p", y_ref.data_ptr()), ("i", rows), ("i", cols),
                       ("i", n), ("i", Q4K_CODE), ("l", row_bytes(DTYPE_Q4_K, cols))])

    def ours():
        assert L.sbk_matmul(DTYPE_Q4_K, w.data_ptr(), rows, cols, n, x.data_ptr(), y_our.data_ptr(), ws.data_ptr(),
                            1, 1, s.cuda_stream) == 0

    ref()
    ours()
    torch.cuda.synchronize()
    yr = y_ref.cpu().numpy().astype(np.float64)
    yo = y_our.cpu().numpy().astype(np.float64)
    rms = float(np.sqrt(np.mean(yo ** 2)))
    assert float(np.abs(yr - yo).max()) <= 1e-3 * rms
    flops = 2.0 * rows * cols * n
    t_ref, t_our = _time(ref, 10), _time(ours, 10)
    print("REFKERN " + json.dumps({
        "case": "Q4_K block GEMM 10944x2048, 512 tokens, f16 operands (configs[4] dense gate)",
        "max_abs_diff_over_rms": float(np.abs(yr - yo).max()) / rms,
        "reference_cvt_f16_iq_matmul_mma_h": {"us": round(t_ref * 1e6, 1), "TFLOPs": round(flops / t_ref / 1e12, 1)},
        "sbk_matmul_f16": {"us": round(t_our * 1e6, 1), "TFLOPs": round(flops / t_our / 1e12, 1)},
        "speedup_vs_reference": round(t_ref / t_our, 2)}))


def test_decode_attention_vs_reference(capamod):
    import torch
    s = torch.cuda.current_stream()
    heads, kvh, hd, ctx = 16, 2, 128, 4096
    kvd = kvh * hd
    g = np.random.default_rng(7)
    kc = torch.from_numpy(g.standard_normal((ctx, kvd)).astype(np.float16).view(np.int16)).cuda()
    vc = torch.from_numpy(g.standard_normal((ctx, kvd)).astype(np.float16).view(np.int16)).cuda()
    q = torch.from_numpy(g.standard_normal(heads * hd).astype(np.float32)).cuda()
    L = lib()
    ws = torch.zeros(int(L.sbk_attn_ws_bytes(heads, kvh, hd, ctx)), dtype=torch.uint8, device="cuda")
    out_ref = torch.empty(heads * hd, device="cuda")
    out_our = torch.empty(heads * hd, device="cuda")
    S_max = (ctx + 255) // 256
    parcial = torch.empty(kvh * S_max * 8 * hd, device="cuda")
    ml = torch.empty(kvh * S_max * 8 * 2, device="cuda")
    scale = float(np.float32(1.0) / np.sqrt(np.float32(hd)))
    rows = []
    for pos in (200, 1000, 4000):
        S = (pos + 1 + 255) // 256
        dpos = torch.tensor([pos], dtype=torch.int32, device="cuda")

        def ref():
            capamod.launch("mo_attn_split", (S, kvh, 1), 256, 0, s.cuda_stream,
                           [("p", q.data_ptr()), ("p", kc.data_ptr()), ("p", vc.data_ptr()), ("p", parcial.data_ptr()),
                            ("p", ml.data_ptr()), ("i", heads), ("i", kvh), ("i", kvd), ("i", pos), ("i", 0),
                            ("f", scale), ("i", S), ("p", 0)])
            capamod.launch("mo_attn_combine", (heads, 1), 128, 0, s.cuda_stream,
                           [("p", parcial.data_ptr()), ("p", ml.data_ptr()), ("p", out_ref.data_ptr()), ("i", heads),
                            ("i", kvh), ("i", S)])

        def ours():
            assert L.sbk_attn_decode(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), out_our.data_ptr(), dpos.data_ptr(),
                                     heads, kvh, hd, ctx, ws.data_ptr(), 0, s.cuda_stream) == 0

        ref()
        ours()
        torch.cuda.synchronize()
        a, b = out_ref.cpu().numpy(), out_our.cpu().numpy()
        assert float(np.abs(a - b).max()) <= 1e-3 * float(np.abs(a).max()), pos
        t_ref, t_our = _time(ref, 20), _time(ours, 20)
        rows.append({"position": pos, "reference_mo_attn_split_combine_us": round(t_ref * 1e6, 2),
                     "sbk_attn_decode_us": round(t_our * 1e6, 2), "speedup": round(t_ref / t_our, 2)})
    print("REFKERN " + json.dumps({"case": "GQA decode attention, 16 q / 2 kv heads x 128, f16 cache of 4096 rows "
                                           "(launch after launch on one stream)", "positions": rows}))
