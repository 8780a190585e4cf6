"""Batched prefill GEMM on the tcgen05 tensor cores (sbk_matmul): Y = X . W^T for Q4_K W.

Two checks per shape:
  * exactness of the tensor-core path: against an f64 product of the same rounded operands
    (W dequantised exactly as crates/sosomodel/src/dequant.rs:150-248, then rounded to the
    operand type; X likewise), within 1e-4 of the output rms -- a wrong tile layout,
    swizzle or descriptor gives O(1) errors;
  * the numerical contract against the exact f64 product of the unrounded operands, per
    output |y - y64| <= bound * max(|y64|, rms(y64)): with f16 operands (11 significant
    bits, the precision of the reference's own mma.sync prefill) the reference's own bound,
    8e-3 (crates/soso-llm-api/tests/cuda_matvec.rs:268-273); with bf16 operands (8 bits)
    the same bound scaled by the 8x coarser rounding step, capped at 3e-2 -- both operands
    carry a relative rounding error of up to 2^-9, so a K-term sum is off by about
    2^-9 * sqrt(2) of its scale, up to ~5 of that over a few hundred thousand outputs.
"""
import numpy as np
import pytest

import oracle
from soso_b200 import synth
from soso_b200._lib import lib
from soso_b200.formats import DTYPE_Q4_K

pytestmark = pytest.mark.gpu
F16, BF16 = 1, 0
BOUND = {F16: 8e-3, BF16: 3e-2}


def bf16_round(a: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32)


def op_round(a: np.ndarray, prec: int) -> np.ndarray:
    return a.astype(np.float16).astype(np.float32) if prec == F16 else bf16_round(a)


def run(w, rows, cols, x, n, prec):
    import torch
    wd = torch.from_numpy(w).cuda()
    xd = torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).cuda()
    y = torch.full((n, rows), float("nan"), device="cuda")
    ws = torch.empty(int(lib().sbk_matmul_ws_bytes(n, cols)), dtype=torch.uint8, device="cuda")
    rc = lib().sbk_matmul(DTYPE_Q4_K, wd.data_ptr(), rows, cols, n, xd.data_ptr(), y.data_ptr(), ws.data_ptr(), prec,
                          1, torch.cuda.current_stream().cuda_stream)
    assert rc == 0, rc
    torch.cuda.synchronize()
    return y.cpu().numpy()


@pytest.mark.parametrize("rows,cols,n", [(128, 256, 256), (256, 2048, 512), (200, 512, 300), (1, 256, 1),
                                         (2048, 2048, 512), (11008, 2048, 512), (384, 4096, 64), (130, 768, 257)])
@pytest.mark.parametrize("prec", [F16, BF16])
def test_prefill_q4k(rows, cols, n, prec):
    g = synth.rng("prefill", rows, cols, n)
    w = synth.model_weights(DTYPE_Q4_K, rows, cols, g)
    x = g.standard_normal((n, cols)).astype(np.float32)
    y = run(w, rows, cols, x, n, prec)
    assert not np.isnan(y).any()
    wf = np.stack([oracle.dequant(DTYPE_Q4_K, w[r * (cols // 256) * 144:(r + 1) * (cols // 256) * 144], cols)
                   for r in range(rows)]).astype(np.float32)
    # exactness of the tensor-core path on the rounded operands
    t_b = op_round(x, prec).astype(np.float64) @ op_round(wf, prec).astype(np.float64).T
    rms_b = float(np.sqrt(np.mean(t_b ** 2)))
    assert float(np.max(np.abs(y - t_b))) <= 1e-4 * rms_b, "tile layout / descriptor error"
    # the numerical contract against the unrounded product
    t = x.astype(np.float64) @ wf.astype(np.float64).T
    rms = float(np.sqrt(np.mean(t ** 2)))
    err = float(np.max(np.abs(y - t) / np.maximum(np.abs(t), rms)))
    assert err <= BOUND[prec], err


def test_prefill_rejects():
    import ctypes
    L = lib()
    p = ctypes.c_void_p(256)
    assert L.sbk_matmul(2, p, 4, 256, 4, p, p, p, 0, 0, None) == -5      # dtype without the GEMM
    assert L.sbk_matmul(DTYPE_Q4_K, p, 4, 100, 4, p, p, p, 0, 0, None) == -1   # cols not whole blocks
    assert L.sbk_matmul(DTYPE_Q4_K, p, 4, 256, 4, p, p, p, 7, 0, None) == -1   # unknown precision
    assert L.sbk_matmul(DTYPE_Q4_K, ctypes.c_void_p(8), 4, 256, 4, p, p, p, 0, 0, None) == -2
