"""The Q4_K matvec entry point that allocates no device memory.

For callers that cannot call cudaMalloc (fixed device-memory budgets, code that
may run during a global-mode graph capture): sbk_matvec_q4k_noalloc takes its
scratch from a fixed array in the library.  Checked here against the regular
sbk_matvec on two calls in a row of different shapes (the second call runs on
the scratch the first one left behind), and its size limit.  Both entry points
run the same kernel over the same grid and sum split rows in the same fixed
order, so their outputs must agree bit for bit.  This file is collected last on
purpose.
"""
import ctypes

import numpy as np
import pytest

import oracle
from soso_b200 import synth
from soso_b200._lib import lib
from soso_b200.formats import DTYPE_Q4_K
from tests._util import MATVEC_REL, matvec_rel_err

pytestmark = pytest.mark.gpu


def test_noalloc_matches_regular_entry_point_twice():
    import torch
    L = lib()
    s = torch.cuda.current_stream().cuda_stream
    for call, (rows, cols) in enumerate([(4096, 4096), (11008, 4096)]):  # two calls in a row
        g = synth.rng("noalloc", call)
        w = synth.random_weights(DTYPE_Q4_K, rows, cols, g)
        x = synth.randn(cols, g)
        wd, xd = torch.from_numpy(w).cuda(), torch.from_numpy(x).cuda()
        y_ref = torch.full((rows,), float("nan"), device="cuda")
        y_na = torch.full((rows,), float("nan"), device="cuda")
        assert L.sbk_matvec(DTYPE_Q4_K, wd.data_ptr(), rows, cols, xd.data_ptr(), y_ref.data_ptr(), 0, s) == 0
        assert L.sbk_matvec_q4k_noalloc(wd.data_ptr(), rows, cols, xd.data_ptr(), y_na.data_ptr(), s) == 0
        torch.cuda.synchronize()
        a, b = y_ref.cpu().numpy(), y_na.cpu().numpy()
        assert not np.isnan(b).any()
        # same results as the regular entry point: identical bits (same kernel, grid and
        # summation order), and so within the matvec tolerance of the tests
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), f"call {call}: outputs differ"
        assert matvec_rel_err(b, a.astype(np.float64)) <= MATVEC_REL
        t = oracle.matvec_f64(DTYPE_Q4_K, w, rows, cols, x)
        ref = matvec_rel_err(oracle.matvec(DTYPE_Q4_K, w, rows, cols, x), t)
        assert matvec_rel_err(b, t) <= max(MATVEC_REL, 1.5 * ref)


def test_noalloc_rejects_oversize():
    L = lib()
    p = ctypes.c_void_p(256)
    assert L.sbk_matvec_q4k_noalloc(p, 262144 + 16, 256, p, p, None) == -8
    assert L.sbk_matvec_q4k_noalloc(p, 16, 100, p, p, None) == -1
