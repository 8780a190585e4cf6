"""sbk_matvec_batch (matvec_lote on device pointers) against the CPU oracle."""
import numpy as np
import pytest

import oracle
from soso_b200 import synth
from soso_b200._lib import SbkMvOp, lib
from soso_b200.formats import DTYPE_Q4_K, DTYPE_Q6_K, DTYPE_Q8_0
from tests._util import MATVEC_REL, matvec_rel_err

pytestmark = pytest.mark.gpu


def run_batch(dt, shapes, seed):
    import torch
    g = np.random.default_rng(seed)
    host, dev = [], []
    for rows, cols in shapes:
        w = synth.random_weights(dt, rows, cols, g)
        x = synth.randn(cols, g)
        host.append((w, x, rows, cols))
        dev.append((torch.from_numpy(w).cuda(), torch.from_numpy(x).cuda(),
                    torch.full((rows,), float("nan"), device="cuda")))
    ops = (SbkMvOp * len(shapes))()
    for i, ((w, x, rows, cols), (wd, xd, yd)) in enumerate(zip(host, dev)):
        ops[i] = SbkMvOp(wd.data_ptr(), rows, cols, xd.data_ptr(), yd.data_ptr())
    rc = lib().sbk_matvec_batch(dt, ops, len(shapes), 1, torch.cuda.current_stream().cuda_stream)
    assert rc == 0, rc
    torch.cuda.synchronize()
    for (w, x, rows, cols), (_, _, yd) in zip(host, dev):
        y = yd.cpu().numpy()
        assert not np.isnan(y).any(), f"{rows}x{cols} unwritten"
        t = oracle.matvec_f64(dt, w, rows, cols, x)
        ref = matvec_rel_err(oracle.matvec(dt, w, rows, cols, x), t)
        err = matvec_rel_err(y, t)
        assert err <= max(MATVEC_REL, 1.5 * ref), f"{rows}x{cols}: {err:.2e} (ref f32 {ref:.2e})"


@pytest.mark.parametrize("shapes", [
    [(11008, 4096), (4096, 4096)] * 4,                     # the bench's mix
    [(256, 2048), (2048, 2048), (1, 256), (33, 512), (17, 4096), (4096, 256)],
    [(16, 256)] * 45,                                      # more than one launch (40 per launch)
    [(151936 // 8, 2048), (7, 768), (1408, 2048)],
])
def test_q4k_batch(shapes):
    run_batch(DTYPE_Q4_K, shapes, len(shapes))


@pytest.mark.parametrize("dt", [DTYPE_Q6_K, DTYPE_Q8_0])
def test_other_dtypes_batch(dt):
    run_batch(dt, [(300, 1024), (77, 2048), (1, 256)], dt)
