"""Repeated large launches of the tensor-core matvec must give bit-identical results.

The kernel is deterministic (fixed split, fixed summation order), so any
difference between repetitions means a consumer read a ring slot before its
TMA copy landed, or after the producer refilled it.  A ring whose slots were
shared by two consumer teams once produced exactly that: one wrong 16-row
group in a few thousand, only under load.  Large shapes, many back-to-back
launches (with programmatic dependent launch) and a batch whose matrices
start at odd stage offsets maximise the exposure; the first repetition is
also checked against the oracle.
"""
import numpy as np
import pytest

import oracle
from soso_b200 import synth
from soso_b200._lib import SbkMvOp, lib
from soso_b200.formats import DTYPE_Q4_K, DTYPE_Q6_K
from tests._util import MATVEC_REL, matvec_rel_err

pytestmark = pytest.mark.gpu
Q6KP = 14
REPS = 24


def _device(w, dt, rows, cols):
    import torch
    src = torch.from_numpy(np.ascontiguousarray(w)).cuda()
    if dt != DTYPE_Q6_K:
        return src, dt
    dst = torch.zeros(int(lib().sbk_row_bytes(Q6KP, cols)) * rows + 64, dtype=torch.uint8, device="cuda")
    assert lib().sbk_q6k_pack(src.data_ptr(), rows, cols, dst.data_ptr(),
                              torch.cuda.current_stream().cuda_stream) == 0
    return dst, Q6KP


@pytest.mark.parametrize("dt,shapes", [
    (DTYPE_Q6_K, [(151936, 2048)]),
    (DTYPE_Q6_K, [(65536, 4096), (2048, 11008), (1, 256), (4096, 4096)]),
    (DTYPE_Q4_K, [(151936, 2048)]),
    (DTYPE_Q4_K, [(11008, 4096), (17, 2048), (4096, 4096), (33, 768), (11008, 2048), (2048, 4096)]),
])
def test_repeated_launches_bit_identical(dt, shapes):
    import torch
    host, dev = [], []
    for i, (rows, cols) in enumerate(shapes):
        g = synth.rng("ring", dt, i, rows, cols)
        w = synth.random_weights(dt, rows, cols, g)
        x = synth.randn(cols, g)
        wd, ddt = _device(w, dt, rows, cols)
        host.append((w, x, rows, cols))
        dev.append((wd, torch.from_numpy(x).cuda(), torch.full((rows,), float("nan"), device="cuda")))
    ops = (SbkMvOp * len(shapes))(*[SbkMvOp(wd.data_ptr(), r, c, xd.data_ptr(), yd.data_ptr())
                                    for (wd, xd, yd), (_, _, r, c) in zip(dev, host)])
    s = torch.cuda.current_stream().cuda_stream
    outs = []
    for rep in range(REPS):
        assert lib().sbk_matvec_batch(ddt, ops, len(shapes), 1, s) == 0
        outs.append(torch.cat([yd for (_, _, yd) in dev]).clone())
    torch.cuda.synchronize()
    first = outs[0].cpu().numpy()
    for rep, o in enumerate(outs[1:], 1):
        diff = np.nonzero(o.cpu().numpy() != first)[0]
        assert diff.size == 0, f"repetition {rep}: {diff.size} outputs differ, first at {diff[:8].tolist()}"
    off = 0
    for w, x, rows, cols in host:
        t = oracle.matvec_f64(dt, w, rows, cols, x)
        ref = matvec_rel_err(oracle.matvec(dt, w, rows, cols, x), t)
        assert matvec_rel_err(first[off:off + rows], t) <= max(MATVEC_REL, 1.5 * ref), (rows, cols)
        off += rows
