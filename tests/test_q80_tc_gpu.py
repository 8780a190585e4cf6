"""Q8_0 on the tensor-core matvec: .som blocks (f32 scale + 32 int8, crates/sosomodel/src/
layout.rs:57-59) read in place when rows are 16-byte aligned (cols a multiple of 128) and
after sbk_q80_pad (SB_DTYPE_Q8_0_R) otherwise; against the oracle's exact dequant with f64
accumulation (crates/soso-llm-core/src/gemm.rs:295-332)."""
import numpy as np
import pytest

import oracle
from soso_b200 import synth
from soso_b200._lib import SbkMvOp, lib
from soso_b200.formats import DTYPE_Q8_0
from tests._util import MATVEC_REL, assert_matvec_close, matvec_rel_err

pytestmark = pytest.mark.gpu
Q80R = 15


def stream():
    import torch
    return torch.cuda.current_stream().cuda_stream


def padded(w, rows, cols):
    import torch
    src = torch.from_numpy(np.ascontiguousarray(w)).cuda()
    dst = torch.full((int(lib().sbk_row_bytes(Q80R, cols)) * rows + 64,), 0xAB, dtype=torch.uint8, device="cuda")
    assert lib().sbk_q80_pad(src.data_ptr(), rows, cols, dst.data_ptr(), stream()) == 0
    return dst


def run(w, rows, cols, x, pad):
    import torch
    wd = padded(w, rows, cols) if pad else torch.from_numpy(w).cuda()
    xd = torch.from_numpy(x).cuda()
    y = torch.full((rows,), float("nan"), device="cuda")
    rc = lib().sbk_matvec(Q80R if pad else DTYPE_Q8_0, wd.data_ptr(), rows, cols, xd.data_ptr(), y.data_ptr(), 1,
                          stream())
    assert rc == 0, rc
    torch.cuda.synchronize()
    return y.cpu().numpy()


def test_pad_bytes():
    rows, cols = 5, 1408 + 32
    w = synth.random_weights(DTYPE_Q8_0, rows, cols, synth.rng("q80pad"))
    got = padded(w, rows, cols).cpu().numpy()
    rb, rbp = cols // 32 * 36, int(lib().sbk_row_bytes(Q80R, cols))
    assert rbp % 16 == 0 and rbp >= rb
    for r in range(rows):
        assert np.array_equal(got[r * rbp:r * rbp + rb], w[r * rb:(r + 1) * rb])
        assert not got[r * rbp + rb:(r + 1) * rbp].any()


@pytest.mark.parametrize("rows,cols,pad,tag", [(4096, 4096, 0, "C1"), (2048, 1408, 0, "C5 expert down"),
                                               (2048, 10944, 1, "C5 dense down"), (2048, 2816, 0, "C5 shared down"),
                                               (4096, 4096, 1, "C1 padded"), (1, 32, 1, "one block"),
                                               (17, 160, 1, "ragged"), (33, 2080, 1, "ragged 2"),
                                               (300, 96, 1, "short")])
def test_q80_tc(rows, cols, pad, tag):
    g = synth.rng("q80tc", rows, cols)
    w = synth.random_weights(DTYPE_Q8_0, rows, cols, g)
    x = synth.randn(cols, g)
    y = run(w, rows, cols, x, pad)
    assert not np.isnan(y).any()
    t = oracle.matvec_f64(DTYPE_Q8_0, w, rows, cols, x)
    ref = matvec_rel_err(oracle.matvec(DTYPE_Q8_0, w, rows, cols, x), t)
    assert matvec_rel_err(y, t) <= max(MATVEC_REL, 1.5 * ref), tag


def test_q80_extreme_activations():
    g = np.random.default_rng(80)
    rows, cols = 256, 2048
    w = synth.model_weights(DTYPE_Q8_0, rows, cols, g)
    for scale in (1e-6, 1.0, 1e8):
        x = (g.standard_normal(cols) * scale).astype(np.float32)
        assert_matvec_close(run(w, rows, cols, x, 0), oracle.matvec_f64(DTYPE_Q8_0, w, rows, cols, x), f"x*{scale}")


def test_q80_batch_repeat_bit_identical():
    import torch
    shapes = [(2048, 1408), (1408, 2048), (2048, 10944), (7, 160), (4096, 4096)]
    host, dev = [], []
    for i, (rows, cols) in enumerate(shapes):
        g = synth.rng("q80batch", i)
        w = synth.random_weights(DTYPE_Q8_0, rows, cols, g)
        x = synth.randn(cols, g)
        host.append((w, x, rows, cols))
        dev.append((padded(w, rows, cols), torch.from_numpy(x).cuda(), torch.full((rows,), float("nan"),
                                                                                   device="cuda")))
    ops = (SbkMvOp * len(shapes))(*[SbkMvOp(wd.data_ptr(), r, c, xd.data_ptr(), yd.data_ptr())
                                    for (wd, xd, yd), (_, _, r, c) in zip(dev, host)])
    outs = []
    for rep in range(8):
        assert lib().sbk_matvec_batch(Q80R, ops, len(shapes), 1, stream()) == 0
        outs.append(torch.cat([yd for (_, _, yd) in dev]).clone())
    torch.cuda.synchronize()
    first = outs[0].cpu().numpy()
    for o in outs[1:]:
        assert np.array_equal(o.cpu().numpy(), first)
    off = 0
    for w, x, rows, cols in host:
        assert_matvec_close(first[off:off + rows], oracle.matvec_f64(DTYPE_Q8_0, w, rows, cols, x), f"{rows}x{cols}")
        off += rows
