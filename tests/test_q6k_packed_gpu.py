"""Q6_K on the tensor-core kernel: the device repacking (sbk_q6k_pack, SB_DTYPE_Q6_K_P)
and the packed matvec against the oracle (exact dequant of the reference-layout
blocks, f64 accumulation; crates/gguf2som/src/lib.rs:1639-1661)."""
import numpy as np
import pytest

import oracle
from soso_b200 import synth
from soso_b200._lib import SbkMvOp, lib
from soso_b200.formats import DTYPE_Q6_K
from tests._util import MATVEC_REL, assert_matvec_close, matvec_rel_err

pytestmark = pytest.mark.gpu
Q6KP = 14


def pack_host(w: np.ndarray, rows: int, cols: int) -> np.ndarray:
    """The packed layout restated on the host: per row, groups of 8 blocks as planes
    [ql 8x128][qh 8x64][sc 8x16][d 8x2]; a last group of m blocks likewise, padded to 16 B."""
    nb = cols // 256
    rbp = int(lib().sbk_row_bytes(Q6KP, cols))
    blk = w.reshape(rows, nb, 210)
    out = np.zeros((rows, rbp), np.uint8)
    for gi in range((nb + 7) // 8):
        m = min(8, nb - 8 * gi)
        g = blk[:, 8 * gi:8 * gi + m]
        o = 1680 * gi
        out[:, o:o + 128 * m] = g[:, :, 0:128].reshape(rows, -1)
        out[:, o + 128 * m:o + 192 * m] = g[:, :, 128:192].reshape(rows, -1)
        out[:, o + 192 * m:o + 208 * m] = g[:, :, 192:208].reshape(rows, -1)
        out[:, o + 208 * m:o + 210 * m] = g[:, :, 208:210].reshape(rows, -1)
    return out.reshape(-1)


def packed_on_device(w, rows, cols):
    import torch
    src = torch.from_numpy(np.ascontiguousarray(w)).cuda()
    dst = torch.zeros(int(lib().sbk_row_bytes(Q6KP, cols)) * rows + 64, dtype=torch.uint8, device="cuda")
    assert lib().sbk_q6k_pack(src.data_ptr(), rows, cols, dst.data_ptr(), torch.cuda.current_stream().cuda_stream) == 0
    torch.cuda.synchronize()
    return dst


def packed_matvec(w, rows, cols, x, pdl=0):
    import torch
    wd = packed_on_device(w, rows, cols)
    xd = torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).cuda()
    yd = torch.full((rows,), float("nan"), device="cuda")
    rc = lib().sbk_matvec(Q6KP, wd.data_ptr(), rows, cols, xd.data_ptr(), yd.data_ptr(), pdl,
                          torch.cuda.current_stream().cuda_stream)
    assert rc == 0, rc
    torch.cuda.synchronize()
    return yd.cpu().numpy()


@pytest.mark.parametrize("rows,cols", [(1, 256), (3, 2048), (17, 2304), (40, 1792), (9, 11008)])
def test_pack_bytes(rows, cols):
    w = synth.random_weights(DTYPE_Q6_K, rows, cols, synth.rng("pack", rows, cols))
    got = packed_on_device(w, rows, cols).cpu().numpy()[:rows * int(lib().sbk_row_bytes(Q6KP, cols))]
    assert np.array_equal(got, pack_host(w, rows, cols))


@pytest.mark.parametrize("rows,cols,tag", [(4096, 11008, "C2"), (151936, 2048, "C2 lm_head"),
                                           (2048, 11008, "C3 ffn_down"), (4096, 4096, "square")])
def test_baseline_shapes_packed(rows, cols, tag):
    g = synth.rng("q6kp", tag, rows, cols)
    w = synth.random_weights(DTYPE_Q6_K, rows, cols, g)
    x = synth.randn(cols, g)
    y = packed_matvec(w, rows, cols, x)
    assert not np.any(np.isnan(y)), "unwritten outputs"
    t = oracle.matvec_f64(DTYPE_Q6_K, w, rows, cols, x)
    ref_err = matvec_rel_err(oracle.matvec(DTYPE_Q6_K, w, rows, cols, x), t)
    err = matvec_rel_err(y, t)
    print(f"{tag} {rows}x{cols}: kernel {err:.2e}, reference-order f32 {ref_err:.2e}")
    assert err <= max(MATVEC_REL, 1.5 * ref_err)


@pytest.mark.parametrize("rows,cols", [(1, 256), (2, 256), (7, 768), (31, 2048), (33, 2304), (100, 1792),
                                       (149, 512), (297, 1280), (5, 12288), (1000, 256)])
def test_edge_shapes_packed(rows, cols):
    g = synth.rng("q6kp.edge", rows, cols)
    w = synth.random_weights(DTYPE_Q6_K, rows, cols, g)
    x = synth.randn(cols, g)
    y = packed_matvec(w, rows, cols, x, pdl=rows % 2)
    assert not np.any(np.isnan(y))
    assert_matvec_close(y, oracle.matvec_f64(DTYPE_Q6_K, w, rows, cols, x), f"Q6_K_P {rows}x{cols}")


def test_model_weights_and_extreme_activations():
    g = np.random.default_rng(61)
    rows, cols = 512, 11008
    w = synth.model_weights(DTYPE_Q6_K, rows, cols, g)
    for scale in (1e-6, 1.0, 1e8):
        x = (g.standard_normal(cols) * scale).astype(np.float32)
        assert_matvec_close(packed_matvec(w, rows, cols, x), oracle.matvec_f64(DTYPE_Q6_K, w, rows, cols, x),
                            f"x*{scale}")


def test_batch_and_determinism():
    import torch
    shapes = [(2048, 11008), (256, 2048), (33, 2304), (4096, 4096), (1, 256)]
    host, dev = [], []
    for i, (rows, cols) in enumerate(shapes):
        g = synth.rng("q6kp.batch", i)
        w = synth.random_weights(DTYPE_Q6_K, rows, cols, g)
        x = synth.randn(cols, g)
        host.append((w, x, rows, cols))
        dev.append((packed_on_device(w, rows, cols), torch.from_numpy(x).cuda(),
                    torch.full((rows,), float("nan"), device="cuda")))
    ops = (SbkMvOp * len(shapes))(*[SbkMvOp(wd.data_ptr(), r, c, xd.data_ptr(), yd.data_ptr())
                                    for (wd, xd, yd), (_, _, r, c) in zip(dev, host)])
    outs = []
    for rep in range(2):
        assert lib().sbk_matvec_batch(Q6KP, ops, len(shapes), rep, torch.cuda.current_stream().cuda_stream) == 0
        torch.cuda.synchronize()
        outs.append([yd.cpu().numpy() for (_, _, yd) in dev])
    for (w, x, rows, cols), y0, y1 in zip(host, outs[0], outs[1]):
        assert np.array_equal(y0, y1)
        assert_matvec_close(y0, oracle.matvec_f64(DTYPE_Q6_K, w, rows, cols, x), f"batch {rows}x{cols}")


def test_rejects_too_many_columns():
    import torch
    rows, cols = 4, 16384
    wd = torch.zeros(int(lib().sbk_row_bytes(Q6KP, cols)) * rows + 64, dtype=torch.uint8, device="cuda")
    x = torch.zeros(cols, device="cuda")
    y = torch.zeros(rows, device="cuda")
    assert lib().sbk_matvec(Q6KP, wd.data_ptr(), rows, cols, x.data_ptr(), y.data_ptr(), 0,
                            torch.cuda.current_stream().cuda_stream) == -5
