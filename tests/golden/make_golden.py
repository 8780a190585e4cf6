"""Generate tests/golden/q4k_ref_blocks.npz from the reference's OWN C decoder.

The reference's plain-C header lxdde/ports/nouveau/q4k_decode.h (demonodojo/soso)
is compiled from its source into oracle/_ref/libq4kref.so by oracle/Makefile
(this container only -- the reference checkout is not on the GPU box).  This
script feeds it seeded random Q4_K / .som Q8_0 blocks and records its outputs,
so the oracle (and through it the CUDA kernels) stay pinned to the reference's
code wherever the tests run.  Run:  python tests/golden/make_golden.py
"""
import ctypes
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

import oracle  # noqa: E402


def main():
    oracle.build(force=True)
    R = oracle.ref_lib()
    if R is None:
        raise SystemExit("oracle/_ref/libq4kref.so missing: the reference checkout is needed to regenerate")
    g = np.random.default_rng(20261201)
    nblk = 64
    q4 = g.integers(0, 256, size=(nblk, 144), dtype=np.uint8)
    # d, dmin: finite f16 in a realistic range, plus a few edge values
    d = g.uniform(1e-4, 2.0, nblk).astype(np.float16)
    dm = g.uniform(1e-4, 2.0, nblk).astype(np.float16)
    d[0], dm[0] = np.float16(0.0), np.float16(0.0)
    d[1], dm[1] = np.float16(6e-8), np.float16(3e-5)  # f16 subnormals
    q4[:, 0:2] = d.view(np.uint8).reshape(nblk, 2)
    q4[:, 2:4] = dm.view(np.uint8).reshape(nblk, 2)
    x = g.standard_normal((nblk, 256)).astype(np.float32)
    u8p = ctypes.POINTER(ctypes.c_uint8)
    f32p = ctypes.POINTER(ctypes.c_float)
    dot_block = np.array([R.ref_q4k_dot_block(q4[i].ctypes.data_as(u8p), x[i].ctypes.data_as(f32p))
                          for i in range(nblk)], dtype=np.float32)
    dot_sub = np.zeros((nblk, 8), dtype=np.float32)
    scmin = np.zeros((nblk, 8, 2), dtype=np.uint8)
    for i in range(nblk):
        for j in range(8):
            xs = np.ascontiguousarray(x[i, j * 32:])
            dot_sub[i, j] = R.ref_q4k_dot_sub(q4[i].ctypes.data_as(u8p), j, xs.ctypes.data_as(f32p))
            sc, m = ctypes.c_ubyte(), ctypes.c_ubyte()
            R.ref_q4k_scale_min(np.ascontiguousarray(q4[i, 4:16]).ctypes.data_as(u8p), j, ctypes.byref(sc),
                                ctypes.byref(m))
            scmin[i, j] = (sc.value, m.value)
    q8 = g.integers(0, 256, size=(nblk, 36), dtype=np.uint8)
    q8[:, 0:4] = g.uniform(1e-3, 0.05, nblk).astype(np.float32).view(np.uint8).reshape(nblk, 4)
    x8 = g.standard_normal((nblk, 32)).astype(np.float32)
    dot8 = np.array([R.ref_q80_dot_block(q8[i].ctypes.data_as(u8p), x8[i].ctypes.data_as(f32p))
                     for i in range(nblk)], dtype=np.float32)
    f16_bits = np.arange(0, 65536, 97, dtype=np.uint16)
    f16_vals = np.array([R.ref_q4k_f16(int(b)) for b in f16_bits], dtype=np.float32)
    np.savez_compressed(os.path.join(HERE, "q4k_ref_blocks.npz"), q4=q4, x=x, dot_block=dot_block,
                        dot_sub=dot_sub, scmin=scmin, q8=q8, x8=x8, dot8=dot8, f16_bits=f16_bits,
                        f16_vals=f16_vals)
    print("wrote q4k_ref_blocks.npz")


if __name__ == "__main__":
    main()
