"""Pin the CPU oracle to the reference before it is trusted as the checker.

Golden vectors restated from the reference's own tests:
  crates/sosomodel/tests/dequant_golden.rs:18-114 (Q4_K scale table, block dot
  -15.875, .som Q8_0 dot 172.59375; duplicated in the reference's C hostcheck
  tools/gsp-hostcheck/main.c:2629-2700),
  crates/gguf2som/src/lib.rs:1866-1889 (Q6_K block of -1.0),
  crates/soso-llm-core/src/quant.rs:408-420 + tools/gsp-hostcheck/main.c:2585-2627
  (row_bytes accept/reject, 5632 cols -> 3168 B),
  crates/soso-llm-core/src/f16.rs:40-55 (f16 cases).
And tests/golden/q4k_ref_blocks.npz, outputs of the reference's C decoder
lxdde/ports/nouveau/q4k_decode.h compiled from source (make_golden.py).
"""
import os

import numpy as np
import pytest

import oracle

GOLD = os.path.join(os.path.dirname(__file__), "golden", "q4k_ref_blocks.npz")


def bloque_q4k():
    """dequant_golden.rs:18-35."""
    b = np.zeros(144, dtype=np.uint8)
    b[0:4] = [0x00, 0x38, 0x00, 0x34]  # d = 0.5, dmin = 0.25
    b[4:16] = [0x41, 0x82, 0xC3, 0x04, 0x45, 0x86, 0xC7, 0x08, 0x9A, 0xBC, 0xDE, 0xF0]
    b[16:] = [(i * 7 + 3) % 256 for i in range(128)]
    return b


def x_256():
    """dequant_golden.rs:37-43."""
    return np.array([((i % 13) - 6.0) * 0.125 for i in range(256)], dtype=np.float32)


def test_q4k_scale_table():
    b = bloque_q4k()
    want = [(1, 5), (2, 6), (3, 7), (4, 8), (26, 25), (44, 43), (62, 61), (0, 15)]
    for j in range(8):
        assert oracle.q4k_scale_min(bytes(b[4:16]), j) == want[j], j


def test_q4k_block_dot_golden():
    b, x = bloque_q4k(), x_256()
    plano = oracle.dequant(oracle.Q4_K, b, 256)
    ref_dot = np.float32(0.0)
    for i in range(256):
        ref_dot = np.float32(ref_dot + plano[i] * x[i])
    porsub = oracle.q4k_dot_ref(b, x)
    assert abs(porsub - ref_dot) <= 1e-3 * max(abs(ref_dot), 1.0)
    assert abs(ref_dot - (-15.875)) <= 1e-2
    # the fused scalar matvec (gemm.rs:428-461) on a 1x256 matrix
    y = oracle.matvec(oracle.Q4_K, b, 1, 256, x)
    assert abs(y[0] - (-15.875)) <= 1e-2


def test_q80_block_dot_golden():
    b = np.zeros(36, dtype=np.uint8)
    b[0:4] = np.array([0.25], dtype=np.float32).view(np.uint8)
    b[4:] = np.array([(i * 9 - 100) for i in range(32)], dtype=np.int64).astype(np.int8).view(np.uint8)
    plano = oracle.dequant(oracle.Q8_0, b, 32)
    xs = np.array([((i % 13) - 6.0) * 0.125 for i in range(32)], dtype=np.float32)
    dot = np.float32(0.0)
    for i in range(32):
        dot = np.float32(dot + plano[i] * xs[i])
    assert abs(dot - 172.59375) <= 1e-3
    y = oracle.matvec(oracle.Q8_0, b, 1, 32, xs)
    assert abs(y[0] - 172.59375) <= 1e-3


def test_q6k_minus_one_block():
    """gguf2som/src/lib.rs:1866-1889: ql/qh zero, scales 1, d = 1/32 -> every element -1.0."""
    q6 = np.zeros(210, dtype=np.uint8)
    q6[192:208] = 1
    d = oracle.f32_to_f16(1.0 / 32.0)
    q6[208], q6[209] = d & 0xFF, d >> 8
    vals = oracle.dequant(oracle.Q6_K, q6, 256)
    assert np.all(vals == -1.0)
    y = oracle.matvec(oracle.Q6_K, q6, 1, 256, np.ones(256, dtype=np.float32))
    assert y[0] == -256.0


def test_row_bytes():
    assert oracle.row_bytes(oracle.Q4_K, 5632) == 3168
    assert oracle.row_bytes(oracle.Q4_K, 4096) == 2304
    assert oracle.row_bytes(oracle.Q4_K, 100) is None
    assert oracle.row_bytes(oracle.Q4_K, 0) is None
    assert oracle.row_bytes(oracle.Q8_0, 4096) == 4608
    assert oracle.row_bytes(oracle.Q8_0, 33) is None
    assert oracle.row_bytes(oracle.Q6_K, 11008) == 9030
    from soso_b200 import formats
    for dt in (oracle.Q8_0, oracle.Q4_K, oracle.Q6_K):
        for cols in (0, 32, 100, 256, 2048, 5632, 11008, 10944):
            assert formats.row_bytes(dt, cols) == oracle.row_bytes(dt, cols)


def test_f16_cases():
    assert oracle.f16_to_f32(0x3C00) == 1.0
    assert oracle.f16_to_f32(0xBC00) == -1.0
    assert oracle.f16_to_f32(0x3800) == 0.5
    assert oracle.f16_to_f32(0) == 0.0
    assert np.isinf(oracle.f16_to_f32(0x7C00))
    assert np.isnan(oracle.f16_to_f32(0x7E00))
    assert abs(oracle.f16_to_f32(0x0001) - 2.0 ** -24) < 1e-10
    for i in range(-1000, 1000):
        v = np.float32(i * 0.37)
        rt = oracle.f16_to_f32(oracle.f32_to_f16(float(v)))
        assert abs(v - rt) <= abs(v) * 1e-3 + 1e-4


@pytest.fixture(scope="module")
def gold():
    return np.load(GOLD)


def test_oracle_matches_reference_c_decoder(gold):
    """oracle.c vs the reference's q4k_decode.h (recorded outputs): bit-exact."""
    q4, x = gold["q4"], gold["x"]
    for i in range(q4.shape[0]):
        assert np.float32(oracle.q4k_dot_ref(q4[i], x[i])) == gold["dot_block"][i], i
        for j in range(8):
            assert oracle.q4k_scale_min(bytes(q4[i, 4:16]), j) == tuple(gold["scmin"][i, j])
    for b, v in zip(gold["f16_bits"], gold["f16_vals"]):
        o = oracle.f16_to_f32(int(b))
        assert (np.isnan(o) and np.isnan(v)) or np.float32(o) == v


def test_oracle_q80_matches_reference_c_decoder(gold):
    """q80_dot_block (q4k_decode.h) sums codes*x then scales once, like gemm.rs:325-328."""
    q8, x8 = gold["q8"], gold["x8"]
    for i in range(q8.shape[0]):
        y = oracle.matvec(oracle.Q8_0, q8[i], 1, 32, x8[i])
        assert np.float32(y[0]) == gold["dot8"][i], i


def test_live_reference_decoder_when_present():
    """In the container that has the reference checkout: also check live."""
    R = oracle.ref_lib()
    if R is None:
        pytest.skip("oracle/_ref not built (reference checkout absent)")
    import ctypes
    g = np.random.default_rng(5)
    for _ in range(32):
        b = g.integers(0, 256, 144, dtype=np.uint8)
        b[0:2] = np.array([g.uniform(0.01, 1)], dtype=np.float16).view(np.uint8)
        b[2:4] = np.array([g.uniform(0.01, 1)], dtype=np.float16).view(np.uint8)
        x = g.standard_normal(256).astype(np.float32)
        r = R.ref_q4k_dot_block(b.ctypes.data_as(ctypes.POINTER(ctypes.c_uint8)),
                                x.ctypes.data_as(ctypes.POINTER(ctypes.c_float)))
        assert np.float32(oracle.q4k_dot_ref(b, x)) == np.float32(r)


def test_q4k_matvec_equals_dequant_dot():
    """quant.rs:332-403: fused matvec agrees with dequantize-then-dot (rel 1e-3)."""
    g = np.random.default_rng(11)
    for cols in (256, 512, 2048):
        rows = 17
        w = oracle.quantize(oracle.Q4_K, g.standard_normal(rows * cols).astype(np.float32))
        x = g.standard_normal(cols).astype(np.float32)
        y = oracle.matvec(oracle.Q4_K, w, rows, cols, x)
        dense = oracle.dequant(oracle.Q4_K, w, rows * cols).reshape(rows, cols)
        ref = dense.astype(np.float64) @ x.astype(np.float64)
        assert np.all(np.abs(y - ref) <= 1e-3 * np.maximum(np.abs(ref), 1.0))


def test_quantizers_roundtrip():
    g = np.random.default_rng(3)
    v = g.standard_normal(4096).astype(np.float32)
    for dt, tol in ((oracle.Q8_0, 0.01), (oracle.Q4_K, 0.2), (oracle.Q6_K, 0.05)):
        w = oracle.quantize(dt, v)
        back = oracle.dequant(dt, w, v.size)
        assert np.sqrt(np.mean((back - v) ** 2)) < tol, dt


def test_cpu_baseline_matches_scalar():
    """AVX2 restatement (gemm.rs:806-894) vs scalar (gemm.rs:315-461): rounding only."""
    g = np.random.default_rng(9)
    from soso_b200 import synth
    for dt, rows, cols in ((oracle.Q4_K, 37, 1024), (oracle.Q8_0, 29, 512), (oracle.Q6_K, 9, 512)):
        w = synth.random_weights(dt, rows, cols, g)
        x = g.standard_normal(cols).astype(np.float32)
        a = oracle.cpu_matvec(dt, w, rows, cols, x, threads=3)
        b = oracle.matvec(dt, w, rows, cols, x)
        t = oracle.matvec_f64(dt, w, rows, cols, x)
        scale = np.sqrt(np.mean(t ** 2))
        assert np.all(np.abs(a - t) <= 1e-4 * np.maximum(np.abs(t), scale)), dt
        assert np.all(np.abs(b - t) <= 1e-4 * np.maximum(np.abs(t), scale)), dt


def test_row_strip():
    """parallel.rs:22-31."""
    for rows in (0, 1, 7, 100, 4096):
        for n in (1, 3, 8, 148):
            spans = [oracle.row_strip(rows, i, n) for i in range(n)]
            assert spans[0][0] == 0 and spans[-1][1] == rows
            for (a, b), (c, d) in zip(spans, spans[1:]):
                assert b == c
            lens = [b - a for a, b in spans]
            assert max(lens) - min(lens) <= 1
