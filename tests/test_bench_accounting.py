"""The arithmetic behind bench.py's roofline fractions, checked on the CPU against counts made
another way: the algorithmic bytes of a Q4_K matvec, the weight bytes one decode token reads
(configs[2] and [3], written out block by block from the architectures BASELINE.json states),
and the FLOPs of a block prefill (summed over decode.shapes, the matrix table the engine is
planned from, plus the causal attention)."""
import dataclasses

import bench
from soso_b200 import decode
from soso_b200.formats import row_bytes


def test_q4k_matvec_algorithmic_bytes():
    # 11008 x 4096: 16 blocks of 144 bytes a row, x and y in f32
    assert bench.algo_bytes(11008, 4096) == 11008 * 16 * 144 + 4096 * 4 + 11008 * 4


def test_weight_bytes_per_token_dense_configs2():
    q4 = lambda rows, cols: rows * (cols // 256) * 144  # noqa: E731
    q6 = lambda rows, cols: rows * (cols // 256) * 210  # noqa: E731
    layer = (q4(2048, 2048) + 2 * q4(256, 2048) + q4(2048, 2048)  # q, k, v, o
             + 2 * q4(11008, 2048) + q6(2048, 11008))              # gate, up (Q4_K), down (Q6_K)
    want = 36 * layer + q6(151936, 2048)                           # + the output matrix (Q6_K)
    assert want == 2_025_166_848
    assert bench.weight_bytes_per_token(decode.QWEN25_3B) == want


def test_weight_bytes_per_token_moe_configs3():
    q4 = lambda rows, cols: rows * (cols // 256) * 144  # noqa: E731
    experts = 8 * (2 * q4(768, 2048) + q4(2048, 768))  # top-8: gate, up, down of each chosen expert
    layer = q4(4096, 2048) + 2 * q4(512, 2048) + q4(2048, 4096) + q4(128, 2048) + experts
    want = 48 * layer + q4(151936, 2048)
    assert want == 1_710_931_968
    assert bench.weight_bytes_per_token(decode.QWEN3_30B_A3B) == want


def _flops_from_shapes(cfg, n):
    """2 x rows x cols a token for every matrix of decode.shapes a token goes through (MoE
    layers: the router and top_k experts), the causal attention 2 x (dqk + dv) per head and
    (query, key) pair, and the output matrix for the last token."""
    fl = 0
    for l in range(cfg.n_layers):
        for name, (rows, cols) in decode.shapes(cfg).items():
            if name.startswith("ffn_") and cfg.is_moe(l):
                continue
            fl += 2 * n * rows * cols
        if cfg.is_moe(l):
            fl += 2 * n * cfg.n_exp * cfg.hidden
            fl += 2 * n * cfg.top_k * 3 * cfg.moe_ffn * cfg.hidden
        pairs = n * (n + 1) // 2
        fl += 2 * cfg.heads * (2 * cfg.head_dim) * pairs
    return fl + 2 * cfg.vocab * cfg.hidden


def test_prefill_flops_dense_and_moe():
    for cfg in (decode.QWEN25_3B, decode.QWEN3_30B_A3B, dataclasses.replace(decode.TINY, n_layers=3)):
        for n in (1, 128, 512):
            assert bench.prefill_flops(cfg, n) == _flops_from_shapes(cfg, n), (cfg.n_layers, n)
