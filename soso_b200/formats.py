"""On-disk block formats of the reference (bytes are used unchanged on device).

crates/sosomodel/src/layout.rs:8-12 (dtype codes), :57-64 (Q8_0 / Q4_K blocks);
Q6_K is GGML block_q6_K (crates/gguf2som/src/lib.rs:1639-1661), code 13 is this
project's extension (the reference has no Q6_K dtype).
"""
DTYPE_F32, DTYPE_Q8_0, DTYPE_Q4_K, DTYPE_Q6_K = 1, 2, 3, 13

# dtype -> (elements per block, bytes per block)
BLOCKS = {DTYPE_Q8_0: (32, 36), DTYPE_Q4_K: (256, 144), DTYPE_Q6_K: (256, 210)}
NAMES = {DTYPE_F32: "F32", DTYPE_Q8_0: "Q8_0", DTYPE_Q4_K: "Q4_K", DTYPE_Q6_K: "Q6_K"}


def row_bytes(dtype: int, cols: int) -> int | None:
    """`sosomodel::dequant::row_bytes` (crates/sosomodel/src/dequant.rs:53-63)."""
    if dtype == DTYPE_F32:
        return cols * 4
    if dtype not in BLOCKS:
        return None
    be, bb = BLOCKS[dtype]
    if cols == 0 or cols % be:
        return None
    return cols // be * bb
