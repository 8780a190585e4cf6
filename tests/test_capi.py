"""CPU-side checks of the C ABI: the library loads without a GPU and exports
exactly what include/*.h declares, with the ctypes signatures matching."""
import ctypes
import glob
import os
import re

from soso_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        src = open(h).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        for m in re.finditer(r"^\s*[A-Za-z_][\w\s\*]*?\b(sbk?_\w+)\s*\(", src, flags=re.M):
            names.add(m.group(1))
    return names


def test_library_loads_and_exports_header():
    L = _lib.lib()
    names = declared_functions()
    assert len(names) >= 10
    for n in sorted(names):
        assert hasattr(L, n), f"{n} declared in include/ but not exported"


def test_ctypes_table_covers_header():
    assert declared_functions() == set(_lib.SIGNATURES), (
        declared_functions() ^ set(_lib.SIGNATURES))


def test_row_bytes_abi_matches_formats():
    from soso_b200 import formats
    L = _lib.lib()
    for dt in (2, 3, 13, 7):
        for cols in (0, 32, 256, 300, 4096, 11008):
            want = formats.row_bytes(dt, cols) or 0
            assert L.sbk_row_bytes(dt, cols) == want


def test_shape_rejections_need_no_gpu():
    """sbk_matvec validates before touching the device."""
    L = _lib.lib()
    p = ctypes.c_void_p(16)
    assert L.sbk_matvec(3, p, 4, 100, p, p, 0, None) == -1      # cols not a block multiple
    assert L.sbk_matvec(7, p, 4, 256, p, p, 0, None) == -1      # dtype without a kernel
    assert L.sbk_matvec(3, ctypes.c_void_p(8), 4, 256, p, p, 0, None) == -2  # misaligned weights
    assert L.sbk_matvec(3, None, 4, 256, p, p, 0, None) == -1


def test_product_has_no_oracle_dependency():
    """The product package must not import or link the oracle."""
    pkg = os.path.join(ROOT, "soso_b200")
    for f in glob.glob(os.path.join(pkg, "**", "*"), recursive=True):
        if f.endswith((".py", ".cu", ".cuh", ".cpp", ".h")):
            txt = open(f, errors="replace").read()
            assert "import oracle" not in txt and "from oracle" not in txt, f
            assert "liboracle" not in txt, f


def test_mla_shape_rejections_need_no_gpu():
    """sbk_mla_absorb / sbk_mla_attn validate before touching the device (every call here
    has exactly one bad argument; the valid remainder is DeepSeek-V2-Lite's shape)."""
    from soso_b200.formats import DTYPE_Q4_K
    L = _lib.lib()
    p = ctypes.c_void_p(256)

    def absorb(k_up=p, dt=DTYPE_Q4_K, heads=16, kv_heads=16, kv_rank=512, qk_nope=128, qk_rope=64, q=p):
        return L.sbk_mla_absorb(q, p, k_up, dt, p, p, p, p, p, heads, kv_heads, kv_rank, qk_nope, qk_rope, 2048,
                                1e4, 0, None)

    assert absorb(q=None) == -1
    assert absorb(dt=8) == -5                  # k_up must be Q4_K
    assert absorb(heads=17, kv_heads=17) == -1  # more heads than the kernels hold
    assert absorb(heads=16, kv_heads=3) == -1  # heads not a multiple of kv_heads
    assert absorb(kv_rank=300) == -1           # latent not whole Q4_K blocks
    assert absorb(qk_nope=257) == -1           # more nope rows than a thread's share covers
    assert absorb(qk_rope=63) == -1            # rope pairs
    assert absorb(k_up=ctypes.c_void_p(8)) == -2

    def attn(latent=p, kv_rank=512, qk_rope=64, ws=p):
        return L.sbk_mla_attn(p, p, latent, p, p, p, 16, 16, kv_rank, 128, qk_rope, 2048, ws, 0, None)

    assert attn(ws=None) == -1
    assert attn(kv_rank=256) == -1             # attention wants kv_rank a multiple of 512
    assert attn(qk_rope=256) == -1
    assert attn(latent=ctypes.c_void_p(8)) == -2
