"""Host-side mirror of the reference's operator boundary, `trait GpuDispatch`.

`CudaGpu` is to this package what `soso_llm_api::cuda::CudaGpu` is to the
reference (crates/soso-llm-api/src/cuda.rs:440, `impl GpuDispatch` :2415-2864):
same method names, argument meaning and results --

* ``True``  (``Ok(true)``):  the op ran on the device and ``out`` is fully written;
* ``False`` (``Ok(false)``): declined (dtype or shape this backend does not take);
* raises ``SbError``  (``Err(())``): the device call failed.

``try_gpu_matvec`` keeps the reference helper's behaviour of turning an error
into "not done" (crates/soso-llm-core/src/gpu.rs:766-788).  There is no CPU
path in here: a declined op is the caller's to compute.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np

from ._lib import SbError, SbMatvecOp, SbStats, SbView, c_f32p, c_u8p, last_error, lib
from .formats import DTYPE_F32, DTYPE_Q4_K, DTYPE_Q8_0


@dataclass
class TensorView:
    """`TensorView { bytes, dtype, elems }` (crates/soso-llm-core/src/layer.rs:26-31)."""
    bytes: np.ndarray  # uint8, the tensor in its on-disk layout
    dtype: int
    elems: int


@dataclass
class MatvecOp:
    """`MatvecOp` (crates/soso-llm-core/src/gpu.rs:189-196)."""
    key: str
    view: TensorView
    rows: int
    cols: int
    x: np.ndarray
    out: np.ndarray


@dataclass
class GpuStats:
    """The `GpuStats` fields this backend fills (gpu.rs:17-36): host-call launches, time and
    bytes; the per-step transfers of the device-resident decode; expert-pool hits / misses
    (always 0: every expert is resident)."""
    launches: int = 0
    total_ns: int = 0
    bytes_up: int = 0
    bytes_down: int = 0
    decode_embed_up: int = 0
    decode_control_up: int = 0
    decode_logits_down: int = 0
    decode_kv_down: int = 0
    decode_steps: int = 0
    stream_hits: int = 0
    stream_misses: int = 0


def _f32_arg(a: np.ndarray, n: int, name: str) -> np.ndarray:
    if not isinstance(a, np.ndarray) or a.dtype != np.float32 or not a.flags.c_contiguous:
        raise TypeError(f"{name} must be a C-contiguous float32 array")
    if a.size < n:
        raise ValueError(f"{name} has {a.size} elements, needs {n}")
    return a


def _view(v: TensorView) -> SbView:
    b = v.bytes
    if not isinstance(b, np.ndarray) or b.dtype != np.uint8 or not b.flags.c_contiguous:
        raise TypeError("TensorView.bytes must be a C-contiguous uint8 array")
    return SbView(b.ctypes.data_as(c_u8p), b.size, v.dtype, v.elems)


class CudaGpu:
    """GpuDispatch over libsosob200.so on one B200."""

    def __init__(self, device: int = 0):
        self._L = lib()
        h = ctypes.c_void_p()
        if self._L.sb_create(device, ctypes.byref(h)) != 0:
            raise SbError(f"sb_create({device}): {last_error()}")
        self._h = h
        self.device = device

    # `CudaGpu::nueva` returns Err when there is no device; Python raises.
    @classmethod
    def nueva(cls, device: int = 0) -> "CudaGpu":
        return cls(device)

    def close(self) -> None:
        if getattr(self, "_h", None):
            self._L.sb_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _check(self, rc: int, what: str) -> bool:
        if rc < 0:
            raise SbError(f"{what}: {last_error()}")
        return rc == 1

    # ---- GpuDispatch ---------------------------------------------------
    def available(self) -> bool:
        return bool(self._h) and self._L.sb_available(self._h) == 1

    def dtype_soportado(self, dtype: int) -> bool:
        return self._L.sb_dtype_supported(self._h, dtype) == 1

    dtype_supported = dtype_soportado

    def matvec(self, key: str, view: TensorView, rows: int, cols: int, x: np.ndarray, out: np.ndarray) -> bool:
        _f32_arg(x, cols, "x")
        _f32_arg(out, rows, "out")
        v = _view(view)
        rc = self._L.sb_matvec(self._h, key.encode(), ctypes.byref(v), rows, cols, x.ctypes.data_as(c_f32p),
                               out.ctypes.data_as(c_f32p))
        return self._check(rc, f"matvec({key})")

    def matmul(self, key: str, view: TensorView, rows: int, cols: int, n: int, x: np.ndarray,
               out: np.ndarray) -> bool:
        _f32_arg(x, n * cols, "x")
        _f32_arg(out, n * rows, "out")
        v = _view(view)
        rc = self._L.sb_matmul(self._h, key.encode(), ctypes.byref(v), rows, cols, n, x.ctypes.data_as(c_f32p),
                               out.ctypes.data_as(c_f32p))
        return self._check(rc, f"matmul({key})")

    def matvec_lote(self, ops: list[MatvecOp], hecho: list[bool]) -> None:
        """`matvec_lote` (gpu.rs:694-701): hecho[i] set for the ops done here."""
        views = [_view(op.view) for op in ops]
        arr = (SbMatvecOp * len(ops))()
        keys = [op.key.encode() for op in ops]
        for i, op in enumerate(ops):
            _f32_arg(op.x, op.cols, "x")
            _f32_arg(op.out, op.rows, "out")
            arr[i] = SbMatvecOp(keys[i], ctypes.pointer(views[i]), op.rows, op.cols, op.x.ctypes.data_as(c_f32p),
                                op.out.ctypes.data_as(c_f32p))
        done = (ctypes.c_uint8 * max(1, len(ops)))()
        rc = self._L.sb_matvec_batch(self._h, arr, len(ops), done)
        self._check(rc, "matvec_lote")
        for i in range(len(ops)):
            if done[i]:
                hecho[i] = True

    def matvec_batch(self, ops: list[MatvecOp]) -> bool:
        """`matvec_batch` (gpu.rs:704-713): True if any op ran."""
        hecho = [False] * len(ops)
        self.matvec_lote(ops, hecho)
        return any(hecho)

    def rmsnorm(self, x: np.ndarray, weight: np.ndarray, eps: float) -> bool:
        _f32_arg(x, 1, "x")
        _f32_arg(weight, x.size, "weight")
        rc = self._L.sb_rmsnorm(self._h, x.ctypes.data_as(c_f32p), weight.ctypes.data_as(c_f32p), x.size, eps)
        return self._check(rc, "rmsnorm")

    def residentes(self) -> int:
        return int(self._L.sb_resident_count(self._h))

    def stats(self) -> GpuStats:
        s = SbStats()
        self._L.sb_get_stats(self._h, ctypes.byref(s))
        return GpuStats(*(getattr(s, f) for f, _ in SbStats._fields_))


def dtype_ofrecible(dtype: int) -> bool:
    """`dtype_ofrecible` (gpu.rs:761-763) as far as this backend goes."""
    return dtype in (DTYPE_F32, DTYPE_Q8_0, DTYPE_Q4_K)


def try_gpu_matvec(gpu, key: str, view: TensorView, rows: int, cols: int, x: np.ndarray, out: np.ndarray) -> bool:
    """`try_gpu_matvec` (gpu.rs:766-788): Err is reported as not done."""
    if not gpu.available() or not gpu.dtype_soportado(view.dtype):
        return False
    if view.elems != rows * cols:
        return False
    try:
        return gpu.matvec(key, view, rows, cols, x, out)
    except SbError:
        return False
