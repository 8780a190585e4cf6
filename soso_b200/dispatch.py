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

from ._lib import (SbError, SbExpertBlock, SbMatvecOp, SbMoeLayerArgs, SbStats, SbView, c_f32p, c_u8p, last_error,
                   lib)
from .formats import DTYPE_F32, DTYPE_Q4_K, DTYPE_Q8_0


@dataclass
class TensorView:
    """`TensorView { bytes, dtype, elems }` (crates/soso-llm-core/src/layer.rs:26-31)."""
    bytes: np.ndarray  # uint8, the tensor in its on-disk layout
    dtype: int
    elems: int


@dataclass
class ExpertoBloque:
    """`ExpertoBloque` (crates/soso-llm-core/src/gpu.rs:175-187): the keys and views of an
    expert's ffn_gate / ffn_up / ffn_down (a view may be None for a resident tensor), the
    block's tokens that chose it, shared or routed, and each token's weight index
    token * top_k + rank."""
    claves: list
    vistas: list
    tokens: np.ndarray
    compartido: bool
    destinos: np.ndarray


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
class MoeNormas:
    """`MoeNormas` (crates/soso-llm-core/src/gpu.rs:279-289): what a MoE layer sends once."""
    attn_norm: np.ndarray
    q_norm: np.ndarray
    k_norm: np.ndarray
    ffn_norm: np.ndarray
    router: np.ndarray  # [n_exp x h] f32
    rope_factores: np.ndarray | None = None


@dataclass
class MoeCapa:
    """`MoeCapa` (crates/soso-llm-core/src/gpu.rs:294-335): one MoE layer of a block of n
    tokens; `hidden` [n x h] f32 in and out.  `flujo` stands for the reference's expert
    provider (streamed experts), which this backend does not take: every expert must be
    resident (gemma_subir)."""
    layer: int
    pos0: int
    n: int
    hidden: np.ndarray
    h: int
    heads: int
    kv_heads: int
    head_dim: int
    ffn: int
    n_exp: int
    top_k: int
    ventana: int
    ctx_max: int
    eps: float
    theta: float
    escala: float
    qk_norm: bool
    rope_mscale: float
    continuar: bool
    encadenar: bool
    clave_q: str
    clave_k: str
    clave_v: str
    clave_o: str
    prefijo: str
    normas: MoeNormas | None = None
    flujo: object = None
    expulsadas: int = 0


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

    def gemma_subir(self, key: str, view: TensorView, rows: int, cols: int) -> bool:
        """`gemma_subir` (gpu.rs:364-368): the tensor resident under its key."""
        v = _view(view)
        return self._check(self._L.sb_upload(self._h, key.encode(), ctypes.byref(v), rows, cols), f"upload({key})")

    def router_topk(self, key: str, w: np.ndarray, xs: np.ndarray, n: int, h: int, n_exp: int, top_k: int,
                    idx: np.ndarray, pesos: np.ndarray) -> bool:
        """`router_topk` (gpu.rs:477-494): idx / pesos [n x top_k] in rank order."""
        _f32_arg(w, n_exp * h, "w")
        _f32_arg(xs, n * h, "xs")
        _f32_arg(pesos, n * top_k, "pesos")
        if idx.dtype != np.int32 or idx.size < n * top_k or not idx.flags.c_contiguous:
            raise TypeError("idx must be a C-contiguous int32 array of n * top_k")
        rc = self._L.sb_router_topk(self._h, key.encode(), w.ctypes.data_as(c_f32p), xs.ctypes.data_as(c_f32p), n, h,
                                    n_exp, top_k, idx.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)),
                                    pesos.ctypes.data_as(c_f32p))
        return self._check(rc, f"router_topk({key})")

    def expertos_bloque(self, xs: np.ndarray, n: int, h: int, ffn: int, top_k: int, pesos: np.ndarray, exps: list,
                        suma: np.ndarray, hecho: list) -> None:
        """`expertos_bloque` (gpu.rs:457-475): exps = ExpertoBloque items; suma [n x h] gets the
        weighted sum (rank order) of the experts resolved here, hecho[i] marks them."""
        _f32_arg(xs, n * h, "xs")
        _f32_arg(pesos, n * top_k, "pesos")
        _f32_arg(suma, n * h, "suma")
        arr = (SbExpertBlock * max(1, len(exps)))()
        keep = []
        for i, e in enumerate(exps):
            keys = [k.encode() for k in e.claves]
            views = [None if v is None else _view(v) for v in e.vistas]
            toks = np.ascontiguousarray(e.tokens, dtype=np.uint32)
            dest = np.ascontiguousarray(e.destinos, dtype=np.uint32)
            keep += [keys, views, toks, dest]
            arr[i].keys = (ctypes.c_char_p * 3)(*keys)
            arr[i].views = (ctypes.POINTER(SbView) * 3)(*[ctypes.pointer(v) if v is not None else None for v in views])
            arr[i].tokens = toks.ctypes.data_as(ctypes.POINTER(ctypes.c_uint32))
            arr[i].n_tokens = toks.size
            arr[i].shared = int(e.compartido)
            arr[i].dests = dest.ctypes.data_as(ctypes.POINTER(ctypes.c_uint32))
        done = (ctypes.c_uint8 * max(1, len(exps)))()
        rc = self._L.sb_experts(self._h, xs.ctypes.data_as(c_f32p), n, h, ffn, top_k, pesos.ctypes.data_as(c_f32p),
                                arr, len(exps), suma.ctypes.data_as(c_f32p), done)
        self._check(rc, "expertos_bloque")
        for i in range(len(exps)):
            if done[i]:
                hecho[i] = True

    def atencion_prefill(self, capa: int, q: np.ndarray, out: np.ndarray, n: int, seq_antes: int, heads: int,
                         kv_heads: int, hd: int, k: np.ndarray, v: np.ndarray, filas_validas: list) -> bool:
        """`atencion_prefill` (gpu.rs:496-517): filas_validas = [rows the device mirrors]."""
        _f32_arg(q, n * heads * hd, "q")
        _f32_arg(out, n * heads * hd, "out")
        kk = np.ascontiguousarray(k, dtype=np.uint16)
        vv = np.ascontiguousarray(v, dtype=np.uint16)
        fv = ctypes.c_size_t(filas_validas[0])
        u16 = ctypes.POINTER(ctypes.c_uint16)
        rc = self._L.sb_attention_prefill(self._h, capa, q.ctypes.data_as(c_f32p), out.ctypes.data_as(c_f32p), n,
                                          seq_antes, heads, kv_heads, hd, kk.ctypes.data_as(u16),
                                          vv.ctypes.data_as(u16), ctypes.byref(fv))
        ok = self._check(rc, "atencion_prefill")
        filas_validas[0] = fv.value
        return ok

    def moe_capa(self, capa: MoeCapa) -> bool:
        """`moe_capa` (gpu.rs:424-429): the whole layer on the device."""
        _f32_arg(capa.hidden, capa.n * capa.h, "hidden")
        keep = []

        def f32(a, n, name):
            if a is None:
                return None
            arr = np.ascontiguousarray(a, dtype=np.float32)
            if arr.size != n:
                raise ValueError(f"{name}: {arr.size} values, want {n}")
            keep.append(arr)
            return arr.ctypes.data
        nm = capa.normas
        a = SbMoeLayerArgs()
        a.layer, a.pos0, a.n, a.hidden = capa.layer, capa.pos0, capa.n, capa.hidden.ctypes.data
        a.h, a.heads, a.kv_heads, a.head_dim = capa.h, capa.heads, capa.kv_heads, capa.head_dim
        a.ffn, a.n_exp, a.top_k, a.window, a.ctx_max = capa.ffn, capa.n_exp, capa.top_k, capa.ventana, capa.ctx_max
        a.eps, a.theta, a.scale, a.qk_norm = capa.eps, capa.theta, capa.escala, int(capa.qk_norm)
        a.rope_mscale, a.cont, a.chain = capa.rope_mscale, int(capa.continuar), int(capa.encadenar)
        a.key_q, a.key_k, a.key_v = capa.clave_q.encode(), capa.clave_k.encode(), capa.clave_v.encode()
        a.key_o, a.prefix = capa.clave_o.encode(), capa.prefijo.encode()
        if nm is not None:
            a.attn_norm = f32(nm.attn_norm, capa.h, "attn_norm")
            a.ffn_norm = f32(nm.ffn_norm, capa.h, "ffn_norm")
            a.q_norm = f32(nm.q_norm, capa.head_dim, "q_norm") if capa.qk_norm else None
            a.k_norm = f32(nm.k_norm, capa.head_dim, "k_norm") if capa.qk_norm else None
            a.router = f32(nm.router, capa.n_exp * capa.h, "router")
            a.rope_factors = f32(nm.rope_factores, capa.head_dim // 2, "rope_factores")
        a.streamed = int(capa.flujo is not None)
        ok = self._check(self._L.sb_moe_layer(self._h, ctypes.byref(a)), "moe_capa")
        capa.expulsadas = int(a.evicted)
        return ok

    def moe_lista(self, layer: int) -> bool:
        return self._check(self._L.sb_moe_ready(self._h, layer), "moe_lista")

    def moe_puede(self, layer: int) -> bool:
        return self._check(self._L.sb_moe_can(self._h, layer), "moe_puede")

    def moe_pendiente(self, layer: int, pos0: int, n: int) -> bool:
        return self._check(self._L.sb_moe_pending(self._h, layer, pos0, n), "moe_pendiente")

    def moe_volcar(self, hidden: np.ndarray) -> None:
        if hidden.dtype != np.float32 or not hidden.flags.c_contiguous:
            raise ValueError("hidden: contiguous float32 wanted")
        self._check(self._L.sb_moe_flush(self._h, hidden.ctypes.data_as(c_f32p), hidden.size), "moe_volcar")

    def moe_descartar(self, layer: int) -> None:
        self._check(self._L.sb_moe_discard(self._h, layer), "moe_descartar")

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
