"""ctypes binding of libsosob200.so -- the only way Python reaches the kernels.

There is no fallback: if the library is missing or cannot be loaded, every
entry point raises.  The declarations follow include/sosob200.h.
"""
from __future__ import annotations

import ctypes
import os

from . import build as _build

c_u8p = ctypes.POINTER(ctypes.c_uint8)
c_f32p = ctypes.POINTER(ctypes.c_float)
c_size = ctypes.c_size_t


class SbView(ctypes.Structure):
    _fields_ = [("bytes", c_u8p), ("len", c_size), ("dtype", ctypes.c_uint8), ("elems", c_size)]


class SbMatvecOp(ctypes.Structure):
    _fields_ = [("key", ctypes.c_char_p), ("view", ctypes.POINTER(SbView)), ("rows", c_size), ("cols", c_size),
                ("x", c_f32p), ("out", c_f32p)]


class SbkMvOp(ctypes.Structure):
    _fields_ = [("w", ctypes.c_void_p), ("rows", c_size), ("cols", c_size), ("x", ctypes.c_void_p),
                ("y", ctypes.c_void_p)]


class SbkXSrc(ctypes.Structure):
    """sbk_xsrc: how a fused batch forms its input (mode SBK_XS_PLAIN 0 / NORM 1 / SWIGLU 2)."""
    _fields_ = [("res", ctypes.c_void_p), ("norm_w", ctypes.c_void_p), ("h_out", ctypes.c_void_p),
                ("eps", ctypes.c_float), ("mode", ctypes.c_int), ("ys", ctypes.c_void_p), ("yw", ctypes.c_void_p),
                ("ny", ctypes.c_int), ("ystride", ctypes.c_int)]


class SbStats(ctypes.Structure):
    _fields_ = [(n, ctypes.c_uint64) for n in ("launches", "total_ns", "bytes_up", "bytes_down", "decode_embed_up",
                                               "decode_control_up", "decode_logits_down", "decode_kv_down",
                                               "decode_steps", "stream_hits", "stream_misses")]


class SbExpertBlock(ctypes.Structure):
    _fields_ = [("keys", ctypes.c_char_p * 3), ("views", ctypes.POINTER(SbView) * 3),
                ("tokens", ctypes.POINTER(ctypes.c_uint32)), ("n_tokens", c_size), ("shared", ctypes.c_int),
                ("dests", ctypes.POINTER(ctypes.c_uint32))]


class SbMoeLayerArgs(ctypes.Structure):
    """sb_moe_layer_args: the MoeCapa mirror (include/sosob200.h)."""
    _fields_ = [("layer", ctypes.c_uint32), ("pos0", c_size), ("n", c_size), ("hidden", ctypes.c_void_p),
                ("h", c_size), ("heads", c_size), ("kv_heads", c_size), ("head_dim", c_size), ("ffn", c_size),
                ("n_exp", c_size), ("top_k", c_size), ("window", c_size), ("ctx_max", c_size),
                ("eps", ctypes.c_float), ("theta", ctypes.c_float), ("scale", ctypes.c_float),
                ("qk_norm", ctypes.c_int), ("rope_mscale", ctypes.c_float), ("cont", ctypes.c_int),
                ("chain", ctypes.c_int), ("key_q", ctypes.c_char_p), ("key_k", ctypes.c_char_p),
                ("key_v", ctypes.c_char_p), ("key_o", ctypes.c_char_p), ("prefix", ctypes.c_char_p),
                ("attn_norm", ctypes.c_void_p), ("q_norm", ctypes.c_void_p), ("k_norm", ctypes.c_void_p),
                ("ffn_norm", ctypes.c_void_p), ("router", ctypes.c_void_p), ("rope_factors", ctypes.c_void_p),
                ("streamed", ctypes.c_int), ("evicted", c_size)]


class SbLayerState(ctypes.Structure):
    _fields_ = [("k", ctypes.c_void_p), ("v", ctypes.c_void_p), ("valid_rows", ctypes.POINTER(ctypes.c_size_t))]


class SbLayerRows(ctypes.Structure):
    _fields_ = [("k", ctypes.c_void_p), ("v", ctypes.c_void_p)]


class SbMat(ctypes.Structure):
    _fields_ = [("key", ctypes.c_char_p), ("view", SbView), ("rows", c_size), ("cols", c_size)]


class SbMoePlan(ctypes.Structure):
    _fields_ = [("n_exp", c_size), ("top_k", c_size), ("ffn", c_size), ("router", SbMat),
                ("experts", ctypes.POINTER(SbMat)), ("shared", ctypes.POINTER(SbMat)), ("shared_gate", c_f32p)]


class SbMlaPlan(ctypes.Structure):
    _fields_ = [("q_rank", c_size), ("kv_rank", c_size), ("qk_nope", c_size), ("qk_rope", c_size), ("v_dim", c_size),
                ("q_down", SbMat), ("q_up", SbMat), ("kv_down", SbMat), ("k_up", SbMat), ("v_up", SbMat)]


class SbLayerPlan(ctypes.Structure):
    _fields_ = [("heads", c_size), ("kv_heads", c_size), ("head_dim", c_size), ("theta", ctypes.c_float),
                ("neox", ctypes.c_int), ("q_norm", c_f32p), ("k_norm", c_f32p), ("qkv_bias", c_f32p),
                ("norm_attn", c_f32p), ("norm_ffn", c_f32p), ("q", SbMat), ("k", SbMat), ("v", SbMat), ("o", SbMat),
                ("gate", SbMat), ("up", SbMat), ("down", SbMat), ("moe", ctypes.POINTER(SbMoePlan)),
                ("mla", ctypes.POINTER(SbMlaPlan)), ("rope_factors", c_f32p), ("rope_mscale", ctypes.c_float)]


class SbDecodePlan(ctypes.Structure):
    _fields_ = [("layers", ctypes.POINTER(SbLayerPlan)), ("n_layers", c_size), ("hidden", c_size), ("vocab", c_size),
                ("ctx", c_size), ("eps", ctypes.c_float), ("final_norm", c_f32p), ("lm_head", SbMat),
                ("embed", SbMat)]


# name -> (restype, argtypes); must match include/sosob200.h
SIGNATURES = {
    "sb_create": (ctypes.c_int, [ctypes.c_int, ctypes.POINTER(ctypes.c_void_p)]),
    "sb_destroy": (None, [ctypes.c_void_p]),
    "sb_available": (ctypes.c_int, [ctypes.c_void_p]),
    "sb_dtype_supported": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_uint8]),
    "sb_matvec": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_char_p, ctypes.POINTER(SbView), c_size, c_size, c_f32p,
                                 c_f32p]),
    "sb_matmul": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_char_p, ctypes.POINTER(SbView), c_size, c_size, c_size,
                                 c_f32p, c_f32p]),
    "sb_matvec_batch": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(SbMatvecOp), c_size, c_u8p]),
    "sb_rmsnorm": (ctypes.c_int, [ctypes.c_void_p, c_f32p, c_f32p, c_size, ctypes.c_float]),
    "sb_resident_count": (c_size, [ctypes.c_void_p]),
    "sb_upload": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_char_p, ctypes.POINTER(SbView), c_size, c_size]),
    "sb_router_topk": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_char_p, c_f32p, c_f32p, c_size, c_size, c_size, c_size,
                                      ctypes.POINTER(ctypes.c_int32), c_f32p]),
    "sb_experts": (ctypes.c_int, [ctypes.c_void_p, c_f32p, c_size, c_size, c_size, c_size, c_f32p,
                                  ctypes.POINTER(SbExpertBlock), c_size, c_f32p, c_u8p]),
    "sb_attention_prefill": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_uint32, c_f32p, c_f32p, c_size, c_size, c_size,
                                            c_size, c_size, ctypes.POINTER(ctypes.c_uint16),
                                            ctypes.POINTER(ctypes.c_uint16), ctypes.POINTER(c_size)]),
    "sb_get_stats": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(SbStats)]),
    "sb_moe_layer": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(SbMoeLayerArgs)]),
    "sb_moe_ready": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_uint32]),
    "sb_moe_can": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_uint32]),
    "sb_moe_pending": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_uint32, c_size, c_size]),
    "sb_moe_flush": (ctypes.c_int, [ctypes.c_void_p, c_f32p, c_size]),
    "sb_moe_discard": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_uint32]),
    "sb_last_error": (ctypes.c_char_p, []),
    "sb_decode_prepare": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(SbDecodePlan)]),
    "sb_decode_token": (ctypes.c_int, [ctypes.c_void_p, c_f32p, c_size, c_f32p, ctypes.POINTER(ctypes.c_uint16)]),
    "sb_group_handle_bytes": (c_size, []),
    "sb_group_create": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]),
    "sb_group_open": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p]),
    "sb_decode_finish": (ctypes.c_int, [ctypes.c_void_p]),
    "sb_decode_greedy": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(ctypes.c_int32), c_size, c_size, c_size,
                                        ctypes.POINTER(ctypes.c_int32)]),
    "sb_decode_upload_state": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(SbLayerState), c_size, c_size]),
    "sb_decode_download_state": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(SbLayerRows), c_size, c_size,
                                                c_f32p]),
    "sb_decode_routes": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(ctypes.c_int32), c_size]),
    "sb_decode_route_trace": (ctypes.c_int, [ctypes.c_void_p, c_size, ctypes.POINTER(ctypes.c_int32), c_size,
                                             ctypes.POINTER(ctypes.c_float), c_size]),
    "sb_decode_prefill": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(ctypes.c_int32), c_size, c_size, c_f32p,
                                         ctypes.POINTER(ctypes.c_int32)]),
    "sbk_row_bytes": (c_size, [ctypes.c_uint8, c_size]),
    "sbk_q6k_pack": (ctypes.c_int, [ctypes.c_void_p, c_size, c_size, ctypes.c_void_p, ctypes.c_void_p]),
    "sbk_q80_pad": (ctypes.c_int, [ctypes.c_void_p, c_size, c_size, ctypes.c_void_p, ctypes.c_void_p]),
    "sbk_swiglu": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, c_size, ctypes.c_int,
                                  ctypes.c_void_p]),
    "sbk_matvec": (ctypes.c_int, [ctypes.c_uint8, ctypes.c_void_p, c_size, c_size, ctypes.c_void_p, ctypes.c_void_p,
                                  ctypes.c_int, ctypes.c_void_p]),
    "sbk_rmsnorm": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                   ctypes.c_void_p, c_size, c_size, ctypes.c_float, ctypes.c_void_p]),
    "sbk_matvec_batch": (ctypes.c_int, [ctypes.c_uint8, ctypes.c_void_p, c_size, ctypes.c_int, ctypes.c_void_p]),
    "sbk_matvec_batch_x": (ctypes.c_int, [ctypes.c_uint8, ctypes.c_void_p, c_size, ctypes.POINTER(SbkXSrc),
                                          ctypes.c_int, ctypes.c_void_p]),
    "sbk_attn_rope_decode": (ctypes.c_int, [ctypes.c_void_p] * 8 + [c_size] * 4 + [ctypes.c_float, ctypes.c_float,
                                                                           ctypes.c_int, ctypes.c_void_p,
                                                                           ctypes.c_int, ctypes.c_void_p]),
    "sbk_attn_rope_decode_yarn": (ctypes.c_int, [ctypes.c_void_p] * 8 + [c_size] * 4 +
                                  [ctypes.c_float, ctypes.c_float, ctypes.c_int, ctypes.c_void_p, ctypes.c_float,
                                   ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p]),
    "sbk_rope_kv_append": (ctypes.c_int, [ctypes.c_void_p] * 7 + [c_size] * 4 + [ctypes.c_float, ctypes.c_float,
                                                                          ctypes.c_int, ctypes.c_int, ctypes.c_void_p]),
    "sbk_rope_kv_append_yarn": (ctypes.c_int, [ctypes.c_void_p] * 7 + [c_size] * 4 +
                                [ctypes.c_float, ctypes.c_float, ctypes.c_int, ctypes.c_void_p, ctypes.c_float,
                                 ctypes.c_int, ctypes.c_void_p]),
    "sbk_attn_ws_bytes": (c_size, [c_size] * 4),
    "sbk_attn_decode": (ctypes.c_int, [ctypes.c_void_p] * 5 + [c_size] * 4 + [ctypes.c_void_p, ctypes.c_int,
                                                                          ctypes.c_void_p]),
    "sbk_router_topk": (ctypes.c_int, [ctypes.c_void_p, c_size, c_size, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
                                       ctypes.c_void_p]),
    "sbk_argmax_ws_bytes": (c_size, []),
    "sbk_argmax": (ctypes.c_int, [ctypes.c_void_p, c_size, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
                                  ctypes.c_void_p]),
    "sbk_embed_row": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_uint8, c_size, c_size, ctypes.c_void_p, ctypes.c_void_p,
                                     ctypes.c_int, ctypes.c_void_p]),
    "sbk_matvec_q4k_noalloc": (ctypes.c_int, [ctypes.c_void_p, c_size, c_size, ctypes.c_void_p, ctypes.c_void_p,
                                              ctypes.c_void_p]),
    "sbk_num_sms": (ctypes.c_int, [ctypes.c_int]),
    "sb_crc32c": (ctypes.c_uint32, [ctypes.c_void_p, c_size]),
    "sb_som_payload": (ctypes.c_int, [ctypes.c_void_p, c_size, ctypes.c_int, ctypes.POINTER(ctypes.c_void_p),
                                      ctypes.POINTER(c_size), ctypes.POINTER(ctypes.c_uint32)]),
    "sbk_matmul_ws_bytes": (c_size, [c_size, c_size]),
    "sbk_mla_ws_bytes": (c_size, [c_size, c_size]),
    "sbk_mla_absorb": (ctypes.c_int, [ctypes.c_void_p] * 3 + [ctypes.c_uint8] + [ctypes.c_void_p] * 5 +
                       [c_size] * 6 + [ctypes.c_float, ctypes.c_int, ctypes.c_void_p]),
    "sbk_mla_attn": (ctypes.c_int, [ctypes.c_void_p] * 6 + [c_size] * 6 + [ctypes.c_void_p, ctypes.c_int,
                                                                         ctypes.c_void_p]),
    "sbk_matmul": (ctypes.c_int, [ctypes.c_uint8, ctypes.c_void_p, c_size, c_size, c_size, ctypes.c_void_p,
                                  ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]),
    "sbk_take_device_error": (ctypes.c_int, [ctypes.c_int, ctypes.POINTER(ctypes.c_uint32)]),
    "sbk_exchange_wait": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_uint, ctypes.c_uint, ctypes.c_void_p,
                                         ctypes.c_void_p]),
}

_L = None


def lib():
    """Load (building first if the sources are newer) and declare the library."""
    global _L
    if _L is None:
        path = _build.LIB
        if not os.path.exists(path) or _build.stale():
            try:
                _build.build()
            except Exception as e:  # no nvcc on this host and no prebuilt library
                if not os.path.exists(path):
                    raise RuntimeError(f"libsosob200.so is missing and could not be built: {e}") from e
        L = ctypes.CDLL(path)
        for name, (res, args) in SIGNATURES.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _L = L
    return _L


def last_error() -> str:
    return (lib().sb_last_error() or b"").decode(errors="replace")


class SbError(RuntimeError):
    """An `Err(())` of the GpuDispatch contract: the call failed on the device."""
