"""ctypes binding of librfx_b200.so (the C ABI declared in include/rfx.h).

The library is built in-tree (``python -m reflex_b200.build`` or
``__graft_entry__.build()``); importing this module fails loudly when it is
missing, so no code path can silently fall back to a CPU implementation.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, Structure, c_double, c_float, c_int, c_long, c_size_t, c_ubyte, c_void_p

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "librfx_b200.so")

RFX_OK = 0
RFX_E_INVAL = 1
RFX_E_CUDA = 2
RFX_E_DEVICE = 3
RFX_E_UNSUPPORTED = 4
RFX_E_STATE = 5

RFX_DTYPE_F32 = 0
RFX_DTYPE_BF16 = 1
RFX_QUANT_I8_SYM = 0
RFX_QUANT_U8_REF = 1
RFX_CHUNK_PI05 = 0
RFX_CHUNK_PI0 = 1
RFX_EMBED_CACHE_POOL_MSE = 0
RFX_EMBED_CACHE_BILINEAR_COS = 1
RFX_KV_RING_TILES = 0
RFX_KV_DENSE = 1

RFX_PRO_LOAD = 0
RFX_PRO_NORM = 1
RFX_EPI_STORE = 0
RFX_EPI_SILU = 1
RFX_EPI_QKV_ROPE = 2
RFX_EPI_RESIDUAL = 3
RFX_EPI_GEGLU = 4
RFX_EPI_GELU = 5

RFX_PACK_QKV_ROPE = 0
RFX_PACK_GATE_UP = 1

RFX_ADARMS_GATE = 0
RFX_ADARMS_SSG = 1


class RfxError(RuntimeError):
    """A librfx_b200 call returned a non-zero status."""

    def __init__(self, code: int, message: str):
        super().__init__(f"rfx error {code}: {message}")
        self.code = code


class KvQuantDesc(Structure):
    _fields_ = [
        ("mode", c_int), ("in_dtype", c_int),
        ("k", c_void_p), ("v", c_void_p),
        ("xs_b", c_long), ("xs_h", c_long), ("xs_l", c_long),
        ("B", c_int), ("H", c_int), ("L", c_int), ("D", c_int),
        ("k_q", c_void_p), ("v_q", c_void_p),
        ("qs_b", c_long), ("qs_h", c_long), ("qs_c", c_long),
        ("capacity", c_int),
        ("k_scale", c_void_p), ("v_scale", c_void_p),
        ("k_zp", c_void_p), ("v_zp", c_void_p),
        ("ss_b", c_long), ("ss_h", c_long), ("ss_c", c_long),
        ("region_base", c_int), ("region_off", c_int), ("region_len", c_int),
    ]


class LinearDesc(Structure):
    _fields_ = [
        ("T", c_int), ("O", c_int), ("K", c_int), ("tokens_per_batch", c_int),
        ("prologue", c_int), ("epilogue", c_int),
        ("w", c_void_p), ("x", c_void_p), ("ldx", c_int),
        ("norm_a1", c_void_p), ("norm_a2", c_void_p), ("norm_b2", c_void_p),
        ("norm_ab_stride", c_long), ("eps", c_float),
        ("y", c_void_p), ("ldy", c_int),
        ("bias", c_void_p), ("gate", c_void_p), ("gate_stride", c_long),
        ("rope_table", c_void_p), ("rope_max_pos", c_int), ("positions", c_void_p),
        ("q_out", c_void_p), ("k_out", c_void_p), ("v_out", c_void_p), ("num_q_heads", c_int),
        ("n_tile", c_int), ("splits", c_int),
        ("y_rows_per_batch", c_int), ("y_row_offset", c_int),
        ("workspace", c_void_p), ("workspace_bytes", c_size_t),
    ]


class AttnDesc(Structure):
    _fields_ = [
        ("B", c_int), ("num_q_heads", c_int), ("head_dim", c_int), ("S", c_int),
        ("capacity", c_int), ("n_ctx", c_int), ("quant_mode", c_int), ("scale_dtype", c_int),
        ("q", c_void_p), ("k_new", c_void_p), ("v_new", c_void_p),
        ("k_ring", c_void_p), ("v_ring", c_void_p),
        ("k_scale", c_void_p), ("v_scale", c_void_p), ("k_zp", c_void_p), ("v_zp", c_void_p),
        ("ctx_valid", c_void_p), ("new_block", c_void_p),
        ("softmax_scale", c_float), ("out", c_void_p),
        ("workspace", c_void_p), ("workspace_bytes", c_size_t), ("kv_splits", c_int), ("kv_source", c_int),
        ("dense_ctx_ready", c_int),
    ]


class TimeCondDesc(Structure):
    _fields_ = [
        ("n_t", c_int), ("t", c_void_p), ("width", c_int),
        ("min_period", c_double), ("max_period", c_double),
        ("w_in", c_void_p), ("b_in", c_void_p), ("w_out", c_void_p), ("b_out", c_void_p),
        ("hidden", c_void_p), ("cond", c_void_p),
    ]


class ModulationDesc(Structure):
    _fields_ = [
        ("mode", c_int), ("n_rows", c_int), ("n_norms", c_int), ("width", c_int),
        ("w", c_void_p), ("b", c_void_p), ("cond", c_void_p),
        ("a2", c_void_p), ("b2", c_void_p), ("gate", c_void_p),
    ]


class ActionIoDesc(Structure):
    _fields_ = [
        ("B", c_int), ("S", c_int), ("S_total", c_int), ("action_dim", c_int), ("width", c_int),
        ("h_row_offset", c_int), ("h", c_void_p),
        ("norm_a1", c_void_p), ("norm_a2", c_void_p), ("norm_b2", c_void_p),
        ("norm_ab_stride", c_long), ("eps", c_float),
        ("w_out", c_void_p), ("b_out", c_void_p), ("x", c_void_p), ("dt", c_float),
        ("w_in", c_void_p), ("b_in", c_void_p),
        ("h_next", c_void_p), ("h_next_ld", c_int),
        ("h_next_rows_per_stream", c_int), ("h_next_row_offset", c_int),
    ]


class CopyRowsDesc(Structure):
    _fields_ = [
        ("dst", c_void_p), ("dst_ld", c_long),
        ("dst_rows_per_group", c_int), ("dst_row_offset", c_int), ("group", c_int),
        ("src", c_void_p), ("src_ld", c_long), ("rows", c_int), ("width", c_int),
    ]


class NormDesc(Structure):
    _fields_ = [
        ("T", c_int), ("K", c_int), ("tokens_per_batch", c_int),
        ("x", c_void_p), ("ldx", c_int),
        ("norm_a1", c_void_p), ("norm_a2", c_void_p), ("norm_b2", c_void_p),
        ("norm_ab_stride", c_long), ("eps", c_float),
        ("y", c_void_p), ("ldy", c_int),
    ]


class PatchesDesc(Structure):
    _fields_ = [
        ("B", c_int), ("C", c_int), ("H", c_int), ("W", c_int), ("patch", c_int),
        ("image", c_void_p), ("out", c_void_p), ("ldo", c_int),
    ]


class LayerNormDesc(Structure):
    _fields_ = [
        ("T", c_int), ("C", c_int),
        ("x", c_void_p), ("ldx", c_int),
        ("w", c_void_p), ("b", c_void_p), ("eps", c_float),
        ("y", c_void_p), ("ldy", c_int),
    ]


class VitAttnDesc(Structure):
    _fields_ = [
        ("B", c_int), ("N", c_int), ("H", c_int), ("D", c_int),
        ("qkv", c_void_p), ("ld_qkv", c_int),
        ("out", c_void_p), ("ld_out", c_int),
        ("scale", c_float),
    ]


class ChunkDesc(Structure):
    _fields_ = [
        ("B", c_int), ("S", c_int), ("num_layers", c_int), ("num_steps", c_int),
        ("width", c_int), ("num_q_heads", c_int), ("mlp_dim", c_int), ("action_dim", c_int),
        ("eps", c_float), ("dt", c_float), ("softmax_scale", c_float),
        ("w_qkv", c_void_p), ("w_o", c_void_p), ("w_gu", c_void_p), ("w_down", c_void_p),
        ("norm_a1", c_void_p), ("mod_a2", c_void_p), ("mod_b2", c_void_p), ("mod_gate", c_void_p),
        ("w_in", c_void_p), ("b_in", c_void_p), ("w_out", c_void_p), ("b_out", c_void_p),
        ("rope_table", c_void_p), ("rope_max_pos", c_int), ("positions", c_void_p),
        ("capacity", c_int), ("n_ctx", c_int), ("quant_mode", c_int), ("scale_dtype", c_int), ("kv_splits", c_int),
        ("k_ring", POINTER(c_void_p)), ("v_ring", POINTER(c_void_p)),
        ("k_scale", POINTER(c_void_p)), ("v_scale", POINTER(c_void_p)),
        ("k_zp", POINTER(c_void_p)), ("v_zp", POINTER(c_void_p)),
        ("ctx_valid", c_void_p), ("x", c_void_p),
        ("variant", c_int), ("state_dim", c_int), ("state", c_void_p), ("w_state", c_void_p), ("b_state", c_void_p),
        ("w_atin", c_void_p), ("b_atin", c_void_p), ("w_atout", c_void_p), ("b_atout", c_void_p),
        ("time_emb", c_void_p), ("new_block", c_void_p),
        ("debug_hidden", c_void_p), ("debug_attn", c_void_p),
    ]


class EmbedCacheDesc(ctypes.Structure):
    _fields_ = [
        ("mode", c_int), ("B", c_int), ("C", c_int), ("H", c_int), ("W", c_int), ("in_dtype", c_int),
        ("pool", c_int), ("threshold", c_float), ("image", c_void_p), ("feat_prev", c_void_p),
        ("feat_new", c_void_p), ("sums", c_void_p), ("state", c_void_p), ("metric", c_void_p),
    ]


# Every entry point declared in include/rfx.h: name -> (argtypes, restype).
SIGNATURES = {
    "rfx_version": ([], c_int),
    "rfx_last_error": ([], ctypes.c_char_p),
    "rfx_device_status": ([c_void_p, POINTER(c_int)], c_int),
    "rfx_set_pdl": ([c_int], c_int),
    "rfx_embed_cache_check": ([POINTER(EmbedCacheDesc), c_void_p], c_int),
    "rfx_set_wait_limit_ns": ([ctypes.c_ulonglong], c_int),
    "rfx_set_trace": ([c_void_p, c_size_t], c_int),
    "rfx_set_chunk_cooperative": ([c_int], c_int),
    "rfx_num_sms": ([POINTER(c_int)], c_int),
    "rfx_kv_quant_append": ([POINTER(KvQuantDesc), c_void_p], c_int),
    "rfx_linear": ([POINTER(LinearDesc), c_void_p], c_int),
    "rfx_pack_weight": ([c_int, c_void_p, c_void_p, c_int, c_int, c_void_p], c_int),
    "rfx_attention": ([POINTER(AttnDesc), c_void_p], c_int),
    "rfx_attention_workspace_size": ([POINTER(AttnDesc), POINTER(c_size_t)], c_int),
    "rfx_linear_workspace_size": ([POINTER(LinearDesc), POINTER(c_size_t)], c_int),
    "rfx_attention_noalloc": ([POINTER(AttnDesc), c_void_p], c_int),
    "rfx_time_cond": ([POINTER(TimeCondDesc), c_void_p], c_int),
    "rfx_modulation": ([POINTER(ModulationDesc), c_void_p], c_int),
    "rfx_action_in": ([POINTER(ActionIoDesc), c_void_p], c_int),
    "rfx_euler_tail": ([POINTER(ActionIoDesc), c_void_p], c_int),
    "rfx_copy_rows": ([POINTER(CopyRowsDesc), c_void_p], c_int),
    "rfx_rms_norm": ([POINTER(NormDesc), c_void_p], c_int),
    "rfx_plan_add_rms_norm": ([c_void_p, POINTER(NormDesc)], c_int),
    "rfx_patches": ([POINTER(PatchesDesc), c_void_p], c_int),
    "rfx_layer_norm": ([POINTER(LayerNormDesc), c_void_p], c_int),
    "rfx_vit_attention": ([POINTER(VitAttnDesc), c_void_p], c_int),
    "rfx_plan_add_patches": ([c_void_p, POINTER(PatchesDesc)], c_int),
    "rfx_plan_add_layer_norm": ([c_void_p, POINTER(LayerNormDesc)], c_int),
    "rfx_plan_add_vit_attention": ([c_void_p, POINTER(VitAttnDesc)], c_int),
    "rfx_plan_add_chunk": ([c_void_p, c_void_p], c_int),
    "rfx_chunk_workspace_size": ([POINTER(ChunkDesc), POINTER(c_size_t)], c_int),
    "rfx_chunk_create": ([POINTER(ChunkDesc), c_void_p, c_size_t, POINTER(c_void_p)], c_int),
    "rfx_chunk_run": ([c_void_p, c_void_p], c_int),
    "rfx_chunk_destroy": ([c_void_p], c_int),
    "rfx_plan_add_barrier": ([c_void_p], c_int),
    "rfx_plan_create": ([POINTER(c_void_p)], c_int),
    "rfx_plan_destroy": ([c_void_p], c_int),
    "rfx_plan_add_linear": ([c_void_p, POINTER(LinearDesc)], c_int),
    "rfx_plan_add_attention": ([c_void_p, POINTER(AttnDesc)], c_int),
    "rfx_plan_add_kv_quant": ([c_void_p, POINTER(KvQuantDesc)], c_int),
    "rfx_plan_add_time_cond": ([c_void_p, POINTER(TimeCondDesc)], c_int),
    "rfx_plan_add_modulation": ([c_void_p, POINTER(ModulationDesc)], c_int),
    "rfx_plan_add_action_in": ([c_void_p, POINTER(ActionIoDesc)], c_int),
    "rfx_plan_add_euler_tail": ([c_void_p, POINTER(ActionIoDesc)], c_int),
    "rfx_plan_add_copy_rows": ([c_void_p, POINTER(CopyRowsDesc)], c_int),
    "rfx_plan_num_launches": ([c_void_p, POINTER(c_int)], c_int),
    "rfx_plan_run": ([c_void_p, c_void_p], c_int),
    "rfx_plan_capture": ([c_void_p, c_void_p], c_int),
    "rfx_plan_replay": ([c_void_p, c_void_p], c_int),
}

_lib = None


def load() -> ctypes.CDLL:
    """Loads librfx_b200.so once; raises if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `python -c 'import __graft_entry__ as g; g.build()'` "
            "(there is no CPU fallback for the rfx kernels)")
    lib = ctypes.CDLL(LIB_PATH)
    for name, (args, res) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = res
    _lib = lib
    return lib


def check(rc: int) -> None:
    if rc != RFX_OK:
        msg = load().rfx_last_error()
        raise RfxError(rc, msg.decode() if msg else "")


def call(name: str, *args) -> None:
    check(getattr(load(), name)(*args))


def ptr(t) -> int | None:
    """Device address of a tensor (None for None)."""
    return None if t is None else t.data_ptr()


__all__ = [n for n in dir() if n.startswith(("RFX_", "Rfx"))] + [
    "KvQuantDesc", "LinearDesc", "AttnDesc", "TimeCondDesc", "ModulationDesc", "ActionIoDesc", "CopyRowsDesc",
    "NormDesc", "ChunkDesc",
    "SIGNATURES", "load", "check", "call", "ptr", "LIB_PATH", "c_ubyte",
]
