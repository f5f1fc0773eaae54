"""KV quantizers, restated bit-exactly in numpy.

``quant_u8_ref`` follows reflex/layers/streaming_attention.py:211-218
(StreamingAttention._quantize): per (batch, head, token) row over head_dim,
uint8 asymmetric with a zero point, every operation rounded to the activation
dtype (bf16 on GPU, fp32 in the CPU config); torch.round is round-half-even.
``dequant_u8_ref`` follows :220-221.

``quant_i8_sym`` is the int8 symmetric per-token/per-head scheme of the
single-layer config (scale = absmax / 127 in fp32, q = clamp(rne(x / scale),
-127, 127)); the reference has no implementation of it.  absmax == 0 gives
scale 0 and q 0.
"""
from __future__ import annotations

import numpy as np

from .bf16 import bf16_round


def _rounder(act_bf16: bool):
    return bf16_round if act_bf16 else (lambda v: np.asarray(v, dtype=np.float32))


def quant_u8_ref(x, act_bf16: bool):
    """x: float32 array [..., D] holding activation-dtype values. Returns (q u8, scale, zp) float32 [..., 1]."""
    r = _rounder(act_bf16)
    x = np.asarray(x, dtype=np.float32)
    mn = x.min(axis=-1, keepdims=True)
    mx = x.max(axis=-1, keepdims=True)
    rng = r(mx - mn)
    rng = np.where(rng < np.float32(1e-5), r(np.float32(1e-5)), rng).astype(np.float32)
    scale = r(rng / np.float32(255.0))
    zp = r(-mn / scale)
    t1 = r(x / scale)
    t2 = r(t1 + zp)
    q = np.clip(np.rint(t2), 0, 255).astype(np.uint8)
    return q, scale.astype(np.float32), zp.astype(np.float32)


def dequant_u8_ref(q, scale, zp, act_bf16: bool):
    r = _rounder(act_bf16)
    return r(r(np.asarray(q, dtype=np.float32) - zp) * scale)


def quant_i8_sym(x):
    """x: float32 [..., D]. Returns (q int8 [..., D], scale float32 [..., 1])."""
    x = np.asarray(x, dtype=np.float32)
    amax = np.abs(x).max(axis=-1, keepdims=True)
    scale = (amax / np.float32(127.0)).astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore"):
        q = np.rint(x / scale)
    q = np.where(amax > 0, np.clip(q, -127, 127), 0).astype(np.int8)
    return q, scale


def dequant_i8_sym(q, scale):
    return np.asarray(q, dtype=np.float32) * scale
