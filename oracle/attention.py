"""Attention restated in fp32 torch (CPU).

``block_mask`` follows reflex/policies/pi05/utils.py:209-215 (token i may
attend to j iff cumsum(att)[j] <= cumsum(att)[i] and both are real tokens).
``attention_fp32`` follows reflex/layers/attention.py:98-164 (scores * scale,
hard mask, a dummy key 0 for fully masked rows, softmax, nan_to_num, PV),
with the single KV head broadcast over the query heads (MQA).
``partitioned_attention`` is the decode branch of StreamingAttention
(reflex/layers/streaming_attention.py:591-627): the suffix keys are appended
after the dequantized context cache and the suffix queries attend over both.
"""
from __future__ import annotations

import torch


def block_mask(pad: torch.Tensor, att: torch.Tensor) -> torch.Tensor:
    """pad [B, N] bool, att [B, N] -> allow [B, 1, N, N] bool."""
    cs = torch.cumsum(att.to(torch.int64), dim=1)
    allow = cs[:, None, :] <= cs[:, :, None]
    allow = allow & (pad[:, None, :] & pad[:, :, None])
    return allow[:, None]


def attention_fp32(q, k, v, allow, scale: float) -> torch.Tensor:
    q, k, v = q.float(), k.float(), v.float()
    scores = torch.matmul(q, k.transpose(-2, -1)) * scale
    if allow is not None:
        allow = allow.expand(scores.shape)
        scores = torch.where(allow, scores, torch.full_like(scores, float("-inf")))
        dead = ~allow.any(dim=-1)
        if dead.any():
            s = scores[dead]
            s[..., 0] = 0.0
            scores[dead] = s
    w = torch.softmax(scores, dim=-1)
    w = torch.nan_to_num(w, nan=0.0, posinf=0.0, neginf=0.0)
    return torch.matmul(w, v)


def partitioned_attention(q, k_ctx, v_ctx, k_suf, v_suf, ctx_pad, suf_att, scale: float) -> torch.Tensor:
    """q [B,H,S,D]; k/v_ctx [B,1,Lc,D] (already dequantized, fp32); k/v_suf [B,1,S,D];
    ctx_pad [B,Lc] bool; suf_att [S] block boundaries of the suffix (context att = 0)."""
    B, H, S, D = q.shape
    Lc = k_ctx.shape[2]
    pad = torch.cat([ctx_pad, torch.ones(B, S, dtype=torch.bool)], dim=1)
    att = torch.cat([torch.zeros(B, Lc, dtype=torch.int64), suf_att.to(torch.int64)[None].expand(B, S)], dim=1)
    allow = block_mask(pad, att)[:, :, Lc:, :]
    k = torch.cat([k_ctx.float(), k_suf.float()], dim=2)
    v = torch.cat([v_ctx.float(), v_suf.float()], dim=2)
    return attention_fp32(q, k, v, allow, scale)
