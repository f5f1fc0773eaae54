"""Action-expert denoising chunk, restated in torch on the CPU.

Follows, function by function:
* create_sinusoidal_pos_embedding      reflex/policies/pi05/utils.py:72-121
* PI05SuffixEmbedder.forward            reflex/policies/pi05/modeling_pi05.py:307-368
* PI0SuffixEmbedder.forward             reflex/policies/pi0/modeling_pi0.py:144-206
* AdaRMSNorm.forward                    reflex/policies/pi05/modeling_pi05.py:73-99
* PI05ModelLayer.forward                reflex/policies/pi05/modeling_pi05.py:563-620
* PI05Attention.forward (fused QKV)     reflex/policies/pi05/modeling_pi05.py:429-494
* RotaryEmbedding / apply_rotary_emb    reflex/layers/rope.py:34-60, 104-132
* attention over [context ; suffix]     reflex/layers/streaming_attention.py:591-627,
                                        reflex/layers/attention.py:98-164
* PI05MLP.forward                       reflex/policies/pi05/modeling_pi05.py:510-534
* denoise_step / Euler loop             reflex/policies/pi05/modeling_pi05.py:1181-1241, 1403-1419
                                        (PI0: reflex/policies/pi0/modeling_pi0.py:740-782, 827-845)
The scale/shift/gate adaRMS variant ("ssg") has no reference source here
(parity unpinned); it follows the published adaRMSNorm formulation
y = rmsnorm(x) * (1 + scale) + shift with a residual gate.

``bf16=False`` is the reference's fp32 path (the parity target).
``bf16=True`` additionally rounds activations to bf16 where the CUDA engine
stores them (norm outputs, GEMM outputs, the residual stream, attention
output): a CPU model of the engine's numerics used to size tolerances.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from .attention import partitioned_attention


def _r(x: torch.Tensor, on: bool) -> torch.Tensor:
    return x.to(torch.bfloat16).to(torch.float32) if on else x


def sinusoid(t: torch.Tensor, dim: int, min_period: float, max_period: float) -> torch.Tensor:
    frac = torch.linspace(0.0, 1.0, dim // 2, dtype=torch.float64)
    period = min_period * (max_period / min_period) ** frac
    scaling = 1.0 / period * 2 * math.pi
    x = scaling[None, :] * t.to(torch.float64)[:, None]
    return torch.cat([torch.sin(x), torch.cos(x)], dim=1)


def linear(x, w, b=None):
    y = x @ w.t()
    return y + b if b is not None else y


def rope(x: torch.Tensor, pos: torch.Tensor, table: torch.Tensor) -> torch.Tensor:
    """x [B, H, L, D], pos [B, L]."""
    cs = table[pos]
    cos, sin = cs.chunk(2, dim=-1)
    cos, sin = cos[:, None], sin[:, None]
    x1, x2 = x.float().chunk(2, dim=-1)
    return torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], dim=-1)


def rms_norm(x, eps):
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps)


def norm(x, cond, wts, name, adarms, eps, bf16):
    """Returns (y, gate): AdaRMSNorm (gate / none) or scale/shift/gate adaRMS."""
    xn = rms_norm(x, eps)
    if adarms == "ssg":
        m = linear(cond, wts[name + ".dense.weight"], wts[name + ".dense.bias"])[:, None, :]
        scale, shift, gate = m.chunk(3, dim=-1)
        y = xn * (1 + scale) + shift
        return _r(y, bf16), _r(gate, bf16)
    y = wts[name + ".weight"] * xn
    if adarms == "gate":
        m = linear(cond, wts[name + ".dense.weight"], wts[name + ".dense.bias"])[:, None, :]
        return _r(y * m, bf16), _r(m, bf16)
    return _r(y, bf16), torch.ones_like(y)


@dataclass
class Context:
    """Dequantized context K/V per layer ([B, 1, Lc, D] fp32) and padding mask."""

    k: list
    v: list
    pad: torch.Tensor  # [B, Lc] bool


def suffix_embed(cfg, wts, state, x_t, t, bf16):
    """-> (embs [B, S_total, W], att row [S_total], cond [B, W] or None)."""
    B = x_t.shape[0]
    temb = sinusoid(t.expand(B), cfg.width, cfg.min_period, cfg.max_period)
    if cfg.variant == "pi05":
        temb = _r(temb.float(), bf16)
        h = _r(torch.nn.functional.silu(_r(linear(temb, wts["time_mlp_in.weight"], wts["time_mlp_in.bias"]), bf16)),
               bf16)
        cond = _r(torch.nn.functional.silu(_r(linear(h, wts["time_mlp_out.weight"], wts["time_mlp_out.bias"]), bf16)),
                  bf16)
        a = _r(linear(_r(x_t, bf16), wts["action_in_proj.weight"], wts["action_in_proj.bias"]), bf16)
        att = torch.zeros(cfg.chunk_size, dtype=torch.int64)
        att[0] = 1
        return a, att, cond
    st = linear(state, wts["state_proj.weight"], wts["state_proj.bias"]).to(torch.bfloat16).float()
    a = _r(linear(_r(x_t, bf16), wts["action_in_proj.weight"], wts["action_in_proj.bias"]), bf16)
    temb = _r(temb.float(), bf16)[:, None, :].expand_as(a)
    at = torch.cat([a, temb], dim=2)
    at = _r(torch.nn.functional.silu(_r(linear(at, wts["action_time_mlp_in.weight"],
                                                wts["action_time_mlp_in.bias"]), bf16)), bf16)
    at = _r(linear(at, wts["action_time_mlp_out.weight"], wts["action_time_mlp_out.bias"]), bf16)
    embs = torch.cat([st[:, None, :], at], dim=1)
    att = torch.zeros(cfg.chunk_size + 1, dtype=torch.int64)
    att[0] = 1
    att[1] = 1
    return embs, att, None


def expert_layer(cfg, wts, l, h, cond, ctx: Context, pos, att, table, bf16, trace=None, kv_out=None):
    p = f"layers.{l}."
    B, S, W = h.shape
    H, D = cfg.num_heads, cfg.head_dim
    res = h
    x, g = norm(h, cond, wts, p + "input_layernorm", cfg.adarms, cfg.eps, bf16)
    wqkv = torch.cat([wts[p + "q_proj.weight"], wts[p + "k_proj.weight"], wts[p + "v_proj.weight"]])
    qkv = _r(linear(x, wqkv), bf16).view(B, S, H + 2, D).permute(0, 2, 1, 3)
    q, k, v = qkv[:, :H], qkv[:, H:H + 1], qkv[:, H + 1:]
    q = _r(rope(q, pos, table), bf16)
    k = _r(rope(k, pos, table), bf16)
    if kv_out is not None:
        kv_out.append((k.clone(), v.clone()))
    o = partitioned_attention(q, ctx.k[l], ctx.v[l], k, v, ctx.pad, att, D ** -0.5)
    o = _r(o, bf16).transpose(1, 2).reshape(B, S, H * D)
    if trace is not None:
        trace.setdefault("attn", []).append(o.clone())
    o = _r(linear(o, wts[p + "o_proj.weight"]), bf16)
    h = _r(res + _r(g * o, bf16), bf16)
    res = h
    x, g = norm(h, cond, wts, p + "post_attention_layernorm", cfg.adarms, cfg.eps, bf16)
    gate = _r(linear(x, wts[p + "gate_proj.weight"]), bf16)
    up = _r(linear(x, wts[p + "up_proj.weight"]), bf16)
    a = _r(_r(torch.nn.functional.gelu(gate, approximate="tanh"), bf16) * up, bf16)
    d = _r(linear(a, wts[p + "down_proj.weight"]), bf16)
    return _r(res + _r(g * d, bf16), bf16)


def denoise_step(cfg, wts, ctx: Context, state, x_t, t, table, bf16=False, hidden=None, trace=None):
    embs, att, cond = suffix_embed(cfg, wts, state, x_t, t, bf16)
    B, S_total, _ = embs.shape
    n_valid = ctx.pad.sum(dim=1)
    pos = (n_valid[:, None] + torch.arange(S_total)[None]).to(torch.int64)
    h = embs
    for l in range(cfg.num_layers):
        h = expert_layer(cfg, wts, l, h, cond, ctx, pos, att, table, bf16, trace)
        if hidden is not None:
            hidden.append(h.clone())
    y, _ = norm(h, cond, wts, "norm", cfg.adarms, cfg.eps, bf16)
    y = y[:, -cfg.chunk_size:]
    return _r(linear(y, wts["action_out_proj.weight"], wts["action_out_proj.bias"]), bf16)


def sample_chunk(cfg, wts, ctx: Context, x0, state=None, table=None, bf16=False, hidden_step0=None,
                 trace_step0=None):
    """10-step Euler chunk; x stays fp32, dt * v_t follows the reference's dtype
    promotion (a bf16 product when v_t is bf16)."""
    if table is None:
        from reflex_b200.synthetic import rope_table
        table = rope_table(cfg.max_position_embeddings, cfg.head_dim, cfg.rope_theta)
    B = x0.shape[0]
    if state is None:
        state = torch.zeros(B, cfg.state_dim)
    dt = torch.tensor(-1.0 / cfg.num_steps, dtype=torch.float32)
    x = x0.clone()
    t = torch.tensor(1.0, dtype=torch.float32)
    for step in range(cfg.num_steps):
        v = denoise_step(cfg, wts, ctx, state, x, t, table, bf16, hidden_step0 if step == 0 else None,
                         trace_step0 if step == 0 else None)
        x = x + _r(dt * v, bf16)
        t = t + dt
    return x


def prefix_frame(cfg, wts, h, ctx: Context, pos, table=None, bf16=False, hidden=None):
    """Streaming frame update of the prefix layers: the new frame's tokens
    [B, n, W] attend bidirectionally to each other and to the cached context
    (pinned prefix + window), layer by layer.  The prefix layers have the
    decoder-layer structure of the expert's (modeling_pi05.py:563-620, the
    prefix stream of PI05ModelLayer) without conditioning.  Attention is the
    non-streaming one (modeling_pi05.py:1379-1401 builds the full prefix
    mask), not the streaming prefill, which returns zeros for the prefix
    (streaming_attention.py:585-587).  Returns (hidden, [(k, v) per layer])
    with the new frame's post-RoPE K/V that the frame appends to each ring."""
    if table is None:
        from reflex_b200.synthetic import rope_table
        table = rope_table(cfg.max_position_embeddings, cfg.head_dim, cfg.rope_theta)
    att = torch.zeros(h.shape[1], dtype=torch.int64)
    att[0] = 1
    kvs = []
    for l in range(cfg.num_layers):
        h = expert_layer(cfg, wts, l, h, None, ctx, pos, att, table, bf16, kv_out=kvs)
        if hidden is not None:
            hidden.append(h.clone())
    return h, kvs
