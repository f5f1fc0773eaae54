"""Seeded synthetic weights and inputs of the action expert (no checkpoint is
available offline).

Every bf16 parameter is generated in fp32 and rounded to bf16 here, so the
fp32 oracle, the reference's own modules and the bf16 CUDA engine all see the
same values.  Norm parameters (input/post-attention/final norm weights and
their AdaRMS ``dense`` layers) stay fp32, following the dtype policy of
reflex/policies/pi05/modeling_pi05.py:919-945.

Initialisation (random-init weights of the right architecture):
* transformer projections: N(0, 0.02) (Gemma initializer_range);
* action / time / state linears: U(-1/sqrt(in), 1/sqrt(in)) weight and bias
  (torch.nn.Linear default);
* norm weights: 1 + N(0, 0.05) (AdaRMSNorm initialises them to one);
* AdaRMS dense: torch.nn.Linear default (fp32).
"""
from __future__ import annotations

import math

import torch

from .config import ExpertConfig


def _bf16(t: torch.Tensor) -> torch.Tensor:
    return t.to(torch.bfloat16).to(torch.float32)


class _Rng:
    def __init__(self, seed: int, device="cpu"):
        self.g = torch.Generator(device=device).manual_seed(seed)
        self.device = device

    def normal(self, *shape, std=1.0):
        return torch.randn(*shape, generator=self.g, device=self.device) * std

    def uniform(self, *shape, bound=1.0):
        return (torch.rand(*shape, generator=self.g, device=self.device) * 2 - 1) * bound


def expert_weights(cfg: ExpertConfig, seed: int = 0, device="cpu") -> dict[str, torch.Tensor]:
    """Returns fp32 tensors (bf16-representable where the parameter is bf16)."""
    r = _Rng(seed, device)
    W, H, D, F, A = cfg.width, cfg.num_heads, cfg.head_dim, cfg.mlp_dim, cfg.action_dim
    w: dict[str, torch.Tensor] = {}

    def lin(name, out_f, in_f, bias=True):
        b = 1.0 / math.sqrt(in_f)
        w[name + ".weight"] = _bf16(r.uniform(out_f, in_f, bound=b))
        if bias:
            w[name + ".bias"] = _bf16(r.uniform(out_f, bound=b))

    lin("action_in_proj", W, A)
    lin("action_out_proj", A, W)
    if cfg.variant == "pi05":
        lin("time_mlp_in", W, W)
        lin("time_mlp_out", W, W)
    else:
        lin("state_proj", W, cfg.state_dim)
        lin("action_time_mlp_in", W, 2 * W)
        lin("action_time_mlp_out", W, W)

    def norm(name):
        w[name + ".weight"] = 1.0 + r.normal(W, std=0.05)
        if cfg.adarms != "none":
            b = 1.0 / math.sqrt(W)
            w[name + ".dense.weight"] = r.uniform(cfg.mod_width, W, bound=b)
            w[name + ".dense.bias"] = r.uniform(cfg.mod_width, bound=b)

    for l in range(cfg.num_layers):
        p = f"layers.{l}."
        w[p + "q_proj.weight"] = _bf16(r.normal(H * D, W, std=0.02))
        w[p + "k_proj.weight"] = _bf16(r.normal(cfg.num_kv_heads * D, W, std=0.02))
        w[p + "v_proj.weight"] = _bf16(r.normal(cfg.num_kv_heads * D, W, std=0.02))
        w[p + "o_proj.weight"] = _bf16(r.normal(W, H * D, std=0.02))
        w[p + "gate_proj.weight"] = _bf16(r.normal(F, W, std=0.02))
        w[p + "up_proj.weight"] = _bf16(r.normal(F, W, std=0.02))
        w[p + "down_proj.weight"] = _bf16(r.normal(W, F, std=0.02))
        norm(p + "input_layernorm")
        norm(p + "post_attention_layernorm")
    norm("norm")
    return w


def prefix_weights(cfg: ExpertConfig, seed: int = 10, device="cpu") -> dict[str, torch.Tensor]:
    """Random-init prefix (VLM) layer weights, same initialisation as the
    expert's layers; norms carry only their weight (no conditioning)."""
    r = _Rng(seed, device)
    W, H, D, F = cfg.width, cfg.num_heads, cfg.head_dim, cfg.mlp_dim
    w: dict[str, torch.Tensor] = {}
    for l in range(cfg.num_layers):
        p = f"layers.{l}."
        w[p + "q_proj.weight"] = _bf16(r.normal(H * D, W, std=0.02))
        w[p + "k_proj.weight"] = _bf16(r.normal(cfg.num_kv_heads * D, W, std=0.02))
        w[p + "v_proj.weight"] = _bf16(r.normal(cfg.num_kv_heads * D, W, std=0.02))
        w[p + "o_proj.weight"] = _bf16(r.normal(W, H * D, std=0.02))
        w[p + "gate_proj.weight"] = _bf16(r.normal(F, W, std=0.02))
        w[p + "up_proj.weight"] = _bf16(r.normal(F, W, std=0.02))
        w[p + "down_proj.weight"] = _bf16(r.normal(W, F, std=0.02))
        w[p + "input_layernorm.weight"] = 1.0 + r.normal(W, std=0.05)
        w[p + "post_attention_layernorm.weight"] = 1.0 + r.normal(W, std=0.05)
    return w


def frame_embeddings(cfg: ExpertConfig, n: int, B: int = 1, seed: int = 11, device="cpu") -> torch.Tensor:
    """A new frame's patch embeddings [B, n, width] ~ N(0, 1) / sqrt(width), bf16-representable."""
    return _bf16(_Rng(seed, device).normal(B, n, cfg.width) / math.sqrt(cfg.width))


def context_kv(cfg: ExpertConfig, n_ctx: int, B: int = 1, seed: int = 1, device="cpu"):
    """Per-layer context K/V [L][B, 1, n_ctx, D] ~ N(0, 1) (post-RoPE keys as the
    prefix layers would have cached them)."""
    r = _Rng(seed, device)
    ks, vs = [], []
    for _ in range(cfg.num_layers):
        ks.append(r.normal(B, cfg.num_kv_heads, n_ctx, cfg.head_dim))
        vs.append(r.normal(B, cfg.num_kv_heads, n_ctx, cfg.head_dim))
    return ks, vs


def noise(cfg: ExpertConfig, B: int = 1, seed: int = 2, device="cpu") -> torch.Tensor:
    """x0 ~ N(0, 1) [B, chunk, action_dim] fp32 (modeling_pi05.py:947-955)."""
    return _Rng(seed, device).normal(B, cfg.chunk_size, cfg.action_dim)


def state(cfg: ExpertConfig, B: int = 1, seed: int = 3, device="cpu") -> torch.Tensor:
    return _Rng(seed, device).normal(B, cfg.state_dim)


def rope_table(max_pos: int, head_dim: int, base: float) -> torch.Tensor:
    """cos | sin table [max_pos, head_dim] in fp32, computed on the CPU exactly as
    RotaryEmbedding.__init__ does (reflex/layers/rope.py:82-101)."""
    inv_freq = 1.0 / (base ** (torch.arange(0, head_dim, 2, dtype=torch.float) / head_dim))
    t = torch.arange(max_pos, dtype=torch.float)
    freqs = torch.einsum("i,j -> ij", t, inv_freq)
    return torch.cat((freqs.cos(), freqs.sin()), dim=-1)


def vision_weights(cfg, seed: int = 20, device="cpu") -> dict[str, torch.Tensor]:
    """Random-init SigLIP tower + projector weights (``cfg``: VisionConfig),
    named as transformers' SiglipVisionModel / PaliGemmaMultiModalProjector
    state dicts.  Linear and patch weights N(0, 0.02) and biases N(0, 0.02),
    bf16-representable; position embeddings N(0, 0.02); LayerNorm weight
    1 + N(0, 0.05) and bias N(0, 0.02), fp32."""
    r = _Rng(seed, device)
    W, F = cfg.width, cfg.mlp_dim
    w: dict[str, torch.Tensor] = {}
    pre = "vision_model."
    w[pre + "embeddings.patch_embedding.weight"] = _bf16(r.normal(W, cfg.channels, cfg.patch, cfg.patch, std=0.02))
    w[pre + "embeddings.patch_embedding.bias"] = _bf16(r.normal(W, std=0.02))
    w[pre + "embeddings.position_embedding.weight"] = _bf16(r.normal(cfg.tokens, W, std=0.02))
    for l in range(cfg.num_layers):
        p = f"{pre}encoder.layers.{l}."
        for name in ("q_proj", "k_proj", "v_proj", "out_proj"):
            w[p + f"self_attn.{name}.weight"] = _bf16(r.normal(W, W, std=0.02))
            w[p + f"self_attn.{name}.bias"] = _bf16(r.normal(W, std=0.02))
        w[p + "mlp.fc1.weight"] = _bf16(r.normal(F, W, std=0.02))
        w[p + "mlp.fc1.bias"] = _bf16(r.normal(F, std=0.02))
        w[p + "mlp.fc2.weight"] = _bf16(r.normal(W, F, std=0.02))
        w[p + "mlp.fc2.bias"] = _bf16(r.normal(W, std=0.02))
        for n in ("layer_norm1", "layer_norm2"):
            w[p + f"{n}.weight"] = 1.0 + r.normal(W, std=0.05)
            w[p + f"{n}.bias"] = r.normal(W, std=0.02)
    w[pre + "post_layernorm.weight"] = 1.0 + r.normal(W, std=0.05)
    w[pre + "post_layernorm.bias"] = r.normal(W, std=0.02)
    w["projector.linear.weight"] = _bf16(r.normal(cfg.proj_dim, W, std=0.02))
    w["projector.linear.bias"] = _bf16(r.normal(cfg.proj_dim, std=0.02))
    return w


def images(cfg, B: int = 1, seed: int = 21, device="cpu") -> torch.Tensor:
    """Normalized camera images [B, 3, H, W] in [-1, 1] (SigLIP's input range),
    fp32."""
    return _Rng(seed, device).uniform(B, cfg.channels, cfg.image, cfg.image)
