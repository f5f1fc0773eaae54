"""SigLIP vision tower + PaliGemma projector (``get_image_features``), restated
in torch on the CPU.  Test infrastructure: the CUDA path is checked against it.

The reference calls the VLM's image embedder at
reflex/policies/pi05/modeling_pi05.py:141-158 (``vlm.model.get_image_features``,
or vision_tower -> multi_modal_projector under bf16 autocast) and :244 (one
call per camera).  The tower comes from transformers (the reference pins a
fork that is not vendored); this restates the published SigLIP architecture as
transformers' modeling_siglip implements it, pinned against the installed
transformers' own modules by tests/golden/make_golden_vision.py:
* SiglipVisionEmbeddings.forward: a stride-14 14x14 convolution with bias
  (patch embedding), patches in row-major grid order, plus a learned position
  embedding per patch;
* SiglipEncoderLayer.forward: x + attn(LayerNorm1(x)), then x + mlp(LayerNorm2(x));
* SiglipAttention (eager): softmax(q k^T * head_dim^-0.5) v per head, q/k/v/out
  projections with bias, no mask;
* SiglipMLP: fc2(gelu_tanh(fc1(x))), both with bias;
* SiglipVisionTransformer.forward: the post LayerNorm after the last layer;
* PaliGemmaMultiModalProjector: one linear with bias, width -> proj_dim.

``bf16=True`` also rounds to bf16 where the CUDA path stores activations
(patch embeddings, LayerNorm outputs, q/k/v, the attention output, the
residual stream, the GELU output, the projector output): a CPU model of the
engine's numerics used to size tolerances.
"""
from __future__ import annotations

import math

import torch


def _r(x: torch.Tensor, on: bool) -> torch.Tensor:
    return x.to(torch.bfloat16).to(torch.float32) if on else x


def gelu_tanh(x: torch.Tensor) -> torch.Tensor:
    return 0.5 * x * (1.0 + torch.tanh(math.sqrt(2.0 / math.pi) * (x + 0.044715 * x * x * x)))


def layer_norm(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor, eps: float) -> torch.Tensor:
    mu = x.mean(-1, keepdim=True)
    var = ((x - mu) ** 2).mean(-1, keepdim=True)
    return (x - mu) * torch.rsqrt(var + eps) * w + b


def patches(cfg, pixels: torch.Tensor) -> torch.Tensor:
    """[B, C, H, W] -> [B, grid*grid, C*P*P]: patch (gy, gx) at row gy*grid+gx,
    its values in (channel, y, x) order, the order of the convolution weight."""
    B, C, H, W = pixels.shape
    P, G = cfg.patch, cfg.grid
    x = pixels[:, :, : G * P, : G * P].reshape(B, C, G, P, G, P)
    return x.permute(0, 2, 4, 1, 3, 5).reshape(B, G * G, C * P * P)


def image_features(cfg, w: dict[str, torch.Tensor], pixels: torch.Tensor, bf16: bool = False,
                   layers: int | None = None, return_hidden: bool = False):
    """[B, 3, 224, 224] fp32 images -> [B, 256, proj_dim] image tokens (and,
    with ``return_hidden``, the post-LayerNorm last hidden state)."""
    pre = "vision_model."
    nl = cfg.num_layers if layers is None else layers
    H, D, Wd = cfg.num_heads, cfg.head_dim, cfg.width
    pw = w[pre + "embeddings.patch_embedding.weight"].reshape(Wd, -1)
    x = patches(cfg, pixels.float()) @ pw.T + w[pre + "embeddings.patch_embedding.bias"]
    x = _r(x, bf16) + w[pre + "embeddings.position_embedding.weight"]
    x = _r(x, bf16)
    B, N, _ = x.shape
    for l in range(nl):
        p = f"{pre}encoder.layers.{l}."
        h = _r(layer_norm(x, w[p + "layer_norm1.weight"], w[p + "layer_norm1.bias"], cfg.eps), bf16)
        q = _r(h @ w[p + "self_attn.q_proj.weight"].T + w[p + "self_attn.q_proj.bias"], bf16)
        k = _r(h @ w[p + "self_attn.k_proj.weight"].T + w[p + "self_attn.k_proj.bias"], bf16)
        v = _r(h @ w[p + "self_attn.v_proj.weight"].T + w[p + "self_attn.v_proj.bias"], bf16)
        q, k, v = (t.reshape(B, N, H, D).transpose(1, 2) for t in (q, k, v))
        s = (q @ k.transpose(-1, -2)) * (D ** -0.5)
        a = torch.softmax(s, dim=-1) @ v
        a = _r(a.transpose(1, 2).reshape(B, N, H * D), bf16)
        o = _r(a @ w[p + "self_attn.out_proj.weight"].T + w[p + "self_attn.out_proj.bias"], bf16)
        x = _r(x + o, bf16)
        h = _r(layer_norm(x, w[p + "layer_norm2.weight"], w[p + "layer_norm2.bias"], cfg.eps), bf16)
        f = _r(h @ w[p + "mlp.fc1.weight"].T + w[p + "mlp.fc1.bias"], bf16)
        f = _r(gelu_tanh(f), bf16)
        o = _r(f @ w[p + "mlp.fc2.weight"].T + w[p + "mlp.fc2.bias"], bf16)
        x = _r(x + o, bf16)
    hid = _r(layer_norm(x, w[pre + "post_layernorm.weight"], w[pre + "post_layernorm.bias"], cfg.eps), bf16)
    out = _r(hid @ w["projector.linear.weight"].T + w["projector.linear.bias"], bf16)
    return (out, hid) if return_hidden else out
