"""Harness that drives the reference's own PyTorch classes (9yc/Reflex) on the
CPU: test infrastructure.  tests/golden/make_golden.py uses it to write the
golden fixtures, and bench.py's reference arm uses it to time the reference's
own code path; the product never imports it.

import_reference(path) imports the `reflex` package from a checkout or a
`pip install --target` directory.  The package imports `lerobot`, which is not
installed: six tiny stub modules stand in for the names it imports (config
base classes, enums and constants); none of them takes part in the
computation.  The Triton KV quantizer is disabled (CPU), so StreamingAttention
uses its torch quantizer (reflex/layers/streaming_attention.py:211-218).

build_reference_model / install_context / run_reference_chunk assemble the
action expert from the reference's PI05ModelLayer / PI0ModelLayer
(reflex/policies/pi05/modeling_pi05.py:537, reflex/policies/pi0/modeling_pi0.py),
AdaRMSNorm (modeling_pi05.py:50-99), the suffix embedders, QKVLinear /
MergedColumnLinear (reflex/layers/linear.py) and the streaming attention
cache, and restate sample_actions' Euler loop (modeling_pi05.py:1403-1419)
around denoise_step (modeling_pi05.py:1181-1241).
"""
from __future__ import annotations

import os
import sys
import types
from types import SimpleNamespace

import torch
from torch import nn


def _stub(name, **attrs):
    m = types.ModuleType(name)
    m.__dict__.update(attrs)
    sys.modules[name] = m
    return m


def import_reference(ref: str):
    """Imports the reference's modules from `ref` (a directory holding the
    `reflex` package)."""
    import enum

    if not ref or not os.path.isdir(os.path.join(ref, "reflex")):
        raise RuntimeError(f"no reflex package under {ref!r}")
    sys.path.insert(0, ref)
    pkg = types.ModuleType("reflex")
    pkg.__path__ = [os.path.join(ref, "reflex")]
    sys.modules["reflex"] = pkg

    class _Cfg:
        def __init__(self, *a, **k):
            pass

        @classmethod
        def register_subclass(cls, *a, **k):
            return lambda c: c

    class FeatureType(enum.Enum):
        STATE = "STATE"
        VISUAL = "VISUAL"
        ACTION = "ACTION"
        ENV = "ENV"

    class NormalizationMode(enum.Enum):
        MIN_MAX = "MIN_MAX"
        MEAN_STD = "MEAN_STD"
        IDENTITY = "IDENTITY"
        QUANTILES = "QUANTILES"

    for n in ("lerobot", "lerobot.configs", "lerobot.optim", "lerobot.policies", "lerobot.utils"):
        _stub(n)
    _stub("lerobot.configs.policies", PreTrainedConfig=_Cfg, T=object)
    _stub("lerobot.configs.types", FeatureType=FeatureType, NormalizationMode=NormalizationMode, PolicyFeature=object)
    _stub("lerobot.optim.optimizers", AdamWConfig=_Cfg)
    _stub("lerobot.optim.schedulers", CosineDecayWithWarmupSchedulerConfig=_Cfg)
    _stub("lerobot.policies.pretrained", PreTrainedPolicy=nn.Module)
    _stub("lerobot.utils.constants", ACTION="action", OBS_STATE="observation.state")
    import reflex.layers.streaming_attention as sam

    sam.HAS_TRITON_QUANT = False
    import reflex.policies.pi0.modeling_pi0 as m0
    import reflex.policies.pi05.modeling_pi05 as m5
    from reflex.layers.attention import Attention
    from reflex.layers.linear import MergedColumnLinear, QKVLinear
    from reflex.policies.pi05.utils import build_attention_mask_and_position_ids

    return SimpleNamespace(sam=sam, m5=m5, m0=m0, Attention=Attention, QKVLinear=QKVLinear,
                           MergedColumnLinear=MergedColumnLinear, build_mask=build_attention_mask_and_position_ids)


# ------------------------------------------------------------ model runs ---
class _AEAttn(nn.Module):
    def __init__(self, R, W, H, D):
        super().__init__()
        self.qkv_proj = R.QKVLinear(W, D, H, 1)
        self.o_proj = nn.Linear(H * D, W, bias=False)
        self.scaling = D ** -0.5
        self.head_dim = D


class _AEMLP(nn.Module):
    def __init__(self, R, W, F):
        super().__init__()
        self.gate_up_proj = R.MergedColumnLinear(W, [F, F])
        self.down_proj = nn.Linear(F, W, bias=False)
        self.act_fn = nn.GELU(approximate="tanh")


class _AELayer(nn.Module):
    def __init__(self, R, norm_cls, W, H, D, F):
        super().__init__()
        self.input_layernorm = norm_cls(W)
        self.post_attention_layernorm = norm_cls(W)
        self.self_attn = _AEAttn(R, W, H, D)
        self.mlp = _AEMLP(R, W, F)


def _ref_config(cfg, streaming):
    text = SimpleNamespace(head_dim=cfg.head_dim, max_position_embeddings=cfg.max_position_embeddings,
                           rope_theta=cfg.rope_theta, num_attention_heads=cfg.num_heads)
    return SimpleNamespace(vlm_config=SimpleNamespace(text_config=text), enable_streaming=streaming,
                           enable_kv_quantization=streaming, max_cache_size=2048, enable_mixed_precision=True,
                           enable_flash_attention=False, max_action_dim=cfg.action_dim, max_state_dim=cfg.state_dim,
                           action_expert_config=SimpleNamespace(hidden_size=cfg.width), min_period=cfg.min_period,
                           max_period=cfg.max_period, state_cond=False, chunk_size=cfg.chunk_size)


def _load_norm(norm, wts, name):
    with torch.no_grad():
        norm.weight.copy_(wts[name + ".weight"])
        if hasattr(norm, "dense") and name + ".dense.weight" in wts:
            norm.dense.weight.copy_(wts[name + ".dense.weight"])
            norm.dense.bias.copy_(wts[name + ".dense.bias"])


def build_reference_model(R, cfg, wts, variant):
    """Reference layer stack over stand-in VLM/expert layer objects.  Norms are the
    in-tree AdaRMSNorm (modeling_pi05.py:50-99)."""
    m = R.m5 if variant == "pi05" else R.m0
    rcfg = _ref_config(cfg, streaming=variant == "pi05")
    W, H, D, F = cfg.width, cfg.num_heads, cfg.head_dim, cfg.mlp_dim
    layers = []
    for l in range(cfg.num_layers):
        vlm = _AELayer(R, R.m5.AdaRMSNorm, 16, 1, 16, 16)  # unused VLM side (hidden state is None)
        vlm.self_attn.scaling = D ** -0.5
        ae = _AELayer(R, R.m5.AdaRMSNorm, W, H, D, F)
        p = f"layers.{l}."
        with torch.no_grad():
            ae.self_attn.qkv_proj.weight.copy_(torch.cat([wts[p + "q_proj.weight"], wts[p + "k_proj.weight"],
                                                          wts[p + "v_proj.weight"]]))
            ae.self_attn.o_proj.weight.copy_(wts[p + "o_proj.weight"])
            ae.mlp.gate_up_proj.weight.copy_(torch.cat([wts[p + "gate_proj.weight"], wts[p + "up_proj.weight"]]))
            ae.mlp.down_proj.weight.copy_(wts[p + "down_proj.weight"])
        _load_norm(ae.input_layernorm, wts, p + "input_layernorm")
        _load_norm(ae.post_attention_layernorm, wts, p + "post_attention_layernorm")
        cls = m.PI05ModelLayer if variant == "pi05" else m.PI0ModelLayer
        layers.append(cls(rcfg, vlm, ae))
    final_norm = R.m5.AdaRMSNorm(W)
    _load_norm(final_norm, wts, "norm")
    out_proj = nn.Linear(W, cfg.action_dim)
    with torch.no_grad():
        out_proj.weight.copy_(wts["action_out_proj.weight"])
        out_proj.bias.copy_(wts["action_out_proj.bias"])
    if variant == "pi05":
        emb = R.m5.PI05SuffixEmbedder(rcfg)
        names = ("action_in_proj", "time_mlp_in", "time_mlp_out")
    else:
        emb = R.m0.PI0SuffixEmbedder(rcfg)
        names = ("action_in_proj", "state_proj", "action_time_mlp_in", "action_time_mlp_out")
    with torch.no_grad():
        for n in names:
            getattr(emb, n).weight.copy_(wts[n + ".weight"])
            getattr(emb, n).bias.copy_(wts[n + ".bias"])
    return SimpleNamespace(layers=layers, norm=final_norm, action_out_proj=out_proj, suffix_embedder=emb, cfg=rcfg)


def quantized_context(R, k, v):
    """Quantizes context K/V with the reference quantizer (fp32 activations)."""
    sa = R.sam.StreamingAttention(scale=1 / 16, quantize_kv_cache=True)
    kq, ks, kz = sa._quantize(k)
    vq, vs, vz = sa._quantize(v)
    return kq, ks, kz, vq, vs, vz


def install_context(R, model, variant, ctx):
    """Puts the quantized context into every layer's cache exactly as
    prefill_source + merge_caches leave it (streaming_attention.py:346-367,511-550)."""
    for l, layer in enumerate(model.layers):
        kq, ks, kz, vq, vs, vz = ctx[l]
        if variant == "pi05":
            a = layer.self_attn.attn
            B, H, Lc, D = kq.shape
            a._init_static_buffer(B, H, D, torch.float32, "cpu")
            a.prefix_k_buffer[:, :, :Lc] = kq
            a.prefix_v_buffer[:, :, :Lc] = vq
            a.prefix_k_scale[:, :, :Lc] = ks
            a.prefix_k_zp[:, :, :Lc] = kz
            a.prefix_v_scale[:, :, :Lc] = vs
            a.prefix_v_zp[:, :, :Lc] = vz
            a.source_length = Lc
            a.merge_caches()
        else:  # PI0 keeps a plain (unquantized) prefix cache: give it the dequantized values
            a = layer.self_attn.attn
            a.k_cache = (kq.float() - kz) * ks
            a.v_cache = (vq.float() - vz) * vs


def run_reference_chunk(R, model, cfg, x0, state, Lc, hooks=None):
    """sample_actions' Euler loop (modeling_pi05.py:1403-1419) around denoise_step
    (modeling_pi05.py:1181-1241; PI0: modeling_pi0.py:740-782, 827-845), restated
    over the reference modules."""
    bsz = x0.shape[0]
    prefix_pad = torch.ones(bsz, Lc, dtype=torch.bool)
    prefix_att = torch.zeros(bsz, Lc)

    def denoise_step(x_t, timestep):
        suffix_embs, suffix_pad, suffix_att, cond = model.suffix_embedder(state, x_t, timestep)
        suffix_embs = suffix_embs.to(torch.float32)
        pad = torch.cat([prefix_pad, suffix_pad], dim=1)
        att = torch.cat([prefix_att, suffix_att.to(prefix_att.dtype)], dim=1)
        full_mask, full_pos = R.build_mask(pad, att, suffix_embs.dtype)
        L_suf = suffix_embs.shape[1]
        mask = full_mask[:, :, -L_suf:, :]
        pos = full_pos[:, -L_suf:]
        hs = [None, suffix_embs]
        conds = [None, cond]
        for i, layer in enumerate(model.layers):
            hs = layer(hs, mask, pos, conds, use_cache=True)
            if hooks is not None:
                hooks.append(hs[1].clone())
        h, _ = model.norm(hs[1], cond=cond)
        out = h[:, -cfg.chunk_size:]
        return model.action_out_proj(out)

    dt = torch.tensor(-1.0 / cfg.num_steps, dtype=torch.float32)
    x_t = x0
    time = torch.tensor(1.0, dtype=torch.float32)
    first = True
    for _ in range(cfg.num_steps):
        v_t = denoise_step(x_t, time.expand(bsz))
        if first and hooks is not None:
            hooks.append(None)  # marks the end of step 0
            first = False
        x_t = x_t + dt * v_t
        time = time + dt
    return x_t


