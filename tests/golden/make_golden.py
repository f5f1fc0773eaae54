"""Generates the golden fixtures of tests/golden/ by running the reference's own
PyTorch code (9yc/Reflex, mounted read-only) on seeded inputs, on the CPU.

Run where the reference is available:
    RFX_REFERENCE=/root/reference python tests/golden/make_golden.py

The reference package imports `lerobot`, which is not installed; six tiny stub
modules stand in for the names it imports (config base classes, enums and
constants) — none of them takes part in the computation.  The Triton KV
quantizer is disabled (CPU), so StreamingAttention uses its torch quantizer
(reflex/layers/streaming_attention.py:211-218).

Fixtures written (numpy .npz):
  quant_u8_ref.npz     reference _quantize on bf16 and fp32 rows (incl. edge rows)
  attention_c1.npz     single partitioned-attention layer (config 1 shapes):
                       full O(N^2) recompute, streaming (fp32 cache), streaming
                       with the uint8 quantized cache, and the quantized cache
  model_pi05_l2.npz    2-layer PI0.5 expert (in-tree AdaRMSNorm), 128-token
                       uint8 context: per-layer hidden states of step 0 and the
                       10-step action chunk
  model_pi05_l18.npz   18-layer PI0.5 expert, 818-token context: action chunk
                       and per-layer statistics of step 0
  model_pi0_l2.npz     2-layer PI0 expert (state token + action-time MLP)
Inputs are regenerated from the recorded seeds by reflex_b200.synthetic; a
SHA-256 of the regenerated inputs is stored next to each output.
"""
from __future__ import annotations

import hashlib
import os
import sys
import types
from types import SimpleNamespace

import numpy as np
import torch
from torch import nn

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
REF = os.environ.get("RFX_REFERENCE", "/root/reference")

from reflex_b200 import synthetic  # noqa: E402
from reflex_b200.config import pi0_config, pi05_config  # noqa: E402


def _stub(name, **attrs):
    m = types.ModuleType(name)
    m.__dict__.update(attrs)
    sys.modules[name] = m
    return m


def import_reference():
    import enum

    sys.path.insert(0, REF)
    pkg = types.ModuleType("reflex")
    pkg.__path__ = [os.path.join(REF, "reflex")]
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


def sha(*ts) -> str:
    h = hashlib.sha256()
    for t in ts:
        h.update(np.ascontiguousarray(t.detach().cpu().float().numpy()).tobytes())
    return h.hexdigest()


# ------------------------------------------------------------- quantizer ---
def edge_rows(D=256):
    rows = [np.zeros(D), np.full(D, 3.25), np.linspace(-1e-6, 1e-6, D), -np.abs(np.linspace(0.1, 7, D)),
            np.linspace(-2.5, 2.5, D), np.r_[np.full(D - 1, 0.5), 127.0], np.r_[np.full(D - 1, -1.0), 1e4],
            np.linspace(0, 255, D), np.r_[np.full(D // 2, 1e-3), np.full(D // 2, -1e-3)]]
    return np.stack(rows).astype(np.float32)


def golden_quant(R):
    sa = R.sam.StreamingAttention(scale=1 / 16, quantize_kv_cache=True)
    g = torch.Generator().manual_seed(11)
    x = torch.randn(1, 1, 300, 256, generator=g) * torch.rand(1, 1, 300, 1, generator=g) * 8
    x[0, 0, :9] = torch.from_numpy(edge_rows())
    out = {"seed": 11, "x_sha": sha(x)}
    for name, dt in (("f32", torch.float32), ("bf16", torch.bfloat16)):
        xi = x.to(dt)
        q, s, z = sa._quantize(xi)
        out[f"q_{name}"] = q.numpy()
        out[f"scale_{name}"] = s.float().numpy()
        out[f"zp_{name}"] = z.float().numpy()
        deq = sa._dequantize(q, s, z)
        out[f"deq16_{name}"] = deq.float().numpy()[:, :, :16]
    np.savez_compressed(os.path.join(HERE, "quant_u8_ref.npz"), **out)


# ----------------------------------------------------------- attention C1 ---
def golden_attention_c1(R):
    """Config 1: B=1, 8 q heads, 1 KV head, D=256; 64 prefix + 512 window
    (576 context) + 50 suffix; Q/K/V ~ N(0,1) fp32."""
    g = torch.Generator().manual_seed(7)
    Lc, S, H, D = 576, 50, 8, 256
    N = Lc + S
    q = torch.randn(1, H, N, D, generator=g)
    k = torch.randn(1, 1, N, D, generator=g)
    v = torch.randn(1, 1, N, D, generator=g)
    pad = torch.ones(1, N, dtype=torch.bool)
    att = torch.zeros(1, N)
    att[0, Lc] = 1
    mask, _ = R.build_mask(pad, att, torch.float32)
    full = R.Attention(scale=1 / 16)(q, k, v, mask, use_cache=False)[:, :, Lc:]
    outs = {"seed": 7, "inputs_sha": sha(q, k, v), "full": full.numpy()}
    for quant in (False, True):
        sa = R.sam.StreamingAttention(scale=1 / 16, enable_streaming=True, quantize_kv_cache=quant)
        sa.prefill_source(k[:, :, :Lc], v[:, :, :Lc])
        sa.merge_caches()
        o = sa(q[:, :, Lc:], k[:, :, Lc:], v[:, :, Lc:], attention_mask=mask[:, :, Lc:], use_cache=True)
        if quant:
            outs["stream_q"] = o.numpy()
            outs["cache_sha"] = sha(*(t[:, :, :Lc] for t in (sa.prefix_k_buffer, sa.prefix_v_buffer,
                                                              sa.prefix_k_scale, sa.prefix_k_zp,
                                                              sa.prefix_v_scale, sa.prefix_v_zp)))
        else:
            outs["stream_vs_full_maxdiff"] = float((o - full).abs().max())
    np.savez_compressed(os.path.join(HERE, "attention_c1.npz"), **outs)


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


def golden_model(R, variant, num_layers, Lc, fname, full_hidden, seed=0):
    cfg = (pi05_config(num_layers=num_layers, adarms="gate") if variant == "pi05"
           else pi0_config(num_layers=num_layers))
    wts = synthetic.expert_weights(cfg, seed=seed)
    ks, vs = synthetic.context_kv(cfg, Lc, seed=seed + 1)
    x0 = synthetic.noise(cfg, seed=seed + 2)
    st = synthetic.state(cfg, seed=seed + 3)
    ctx = [quantized_context(R, ks[l], vs[l]) for l in range(num_layers)]
    model = build_reference_model(R, cfg, wts, variant)
    install_context(R, model, variant, ctx)
    hooks = []
    with torch.no_grad():
        x = run_reference_chunk(R, model, cfg, x0, st, Lc, hooks)
    step0 = hooks[:hooks.index(None)]
    out = {"seed": seed, "num_layers": num_layers, "n_ctx": Lc, "variant": variant,
           "weights_sha": sha(*[wts[k] for k in sorted(wts)]), "inputs_sha": sha(*ks, *vs, x0, st),
           "actions": x.numpy(), "ctx_sha": sha(*[t for c in ctx for t in c])}
    if full_hidden:
        out["hidden_step0"] = np.stack([h.numpy() for h in step0])
    else:
        out["hidden_step0_absmax"] = np.array([h.abs().max().item() for h in step0])
        out["hidden_step0_mean"] = np.array([h.mean().item() for h in step0])
        out["hidden_step0_l2"] = np.array([h.norm().item() for h in step0])
    np.savez_compressed(os.path.join(HERE, fname), **out)


def main():
    torch.set_num_threads(os.cpu_count() or 1)
    R = import_reference()
    golden_quant(R)
    golden_attention_c1(R)
    golden_model(R, "pi05", 2, 128, "model_pi05_l2.npz", full_hidden=True)
    golden_model(R, "pi0", 2, 128, "model_pi0_l2.npz", full_hidden=True)
    golden_model(R, "pi05", 18, 818, "model_pi05_l18.npz", full_hidden=False)
    for f in sorted(os.listdir(HERE)):
        if f.endswith(".npz"):
            print(f, os.path.getsize(os.path.join(HERE, f)))


if __name__ == "__main__":
    main()
