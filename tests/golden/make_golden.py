"""Generates the golden fixtures of tests/golden/ by running the reference's own
PyTorch code (9yc/Reflex, mounted read-only) on seeded inputs, on the CPU.

Run where the reference is available, with RFX_REFERENCE naming its checkout
(the script refuses to run without it):
    RFX_REFERENCE=<path to the Reflex checkout> python tests/golden/make_golden.py

The reference's classes are driven by oracle/reference_harness.py (stub
modules for the absent `lerobot`; the torch KV quantizer of
reflex/layers/streaming_attention.py:211-218 on the CPU).

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

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
REF = os.environ.get("RFX_REFERENCE")
if not REF and __name__ == "__main__":
    sys.exit("make_golden.py: set RFX_REFERENCE to the Reflex checkout (read-only is fine)")

from reflex_b200 import synthetic  # noqa: E402
from reflex_b200.config import pi0_config, pi05_config  # noqa: E402
from oracle import reference_harness as H  # noqa: E402


def import_reference():
    if not REF:
        raise RuntimeError("set RFX_REFERENCE to the Reflex checkout")
    return H.import_reference(REF)


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


def golden_model(R, variant, num_layers, Lc, fname, full_hidden, seed=0):
    cfg = (pi05_config(num_layers=num_layers, adarms="gate") if variant == "pi05"
           else pi0_config(num_layers=num_layers))
    wts = synthetic.expert_weights(cfg, seed=seed)
    ks, vs = synthetic.context_kv(cfg, Lc, seed=seed + 1)
    x0 = synthetic.noise(cfg, seed=seed + 2)
    st = synthetic.state(cfg, seed=seed + 3)
    ctx = [H.quantized_context(R, ks[l], vs[l]) for l in range(num_layers)]
    model = H.build_reference_model(R, cfg, wts, variant)
    H.install_context(R, model, variant, ctx)
    hooks = []
    with torch.no_grad():
        x = H.run_reference_chunk(R, model, cfg, x0, st, Lc, hooks)
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
