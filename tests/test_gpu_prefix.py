"""Streaming frame update of the prefix layers (PrefixEngine) against the fp32
oracle: the new frame's hidden states (max abs <= 2e-2 * max(1, |h|max), the
bf16 residual-stream tolerance) and the K/V it appends to each ring
(dequantized, within half a quantization step of the fp32 K/V plus
2e-2 * max(1, |K/V|max): the K/V of layer l > 0 inherit the bf16 residual
stream's error, like the hidden states), with the pinned prefix and the
surviving frame untouched.
"""
import numpy as np
import pytest
import torch

from oracle import quant as oq
from oracle.model import Context, prefix_frame
from reflex_b200 import kernels as K
from reflex_b200 import _lib as L
from reflex_b200 import synthetic
from reflex_b200.config import vlm_config

pytestmark = pytest.mark.gpu


def _deq(ring, a, b):
    k = oq.dequant_i8_sym(ring.k_q[:, :, a:b].cpu().numpy(), ring.k_scale[:, :, a:b, None].cpu().numpy())
    v = oq.dequant_i8_sym(ring.v_q[:, :, a:b].cpu().numpy(), ring.v_scale[:, :, a:b, None].cpu().numpy())
    return torch.from_numpy(k), torch.from_numpy(v)


@pytest.mark.parametrize("layers,flen", [(2, 128), (4, 768)])
def test_frame_update_matches_oracle(layers, flen):
    """(4, 768): the streaming configuration's frame of 3 cameras x 256
    tokens, through four Gemma-2B-shape prefix layers."""
    from reflex_b200.prefix import PrefixEngine
    cfg = vlm_config(num_layers=layers)
    B, pinned = 1, 48
    cap = pinned + 2 * flen
    wts = synthetic.prefix_weights(cfg, seed=10)
    rings = [K.KVRing.allocate(B, 1, cap, 256, L.RFX_QUANT_I8_SYM, scale_dtype=torch.float32)
             for _ in range(cfg.num_layers)]
    eng = PrefixEngine(cfg, wts, rings, pinned=pinned, frame_len=flen, window_frames=2, batch=B)
    ks, vs = synthetic.context_kv(cfg, pinned + 2 * flen, B=B, seed=12)
    for l in range(cfg.num_layers):
        eng.load_context(l, ks[l], vs[l])
    before = [(r.k_q.clone(), r.v_q.clone()) for r in rings]
    eng.frames = 1  # the next frame replaces frame slot 1; context = pinned + slot 0
    emb = synthetic.frame_embeddings(cfg, flen, B=B, seed=13)
    eng.run(emb.cuda())
    torch.cuda.synchronize()
    assert K.device_status() == 0
    # oracle: the context the frame sees is the dequantized pinned prefix + slot 0
    ctx_k, ctx_v = [], []
    for l in range(cfg.num_layers):
        k, v = _deq(rings[l], 0, pinned + flen)
        ctx_k.append(k)
        ctx_v.append(v)
    ctx = Context(ctx_k, ctx_v, torch.ones(B, pinned + flen, dtype=torch.bool))
    pos = (pinned + flen + torch.arange(flen))[None].expand(B, -1)
    with torch.no_grad():
        h_ref, kvs = prefix_frame(cfg, wts, emb.float(), ctx, pos)
    h = eng.h.view(B, flen, -1).float().cpu()
    err = (h - h_ref).abs().max().item()
    print(f"frame update: hidden maxerr {err:.4f} (|h|max {h_ref.abs().max().item():.2f})")
    assert err <= 2e-2 * max(1.0, h_ref.abs().max().item())
    base = pinned + flen
    for l in range(cfg.num_layers):
        kq, vq = _deq(rings[l], base, base + flen)
        k_ref, v_ref = kvs[l]
        for got, ref in ((kq, k_ref), (vq, v_ref)):
            step = ref.abs().amax(dim=-1, keepdim=True) / 127
            excess = ((got - ref).abs() - 0.5 * step).max().item()
            print(f"layer {l}: appended K/V excess over half a step {excess:.4f}")
            assert excess <= 2e-2 * max(1.0, ref.abs().max().item())
        # the pinned prefix and the surviving frame are untouched
        assert torch.equal(rings[l].k_q[:, :, :base], before[l][0][:, :, :base])
        assert torch.equal(rings[l].v_q[:, :, :base], before[l][1][:, :, :base])
    assert np.isfinite(h.numpy()).all()
