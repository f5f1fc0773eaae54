"""Generates tests/golden/vision_l2.npz: image tokens of a 2-layer SigLIP tower
(full SigLIP-So400m widths) + PaliGemma projector, computed by the installed
transformers' own SiglipVisionModel and PaliGemmaMultiModalProjector in fp32 on
the CPU, from the seeded weights and image of reflex_b200.synthetic.

The reference reaches these modules through ``vlm.model.get_image_features``
(reflex/policies/pi05/modeling_pi05.py:141-158) of a pinned transformers fork
that is not vendored; the installed transformers stands in for it.

    python tests/golden/make_golden_vision.py

Stored: the seeds, a SHA-256 of the regenerated weights and image, the post
LayerNorm hidden state and the projected image tokens of the first 64 patches
(fp32), and per-token means and norms of all 256.
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

from reflex_b200 import synthetic  # noqa: E402
from reflex_b200.config import VisionConfig  # noqa: E402

LAYERS, W_SEED, IMG_SEED = 2, 20, 21


def sha(ts) -> str:
    h = hashlib.sha256()
    for t in ts:
        h.update(np.ascontiguousarray(t.detach().cpu().float().numpy()).tobytes())
    return h.hexdigest()


def main() -> None:
    from transformers import PaliGemmaConfig, SiglipVisionConfig
    from transformers.models.paligemma.modeling_paligemma import PaliGemmaMultiModalProjector
    from transformers.models.siglip.modeling_siglip import SiglipVisionModel

    cfg = VisionConfig(num_layers=LAYERS)
    w = synthetic.vision_weights(cfg, seed=W_SEED)
    img = synthetic.images(cfg, B=1, seed=IMG_SEED)
    vc = SiglipVisionConfig(hidden_size=cfg.width, intermediate_size=cfg.mlp_dim, num_hidden_layers=LAYERS,
                            num_attention_heads=cfg.num_heads, num_channels=cfg.channels, image_size=cfg.image,
                            patch_size=cfg.patch, hidden_act="gelu_pytorch_tanh", layer_norm_eps=cfg.eps,
                            vision_use_head=False, attn_implementation="eager")
    tower = SiglipVisionModel(vc).eval()
    sd = {k: v for k, v in w.items() if k.startswith("vision_model.")}
    missing, unexpected = tower.load_state_dict(sd, strict=False)
    assert not unexpected and all("position_ids" in m for m in missing), (missing, unexpected)
    pc = PaliGemmaConfig(vision_config=vc.to_dict(), projection_dim=cfg.proj_dim)
    proj = PaliGemmaMultiModalProjector(pc).eval()
    proj.linear.weight.data.copy_(w["projector.linear.weight"])
    proj.linear.bias.data.copy_(w["projector.linear.bias"])
    with torch.no_grad():
        hid = tower(img).last_hidden_state
        out = proj(hid)
    np.savez_compressed(
        os.path.join(HERE, "vision_l2.npz"),
        layers=LAYERS, w_seed=W_SEED, img_seed=IMG_SEED,
        inputs_sha=sha([w[k] for k in sorted(w)] + [img]),
        hidden64=hid[0, :64].numpy().astype(np.float32), tokens64=out[0, :64].numpy().astype(np.float32),
        tok_mean=out[0].mean(-1).numpy().astype(np.float32), tok_norm=out[0].norm(dim=-1).numpy().astype(np.float32),
    )
    print("wrote vision_l2.npz", tuple(out.shape), float(out.abs().max()))


if __name__ == "__main__":
    main()
