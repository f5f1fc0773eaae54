"""CPU restatement of the reference's observation-embedding cache checks
(test infrastructure; the product never imports it).

pool_mse: PI05PrefixEmbedder.forward, reflex/policies/pi05/modeling_pi05.py:
214-229 -- F.adaptive_avg_pool2d(img, (32, 32)), F.mse_loss(..., 'none')
.mean(dim=(1, 2, 3)), hit iff (mse < 1 - threshold_score).all().
bilinear_cos: LastFrameCache, reflex/optimizations/dynamic_embedding_cache.py:
316-345 -- F.interpolate(image, (16, 16), mode='bilinear',
align_corners=False).flatten(1), F.normalize both, per-image dot, mean over
the batch, hit iff mean >= threshold.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F


def pool_features(img: torch.Tensor, pool: int = 32) -> torch.Tensor:
    return F.adaptive_avg_pool2d(img.float(), (pool, pool))


def pool_mse(new: torch.Tensor, prev: torch.Tensor) -> torch.Tensor:
    return F.mse_loss(new, prev, reduction="none").mean(dim=(1, 2, 3))


def bilinear_features(img: torch.Tensor, size: int = 16) -> torch.Tensor:
    return F.interpolate(img.float(), size=(size, size), mode="bilinear", align_corners=False)


def cosine(new: torch.Tensor, prev: torch.Tensor) -> torch.Tensor:
    a, b = F.normalize(new.flatten(1), dim=-1), F.normalize(prev.flatten(1), dim=-1)
    return (a * b).sum(dim=-1)
