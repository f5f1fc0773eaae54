"""Observation-embedding cache with the similarity gate on the GPU
(rfx_embed_cache_check): a camera's embedding is reused while its image stays
close to the last one that was embedded.

``EmbeddingCache.embed(images, img_embedder)`` follows the cache of
PI05PrefixEmbedder.forward (reflex/policies/pi05/modeling_pi05.py:173-247):
per camera, the image is average-pooled to 32 x 32 and compared with the
stored pooled image by mean squared error; below ``1 - threshold_score``
(for every image of the batch) the last embedding is reused, otherwise the
embedder runs and the new pooled image and embedding are stored.  A change
in the number of cameras resets the cache.  ``mode="cosine"`` gives
LastFrameCache's check instead (reflex/optimizations/
dynamic_embedding_cache.py:284-392: bilinear 16 x 16 features, hit when the
batch-mean cosine similarity reaches ``threshold_score``).

Only the decision (one int per camera) is read back to the host; the pooling
and comparison never leave the GPU.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib as L
from . import kernels as K


class _Slot:
    def __init__(self, B: int, C: int, pool: int, device):
        self.feat_prev = torch.zeros(B, C, pool, pool, dtype=torch.float32, device=device)
        self.feat_new = torch.zeros_like(self.feat_prev)
        self.sums = torch.zeros(B, 3, dtype=torch.float32, device=device)
        self.state = torch.zeros(2, dtype=torch.int32, device=device)
        self.metric = torch.zeros(B, dtype=torch.float32, device=device)
        self.embedding = None


class EmbeddingCache:
    def __init__(self, threshold_score: float = 0.98, mode: str = "mse", pool: int | None = None):
        if mode not in ("mse", "cosine"):
            raise ValueError("mode must be 'mse' or 'cosine'")
        self.mode = mode
        self.pool = pool or (32 if mode == "mse" else 16)
        # the reference turns a similarity score into an MSE bound (pixels in [-1, 1])
        self.threshold = (1.0 - threshold_score) if mode == "mse" else threshold_score
        self.stats = {"total_requests": 0, "cache_hits": 0, "cache_misses": 0}
        self.reset_cache()

    def reset_cache(self) -> None:
        self.slots: list[_Slot | None] = []

    def check(self, i: int, image: torch.Tensor) -> bool:
        """Runs the gate of camera slot i on image [B, C, H, W] (fp32 / bf16);
        True when the stored embedding may be reused.  On a miss the new
        features are stored."""
        if not image.is_cuda:
            raise ValueError("EmbeddingCache runs on the GPU: pass a CUDA image")
        B, C, H, W = image.shape
        s = self.slots[i]
        if s is None or s.feat_prev.shape[:2] != (B, C):
            s = self.slots[i] = _Slot(B, C, self.pool, image.device)
        img = image.contiguous()
        d = L.EmbedCacheDesc()
        d.mode = L.RFX_EMBED_CACHE_POOL_MSE if self.mode == "mse" else L.RFX_EMBED_CACHE_BILINEAR_COS
        d.B, d.C, d.H, d.W = B, C, H, W
        d.in_dtype = K._dtype_code(img)
        d.pool, d.threshold = self.pool, self.threshold
        d.image = img.data_ptr()
        d.feat_prev, d.feat_new, d.sums = s.feat_prev.data_ptr(), s.feat_new.data_ptr(), s.sums.data_ptr()
        d.state, d.metric = s.state.data_ptr(), s.metric.data_ptr()
        L.call("rfx_embed_cache_check", ctypes.byref(d), K._stream())
        return bool(s.state[1].item()) and s.embedding is not None

    def embed(self, images: list, img_embedder) -> list:
        """Embeddings of every camera image, reusing cached ones on a hit."""
        if len(self.slots) != len(images):
            self.reset_cache()
            self.slots = [None] * len(images)
        out = []
        for i, img in enumerate(images):
            self.stats["total_requests"] += 1
            if self.check(i, img):
                self.stats["cache_hits"] += 1
                out.append(self.slots[i].embedding)
                continue
            self.stats["cache_misses"] += 1
            emb = img_embedder(img)
            self.slots[i].embedding = emb.detach()
            out.append(emb)
        return out
