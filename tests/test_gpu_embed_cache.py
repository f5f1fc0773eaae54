"""Observation-embedding cache gate (rfx_embed_cache_check through the C ABI)
against the CPU restatement of the reference's checks (oracle/embed_cache.py):
pooled / resampled features within 1e-5 relative of torch's, the per-image
mse / cosine within 1e-4 relative, identical hit decisions away from the
threshold, and EmbeddingCache's reuse and reset behaviour."""
import pytest
import torch

from oracle import embed_cache as oe

pytestmark = pytest.mark.gpu


def _img(B, C, H, W, seed, dtype=torch.float32):
    g = torch.Generator().manual_seed(seed)
    return (torch.rand(B, C, H, W, generator=g) * 2 - 1).to(dtype)


@pytest.mark.parametrize("H,W", [(224, 224), (250, 333), (32, 40)])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_pool_mse_gate_matches_reference(H, W, dtype):
    from reflex_b200.embedding_cache import EmbeddingCache
    cache = EmbeddingCache(threshold_score=0.98, mode="mse")
    cache.slots = [None]
    a = _img(2, 3, H, W, 1, dtype)
    assert not cache.check(0, a.cuda())  # nothing stored: miss, features stored
    s = cache.slots[0]
    ref_a = oe.pool_features(a)
    assert torch.allclose(s.feat_prev.cpu(), ref_a, rtol=1e-5, atol=1e-6)
    s.embedding = torch.zeros(1)  # as after the embedder ran
    # a uniform shift survives the pooling: mse = shift^2 against the 0.02 bound
    for shift, want_hit in ((0.05, True), (0.3, False)):
        b = (a.float() + shift + 0.01 * _img(2, 3, H, W, 2)).to(dtype)
        got = cache.check(0, b.cuda())
        ref_b = oe.pool_features(b)
        mse = oe.pool_mse(ref_b, ref_a)
        assert torch.allclose(s.metric.cpu(), mse, rtol=1e-4, atol=1e-9)
        assert got == bool((mse < cache.threshold).all()) == want_hit
    # the miss stored the new features; the hit before it kept the old ones
    assert torch.allclose(s.feat_prev.cpu(), ref_b, rtol=1e-5, atol=1e-6)


def test_cosine_gate_matches_reference():
    from reflex_b200.embedding_cache import EmbeddingCache
    cache = EmbeddingCache(threshold_score=0.99, mode="cosine")
    cache.slots = [None]
    a = _img(3, 3, 224, 224, 5)
    cache.check(0, a.cuda())
    s = cache.slots[0]
    ref_a = oe.bilinear_features(a)
    assert torch.allclose(s.feat_prev.cpu(), ref_a, rtol=1e-5, atol=1e-6)
    s.embedding = torch.zeros(1)
    for noise in (0.01, 2.0):
        b = a + noise * _img(3, 3, 224, 224, 6)
        got = cache.check(0, b.cuda())
        sim = oe.cosine(oe.bilinear_features(b), ref_a)
        assert torch.allclose(s.metric.cpu(), sim, rtol=1e-4)
        assert got == bool(sim.mean() >= cache.threshold)


def test_embedding_cache_reuse_and_reset():
    from reflex_b200.embedding_cache import EmbeddingCache
    calls = []

    def embedder(img):
        calls.append(1)
        return img.mean(dim=(2, 3)) + len(calls)

    cache = EmbeddingCache(threshold_score=0.98)
    cams = [_img(1, 3, 224, 224, 10).cuda(), _img(1, 3, 224, 224, 11).cuda()]
    e1 = cache.embed(cams, embedder)
    assert len(calls) == 2
    e2 = cache.embed([c + 0.01 for c in cams], embedder)  # tiny change: both reused
    assert len(calls) == 2 and all(torch.equal(x, y) for x, y in zip(e1, e2))
    e3 = cache.embed([cams[0], cams[1] + 0.5], embedder)  # camera 1 changed (mse 0.25)
    assert len(calls) == 3 and torch.equal(e3[0], e1[0]) and not torch.equal(e3[1], e1[1])
    cache.embed(cams[:1], embedder)  # one camera fewer: the cache resets
    assert len(calls) == 4
    assert cache.stats == {"total_requests": 7, "cache_hits": 3, "cache_misses": 4}
