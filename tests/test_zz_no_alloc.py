"""rfx_attention_noalloc (split-KV partials in the library's static scratch)
against rfx_attention with a caller workspace, through the C ABI.

Both calls run the same kernels with the same split count, so the outputs
agree to the test tolerance of 0 (bit-identical).  The file is named to be
collected last, so it runs both alone and after every other GPU test.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

TOL = 0.0


@pytest.fixture(scope="module")
def K():
    from reflex_b200 import kernels
    return kernels


@pytest.fixture(scope="module")
def L():
    from reflex_b200 import _lib
    return _lib


def _case(K, L, B, n_ctx, S, seed):
    g = torch.Generator().manual_seed(seed)
    r = lambda *s: torch.randn(*s, generator=g)  # noqa: E731
    Hq, D, cap = 8, 256, 1024
    ring = K.KVRing.allocate(B, 1, cap, D, L.RFX_QUANT_I8_SYM, scale_dtype=torch.float32)
    K.kv_quant_append(r(B, 1, n_ctx, D).bfloat16().cuda(), r(B, 1, n_ctx, D).bfloat16().cuda(), ring, 0, 0, cap)
    q = r(B, Hq, S, D).bfloat16().cuda()
    ks = r(B, S, D).bfloat16().cuda()
    vs = r(B, S, D).bfloat16().cuda()
    return dict(q=q, k_new=ks, v_new=vs, ring=ring, n_ctx=n_ctx, softmax_scale=1 / 16)


def _run_both(K, L, case, splits):
    B, Hq, S, D = case["q"].shape
    out_ref = torch.empty(B * S, Hq * D, dtype=torch.bfloat16, device="cuda")
    out_na = torch.full_like(out_ref, float("nan"))
    K.attention(out=out_ref, kv_splits=splits, **case)
    d = K.attention_desc(out=out_na, kv_splits=splits, **case)
    assert K.attention_workspace_bytes(d) > 0  # the split-KV path (scratch in use)
    L.call("rfx_attention_noalloc", ctypes.byref(d), K._stream())
    torch.cuda.synchronize()
    return out_ref, out_na


@pytest.mark.parametrize("B,n_ctx,S,splits", [(1, 818, 10, 0), (4, 818, 10, 0), (2, 600, 50, 5)])
def test_noalloc_matches_workspace_path_twice(K, L, B, n_ctx, S, splits):
    for call in range(2):  # two calls in a row, fresh inputs each time
        case = _case(K, L, B, n_ctx, S, seed=100 * call + B)
        ref, got = _run_both(K, L, case, splits)
        err = (got.float() - ref.float()).abs().max().item()
        assert err <= TOL, f"call {call}: max abs diff {err}"
    assert K.device_status() == 0


def test_noalloc_rejects_oversize(K, L):
    case = _case(K, L, 8, 900, 10, seed=7)
    B, Hq, S, D = case["q"].shape
    out = torch.empty(B * S, Hq * D, dtype=torch.bfloat16, device="cuda")
    d = K.attention_desc(out=out, kv_splits=15, **case)  # 8 CTAs x 15 splits > 63
    assert K.attention_workspace_bytes(d) > 8 << 20
    with pytest.raises(L.RfxError, match="static scratch"):
        L.call("rfx_attention_noalloc", ctypes.byref(d), K._stream())
