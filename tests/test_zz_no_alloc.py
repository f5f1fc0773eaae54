"""rfx_attention_noalloc (scratch in the library's static device array, no
allocation) against rfx_attention with a caller workspace, through the C ABI.

The entry point is for hosts that may not allocate device memory once they
run (a memory pool that owns every device byte from start-up, or a control
loop that forbids cudaMalloc because it can synchronize the device).  Both
calls run the same kernels with the same split count, so the outputs agree
to the test tolerance of 0 (bit-identical); with an automatic split count the
no-allocation call may pick fewer splits to fit its scratch, and the test
compares it with the workspace path at that count.  The file is named to be
collected last, so it runs both alone and after every other GPU test.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

TOL = 0.0
SCRATCH_USABLE = (8 << 20) - 1024


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
    Hq, D, cap = 8, 256, max(1024, n_ctx)
    ring = K.KVRing.allocate(B, 1, cap, D, L.RFX_QUANT_I8_SYM, scale_dtype=torch.float32)
    K.kv_quant_append(r(B, 1, n_ctx, D).bfloat16().cuda(), r(B, 1, n_ctx, D).bfloat16().cuda(), ring, 0, 0, cap)
    q = r(B, Hq, S, D).bfloat16().cuda()
    ks = r(B, S, D).bfloat16().cuda()
    vs = r(B, S, D).bfloat16().cuda()
    return dict(q=q, k_new=ks, v_new=vs, ring=ring, n_ctx=n_ctx, softmax_scale=1 / 16)


def _fitting_splits(K, L, case, out, source):
    """The split count the no-allocation call uses with kv_splits = 0: the
    library's automatic count (one per key block, at most SMs / query-tile
    CTAs and 32), lowered until the scratch fits."""
    B, Hq, S, _ = case["q"].shape
    n_blocks = (case["n_ctx"] + 63) // 64 + (S + 63) // 64
    q_tiles = (Hq * S + 127) // 128
    nsm = ctypes.c_int(0)
    L.call("rfx_num_sms", ctypes.byref(nsm))
    s = min(32, n_blocks, max(1, min(n_blocks, nsm.value // (B * q_tiles))))
    while s > 1:
        d = K.attention_desc(out=out, kv_splits=s, kv_source=source, **case)
        if K.attention_workspace_bytes(d) <= SCRATCH_USABLE:
            break
        s -= 1
    return s


def _run_both(K, L, case, splits, source=0):
    B, Hq, S, D = case["q"].shape
    out_ref = torch.empty(B * S, Hq * D, dtype=torch.bfloat16, device="cuda")
    out_na = torch.full_like(out_ref, float("nan"))
    ref_splits = splits if splits > 0 else _fitting_splits(K, L, case, out_ref, source)
    K.attention(out=out_ref, kv_splits=ref_splits, kv_source=source, **case)
    d = K.attention_desc(out=out_na, kv_splits=splits, kv_source=source, **case)
    L.call("rfx_attention_noalloc", ctypes.byref(d), K._stream())
    torch.cuda.synchronize()
    return out_ref, out_na


@pytest.mark.parametrize("B,n_ctx,S,splits,source", [
    (1, 818, 10, 0, 0),
    (4, 818, 10, 0, 0),
    (2, 600, 50, 5, 0),
    (2, 2048, 10, 0, 0),   # the automatic split count (32) would not fit: it shrinks
    (1, 2048, 50, 0, 0),
    (1, 818, 50, 0, 1),    # dense key source: the key copy lives in the scratch too
    (2, 600, 10, 4, 1),
])
def test_noalloc_matches_workspace_path_twice(K, L, B, n_ctx, S, splits, source):
    for call in range(2):  # two calls in a row, fresh inputs each time
        case = _case(K, L, B, n_ctx, S, seed=100 * call + B)
        ref, got = _run_both(K, L, case, splits, source)
        assert torch.isfinite(got.float()).all(), f"call {call}: output not fully written"
        err = (got.float() - ref.float()).abs().max().item()
        assert err <= TOL, f"call {call}: max abs diff {err}"
    assert K.device_status() == 0


def test_noalloc_rejects_oversize(K, L):
    case = _case(K, L, 8, 900, 10, seed=7)
    B, Hq, S, D = case["q"].shape
    out = torch.empty(B * S, Hq * D, dtype=torch.bfloat16, device="cuda")
    d = K.attention_desc(out=out, kv_splits=15, **case)  # 8 CTAs x 15 splits > 63
    assert K.attention_workspace_bytes(d) > SCRATCH_USABLE
    with pytest.raises(L.RfxError, match="static scratch"):
        L.call("rfx_attention_noalloc", ctypes.byref(d), K._stream())
