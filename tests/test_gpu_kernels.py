"""Kernel-level parity of the CUDA path (through the C ABI) against the oracle.

Bit-exact for the KV quantizers; the bf16 GEMMs and attention against an
fp32 torch computation on the same bf16 inputs with the tolerance stated in
each test.
"""
import ctypes
import math

import numpy as np
import pytest
import torch

from oracle import quant as oq
from oracle.attention import partitioned_attention
from oracle.bf16 import bf16_round

pytestmark = pytest.mark.gpu

# Tolerance of a bf16 kernel output against the fp32 computation of the same
# bf16 inputs: 1e-2 absolute + 1e-2 relative (one bf16 ulp is 2^-8 relative).
ATOL, RTOL = 1e-2, 1e-2


@pytest.fixture(scope="module")
def K():
    from reflex_b200 import kernels
    return kernels


@pytest.fixture(scope="module")
def L():
    from reflex_b200 import _lib
    return _lib


def gen(seed):
    g = torch.Generator().manual_seed(seed)
    return lambda *shape, std=1.0: torch.randn(*shape, generator=g) * std


# ------------------------------------------------------------- quantizers ---
def _edge_rows(D=256):
    rows = [np.zeros(D), np.full(D, 3.25), np.linspace(-1e-6, 1e-6, D), -np.abs(np.linspace(0.1, 7, D)),
            np.linspace(-2.5, 2.5, D), np.r_[np.full(D - 1, 0.5), 127.0], np.r_[np.full(D - 1, -1.0), 1e4]]
    return np.stack(rows).astype(np.float32)


@pytest.mark.parametrize("mode", ["i8", "u8"])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_kv_quant_bit_exact(K, L, mode, dtype):
    B, H, Lnew, D, cap = 2, 1, 77, 256, 160
    r = gen(1)
    k = r(B, H, Lnew, D) * 3
    v = r(B, H, Lnew, D)
    k[0, 0, :7] = torch.from_numpy(_edge_rows())
    k = k.to(dtype).cuda()
    v = v.to(dtype).cuda()
    qm = L.RFX_QUANT_I8_SYM if mode == "i8" else L.RFX_QUANT_U8_REF
    ring = K.KVRing.allocate(B, H, cap, D, qm, scale_dtype=dtype)
    # window region [32, 160) with an append that wraps around its end
    base, off, rlen = 32, 100, 128
    K.kv_quant_append(k, v, ring, base, off, rlen)
    torch.cuda.synchronize()
    slots = base + (off + np.arange(Lnew)) % rlen
    for src, q, s, z in ((k, ring.k_q, ring.k_scale, ring.k_zp), (v, ring.v_q, ring.v_scale, ring.v_zp)):
        x = src.float().cpu().numpy()
        if mode == "i8":
            eq, es = oq.quant_i8_sym(x)
        else:
            eq, es, ez = oq.quant_u8_ref(x, act_bf16=dtype == torch.bfloat16)
            np.testing.assert_array_equal(z.float().cpu().numpy()[:, :, slots], ez[..., 0])
        np.testing.assert_array_equal(q.cpu().numpy()[:, :, slots], eq)
        np.testing.assert_array_equal(s.float().cpu().numpy()[:, :, slots], es[..., 0])


def _near_tie_rows(D=256, n=96, seed=3):
    """Rows whose quotients x / scale sit on or within a few ulps of
    half-integers (the int8 quantizer rounds them from a product with the
    reciprocal and must fall back to the exact divide there), over scales from
    normal down to denormal (where the reciprocal overflows)."""
    rng = np.random.default_rng(seed)
    f32 = np.float32
    rows = []
    for i in range(n):
        amax = f32(10.0 ** rng.uniform(-41, 30)) if i % 4 else f32(127.0) * f32(rng.uniform(0.05, 2.0))
        s = f32(amax / f32(127))
        k = rng.integers(-127, 127, D).astype(f32) + f32(0.5)
        x = (k * s).astype(f32)
        x = (x.view(np.int32) + rng.integers(-3, 4, D).astype(np.int32)).view(f32)
        x = np.clip(x, -amax, amax)
        x[0] = amax
        rows.append(x)
    return np.stack(rows).astype(np.float32)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_kv_quant_i8_near_ties(K, L, dtype):
    """int8 scheme, bit-exact against the oracle on quotients at and next to
    rounding boundaries, denormal scales included."""
    x = torch.from_numpy(_near_tie_rows()).to(dtype)
    B, Lnew = 2, x.shape[0] // 2
    k = x.reshape(B, 1, Lnew, 256).contiguous()
    v = torch.flip(k, dims=[2]).contiguous()
    ring = K.KVRing.allocate(B, 1, Lnew, 256, L.RFX_QUANT_I8_SYM, scale_dtype=torch.float32)
    K.kv_quant_append(k.cuda(), v.cuda(), ring)
    torch.cuda.synchronize()
    for src, q, s in ((k, ring.k_q, ring.k_scale), (v, ring.v_q, ring.v_scale)):
        eq, es = oq.quant_i8_sym(src.float().numpy())
        np.testing.assert_array_equal(q.cpu().numpy(), eq)
        np.testing.assert_array_equal(s.cpu().numpy(), es[..., 0])


# ------------------------------------------------------------------ linear ---
def _mm(x, w):
    return x.float() @ w.float().t()


@pytest.mark.parametrize("T,n_tile,splits", [(50, 0, 0), (1, 64, 1), (50, 64, 2), (50, 64, 8), (100, 64, 8),
                                             (100, 128, 4), (200, 256, 2), (400, 0, 0)])
def test_linear_store(K, T, n_tile, splits):
    r = gen(2)
    O, Kd = 512, 1024
    x = r(T, Kd).bfloat16().cuda()
    w = r(O, Kd, std=0.03).bfloat16().cuda()
    bias = r(O, std=0.1).cuda()
    y = torch.empty(T, O, dtype=torch.bfloat16, device="cuda")
    K.linear(w=w, x=x, T=T, S=T, y=y, bias=bias, n_tile=n_tile, splits=splits)
    ref = _mm(x, w).cpu() + bias.cpu()
    torch.testing.assert_close(y.float().cpu(), ref, atol=ATOL, rtol=RTOL)


@pytest.mark.parametrize("epi", ["store", "residual", "geglu", "qkv",
                                 "store_wide", "residual_wide", "geglu_wide", "qkv_wide"])
@pytest.mark.parametrize("B,S", [(1, 300), (2, 384), (1, 768)])
def test_linear_many_tokens_persistent_tiles(K, L, epi, B, S):
    """T > 128 tokens with the load prologue run the persistent tile kernel (two
    TMEM accumulators, a tile's epilogue under the next tile's mainloop).  Each
    output sums the same k-steps in the same order as in the per-tile kernel
    without split-K, so the outputs are bit-identical to it for every
    epilogue, with ragged last token tiles and several batches; the store
    epilogue is also checked against the fp32 product.  The token tile width
    (the MMA's N) does not change a result bit, so the reference is the
    per-tile kernel at 128-token tiles for all of them; the persistent kernel
    picks 128-token tiles at 4096 rows x 300 tokens, 192 at 4096 x 768 and
    16384 x 300, 256 at 16384 x 768 (the *_wide cases have 16384 rows)."""
    r = gen(6)
    T, Kd, Hq, D = B * S, 1024, 8, 256
    x = r(T, Kd).bfloat16().cuda()
    wide = epi.endswith("_wide")
    epi = epi.replace("_wide", "")
    # output rows (2F for gate/up): enough 128-token tiles for the persistent kernel
    O = 16384 if wide else 4096
    Hq = 62 if wide else 14  # QKV: (Hq + 2) x 256 = 16384 or 4096 rows

    def run(tiling):
        kw = dict(w=w, x=x, T=T, S=S, n_tile=tiling[0], splits=tiling[1])
        if epi == "store":
            y = torch.empty(T, O, dtype=torch.bfloat16, device="cuda")
            K.linear(y=y, bias=bias, **kw)
            return [y]
        if epi == "residual":
            y = y0.clone()
            K.linear(epilogue=L.RFX_EPI_RESIDUAL, y=y, gate=gate, gate_stride=O, **kw)
            return [y]
        if epi == "geglu":
            y = torch.empty(T, O // 2, dtype=torch.bfloat16, device="cuda")
            K.linear(epilogue=L.RFX_EPI_GEGLU, y=y, **kw)
            return [y]
        q = torch.empty(B, Hq, S, D, dtype=torch.bfloat16, device="cuda")
        k = torch.empty(T, D, dtype=torch.bfloat16, device="cuda")
        v = torch.empty(T, D, dtype=torch.bfloat16, device="cuda")
        K.linear(epilogue=L.RFX_EPI_QKV_ROPE, rope_table=tab, positions=pos, q_out=q, k_out=k, v_out=v,
                 num_q_heads=Hq, **kw)
        return [q, k, v]

    if epi == "store":
        w = r(O, Kd, std=0.03).bfloat16().cuda()
        bias = r(O, std=0.1).cuda()
    elif epi == "residual":
        w = r(O, Kd, std=0.03).bfloat16().cuda()
        gate = torch.from_numpy(bf16_round(r(B, O).numpy())).cuda()
        y0 = r(T, O).bfloat16().cuda()
    elif epi == "geglu":
        w = K.pack_weight(L.RFX_PACK_GATE_UP, r(O, Kd, std=0.03).bfloat16().cuda())
    else:
        O = (Hq + 2) * D
        w = K.pack_weight(L.RFX_PACK_QKV_ROPE, r(O, Kd, std=0.03).bfloat16().cuda())
        tab = rope_table().cuda()
        pos = (100 + torch.arange(S, dtype=torch.int32)).repeat(B).cuda()
    nsm = torch.cuda.get_device_properties(0).multi_processor_count
    assert 2 * (O // 128) * ((T + 127) // 128) >= nsm  # the persistent kernel serves these shapes
    got = run((0, 0))       # persistent tile kernel
    ref = run((128, 1))     # per-tile kernel
    torch.cuda.synchronize()
    assert K.device_status() == 0
    for a, b in zip(got, ref):
        assert torch.equal(a, b), f"max diff {(a.float() - b.float()).abs().max().item()}"
    if epi == "store":
        torch.testing.assert_close(got[0].float().cpu(), _mm(x, w).cpu() + bias.cpu(), atol=ATOL, rtol=RTOL)


@pytest.mark.gpu
@pytest.mark.parametrize("epi", ["store", "residual", "geglu", "qkv"])
@pytest.mark.parametrize("B,S", [(1, 768), (2, 300)])
def test_linear_split_k_workspace(K, L, epi, B, S):
    """With a zero-filled workspace, a many-token GEMM whose tiles leave SMs
    idle (a 2048-row weight at 600 or 768 tokens: 80 or 96 tiles of 128
    tokens, K = 8192) splits K over three CTAs per tile (ragged: 128 k-steps
    as 42/43/43);
    the last split to arrive sums the fp32 partials in split order and runs
    the fused epilogue.  Checked against the fp32 product (store), against the
    unsplit persistent kernel within bf16 rounding (every epilogue), for
    run-to-run bit identity over back-to-back launches on one stream, and for
    counters left at zero.  A workspace one byte short disables the split and
    gives the unsplit result exactly."""
    r = gen(7)
    T, Kd, D = B * S, 8192, 256
    Hq = 6  # QKV: (6 + 2) x 256 = 2048 rows
    O = 2048
    x = r(T, Kd).bfloat16().cuda()
    if epi == "geglu":
        w = K.pack_weight(L.RFX_PACK_GATE_UP, r(O, Kd, std=0.011).bfloat16().cuda())
    elif epi == "qkv":
        w = K.pack_weight(L.RFX_PACK_QKV_ROPE, r(O, Kd, std=0.011).bfloat16().cuda())
        tab = rope_table().cuda()
        pos = (100 + torch.arange(S, dtype=torch.int32)).repeat(B).cuda()
    else:
        w = r(O, Kd, std=0.011).bfloat16().cuda()
    bias = r(O, std=0.1).cuda()
    gate = torch.from_numpy(bf16_round(r(B, O).numpy())).cuda()
    y0 = r(T, O).bfloat16().cuda()

    def run(ws):
        kw = dict(w=w, x=x, T=T, S=S, workspace=ws)
        if epi == "store":
            outs = [torch.empty(T, O, dtype=torch.bfloat16, device="cuda")]
            K.linear(y=outs[0], bias=bias, **kw)
        elif epi == "residual":
            outs = [y0.clone()]
            K.linear(epilogue=L.RFX_EPI_RESIDUAL, y=outs[0], gate=gate, gate_stride=O, **kw)
        elif epi == "geglu":
            outs = [torch.empty(T, O // 2, dtype=torch.bfloat16, device="cuda")]
            K.linear(epilogue=L.RFX_EPI_GEGLU, y=outs[0], **kw)
        else:
            outs = [torch.empty(B, Hq, S, D, dtype=torch.bfloat16, device="cuda"),
                    torch.empty(T, D, dtype=torch.bfloat16, device="cuda"),
                    torch.empty(T, D, dtype=torch.bfloat16, device="cuda")]
            K.linear(epilogue=L.RFX_EPI_QKV_ROPE, rope_table=tab, positions=pos, q_out=outs[0], k_out=outs[1],
                     v_out=outs[2], num_q_heads=Hq, **kw)
        return outs

    tiles = (O // 128) * ((T + 127) // 128)
    ctr_bytes = 65536  # the fixed counter block
    probe = K.linear_desc(w=w, x=x, T=T, S=S, y=torch.empty(T, O, dtype=torch.bfloat16, device="cuda"))
    need = K.linear_workspace_bytes(probe)
    nsm = torch.cuda.get_device_properties(0).multi_processor_count
    if nsm == 148:
        assert need == ctr_bytes + tiles * 3 * 128 * 128 * 4
    assert need > 0
    ws = K.linear_workspace(need, "cuda")
    assert ws.data_ptr() % 256 == 0
    plain = run(None)
    split = [run(ws) for _ in range(3)]  # back-to-back on one stream (PDL overlap)
    short = run(ws[:need - 1])
    torch.cuda.synchronize()
    assert K.device_status() == 0
    assert int(ws[:ctr_bytes].count_nonzero()) == 0  # counters back at zero
    for later in split[1:]:
        for a, b in zip(split[0], later):
            assert torch.equal(a, b)
    for a, b in zip(short, plain):
        assert torch.equal(a, b)
    for a, b in zip(split[0], plain):
        # bf16 roundings of two fp32 sums: a one-ulp flip of a RoPE input
        # (outputs of std ~1) moves a cancelling output by up to two ulps
        torch.testing.assert_close(a.float(), b.float(), atol=3e-2, rtol=1.6e-2)
    if epi == "store":
        torch.testing.assert_close(split[0][0].float().cpu(), _mm(x, w).cpu() + bias.cpu(), atol=ATOL, rtol=RTOL)


def _norm_ref(x, a1, a2, b2, S, eps=1e-6):
    xf = x.float().cpu()
    rstd = torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    b = torch.arange(x.shape[0]) // S
    y = (xf * rstd) * a1.cpu()
    if a2 is not None:
        y = y * a2.cpu()[b]
    if b2 is not None:
        y = y + b2.cpu()[b]
    return y.bfloat16()


@pytest.mark.parametrize("epi", ["residual", "geglu", "silu"])
def test_linear_norm_prologue_epilogues(K, L, epi):
    r = gen(3)
    B, S, Kd = 2, 50, 1024
    T = B * S
    x = r(T, Kd).bfloat16().cuda()
    a1 = (1 + r(Kd, std=0.1)).cuda()
    a2 = (1 + r(B, Kd, std=0.2)).cuda()
    b2 = r(B, Kd, std=0.1).cuda()
    xn = _norm_ref(x, a1, a2, b2, S)
    if epi == "residual":
        O = 1024
        w = r(O, Kd, std=0.03).bfloat16().cuda()
        gate = bf16_round(r(B, O).numpy())
        gate = torch.from_numpy(gate).cuda()
        y = r(T, O).bfloat16().cuda()
        y0 = y.clone().cpu().float()
        K.linear(w=w, x=x, T=T, S=S, prologue=L.RFX_PRO_NORM, epilogue=L.RFX_EPI_RESIDUAL, y=y, norm_a1=a1,
                 norm_a2=a2, norm_b2=b2, norm_ab_stride=Kd, gate=gate, gate_stride=O)
        acc = _mm(xn, w.cpu()).bfloat16().float()
        g = gate.cpu()[torch.arange(T) // S]
        ref = (y0 + (g * acc).bfloat16().float())
    elif epi == "geglu":
        F = 2048
        wg = r(F, Kd, std=0.03).bfloat16()
        wu = r(F, Kd, std=0.03).bfloat16()
        w = K.pack_weight(L.RFX_PACK_GATE_UP, torch.cat([wg, wu]).cuda())
        y = torch.empty(T, F, dtype=torch.bfloat16, device="cuda")
        K.linear(w=w, x=x, T=T, S=S, prologue=L.RFX_PRO_NORM, epilogue=L.RFX_EPI_GEGLU, y=y, norm_a1=a1,
                 norm_a2=a2, norm_b2=b2, norm_ab_stride=Kd)
        gg = _mm(xn, wg).bfloat16().float()
        uu = _mm(xn, wu).bfloat16().float()
        ref = torch.nn.functional.gelu(gg, approximate="tanh").bfloat16().float() * uu
    else:
        O = 1024
        w = r(O, Kd, std=0.03).bfloat16().cuda()
        bias = r(O, std=0.1).cuda()
        y = torch.empty(T, O, dtype=torch.bfloat16, device="cuda")
        K.linear(w=w, x=x, T=T, S=S, prologue=L.RFX_PRO_NORM, epilogue=L.RFX_EPI_SILU, y=y, norm_a1=a1,
                 norm_a2=a2, norm_b2=b2, norm_ab_stride=Kd, bias=bias)
        ref = torch.nn.functional.silu((_mm(xn, w.cpu()) + bias.cpu()).bfloat16().float())
    torch.cuda.synchronize()
    torch.testing.assert_close(y.float().cpu(), ref, atol=ATOL, rtol=RTOL)


@pytest.mark.parametrize("K_,shared", [(1024, True), (2048, False)])
def test_rms_norm_exact(K, K_, shared):
    """The norm kernel rounds once to bf16 like AdaRMSNorm (reflex/policies/pi05/modeling_pi05.py:73-99);
    against the fp32 torch computation it may differ by one bf16 ulp (summation order of mean(x^2))."""
    r = gen(8)
    B, S = 3, 50
    x = (r(B * S, K_) * 2).bfloat16().cuda()
    a1 = (1 + r(K_, std=0.1)).cuda()
    a2 = (1 + r(1 if shared else B, K_, std=0.2)).cuda()
    b2 = r(1 if shared else B, K_, std=0.1).cuda()
    y = torch.empty_like(x)
    K.rms_norm(x=x, y=y, S=S, norm_a1=a1, norm_a2=a2, norm_b2=b2, norm_ab_stride=0 if shared else K_)
    torch.cuda.synchronize()
    xf = x.float().cpu()
    rstd = torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6)
    bidx = torch.zeros(B * S, dtype=torch.long) if shared else torch.arange(B * S) // S
    ref = ((xf * rstd) * a1.cpu()) * a2.cpu()[bidx] + b2.cpu()[bidx]
    diff = (y.float().cpu() - ref.bfloat16().float()).abs()
    ulp = ref.abs().clamp_min(1e-30) * 2 ** -7
    assert (diff <= ulp + 1e-6).all()


def rope_table(max_pos=8192, D=256, base=10000.0):
    inv = 1.0 / (base ** (torch.arange(0, D, 2, dtype=torch.float) / D))
    t = torch.arange(max_pos, dtype=torch.float)
    f = torch.einsum("i,j->ij", t, inv)
    return torch.cat([f.cos(), f.sin()], dim=-1)


def test_linear_qkv_rope(K, L):
    r = gen(4)
    B, S, Kd, Hq, D = 2, 50, 1024, 8, 256
    T = B * S
    x = r(T, Kd).bfloat16().cuda()
    a1 = (1 + r(Kd, std=0.1)).cuda()
    wqkv = r((Hq + 2) * D, Kd, std=0.03).bfloat16()
    w = K.pack_weight(L.RFX_PACK_QKV_ROPE, wqkv.cuda())
    tab = rope_table().cuda()
    pos = (818 + torch.arange(S, dtype=torch.int32)).repeat(B).cuda()
    q = torch.empty(B, Hq, S, D, dtype=torch.bfloat16, device="cuda")
    k = torch.empty(T, D, dtype=torch.bfloat16, device="cuda")
    v = torch.empty(T, D, dtype=torch.bfloat16, device="cuda")
    K.linear(w=w, x=x, T=T, S=S, prologue=L.RFX_PRO_NORM, epilogue=L.RFX_EPI_QKV_ROPE, norm_a1=a1,
             rope_table=tab, positions=pos, q_out=q, k_out=k, v_out=v, num_q_heads=Hq)
    torch.cuda.synchronize()
    xn = _norm_ref(x, a1, None, None, S)
    out = _mm(xn, wqkv).bfloat16().view(T, Hq + 2, D)
    cs = tab.cpu()[pos.cpu().long()]
    cos, sin = cs[:, None, :128], cs[:, None, 128:]

    def rope(t):
        t1, t2 = t.float().chunk(2, -1)
        return torch.cat([t1 * cos - t2 * sin, t2 * cos + t1 * sin], -1)

    qr = rope(out[:, :Hq]).view(B, S, Hq, D).permute(0, 2, 1, 3)
    kr = rope(out[:, Hq:Hq + 1])[:, 0]
    torch.testing.assert_close(q.float().cpu(), qr, atol=ATOL, rtol=RTOL)
    torch.testing.assert_close(k.float().cpu(), kr, atol=ATOL, rtol=RTOL)
    torch.testing.assert_close(v.float().cpu(), out[:, Hq + 1].float(), atol=ATOL, rtol=RTOL)


# --------------------------------------------------------------- attention ---
@pytest.mark.parametrize("mode", ["i8", "u8"])
@pytest.mark.parametrize("n_ctx,S,splits", [(576, 50, 0), (818, 50, 1), (818, 50, 3), (100, 50, 0), (0, 50, 0),
                                            (1584, 51, 0)])
def test_attention_partitioned(K, L, mode, n_ctx, S, splits):
    r = gen(5)
    B, Hq, D, cap = 2, 8, 256, max(64, n_ctx + 64)
    qm = L.RFX_QUANT_I8_SYM if mode == "i8" else L.RFX_QUANT_U8_REF
    ring = K.KVRing.allocate(B, 1, cap, D, qm, scale_dtype=torch.bfloat16)
    kc = r(B, 1, n_ctx, D).bfloat16()
    vc = r(B, 1, n_ctx, D).bfloat16()
    if n_ctx:
        K.kv_quant_append(kc.cuda(), vc.cuda(), ring, 0, 0, cap)
    q = r(B, Hq, S, D).bfloat16()
    ks = r(B, S, D).bfloat16()
    vs = r(B, S, D).bfloat16()
    # PI0-style suffix block ids: first token its own block when S == 51
    blk = torch.zeros(S, dtype=torch.int32)
    blk[1:] = 1 if S == 51 else 0
    out = torch.empty(B * S, Hq * D, dtype=torch.bfloat16, device="cuda")
    K.attention(q=q.cuda(), k_new=ks.cuda(), v_new=vs.cuda(), ring=ring, n_ctx=n_ctx, out=out,
                softmax_scale=1 / 16, new_block=blk.cuda(), kv_splits=splits)
    torch.cuda.synchronize()
    # oracle: dequantize what the GPU stored, then fp32 attention
    if mode == "i8":
        kd = oq.dequant_i8_sym(ring.k_q.cpu().numpy(), ring.k_scale.cpu().numpy()[..., None])
        vd = oq.dequant_i8_sym(ring.v_q.cpu().numpy(), ring.v_scale.cpu().numpy()[..., None])
    else:
        kd = oq.dequant_u8_ref(ring.k_q.cpu().numpy(), ring.k_scale.float().cpu().numpy()[..., None],
                               ring.k_zp.float().cpu().numpy()[..., None], True)
        vd = oq.dequant_u8_ref(ring.v_q.cpu().numpy(), ring.v_scale.float().cpu().numpy()[..., None],
                               ring.v_zp.float().cpu().numpy()[..., None], True)
    kd = torch.from_numpy(kd)[:, :, :n_ctx]
    vd = torch.from_numpy(vd)[:, :, :n_ctx]
    att = torch.zeros(S, dtype=torch.int64)
    att[0] = 1
    if S == 51:
        att[1] = 1
    ref = partitioned_attention(q, kd, vd, ks[:, None], vs[:, None], torch.ones(B, n_ctx, dtype=torch.bool), att,
                                1 / 16)
    ref = ref.permute(0, 2, 1, 3).reshape(B * S, Hq * D)
    err = (out.float().cpu() - ref).abs().max().item()
    assert err <= 2e-2, f"max abs err {err}"
    assert K.device_status() == 0


@pytest.mark.parametrize("mode", ["i8", "u8"])
@pytest.mark.parametrize("n_ctx,S,splits", [(1584, 200, 0), (300, 100, 1), (0, 64, 0), (818, 50, 3), (2100, 51, 0)])
def test_attention_dense_source_matches_ring_tiles_and_oracle(K, L, mode, n_ctx, S, splits):
    """RFX_KV_DENSE (one dequantize pass, then TMA-fed bf16/f16 tiles with two key
    blocks in flight) against the in-kernel conversion path on the same inputs,
    and both against fp32 attention over the dequantized context (2e-2), with a
    masked context range (an evicted frame); the new keys form one bidirectional
    block, or (S = 51, PI0) a state token in its own block before the actions."""
    r = gen(9)
    B, Hq, D, cap = 1, 8, 256, max(64, n_ctx + 64)
    qm = L.RFX_QUANT_I8_SYM if mode == "i8" else L.RFX_QUANT_U8_REF
    ring = K.KVRing.allocate(B, 1, cap, D, qm, scale_dtype=torch.float32 if mode == "i8" else torch.bfloat16)
    kc, vc = r(B, 1, n_ctx, D).bfloat16(), r(B, 1, n_ctx, D).bfloat16()
    if n_ctx:
        K.kv_quant_append(kc.cuda(), vc.cuda(), ring, 0, 0, cap)
    valid = torch.ones(B, cap, dtype=torch.uint8)
    valid[:, n_ctx // 3: 2 * n_ctx // 3] = 0
    q = r(B, Hq, S, D).bfloat16()
    kn, vn = r(B, S, D).bfloat16(), r(B, S, D).bfloat16()
    blk = None
    if S == 51:
        blk = torch.zeros(S, dtype=torch.int32)
        blk[1:] = 1
    outs = []
    for src in (L.RFX_KV_RING_TILES, L.RFX_KV_DENSE):
        out = torch.empty(B * S, Hq * D, dtype=torch.bfloat16, device="cuda")
        K.attention(q=q.cuda(), k_new=kn.cuda(), v_new=vn.cuda(), ring=ring, n_ctx=n_ctx, out=out,
                    softmax_scale=1 / 16, ctx_valid=valid.cuda(), kv_splits=splits, kv_source=src,
                    new_block=None if blk is None else blk.cuda())
        torch.cuda.synchronize()
        outs.append(out.float().cpu())
    assert K.device_status() == 0
    d_paths = (outs[0] - outs[1]).abs().max().item()
    if mode == "i8":
        kd = oq.dequant_i8_sym(ring.k_q.cpu().numpy(), ring.k_scale.cpu().numpy()[..., None])
        vd = oq.dequant_i8_sym(ring.v_q.cpu().numpy(), ring.v_scale.cpu().numpy()[..., None])
    else:
        kd = oq.dequant_u8_ref(ring.k_q.cpu().numpy(), ring.k_scale.float().cpu().numpy()[..., None],
                               ring.k_zp.float().cpu().numpy()[..., None], True)
        vd = oq.dequant_u8_ref(ring.v_q.cpu().numpy(), ring.v_scale.float().cpu().numpy()[..., None],
                               ring.v_zp.float().cpu().numpy()[..., None], True)
    kd = torch.from_numpy(kd)[:, :, :n_ctx]
    vd = torch.from_numpy(vd)[:, :, :n_ctx]
    att = torch.zeros(S, dtype=torch.int64)
    att[0] = 1
    if S == 51:
        att[1] = 1
    ref = partitioned_attention(q, kd, vd, kn[:, None], vn[:, None], valid[:, :n_ctx].bool(), att, 1 / 16)
    ref = ref.permute(0, 2, 1, 3).reshape(B * S, Hq * D)
    errs = [(o - ref).abs().max().item() for o in outs]
    print(f"dense vs ring tiles {d_paths:.2e}; vs oracle ring {errs[0]:.2e} dense {errs[1]:.2e}")
    assert d_paths <= 2e-3
    assert max(errs) <= 2e-2



@pytest.mark.parametrize("mode", ["i8", "u8"])
def test_attention_dense_context_kept_across_calls(K, L, mode):
    """dense_ctx_ready: a second call on the same workspace with new queries
    and new keys converts only the new keys and gives bit-identical output to
    a call that converts everything (the engine's steps 1.. of a chunk); B = 3
    streams, a masked context range."""
    r = gen(12)
    B, Hq, D, S, n_ctx = 3, 8, 256, 50, 700
    cap = n_ctx + 64
    qm = L.RFX_QUANT_I8_SYM if mode == "i8" else L.RFX_QUANT_U8_REF
    ring = K.KVRing.allocate(B, 1, cap, D, qm, scale_dtype=torch.float32 if mode == "i8" else torch.bfloat16)
    K.kv_quant_append(r(B, 1, n_ctx, D).bfloat16().cuda(), r(B, 1, n_ctx, D).bfloat16().cuda(), ring, 0, 0, cap)
    valid = torch.ones(B, cap, dtype=torch.uint8)
    valid[1, 100:300] = 0
    step_inputs = [(r(B, Hq, S, D).bfloat16().cuda(), r(B * S, D).bfloat16().cuda(), r(B * S, D).bfloat16().cuda())
                   for _ in range(2)]
    kw = dict(ring=ring, n_ctx=n_ctx, softmax_scale=1 / 16, ctx_valid=valid.cuda(), kv_source=L.RFX_KV_DENSE)
    d0 = K.attention_desc(q=step_inputs[0][0], k_new=step_inputs[0][1], v_new=step_inputs[0][2],
                          out=torch.empty(B * S, Hq * D, dtype=torch.bfloat16, device="cuda"), **kw)
    need = K.attention_workspace_bytes(d0)
    ws_keep = torch.empty(need + 1024, dtype=torch.uint8, device="cuda")
    outs = {}
    for name, ready in (("kept", (0, 1)), ("full", (0, 0))):
        ws = ws_keep if name == "kept" else torch.empty(need + 1024, dtype=torch.uint8, device="cuda")
        for i, (q, kn, vn) in enumerate(step_inputs):
            out = torch.empty(B * S, Hq * D, dtype=torch.bfloat16, device="cuda")
            d = K.attention_desc(q=q, k_new=kn, v_new=vn, out=out, **kw)
            d.workspace, d.workspace_bytes = K.aligned_ptr(ws, 1024), need
            d.dense_ctx_ready = ready[i]
            L.call("rfx_attention", ctypes.byref(d), K._stream())
            outs[(name, i)] = out
    torch.cuda.synchronize()
    assert K.device_status() == 0
    assert torch.equal(outs[("kept", 1)], outs[("full", 1)])
    assert not torch.equal(outs[("kept", 0)], outs[("kept", 1)])

# ------------------------------------------------------ conditioning heads ---
def test_time_cond_matches_fp64_embedding_and_mlp(K):
    from oracle.model import sinusoid
    r = gen(11)
    W, n_t = 1024, 10
    t = torch.linspace(1.0, 0.1, n_t, dtype=torch.float32)
    w_in, w_out = (r(W, W) * 0.03).bfloat16().float(), (r(W, W) * 0.03).bfloat16().float()
    b_in, b_out = (r(W) * 0.1).bfloat16().float(), (r(W) * 0.1).bfloat16().float()
    dev = lambda a: a.bfloat16().cuda()  # noqa: E731
    hid = torch.empty(n_t, W, dtype=torch.bfloat16, device="cuda")
    cond = torch.empty(n_t, W, dtype=torch.bfloat16, device="cuda")
    # embedding alone: bf16 of the fp64 sinusoid.  fp64 pow/sin differ between
    # libraries by an ulp, which only shows where sin/cos is ~1e-13 (t * 2pi /
    # period a multiple of pi); everywhere else the bf16 values are identical.
    K.time_cond(t=t.cuda(), w_in=None, b_in=None, w_out=None, b_out=None, hidden=hid, cond=cond,
                min_period=4e-3, max_period=4.0)
    torch.cuda.synchronize()
    emb = sinusoid(t, W, 4e-3, 4.0).to(torch.bfloat16)
    got = cond.cpu()
    diff = (got.double() - emb.double()).abs()
    assert diff.max().item() <= 1e-9
    assert (got != emb).sum().item() <= 4
    # full: silu(W_out silu(W_in e + b_in) + b_out), bf16 after each layer
    K.time_cond(t=t.cuda(), w_in=dev(w_in), b_in=dev(b_in), w_out=dev(w_out), b_out=dev(b_out), hidden=hid,
                cond=cond, min_period=4e-3, max_period=4.0)
    torch.cuda.synchronize()
    silu = torch.nn.functional.silu
    h1 = silu((emb.float() @ w_in.t() + b_in).bfloat16().float()).bfloat16()
    ref = silu((h1.float() @ w_out.t() + b_out).bfloat16().float())
    err = (cond.float().cpu() - ref).abs().max().item()
    assert err <= ATOL, err


@pytest.mark.parametrize("mode", ["ssg", "gate"])
def test_modulation_fp32_dense(K, L, mode):
    r = gen(12)
    W, n_rows, n_norms = 1024, 10, 5
    m = L.RFX_ADARMS_SSG if mode == "ssg" else L.RFX_ADARMS_GATE
    out = 3 * W if mode == "ssg" else W
    w = r(n_norms * out, W) * 0.03
    b = r(n_norms * out) * 0.1
    cond = r(n_rows, W).bfloat16()
    a2 = torch.zeros(n_rows, n_norms, W, device="cuda")
    b2 = torch.zeros_like(a2)
    gate = torch.zeros_like(a2)
    K.modulation(mode=m, w=w.cuda(), b=b.cuda(), cond=cond.cuda(), a2=a2, b2=b2, gate=gate, n_norms=n_norms)
    torch.cuda.synchronize()
    dense = (cond.double() @ w.double().t() + b.double()).view(n_rows, n_norms, out)
    if mode == "ssg":
        ref_a2, ref_b2, ref_g = 1 + dense[..., :W], dense[..., W:2 * W], dense[..., 2 * W:]
    else:
        ref_a2, ref_b2, ref_g = dense, torch.zeros_like(dense), dense
    assert (a2.cpu().double() - ref_a2).abs().max().item() <= 1e-4
    assert (b2.cpu().double() - ref_b2).abs().max().item() <= 1e-4
    # the gate is stored bf16-rounded: within half a bf16 ulp (2^-8 relative) plus the fp32 dot-product error
    assert ((gate.cpu().double() - ref_g).abs() <= ref_g.abs() * 2.0 ** -8 + 1e-4).all()
    assert torch.equal(gate.cpu(), gate.cpu().bfloat16().float())
