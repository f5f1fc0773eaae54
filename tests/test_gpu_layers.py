"""The Reflex layer mirrors through the C ABI against the oracle.

StreamingAttention: prefill (main and pending), commit, eviction, merge of a
source slice and decode with a block-causal suffix mask, against fp32
attention over the dequantized source (max abs error <= 2e-2, the bf16
attention tolerance).  fused_quantize_store: bit-exact against the oracle's
restatement of the reference quantizer.  QKVLinear / MergedColumnLinear:
against the fp32 product of the same bf16 operands (1e-2 abs + 1e-2 rel).
"""
import numpy as np
import pytest
import torch

from oracle import quant as oq
from oracle.attention import partitioned_attention

pytestmark = pytest.mark.gpu


def gen(seed):
    g = torch.Generator().manual_seed(seed)
    return lambda *s: torch.randn(*s, generator=g)


def _dequant(a):
    """The source tokens [0, source_length) in logical order, dequantized (fp32)."""
    r = a.ring
    sl = a.source_slots(0, a.source_length).to(r.k_q.device)
    g = lambda t: t[:, :, sl]  # noqa: E731
    if r.k_zp is None:  # int8 symmetric
        kd = oq.dequant_i8_sym(g(r.k_q).cpu().numpy(), g(r.k_scale)[..., None].cpu().numpy())
        vd = oq.dequant_i8_sym(g(r.v_q).cpu().numpy(), g(r.v_scale)[..., None].cpu().numpy())
        return torch.from_numpy(kd), torch.from_numpy(vd)
    kd = oq.dequant_u8_ref(g(r.k_q).cpu().numpy(), g(r.k_scale)[..., None].float().cpu().numpy(),
                           g(r.k_zp)[..., None].float().cpu().numpy(), True)
    vd = oq.dequant_u8_ref(g(r.v_q).cpu().numpy(), g(r.v_scale)[..., None].float().cpu().numpy(),
                           g(r.v_zp)[..., None].float().cpu().numpy(), True)
    return torch.from_numpy(kd), torch.from_numpy(vd)


def test_fused_quantize_store_bit_exact():
    from reflex_b200.layers import fused_quantize_store
    r = gen(1)
    B, H, Ln, D, cap = 2, 1, 37, 256, 96
    x = (r(B, H, Ln, D) * 2).bfloat16()
    cache = torch.zeros(B, H, cap, D, dtype=torch.uint8, device="cuda")
    scale = torch.zeros(B, H, cap, 1, dtype=torch.bfloat16, device="cuda")
    zp = torch.zeros_like(scale)
    fused_quantize_store(x.cuda(), cache, scale, zp, cache_start_idx=11)
    torch.cuda.synchronize()
    q, s, z = oq.quant_u8_ref(x.float().numpy(), True)
    assert np.array_equal(cache[:, :, 11:11 + Ln].cpu().numpy(), q)
    assert np.array_equal(scale[:, :, 11:11 + Ln].float().cpu().numpy(), s)
    assert np.array_equal(zp[:, :, 11:11 + Ln].float().cpu().numpy(), z)
    assert int(cache[:, :, :11].abs().sum()) == 0


@pytest.mark.parametrize("masked,quantize", [(False, True), (True, True), (True, False)])
def test_streaming_attention_lifecycle(masked, quantize):
    """quantize=True: the reference's uint8 source cache; quantize=False (the
    reference's default): the source kept as int8 with per-token scales."""
    from reflex_b200.layers import StreamingAttention
    r = gen(2)
    B, Hq, D, S = 2, 8, 256, 51
    a = StreamingAttention(D ** -0.5, max_cache_size=1024, quantize_kv_cache=quantize)
    k1, v1 = r(B, 1, 300, D).bfloat16(), r(B, 1, 300, D).bfloat16()
    k2, v2 = r(B, 1, 200, D).bfloat16(), r(B, 1, 200, D).bfloat16()
    a.prefill_source(k1.cuda(), v1.cuda())
    a.prefill_source(k2.cuda(), v2.cuda(), cache_slot="pending")
    assert a.source_length == 300
    a.commit_pending_source()
    assert a.source_length == 500
    a.evict_source_prefix(120)
    assert a.source_length == 380
    q = r(B, Hq, S, D).bfloat16()
    ks, vs = r(B, 1, S, D).bfloat16(), r(B, 1, S, D).bfloat16()
    blocks = torch.zeros(S, dtype=torch.int64)
    blocks[1:] = 1 if masked else 0
    start = 40  # decode attends to the source slice [40, 380)
    mask = None
    if masked:
        n_src = 380 - start
        suf = blocks[None, :] <= blocks[:, None]
        m = torch.cat([torch.ones(S, n_src, dtype=torch.bool), suf], dim=1)
        m[:, 7] = False  # one padded source token
        mask = m[None, None].expand(B, 1, -1, -1).contiguous().cuda()
    out = a.forward(q.cuda(), ks.cuda(), vs.cuda(), attention_mask=mask, merge_before_decode=True,
                    source_slice_start=start)
    torch.cuda.synchronize()
    kd, vd = _dequant(a)
    kd, vd = kd[:, :, start:], vd[:, :, start:]
    pad = torch.ones(B, kd.shape[2], dtype=torch.bool)
    if masked:
        pad[:, 7] = False
    att = torch.zeros(S, dtype=torch.int64)
    att[0] = 1
    if masked:
        att[1] = 1
    ref = partitioned_attention(q.float(), kd, vd, ks.float(), vs.float(), pad, att, D ** -0.5)
    err = (out.float().cpu() - ref).abs().max().item()
    assert err <= 2e-2, err
    # the surviving source tokens keep their quantized values after the eviction
    kd_all, _ = _dequant(a)
    both = torch.cat([k1, k2], 2).float().numpy()
    if quantize:
        k_ref = oq.dequant_u8_ref(*oq.quant_u8_ref(both, True), True)
    else:
        k_ref = oq.dequant_i8_sym(*oq.quant_i8_sym(both))
        # against the unquantized source: int8 keys / values cost at most absmax / 254 per value
        ref_exact = partitioned_attention(q.float(), torch.cat([k1, k2], 2)[:, :, 120 + start:500].float(),
                                          torch.cat([v1, v2], 2)[:, :, 120 + start:500].float(), ks.float(),
                                          vs.float(), pad, att, D ** -0.5)
        assert (out.float().cpu() - ref_exact).abs().max().item() <= 5e-2
    assert np.array_equal(kd_all.numpy(), k_ref[:, :, 120:500])
    # the same mask object again: its structure comes from the cache
    if masked:
        hits = a.cache_stats["mask_cache_hits"]
        out2 = a.forward(q.cuda(), ks.cuda(), vs.cuda(), attention_mask=mask)
        assert a.cache_stats["mask_cache_hits"] == hits + 1
        assert torch.equal(out2, out)


def test_streaming_attention_wrapping_ring():
    """Appends after evictions wrap around the ring; decode over the wrapped
    source matches attention over the logical source order."""
    from reflex_b200.layers import StreamingAttention
    r = gen(4)
    B, Hq, D, S, cap = 1, 8, 256, 50, 512
    a = StreamingAttention(D ** -0.5, max_cache_size=cap)
    ks_all, vs_all = [], []
    for _ in range(4):  # four frames of 200 tokens, keeping the last two
        k, v = r(B, 1, 200, D).bfloat16(), r(B, 1, 200, D).bfloat16()
        if a.source_length + 200 > cap:
            a.evict_source_prefix(200)
            ks_all, vs_all = ks_all[1:], vs_all[1:]
        a.prefill_source(k.cuda(), v.cuda())
        ks_all.append(k)
        vs_all.append(v)
    assert a.source_length == 400 and a._head == 400  # slots 400..511 then 0..287
    a.merge_caches()
    q = r(B, Hq, S, D).bfloat16()
    kn, vn = r(B, 1, S, D).bfloat16(), r(B, 1, S, D).bfloat16()
    out = a.forward(q.cuda(), kn.cuda(), vn.cuda())
    torch.cuda.synchronize()
    kd, vd = _dequant(a)
    src = torch.cat(ks_all, 2).float().numpy()
    assert np.array_equal(kd.numpy(), oq.dequant_i8_sym(*oq.quant_i8_sym(src)))
    att = torch.zeros(S, dtype=torch.int64)
    att[0] = 1
    ref = partitioned_attention(q.float(), kd, vd, kn.float(), vn.float(), torch.ones(B, 400, dtype=torch.bool),
                                att, D ** -0.5)
    assert (out.float().cpu() - ref).abs().max().item() <= 2e-2


def test_qkv_and_merged_linear():
    from reflex_b200.layers import MergedColumnLinear, QKVLinear
    r = gen(3)
    B, Lx, Hd = 2, 50, 1024
    x = (r(B, Lx, Hd)).bfloat16()
    qkv = QKVLinear(Hd, 256, 8, 1).to(device="cuda", dtype=torch.bfloat16)
    with torch.no_grad():
        qkv.weight.copy_((r(*qkv.weight.shape) * 0.03).bfloat16())
    q, k, v = qkv.forward(x.cuda())
    y = x.float().reshape(-1, Hd) @ qkv.weight.float().cpu().t()
    ref_q = y[:, :2048].view(B, Lx, 8, 256).transpose(1, 2)
    ref_k = y[:, 2048:2304].view(B, Lx, 1, 256).transpose(1, 2)
    ref_v = y[:, 2304:].view(B, Lx, 1, 256).transpose(1, 2)
    for got, ref in ((q, ref_q), (k, ref_k), (v, ref_v)):
        assert got.shape == ref.shape
        assert torch.allclose(got.float().cpu(), ref, atol=1e-2, rtol=1e-2)
    mc = MergedColumnLinear(Hd, [4096, 4096], bias=True).to(device="cuda", dtype=torch.bfloat16)
    with torch.no_grad():
        mc.weight.copy_((r(*mc.weight.shape) * 0.03).bfloat16())
        mc.bias.copy_(r(8192) * 0.1)
    g, u = mc.forward(x.cuda())
    y = x.float().reshape(-1, Hd) @ mc.weight.float().cpu().t() + mc.bias.float().cpu()
    assert g.shape == (B, Lx, 4096) and u.shape == (B, Lx, 4096)
    assert torch.allclose(g.float().cpu().reshape(-1, 4096), y[:, :4096], atol=1e-2, rtol=1e-2)
    assert torch.allclose(u.float().cpu().reshape(-1, 4096), y[:, 4096:], atol=1e-2, rtol=1e-2)
