"""CPU: the oracle against the golden vectors produced by the reference's own code.

The uint8 quantizer must match bit for bit; attention, per-layer hidden states
and action chunks within fp32 rounding (atol 1e-4, the reference and the
oracle differ only in summation order).
"""
import hashlib
import os

import numpy as np
import pytest
import torch

from oracle import quant as oq
from oracle.attention import block_mask, partitioned_attention
from oracle.bf16 import bf16_round
from oracle.model import Context, sample_chunk
from reflex_b200 import synthetic
from reflex_b200.config import pi0_config, pi05_config

GOLD = os.path.join(os.path.dirname(__file__), "golden")
FP32_ATOL = 1e-4


def sha(*ts):
    h = hashlib.sha256()
    for t in ts:
        h.update(np.ascontiguousarray(t.detach().cpu().float().numpy()).tobytes())
    return h.hexdigest()


def load(name):
    return np.load(os.path.join(GOLD, name), allow_pickle=False)


def edge_rows(D=256):
    rows = [np.zeros(D), np.full(D, 3.25), np.linspace(-1e-6, 1e-6, D), -np.abs(np.linspace(0.1, 7, D)),
            np.linspace(-2.5, 2.5, D), np.r_[np.full(D - 1, 0.5), 127.0], np.r_[np.full(D - 1, -1.0), 1e4],
            np.linspace(0, 255, D), np.r_[np.full(D // 2, 1e-3), np.full(D // 2, -1e-3)]]
    return np.stack(rows).astype(np.float32)


def quant_inputs():
    g = torch.Generator().manual_seed(11)
    x = torch.randn(1, 1, 300, 256, generator=g) * torch.rand(1, 1, 300, 1, generator=g) * 8
    x[0, 0, :9] = torch.from_numpy(edge_rows())
    return x


# ------------------------------------------------------------- quantizers ---
@pytest.mark.parametrize("name,dtype", [("f32", torch.float32), ("bf16", torch.bfloat16)])
def test_u8_ref_quantizer_bit_exact(name, dtype):
    g = load("quant_u8_ref.npz")
    x = quant_inputs()
    assert sha(x) == str(g["x_sha"])
    xi = x.to(dtype).float().numpy()
    q, s, z = oq.quant_u8_ref(xi, act_bf16=dtype == torch.bfloat16)
    np.testing.assert_array_equal(q, g[f"q_{name}"])
    np.testing.assert_array_equal(s, g[f"scale_{name}"])
    np.testing.assert_array_equal(z, g[f"zp_{name}"])
    deq = oq.dequant_u8_ref(q, s, z, act_bf16=dtype == torch.bfloat16)
    np.testing.assert_array_equal(deq[:, :, :16], g[f"deq16_{name}"])


def test_i8_sym_known_answers():
    # hand-derived from scale = absmax / 127, q = rne(x / scale)
    x = np.zeros((4, 256), np.float32)
    x[0, :4] = [127.0, -63.5, 0.5, 1.5]          # scale 1: rne(0.5)=0, rne(1.5)=2, rne(-63.5)=-64
    x[1, :3] = [2.54, -1.27, 0.01]              # scale 0.02: 127, -63.5 -> -64 (ties to even), 0.5 -> 0
    x[3, :] = -3.0                              # constant row: every value -> -127
    q, s = oq.quant_i8_sym(x)
    assert s[0, 0] == np.float32(1.0) and list(q[0, :4]) == [127, -64, 0, 2]
    assert s[1, 0] == np.float32(2.54) / np.float32(127.0)
    assert q[1, 0] == 127 and q[1, 1] == np.int8(np.rint(np.float32(-1.27) / s[1, 0])) and q[1, 2] == np.int8(
        np.rint(np.float32(0.01) / s[1, 0]))
    assert s[2, 0] == 0 and not q[2].any()      # all-zero row: scale 0, q 0
    assert (q[3] == -127).all()
    # dequantization error is at most half a step
    xs = np.random.default_rng(0).standard_normal((64, 256)).astype(np.float32)
    q, s = oq.quant_i8_sym(xs)
    assert np.abs(oq.dequant_i8_sym(q, s) - xs).max() <= (s.max() * 0.5 + 1e-6)


def test_bf16_rounding_matches_torch():
    x = torch.randn(10000) * torch.logspace(-8, 8, 10000)
    np.testing.assert_array_equal(bf16_round(x.numpy()), x.to(torch.bfloat16).float().numpy())


# -------------------------------------------------------------- attention ---
def c1_inputs():
    g = torch.Generator().manual_seed(7)
    Lc, S, H, D = 576, 50, 8, 256
    q = torch.randn(1, H, Lc + S, D, generator=g)
    k = torch.randn(1, 1, Lc + S, D, generator=g)
    v = torch.randn(1, 1, Lc + S, D, generator=g)
    return q, k, v, Lc, S


def test_attention_c1_full_and_streaming():
    g = load("attention_c1.npz")
    q, k, v, Lc, S = c1_inputs()
    assert sha(q, k, v) == str(g["inputs_sha"])
    assert float(g["stream_vs_full_maxdiff"]) <= 1e-5  # the reference's own streaming == full recompute
    att = torch.zeros(S, dtype=torch.int64)
    att[0] = 1
    pad = torch.ones(1, Lc, dtype=torch.bool)
    out = partitioned_attention(q[:, :, Lc:], k[:, :, :Lc], v[:, :, :Lc], k[:, :, Lc:], v[:, :, Lc:], pad, att, 1 / 16)
    np.testing.assert_allclose(out.numpy(), g["full"], atol=1e-5, rtol=0)
    # uint8 quantized context: the oracle's cache equals the reference's, and so does the output
    kq, ks, kz = oq.quant_u8_ref(k[:, :, :Lc].numpy(), act_bf16=False)
    vq, vs, vz = oq.quant_u8_ref(v[:, :, :Lc].numpy(), act_bf16=False)
    T = torch.from_numpy
    assert sha(T(kq), T(vq), T(ks), T(kz), T(vs), T(vz)) == str(g["cache_sha"])
    kd = T(oq.dequant_u8_ref(kq, ks, kz, False))
    vd = T(oq.dequant_u8_ref(vq, vs, vz, False))
    outq = partitioned_attention(q[:, :, Lc:], kd, vd, k[:, :, Lc:], v[:, :, Lc:], pad, att, 1 / 16)
    np.testing.assert_allclose(outq.numpy(), g["stream_q"], atol=1e-5, rtol=0)


def test_block_mask_rule():
    pad = torch.tensor([[True, True, False, True, True]])
    att = torch.tensor([[0, 0, 0, 1, 1]])
    m = block_mask(pad, att)[0, 0]
    assert m[3, 0] and m[3, 1] and not m[3, 2] and m[3, 3] and not m[3, 4]  # block 1 cannot see block 2
    assert m[4].tolist() == [True, True, False, True, True]
    assert not m[2].any()


# ------------------------------------------------------------------ model ---
def model_case(name):
    g = load(name)
    variant = str(g["variant"])
    nl, Lc, seed = int(g["num_layers"]), int(g["n_ctx"]), int(g["seed"])
    cfg = pi05_config(num_layers=nl, adarms="gate") if variant == "pi05" else pi0_config(num_layers=nl)
    wts = synthetic.expert_weights(cfg, seed=seed)
    assert sha(*[wts[k] for k in sorted(wts)]) == str(g["weights_sha"])
    ks, vs = synthetic.context_kv(cfg, Lc, seed=seed + 1)
    x0 = synthetic.noise(cfg, seed=seed + 2)
    st = synthetic.state(cfg, seed=seed + 3)
    assert sha(*ks, *vs, x0, st) == str(g["inputs_sha"])
    T = torch.from_numpy
    kd, vd, parts = [], [], []
    for l in range(nl):
        kq, kS, kz = oq.quant_u8_ref(ks[l].numpy(), False)
        vq, vS, vz = oq.quant_u8_ref(vs[l].numpy(), False)
        parts += [T(kq), T(kS), T(kz), T(vq), T(vS), T(vz)]
        kd.append(T(oq.dequant_u8_ref(kq, kS, kz, False)))
        vd.append(T(oq.dequant_u8_ref(vq, vS, vz, False)))
    assert sha(*parts) == str(g["ctx_sha"])
    ctx = Context(kd, vd, torch.ones(1, Lc, dtype=torch.bool))
    return g, cfg, wts, ctx, x0, st


@pytest.mark.parametrize("name", ["model_pi05_l2.npz", "model_pi0_l2.npz"])
def test_model_small_matches_reference(name):
    g, cfg, wts, ctx, x0, st = model_case(name)
    hidden = []
    with torch.no_grad():
        x = sample_chunk(cfg, wts, ctx, x0, st, hidden_step0=hidden)
    for l, h in enumerate(hidden):
        np.testing.assert_allclose(h.numpy(), g["hidden_step0"][l], atol=FP32_ATOL, rtol=0, err_msg=f"layer {l}")
    np.testing.assert_allclose(x.numpy(), g["actions"], atol=FP32_ATOL, rtol=0)


def test_model_18_layers_matches_reference():
    g, cfg, wts, ctx, x0, st = model_case("model_pi05_l18.npz")
    torch.set_num_threads(os.cpu_count() or 1)
    hidden = []
    with torch.no_grad():
        x = sample_chunk(cfg, wts, ctx, x0, st, hidden_step0=hidden)
    np.testing.assert_allclose([h.abs().max().item() for h in hidden], g["hidden_step0_absmax"], rtol=1e-4)
    np.testing.assert_allclose([h.norm().item() for h in hidden], g["hidden_step0_l2"], rtol=1e-4)
    np.testing.assert_allclose(x.numpy(), g["actions"], atol=FP32_ATOL, rtol=0)


def test_vision_tower_matches_transformers_siglip():
    """The SigLIP tower + projector restatement against the installed
    transformers' SiglipVisionModel / PaliGemmaMultiModalProjector (2 layers at
    full widths, seeded weights and image; tests/golden/make_golden_vision.py)."""
    from oracle import vision as ov
    from reflex_b200.config import VisionConfig

    g = np.load(os.path.join(GOLD, "vision_l2.npz"))
    cfg = VisionConfig(num_layers=int(g["layers"]))
    w = synthetic.vision_weights(cfg, seed=int(g["w_seed"]))
    img = synthetic.images(cfg, B=1, seed=int(g["img_seed"]))
    assert sha(*([w[k] for k in sorted(w)] + [img])) == str(g["inputs_sha"])
    with torch.no_grad():
        out, hid = ov.image_features(cfg, w, img, return_hidden=True)
    assert (hid[0, :64] - torch.from_numpy(g["hidden64"])).abs().max().item() < FP32_ATOL
    assert (out[0, :64] - torch.from_numpy(g["tokens64"])).abs().max().item() < FP32_ATOL
    assert (out[0].norm(dim=-1) - torch.from_numpy(g["tok_norm"])).abs().max().item() < 1e-3
    assert (out[0].mean(-1) - torch.from_numpy(g["tok_mean"])).abs().max().item() < FP32_ATOL


def test_vision_patch_rows_are_the_convolution():
    """The patch rows the CUDA path feeds to its GEMM, times the reshaped
    convolution weight, equal the stride-14 14 x 14 convolution itself (the
    order of pixels within a row matches the weight's (channel, y, x) order)."""
    from oracle import vision as ov
    from reflex_b200.config import VisionConfig

    cfg = VisionConfig(num_layers=1, image=56)
    w = synthetic.vision_weights(cfg, seed=3)
    img = synthetic.images(cfg, B=2, seed=4)
    pw = w["vision_model.embeddings.patch_embedding.weight"]
    conv = torch.nn.functional.conv2d(img, pw, w["vision_model.embeddings.patch_embedding.bias"], stride=cfg.patch)
    ref = conv.flatten(2).transpose(1, 2)
    got = ov.patches(cfg, img) @ pw.reshape(cfg.width, -1).T + w["vision_model.embeddings.patch_embedding.bias"]
    assert (got - ref).abs().max().item() < 1e-4
