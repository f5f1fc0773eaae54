"""Policy-level entry points (reflex_b200.policy) and the layer mirrors under
the reference's fusion init, on the GPU, against the reference's own fp32
goldens and the fp32 oracle.

* Fusion init: the reference's init_qkv_fusion_from_existing /
  init_mlp_fusion_from_existing sequence (reflex/policies/pi05/
  modeling_pi05.py:843-866, 883-917: construct QKVLinear / MergedColumnLinear,
  .to(device, dtype), copy the projections into row slices under no_grad,
  drop the originals) run on the rfx mirrors; the fused state dict then
  drives the engine, whose step-0 hidden states and actions match the
  golden 2-layer PI0.5 chunk (hidden 2e-2 * max(1, |h|max), actions 2e-2).
* PI05Model.sample_actions / denoise_step and PI0Model.sample_actions with
  the prefix already in the rings (the reference's cached-prefix decode).
* PI05Model with prefix-layer weights: instruction and frame embeddings
  through the prefix layers into the rings, then the chunk, against the
  oracle run stage by stage over the same quantized context.
* PI05Policy.select_action's action queue.
"""
import os

import numpy as np
import pytest
import torch
from torch import nn

from oracle import quant as oq
from oracle.model import Context, denoise_step, prefix_frame, sample_chunk
from reflex_b200 import synthetic
from reflex_b200.config import pi0_config, pi05_config, vlm_config

from test_gpu_model import GOLD, TOL, hidden_tol, make_case, report, write_ring

pytestmark = pytest.mark.gpu


def _fuse_like_reference(wts, cfg):
    """The fusion init of modeling_pi05.py:843-866 / 883-917 on separate
    nn.Linear projections, with the rfx mirrors as QKVLinear /
    MergedColumnLinear; returns the state dict the fused layers leave."""
    from reflex_b200.layers import MergedColumnLinear, QKVLinear
    W, H, D, F = cfg.width, cfg.num_heads, cfg.head_dim, cfg.mlp_dim
    sd = {k: v for k, v in wts.items() if not any(s in k for s in ("q_proj", "k_proj", "v_proj", "gate_proj",
                                                                    "up_proj"))}
    for l in range(cfg.num_layers):
        p = f"layers.{l}."
        attn = nn.Module()
        for n, rows in (("q_proj", H * D), ("k_proj", D), ("v_proj", D)):
            lin = nn.Linear(W, rows, bias=False).to(device="cuda", dtype=torch.bfloat16)
            with torch.no_grad():
                lin.weight.copy_(wts[p + n + ".weight"])
            setattr(attn, n, lin)
        qkv = QKVLinear(hidden_size=W, head_size=D, total_num_heads=H, total_num_kv_heads=1,
                        bias=attn.q_proj.bias is not None)
        attn.qkv_proj = qkv
        qkv.to(device=attn.q_proj.weight.device, dtype=attn.q_proj.weight.dtype)
        with torch.no_grad():
            out_w = qkv.weight
            q_span, kv_span = H * D, D
            out_w[:q_span].copy_(attn.q_proj.weight)
            out_w[q_span:q_span + kv_span].copy_(attn.k_proj.weight)
            out_w[q_span + kv_span:].copy_(attn.v_proj.weight)
        for n in ("q_proj", "k_proj", "v_proj"):
            delattr(attn, n)
        mlp = nn.Module()
        mlp.gate_proj = nn.Linear(W, F, bias=False).to(device="cuda", dtype=torch.bfloat16)
        mlp.up_proj = nn.Linear(W, F, bias=False).to(device="cuda", dtype=torch.bfloat16)
        with torch.no_grad():
            mlp.gate_proj.weight.copy_(wts[p + "gate_proj.weight"])
            mlp.up_proj.weight.copy_(wts[p + "up_proj.weight"])
        gate_up = MergedColumnLinear(W, [F, F], bias=False)
        mlp.gate_up_proj = gate_up
        gate_up.to(device=mlp.gate_proj.weight.device, dtype=mlp.gate_proj.weight.dtype)
        with torch.no_grad():
            gate_up.weight[:F].copy_(mlp.gate_proj.weight)
            gate_up.weight[F:].copy_(mlp.up_proj.weight)
        delattr(mlp, "gate_proj")
        delattr(mlp, "up_proj")
        sd[p + "qkv_proj.weight"] = attn.qkv_proj.state_dict()["weight"]
        sd[p + "gate_up_proj.weight"] = mlp.gate_up_proj.state_dict()["weight"]
    return sd


def test_fusion_init_on_mirrors_gives_golden_layers():
    from reflex_b200.expert import ActionExpertEngine
    g = np.load(os.path.join(GOLD, "model_pi05_l2.npz"))
    nl, n_ctx = int(g["num_layers"]), int(g["n_ctx"])
    cfg = pi05_config(num_layers=nl, adarms="gate", quant_mode="u8_ref")
    wts, ctx, parts, x0, st = make_case(cfg, n_ctx)
    sd = _fuse_like_reference(wts, cfg)
    assert not any("q_proj" in k or "gate_proj" in k for k in sd)
    eng = ActionExpertEngine(cfg, sd, capacity=256, n_ctx=n_ctx, scale_dtype=torch.float32)
    for l, p in enumerate(parts):
        write_ring(eng.rings[l], *p)
    eng.set_inputs(x0.cuda())
    hid = []
    eng.run_eager(lambda tag: hid.append(eng.h.view(1, eng.St, -1).float().cpu())
                  if tag[0] == "layer" and tag[1] == 0 else None)
    torch.cuda.synchronize()
    ref_h = [torch.from_numpy(h) for h in g["hidden_step0"]]
    report("fusion-init", ref_h, hid)
    for l in range(nl):
        assert (hid[l] - ref_h[l]).abs().max().item() <= hidden_tol(ref_h[l])
    err = (eng.x.float().cpu() - torch.from_numpy(g["actions"])).abs().max().item()
    print(f"fusion-init actions maxerr vs reference fp32: {err:.5f}")
    assert err <= TOL


def _model_with_cached_prefix(cfg, n_ctx, cls):
    wts, ctx, parts, x0, st = make_case(cfg, n_ctx)
    m = cls(cfg, wts, n_lang=n_ctx, capacity=256)
    for l, p in enumerate(parts):
        write_ring(m.engine.rings[l], *p)
    m.set_prefix(n_ctx, instruction=True, frames=0)
    return m, wts, ctx, x0, st


@pytest.mark.parametrize("name", ["model_pi05_l2.npz", "model_pi0_l2.npz"])
def test_sample_actions_over_cached_prefix_matches_golden(name):
    from reflex_b200.policy import PI0Model, PI05Model
    g = np.load(os.path.join(GOLD, name))
    nl, n_ctx = int(g["num_layers"]), int(g["n_ctx"])
    if str(g["variant"]) == "pi05":
        cfg, cls = pi05_config(num_layers=nl, adarms="gate", quant_mode="u8_ref"), PI05Model
    else:
        cfg, cls = pi0_config(num_layers=nl, quant_mode="u8_ref"), PI0Model
    m, wts, ctx, x0, st = _model_with_cached_prefix(cfg, n_ctx, cls)
    for _ in range(2):  # the second call replays the same chunk
        a = m.sample_actions(None, None, None, None, st.cuda(), noise=x0.cuda())
        torch.cuda.synchronize()
        err = (a.float().cpu() - torch.from_numpy(g["actions"])).abs().max().item()
        print(f"{name} sample_actions maxerr vs reference fp32: {err:.5f}")
        assert err <= TOL


def test_denoise_step_matches_oracle_velocity():
    from reflex_b200.policy import PI05Model
    cfg = pi05_config(num_layers=2, adarms="gate", quant_mode="u8_ref")
    n_ctx = 128
    m, wts, ctx, x0, st = _model_with_cached_prefix(cfg, n_ctx, PI05Model)
    table = synthetic.rope_table(cfg.max_position_embeddings, cfg.head_dim, cfg.rope_theta)
    pad = torch.ones(1, n_ctx, dtype=torch.bool)
    for t in (1.0, 0.35):
        v = m.denoise_step(pad.cuda(), torch.zeros(1, n_ctx).cuda(), st.cuda(), x0.cuda(),
                           torch.tensor([t]).cuda())
        with torch.no_grad():
            v_ref = denoise_step(cfg, wts, ctx, st, x0, torch.tensor([t]), table)
        err = (v.float().cpu() - v_ref).abs().max().item()
        print(f"denoise_step t={t}: v maxerr vs fp32 oracle {err:.5f}")
        assert err <= TOL
    # a padded prefix token: the suffix must not see it
    pad[0, 5] = False
    v = m.denoise_step(pad.cuda(), torch.zeros(1, n_ctx).cuda(), st.cuda(), x0.cuda(), torch.tensor([1.0]).cuda())
    with torch.no_grad():
        v_ref = denoise_step(cfg, wts, Context(ctx.k, ctx.v, pad), st, x0, torch.tensor([1.0]), table)
    assert (v.float().cpu() - v_ref).abs().max().item() <= TOL


def test_streaming_prefill_then_chunk_matches_oracle():
    """Instruction (16 tokens) and two frames (64 tokens each, window 2)
    through 2 prefix layers into the rings, then a 2-layer PI0.5 chunk."""
    from reflex_b200.policy import PI05Model
    cfg = pi05_config(num_layers=2, adarms="gate", quant_mode="i8_sym")
    vcfg = vlm_config(num_layers=2)
    n_lang, flen, win = 16, 64, 2
    wts = synthetic.expert_weights(cfg, seed=0)
    pw = synthetic.prefix_weights(vcfg, seed=10)
    m = PI05Model(cfg, wts, prefix_cfg=vcfg, prefix_weights=pw, n_lang=n_lang, frame_len=flen, window_frames=win)
    lang = synthetic.frame_embeddings(vcfg, n_lang, seed=21)
    frames = [synthetic.frame_embeddings(vcfg, flen, seed=22 + i) for i in range(3)]
    x0 = synthetic.noise(cfg, seed=2)
    a = m.sample_actions(frames[0].cuda(), None, lang.cuda(), None, None, noise=x0.cuda())
    for f in frames[1:]:  # the third frame evicts the first
        a = m.sample_actions(f.cuda(), None, None, None, None, noise=x0.cuda(), incremental_input=True)
    torch.cuda.synchronize()
    assert m.prefix_length == n_lang + win * flen
    # oracle over the context the rings hold (dequantized): the chunk
    rings = m.engine.rings
    n = m.prefix_length
    kd = [torch.from_numpy(oq.dequant_i8_sym(r.k_q[:, :, :n].cpu().numpy(), r.k_scale[:, :, :n, None].cpu().numpy()))
          for r in rings]
    vd = [torch.from_numpy(oq.dequant_i8_sym(r.v_q[:, :, :n].cpu().numpy(), r.v_scale[:, :, :n, None].cpu().numpy()))
          for r in rings]
    with torch.no_grad():
        x_ref = sample_chunk(cfg, wts, Context(kd, vd, torch.ones(1, n, dtype=torch.bool)), x0)
    err = (a.float().cpu() - x_ref).abs().max().item()
    print(f"streaming prefill + chunk: actions maxerr vs fp32 oracle {err:.5f}")
    assert err <= TOL
    # the ring holds the instruction's and the newest frames' K/V: check the
    # last frame (slot 0 after three frames) against the oracle's frame pass
    # over the instruction and the second frame
    with torch.no_grad():
        ctx = Context([k[:, :, :n_lang + 2 * flen] for k in kd], [v[:, :, :n_lang + 2 * flen] for v in vd],
                      torch.ones(1, n_lang + 2 * flen, dtype=torch.bool))
        keep = torch.cat([torch.arange(n_lang), torch.arange(n_lang + flen, n_lang + 2 * flen)])
        ctx = Context([k[:, :, keep] for k in ctx.k], [v[:, :, keep] for v in ctx.v],
                      torch.ones(1, n_lang + flen, dtype=torch.bool))
        pos = (n_lang + flen + torch.arange(flen))[None]
        _, kvs = prefix_frame(vcfg, pw, frames[2].float(), ctx, pos)
    for l in range(vcfg.num_layers):
        got = kd[l][:, :, n_lang:n_lang + flen]
        ref = kvs[l][0]
        assert (got - ref).abs().max().item() <= 2e-2 * max(1.0, ref.abs().max().item()) + \
            ref.abs().amax().item() / 127


def test_select_action_queue():
    from reflex_b200.policy import PI05Model, PI05Policy
    cfg = pi05_config(num_layers=1, adarms="gate", quant_mode="u8_ref", chunk_size=8)
    m, wts, ctx, x0, st = _model_with_cached_prefix(cfg, 64, PI05Model)
    pol = PI05Policy(m, n_action_steps=5, action_dim=7)
    x0 = x0.cuda()
    chunk = pol.predict_action_chunk({}, noise=x0)
    assert chunk.shape == (1, 5, 7)
    acts = [pol.select_action({}, noise=x0) for _ in range(6)]
    assert all(a.shape == (1, 7) for a in acts)
    for i in range(5):  # the first five come from one chunk, the sixth from a new one
        assert torch.equal(acts[i], chunk[:, i])
    assert torch.equal(acts[5], chunk[:, 0])
    pol.reset()
    assert len(pol._action_queue) == 0


def test_sample_actions_from_camera_images():
    """Camera images through the model's vision tower (SigLIP + projector,
    2 layers at full widths) give the same actions as passing that tower's
    image tokens (the path the other tests check against the oracle), with
    the cameras' tokens concatenated in camera order."""
    from reflex_b200.config import VisionConfig
    from reflex_b200.policy import PI05Model
    from reflex_b200.vision import VisionTower
    cfg = pi05_config(num_layers=2, adarms="gate", quant_mode="i8_sym")
    vcfg = vlm_config(num_layers=2)
    viscfg = VisionConfig(num_layers=2)
    tower = VisionTower(viscfg, synthetic.vision_weights(viscfg, seed=40), max_images=2)
    n_lang, ncam = 16, 2
    wts = synthetic.expert_weights(cfg, seed=0)
    pw = synthetic.prefix_weights(vcfg, seed=10)
    kw = dict(prefix_cfg=vcfg, prefix_weights=pw, n_lang=n_lang, frame_len=ncam * viscfg.tokens, window_frames=2)
    with_tower = PI05Model(cfg, wts, vision=tower, **kw)
    plain = PI05Model(cfg, wts, **kw)
    lang = synthetic.frame_embeddings(vcfg, n_lang, seed=21).cuda()
    cams = [synthetic.images(viscfg, B=1, seed=50 + i) for i in range(ncam)]
    x0 = synthetic.noise(cfg, seed=2).cuda()
    a1 = with_tower.sample_actions([c.cuda() for c in cams], None, lang, None, None, noise=x0).clone()
    tokens = tower.get_image_features(torch.cat(cams).cuda()).reshape(1, ncam * viscfg.tokens, -1).clone()
    a2 = plain.sample_actions(tokens, None, lang, None, None, noise=x0)
    torch.cuda.synchronize()
    assert torch.equal(a1, a2)
    with pytest.raises(ValueError):
        plain.sample_actions(torch.stack(cams, 1).cuda(), None, None, None, None, noise=x0, incremental_input=True)
