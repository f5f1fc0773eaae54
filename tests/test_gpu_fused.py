"""The persistent chunk executor (rfx_chunk) against the fp32 oracle and the
per-op engine, through the C ABI.

Tolerances are those of the per-op engine: denoised actions within max abs
2e-2 of the fp32 path.  Split GEMM partials are summed in a fixed order, so
replays of the same chunk are bit-identical.
"""
import os

import numpy as np
import pytest
import torch

from oracle.model import sample_chunk
from reflex_b200 import kernels
from reflex_b200.config import pi0_config, pi05_config

from test_gpu_model import GOLD, TOL, hidden_tol, make_case, make_engine, report

pytestmark = pytest.mark.gpu


def run_chunk(eng, x0, st=None):
    eng.set_inputs(x0.cuda(), None if st is None else st.cuda())
    eng.run_eager()
    torch.cuda.synchronize()
    assert kernels.device_status() == 0
    return eng.x.float().cpu()


@pytest.mark.parametrize("adarms,quant,n_ctx", [("gate", "u8_ref", 200), ("ssg", "i8_sym", 300), ("ssg", "i8_sym", 0)])
def test_fused_small_matches_oracle_and_per_op_engine(adarms, quant, n_ctx):
    cfg = pi05_config(num_layers=2, adarms=adarms, quant_mode=quant)
    wts, ctx, parts, x0, st = make_case(cfg, n_ctx)
    fused = make_engine(cfg, wts, parts, n_ctx, fused=True)
    xf = run_chunk(fused, x0)
    per_op = make_engine(cfg, wts, parts, n_ctx)
    xp = run_chunk(per_op, x0)
    with torch.no_grad():
        x32 = sample_chunk(cfg, wts, ctx, x0, st)
    e_oracle = (xf - x32).abs().max().item()
    e_per_op = (xf - xp).abs().max().item()
    print(f"fused {adarms}/{quant}/{n_ctx}: vs fp32 oracle {e_oracle:.5f}, vs per-op engine {e_per_op:.5f}")
    assert e_oracle <= TOL
    assert e_per_op <= TOL


def test_fused_c2_full_size():
    """18 layers, 818-token int8 context, scale/shift/gate adaRMS (the benchmark workload)."""
    cfg = pi05_config(adarms="ssg", quant_mode="i8_sym")
    n_ctx = 818
    wts, ctx, parts, x0, st = make_case(cfg, n_ctx)
    eng = make_engine(cfg, wts, parts, n_ctx, capacity=1024, fused=True)
    xf = run_chunk(eng, x0)
    torch.set_num_threads(os.cpu_count() or 1)
    with torch.no_grad():
        x32 = sample_chunk(cfg, wts, ctx, x0, st)
    err = (xf - x32).abs().max().item()
    print(f"fused c2: actions maxerr vs fp32 oracle {err:.5f}")
    assert err <= TOL


@pytest.mark.parametrize("adarms,quant", [("gate", "u8_ref"), ("ssg", "i8_sym")])
def test_fused_c2_full_size_per_layer(adarms, quant):
    """18 layers, 818-token context through the persistent executor, with the
    first step's hidden states and attention outputs of every layer checked
    against the fp32 oracle (gate / u8_ref is the variant the reference's
    own goldens pin; ssg / i8_sym is the benchmark's)."""
    cfg = pi05_config(adarms=adarms, quant_mode=quant)
    n_ctx = 818
    wts, ctx, parts, x0, st = make_case(cfg, n_ctx)
    eng = make_engine(cfg, wts, parts, n_ctx, capacity=1024, fused=True)
    eng.enable_chunk_debug()
    xf = run_chunk(eng, x0)
    torch.set_num_threads(os.cpu_count() or 1)
    h32, trace = [], {}
    with torch.no_grad():
        x32 = sample_chunk(cfg, wts, ctx, x0, st, hidden_step0=h32, trace_step0=trace)
    hid = [eng.dbg_h[l].view(1, eng.St, -1).float().cpu() for l in range(cfg.num_layers)]
    att = [eng.dbg_attn[l].view(1, eng.St, -1).float().cpu() for l in range(cfg.num_layers)]
    report(f"fused-c2-{adarms}-{quant}", h32, hid, trace["attn"], att)
    for l in range(cfg.num_layers):
        assert (hid[l] - h32[l]).abs().max().item() <= hidden_tol(h32[l]), f"layer {l}"
        assert (att[l] - trace["attn"][l]).abs().max().item() <= TOL, f"layer {l}"
    err = (xf - x32).abs().max().item()
    print(f"fused c2 {adarms}/{quant}: actions maxerr vs fp32 oracle {err:.5f}")
    assert err <= TOL


def test_fused_graph_replay_is_deterministic():
    cfg = pi05_config(num_layers=4)
    wts, ctx, parts, x0, st = make_case(cfg, 300)
    eng = make_engine(cfg, wts, parts, 300, fused=True)
    ref = run_chunk(eng, x0)
    eng.capture()
    for _ in range(3):
        eng.set_inputs(x0.cuda())
        eng.launch_chunk()
        torch.cuda.synchronize()
        assert torch.equal(eng.x.float().cpu(), ref)
    assert kernels.device_status() == 0


def test_dependency_wait_timeout_aborts_cleanly_and_next_chunk_runs():
    """A wait on another CTA's phase counter that runs out: with the bound
    cut to 2 us (every chunk has waits far longer than that), the executor
    records the timeout in the device status word, every role leaves, drains
    its copies and MMAs and frees TMEM, and the launch returns; with the
    default bound back, the next chunk is bit-identical to one before."""
    import ctypes

    from reflex_b200 import _lib as L
    cfg = pi05_config(num_layers=2)
    wts, ctx, parts, x0, st = make_case(cfg, 200)
    eng = make_engine(cfg, wts, parts, 200, fused=True)
    ref = run_chunk(eng, x0)
    try:
        L.call("rfx_set_wait_limit_ns", ctypes.c_ulonglong(2000))  # taken at each launch
        eng.set_inputs(x0.cuda())
        eng.run_eager()
        torch.cuda.synchronize()
        assert kernels.device_status() == 8  # the executor's dependency-timeout code
    finally:
        L.call("rfx_set_wait_limit_ns", ctypes.c_ulonglong(0))
    eng.set_inputs(x0.cuda())
    eng.run_eager()
    torch.cuda.synchronize()
    assert kernels.device_status() == 0
    assert torch.equal(eng.x.float().cpu(), ref)


# ------------------------------------------------------------------ PI0 ---
def _debug_rows(eng, cfg):
    hid = [eng.dbg_h[l].view(eng.B, eng.St, -1).float().cpu() for l in range(cfg.num_layers)]
    att = [eng.dbg_attn[l].view(eng.B, eng.St, -1).float().cpu() for l in range(cfg.num_layers)]
    return hid, att


def test_fused_pi0_small_vs_reference_golden():
    """PI0 on the persistent executor (state token first, block-causal new
    keys, the [action, time] MLP as two GEMM phases per step) against the
    reference's own fp32 outputs (golden model_pi0_l2: 2 layers, uint8
    context) and the oracle's attention trace."""
    g = np.load(os.path.join(GOLD, "model_pi0_l2.npz"))
    nl, n_ctx = int(g["num_layers"]), int(g["n_ctx"])
    cfg = pi0_config(num_layers=nl, quant_mode="u8_ref")
    wts, ctx, parts, x0, st = make_case(cfg, n_ctx)
    eng = make_engine(cfg, wts, parts, n_ctx, fused=True)
    eng.enable_chunk_debug()
    x = run_chunk(eng, x0, st)
    trace = {}
    with torch.no_grad():
        sample_chunk(cfg, wts, ctx, x0, st, trace_step0=trace)
    ref_h = [torch.from_numpy(h) for h in g["hidden_step0"]]
    hid, att = _debug_rows(eng, cfg)
    report("fused-pi0-golden", ref_h, hid, trace["attn"], att)
    for l in range(nl):
        assert (hid[l] - ref_h[l]).abs().max().item() <= hidden_tol(ref_h[l]), f"layer {l}"
        assert (att[l] - trace["attn"][l]).abs().max().item() <= TOL, f"layer {l}"
    err = (x - torch.from_numpy(g["actions"])).abs().max().item()
    print(f"fused pi0 golden: actions maxerr vs reference fp32 {err:.5f}")
    assert err <= TOL


@pytest.mark.parametrize("quant,n_ctx", [("i8_sym", 300), ("u8_ref", 0)])
def test_fused_pi0_matches_oracle_and_per_op_engine(quant, n_ctx):
    cfg = pi0_config(num_layers=2, quant_mode=quant)
    wts, ctx, parts, x0, st = make_case(cfg, n_ctx)
    xf = run_chunk(make_engine(cfg, wts, parts, n_ctx, fused=True), x0, st)
    xp = run_chunk(make_engine(cfg, wts, parts, n_ctx), x0, st)
    with torch.no_grad():
        x32 = sample_chunk(cfg, wts, ctx, x0, st)
    e_oracle = (xf - x32).abs().max().item()
    e_per_op = (xf - xp).abs().max().item()
    print(f"fused pi0 {quant}/{n_ctx}: vs fp32 oracle {e_oracle:.5f}, vs per-op engine {e_per_op:.5f}")
    assert e_oracle <= TOL
    assert e_per_op <= TOL


def test_fused_pi0_long_context_full_size():
    """PI0 over 6344 int8 context tokens (200-token prefix + 8 frames x 3
    cameras x 256), 18 layers, 10 steps on the persistent executor, per layer
    against the fp32 oracle, with the bf16-storage drift bound of the per-op
    engine's test (the oracle with every op rounded to bf16)."""
    cfg = pi0_config(quant_mode="i8_sym")
    n_ctx = 200 + 8 * 3 * 256
    wts, ctx, parts, x0, st = make_case(cfg, n_ctx)
    eng = make_engine(cfg, wts, parts, n_ctx, capacity=(n_ctx + 63) // 64 * 64, fused=True)
    eng.enable_chunk_debug()
    x = run_chunk(eng, x0, st)
    torch.set_num_threads(os.cpu_count() or 1)
    h32, hbf, trace = [], [], {}
    with torch.no_grad():
        x32 = sample_chunk(cfg, wts, ctx, x0, st, hidden_step0=h32, trace_step0=trace)
        xbf = sample_chunk(cfg, wts, ctx, x0, st, bf16=True, hidden_step0=hbf)
    hid, att = _debug_rows(eng, cfg)
    report("fused-pi0-6344", h32, hid, trace["attn"], att)
    for l in range(cfg.num_layers):
        drift = (hbf[l] - h32[l]).abs().max().item()
        assert (hid[l] - h32[l]).abs().max().item() <= max(hidden_tol(h32[l]), 1.5 * drift), f"layer {l}"
        assert (att[l] - trace["attn"][l]).abs().max().item() <= TOL, f"layer {l}"
    err = (x - x32).abs().max().item()
    drift = (xbf - x32).abs().max().item()
    print(f"fused pi0-6344 actions maxerr vs fp32 oracle: {err:.5f} (bf16 oracle: {drift:.5f})")
    assert err <= max(TOL, 1.5 * drift)


def test_fused_pi0_graph_replay_is_deterministic():
    cfg = pi0_config(num_layers=3, quant_mode="i8_sym")
    wts, ctx, parts, x0, st = make_case(cfg, 300)
    eng = make_engine(cfg, wts, parts, 300, fused=True)
    ref = run_chunk(eng, x0, st)
    eng.capture()
    for _ in range(3):
        eng.set_inputs(x0.cuda(), st.cuda())
        eng.launch_chunk()
        torch.cuda.synchronize()
        assert torch.equal(eng.x.float().cpu(), ref)
    assert kernels.device_status() == 0


# ------------------------------------------------- several streams, masks ---
@pytest.mark.parametrize("variant,B,chunk", [("pi05", 4, 12), ("pi0", 3, 16)])
def test_fused_several_streams_match_per_op_engine(variant, B, chunk):
    """B streams in one executor launch (B * tokens <= 64): every stream's own
    context ring, query tiles and new-key block; against the per-op engine and
    the fp32 oracle on the same inputs."""
    cfg = (pi05_config(num_layers=2, quant_mode="i8_sym", chunk_size=chunk) if variant == "pi05"
           else pi0_config(num_layers=2, quant_mode="i8_sym", chunk_size=chunk))
    n_ctx = 150
    wts, ctx, parts, x0, st = make_case(cfg, n_ctx, B=B)
    xf = run_chunk(make_engine(cfg, wts, parts, n_ctx, B=B, fused=True), x0, st)
    xp = run_chunk(make_engine(cfg, wts, parts, n_ctx, B=B), x0, st)
    with torch.no_grad():
        x32 = sample_chunk(cfg, wts, ctx, x0, st)
    e_oracle = (xf - x32).abs().max().item()
    e_per_op = (xf - xp).abs().max().item()
    print(f"fused {variant} B={B}: vs fp32 oracle {e_oracle:.5f}, vs per-op engine {e_per_op:.5f}")
    assert e_oracle <= TOL
    assert e_per_op <= TOL


@pytest.mark.parametrize("variant", ["pi05", "pi0"])
def test_fused_context_mask_matches_per_op_engine(variant):
    """A per-slot context mask (padded prefix tokens, an evicted range) on the
    executor against the per-op engine with the same mask."""
    cfg = (pi05_config(num_layers=2, quant_mode="u8_ref", adarms="gate", chunk_size=16) if variant == "pi05"
           else pi0_config(num_layers=2, quant_mode="u8_ref", chunk_size=16))
    B, n_ctx = 2, 260
    wts, ctx, parts, x0, st = make_case(cfg, n_ctx, B=B)
    valid = torch.ones(B, n_ctx, dtype=torch.bool)
    valid[0, 40:100] = False
    valid[1, 250:] = False
    outs = []
    for fused in (True, False):
        eng = make_engine(cfg, wts, parts, n_ctx, B=B, fused=fused)
        eng.set_context_mask(valid.cuda())
        outs.append(run_chunk(eng, x0, st))
    from oracle.model import Context
    with torch.no_grad():
        x32 = sample_chunk(cfg, wts, Context(ctx.k, ctx.v, valid), x0, st)
    err = (outs[0] - outs[1]).abs().max().item()
    e_oracle = (outs[0] - x32).abs().max().item()
    print(f"fused {variant} with a context mask: vs per-op engine {err:.5f}, vs fp32 oracle {e_oracle:.5f}")
    assert err <= TOL
    assert e_oracle <= TOL
    assert kernels.device_status() == 0
