"""The persistent chunk executor (rfx_chunk) against the fp32 oracle and the
per-op engine, through the C ABI.

Tolerances are those of the per-op engine: denoised actions within max abs
2e-2 of the fp32 path.  Split GEMM partials are summed in a fixed order, so
replays of the same chunk are bit-identical.
"""
import os

import pytest
import torch

from oracle.model import sample_chunk
from reflex_b200 import kernels
from reflex_b200.config import pi05_config

from test_gpu_model import TOL, make_case, make_engine

pytestmark = pytest.mark.gpu


def run_chunk(eng, x0):
    eng.set_inputs(x0.cuda())
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
