"""bench.py's reference arm runs the reference's own computation: the
`pip install --target baseline/_ref` copy of Reflex, driven through the
harness the arm uses, reproduces the golden 2-layer PI0.5 chunk that
tests/golden/make_golden.py computed from the reference checkout (same seeded
weights, context, noise and state); that test is skipped where the install
is absent (it is git-ignored).  The arm's JSON line carries the contract's
keys either way (without the install it times the oracle port).  CPU only.
"""
import os

import numpy as np
import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_DIR = os.path.join(ROOT, "baseline", "_ref")
GOLD = os.path.join(ROOT, "tests", "golden", "model_pi05_l2.npz")


@pytest.mark.skipif(not os.path.isdir(os.path.join(REF_DIR, "reflex")), reason="baseline/_ref not installed")
def test_reference_arm_reproduces_golden_chunk():
    import contextlib
    import sys

    from oracle import reference_harness as H
    from reflex_b200 import synthetic
    from reflex_b200.config import pi05_config

    g = np.load(GOLD)
    nl, n_ctx, seed = int(g["num_layers"]), int(g["n_ctx"]), int(g["seed"])
    with contextlib.redirect_stdout(sys.stderr):  # the reference prints banners
        R = H.import_reference(REF_DIR)
        cfg = pi05_config(num_layers=nl, adarms="gate")
        wts = synthetic.expert_weights(cfg, seed=seed)
        ks, vs = synthetic.context_kv(cfg, n_ctx, seed=seed + 1)
        ctx = [H.quantized_context(R, ks[l], vs[l]) for l in range(nl)]
        model = H.build_reference_model(R, cfg, wts, "pi05")
        H.install_context(R, model, "pi05", ctx)
        x0, st = synthetic.noise(cfg, seed=seed + 2), synthetic.state(cfg, seed=seed + 3)
        with torch.no_grad():
            x = H.run_reference_chunk(R, model, cfg, x0, st, n_ctx)
    err = (x - torch.from_numpy(g["actions"])).abs().max().item()
    assert err <= 1e-5, err


def test_reference_arm_json_line():
    """`bench.py --impl reference` prints one JSON line with the contract's
    keys (here with 2 layers and one chunk, to keep the CPU suite short)."""
    import json
    import subprocess
    import sys

    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1",
                          "--warmup", "0", "--layers", "2"], capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.strip()]
    assert len(lines) == 1, out.stdout
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["unit"] == "ms" and d["higher_is_better"] is False
    assert d["value"] > 0 and d["n_gpus"] == 1 and d["steps"] == 1
    assert d["cpu_baseline"]["kind"] in ("reference", "port") and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"] == {"value": d["value"], "unit": "ms", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    assert d["config"]["workload"]
