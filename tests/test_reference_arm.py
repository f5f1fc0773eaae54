"""bench.py's reference arm runs the reference's own computation: the
`pip install --target baseline/_ref` copy of Reflex, driven through the
harness the arm uses, reproduces the golden 2-layer PI0.5 chunk that
tests/golden/make_golden.py computed from the reference checkout (same seeded
weights, context, noise and state).  CPU only; skipped where the install is
absent (it is git-ignored).
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
