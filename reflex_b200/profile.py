"""Runs the kernels of one denoising layer in isolation, for profilers.

    python -m reflex_b200.profile [--layers 2] [--reps 3] [--ops qkv,attn,o,gu,down,tail,time,mod]
    python -m reflex_b200.profile --layers 18 --chunk   # one eager chunk, then one graph replay
    python -m reflex_b200.profile --layers 2 --chunk --fused   # the same through the chunk executor

Builds the PI0.5 engine at the benchmark's shapes (width 1024, 8x256 heads,
818-token int8 context, 50 action tokens) with a few layers, runs one chunk to
warm up, then launches the requested ops of step 0 / layer 0 `reps` times each
through the direct C entry points, in the order given.  Only the measured
launches sit inside cudaProfilerStart/Stop (profile with
`ncu --profile-from-start off`).  Device memory stays
well under 1 GB, so a profiler capture of a handful of launches ends quickly.
"""
from __future__ import annotations

import argparse

import torch

from . import kernels as K
from . import synthetic
from .config import pi05_config
from .expert import ActionExpertEngine


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--layers", type=int, default=2)
    ap.add_argument("--reps", type=int, default=3)
    ap.add_argument("--ops", default="qkv,attn,o,gu,down,tail")
    ap.add_argument("--n-ctx", type=int, default=818)
    ap.add_argument("--streams", type=int, default=1)
    ap.add_argument("--chunk", action="store_true", help="run whole chunks instead of single ops")
    ap.add_argument("--fused", action="store_true", help="with --chunk: the persistent chunk executor")
    args = ap.parse_args()
    cfg = pi05_config(num_layers=args.layers, adarms="ssg")
    wts = synthetic.expert_weights(cfg, seed=0, device="cuda")
    eng = ActionExpertEngine(cfg, wts, batch=args.streams, capacity=1024, n_ctx=args.n_ctx,
                             scale_dtype=torch.float32, fused=args.chunk and args.fused)
    ks, vs = synthetic.context_kv(cfg, args.n_ctx, B=args.streams, seed=1, device="cuda")
    for l in range(cfg.num_layers):
        eng.load_context(l, ks[l], vs[l])
    eng.set_inputs(synthetic.noise(cfg, B=args.streams, seed=2, device="cuda"))
    eng.run_eager()
    torch.cuda.synchronize()
    if args.chunk:
        print("launches per chunk", eng.num_launches)
        eng.capture()
        torch.cuda.synchronize()
        torch.cuda.profiler.start()
        eng.launch_chunk()
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()
        print("ok", K.device_status())
        return
    by_tag = {}
    for kind, desc, tag in eng.ops:
        if tag is not None and tag[1] == 0 and (len(tag) < 3 or tag[2] == 0):
            by_tag[tag[0]] = (kind, desc)
    for kind, desc, tag in eng.ops:
        if kind in ("time", "mod"):  # the per-chunk conditioning heads
            by_tag[kind] = (kind, desc)
    names = {"qkv": "qkv", "attn": "attn", "o": "o", "gu": "gu", "down": "layer", "tail": "step", "time": "time",
             "mod": "mod"}
    torch.cuda.profiler.start()
    for op in args.ops.split(","):
        kind, desc = by_tag[names[op]]
        for _ in range(args.reps):
            K.Plan.run_direct(desc, kind if kind in ("in", "tail") else None)
    torch.cuda.synchronize()
    torch.cuda.profiler.stop()
    print("ok", K.device_status())


if __name__ == "__main__":
    main()
