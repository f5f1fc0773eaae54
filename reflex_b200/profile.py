"""Runs the kernels of one denoising layer in isolation, for profilers.

    python -m reflex_b200.profile [--layers 2] [--reps 3] [--ops qkv,attn,o,gu,down,tail,time,mod]
    python -m reflex_b200.profile --layers 18 --chunk   # one eager chunk, then one graph replay
    python -m reflex_b200.profile --layers 2 --chunk --fused   # the same through the chunk executor
    python -m reflex_b200.profile --layers 18 --chunk --fused --trace   # per-phase timeline of the executor
    python -m reflex_b200.profile --frame --ops qkv,attn,gu,down   # frame-update ops (768 tokens, Gemma-2B layer)
    python -m reflex_b200.profile --quant-bulk --reps 20   # int8 quantize-append of 64 streams x 2048 tokens

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
    ap.add_argument("--variant", default="pi05", choices=["pi05", "pi0"],
                    help="pi0: 1 state + 50 action tokens, plain RMSNorm (the long-context configuration)")
    ap.add_argument("--streams", type=int, default=1)
    ap.add_argument("--chunk", action="store_true", help="run whole chunks instead of single ops")
    ap.add_argument("--fused", action="store_true", help="with --chunk: the persistent chunk executor")
    ap.add_argument("--trace", action="store_true",
                    help="with --chunk --fused: %%globaltimer stamps of every task of the first Euler step "
                         "(needs a library built with make -C reflex_b200/csrc EXTRA_NVFLAGS=-DRFX_TRACE)")
    ap.add_argument("--trace-out", default=None, help="with --trace: also save the raw stamps (.npy)")
    ap.add_argument("--noncoop", action="store_true",
                    help="with --chunk --fused: launch the executor without the cooperative attribute (profilers "
                         "that cannot replay cooperative launches) and with 20 ms bounds on its cross-CTA waits")
    ap.add_argument("--frame", action="store_true",
                    help="the ops of one prefix layer of the streaming frame update (768 new tokens over a 48-token "
                         "pinned prefix and a 2-frame window)")
    ap.add_argument("--quant-bulk", action="store_true",
                    help="time the int8 quantize-append of a 64-stream x 2048-token prefill (larger than L2)")
    args = ap.parse_args()
    if args.quant_bulk:
        quant_bulk(args.reps)
        return
    if args.noncoop:
        from . import _lib as L
        L.call("rfx_set_chunk_cooperative", 0)
        L.call("rfx_set_wait_limit_ns", 20_000_000)
    if args.frame:
        frame_ops(args.ops, args.reps)
        return
    if args.variant == "pi0":
        from .config import pi0_config
        cfg = pi0_config(num_layers=args.layers)
    else:
        cfg = pi05_config(num_layers=args.layers, adarms="ssg")
    wts = synthetic.expert_weights(cfg, seed=0, device="cuda")
    eng = ActionExpertEngine(cfg, wts, batch=args.streams, capacity=max(1024, (args.n_ctx + 63) // 64 * 64),
                             n_ctx=args.n_ctx,
                             scale_dtype=torch.float32, fused=args.chunk and args.fused)
    ks, vs = synthetic.context_kv(cfg, args.n_ctx, B=args.streams, seed=1, device="cuda")
    for l in range(cfg.num_layers):
        eng.load_context(l, ks[l], vs[l])
    eng.set_inputs(synthetic.noise(cfg, B=args.streams, seed=2, device="cuda"),
                   synthetic.state(cfg, B=args.streams, seed=3, device="cuda") if cfg.variant == "pi0" else None)
    eng.run_eager()
    torch.cuda.synchronize()
    if args.chunk and args.fused and args.trace:
        trace_chunk(eng, out=args.trace_out)
        return
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


def quant_bulk(reps: int, streams: int = 64, tokens: int = 2048, sets: int = 3) -> None:
    """Times a bulk int8 quantize-append: K and V of `streams` rings x `tokens`
    bf16 tokens (one head of 256) into rings of the same capacity, the prefill of
    a multi-stream batch.  `sets` input sets are cycled so that no launch finds
    its input in L2 (each set is 2 x streams x tokens x 512 B, 134 MB at the
    defaults).  Prints the CUDA-event time per launch and the achieved bandwidth
    over the algorithmic bytes: per (token, head) row 512 B read, 256 B + a
    4-byte fp32 scale written."""
    from . import _lib as L

    g = torch.Generator(device="cuda").manual_seed(5)
    ring = K.KVRing.allocate(streams, 1, tokens, 256, L.RFX_QUANT_I8_SYM, scale_dtype=torch.float32)
    xs = [(torch.randn(streams, 1, tokens, 256, generator=g, device="cuda").bfloat16(),
           torch.randn(streams, 1, tokens, 256, generator=g, device="cuda").bfloat16()) for _ in range(sets)]
    for k, v in xs:
        K.kv_quant_append(k, v, ring)
    torch.cuda.synchronize()
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(reps + 1)]
    torch.cuda.profiler.start()
    evs[0].record()
    for i in range(reps):
        k, v = xs[i % sets]
        K.kv_quant_append(k, v, ring)
        evs[i + 1].record()
    torch.cuda.synchronize()
    torch.cuda.profiler.stop()
    per = sorted(evs[i].elapsed_time(evs[i + 1]) for i in range(reps))
    med = per[len(per) // 2]
    rows = 2 * streams * tokens
    nbytes = rows * (512 + 256 + 4)
    print(f"quant bulk {streams}x{tokens} tokens, K+V: {med * 1e3:.1f} us per launch (median of {reps}), "
          f"{nbytes / 1e6:.1f} MB algorithmic, {nbytes / (med * 1e-3) / 1e9:.0f} GB/s")
    print("status", K.device_status())


def frame_ops(ops: str, reps: int) -> None:
    """Launches the requested ops (norm, qkv, attn, o, norm2, gu, down, quant) of
    layer 0 of a one-layer frame update `reps` times each, between
    cudaProfilerStart/Stop, after one warm-up run of every op."""
    from . import _lib as L
    from .config import vlm_config
    from .prefix import PrefixEngine

    cfg = vlm_config(num_layers=1)
    pinned, flen = 48, 768
    wts = synthetic.prefix_weights(cfg, seed=10)
    rings = [K.KVRing.allocate(1, 1, 2048, 256, L.RFX_QUANT_I8_SYM, scale_dtype=torch.float32)]
    eng = PrefixEngine(cfg, wts, rings, pinned=pinned, frame_len=flen, window_frames=2, batch=1)
    ks, vs = synthetic.context_kv(cfg, pinned + 2 * flen, B=1, seed=12)
    eng.load_context(0, ks[0], vs[0])
    eng.set_frame(synthetic.frame_embeddings(cfg, flen, B=1, seed=13).cuda())
    names = ["norm", "qkv", "attn", "o", "norm2", "gu", "down", "quant"]
    layer = [d for kind, d, _ in eng.ops(0) if kind != "barrier"]
    for d in layer:
        K.Plan.run_direct(d)
    torch.cuda.synchronize()
    torch.cuda.profiler.start()
    for op in ops.split(","):
        for _ in range(reps):
            K.Plan.run_direct(layer[names.index(op)])
    torch.cuda.synchronize()
    torch.cuda.profiler.stop()
    print("ok", K.device_status())


# task types and trace slots of the chunk executor (csrc/chunk.cu): per task 16
# u64: [0] start, [1] inputs ready / accumulator ready, [2] end, [3] producer
# saw the input, [4] task words x | y << 32, [6] accumulator read out,
# [8] own rows stored, [9] peer partial arrived, [10] / [11] first / last
# operand stage seen by the MMA issuer, [12] epilogue done.
_TASKS = {1: "qkv", 2: "o", 3: "gu", 4: "down", 5: "attn", 6: "comb", 7: "fin_o", 8: "fin_d"}
_ORDER = ["qkv", "attn", "comb", "o", "fin_o", "gu", "down", "fin_d"]


def trace_chunk(eng, per_cta: int = 256, out: str | None = None) -> None:
    """Runs one chunk with task tracing on and prints, for the first Euler step,
    the per-layer phase timeline and the median segments of the GEMM tasks."""
    import numpy as np

    from . import _lib as L

    nsm = torch.cuda.get_device_properties(0).multi_processor_count
    buf = torch.zeros(nsm * per_cta * 16, dtype=torch.int64, device="cuda")
    for _ in range(2):
        eng.run_eager()
    torch.cuda.synchronize()
    L.call("rfx_set_trace", buf.data_ptr(), buf.numel() * 8)
    eng.run_eager()
    torch.cuda.synchronize()
    L.call("rfx_set_trace", None, 0)
    print("status", K.device_status())
    tr = buf.view(nsm, per_cta, 16).cpu().numpy().astype(np.int64)
    if out:
        np.save(out, tr)
    rows = []
    for c in range(nsm):
        for i in range(per_cta):
            if tr[c, i, 0] == 0:
                continue
            w = int(tr[c, i, 4] & 0xFFFFFFFF)
            rows.append((_TASKS.get(w & 0xFF, "?"), (w >> 8) & 0xFF, tr[c, i]))
    t0 = min(r[2][0] for r in rows)
    us = lambda v: (v - t0) / 1e3  # noqa: E731
    print("layer phase  tasks  last_input_ready  last_end  median(end - ready) [us from the chunk start]")
    ends = []
    for layer in range(eng.cfg.num_layers):
        for name in _ORDER:
            rs = [r[2] for r in rows if r[0] == name and r[1] == layer]
            if not rs:
                continue
            ready = [x[1] for x in rs if x[1] > 0]
            if layer < 3:
                print(f"{layer:5d} {name:6s} {len(rs):5d} {us(max(ready)) if ready else 0:17.2f} "
                      f"{us(max(x[2] for x in rs)):9.2f} {np.median([(x[2] - x[1]) / 1e3 for x in rs if x[1]]):10.2f}")
            if name == "fin_d":
                ends.append(us(max(x[2] for x in rs)))
    if len(ends) > 2:
        print("layer time (us, median over layers): %.2f" % float(np.median(np.diff(ends))))

    def seg(name, a, b):
        v = [(r[2][b] - r[2][a]) / 1e3 for r in rows if r[0] == name and r[2][a] and r[2][b]]
        return float(np.median(v)) if v else float("nan")

    for name in ["qkv", "o", "gu", "down"]:
        print(f"{name:5s} producer saw input -> first stage {seg(name, 3, 10):.2f}, first -> last stage "
              f"{seg(name, 10, 11):.2f}, last stage -> accumulator ready {seg(name, 11, 1):.2f}, "
              f"accumulator -> stored {seg(name, 1, 6):.2f}, stored -> end {seg(name, 6, 2):.2f} us")
        print(f"{'':5s} weights issued (last) -> producer saw input {seg(name, 13, 3):.2f}, armed weights issued -> "
              f"saw input {seg(name, 7, 3):.2f}, MMA waited on stages 2..n: "
              f"{float(np.median([r[2][14] / 1e3 for r in rows if r[0] == name])):.2f} us")
        print(f"{'':5s} read out -> own rows stored {seg(name, 6, 8):.2f}, -> peer partial arrived "
              f"{seg(name, 8, 9):.2f}, -> epilogue done {seg(name, 9, 12):.2f}, -> end {seg(name, 12, 2):.2f}, "
              f"task start -> producer saw input {seg(name, 0, 3):.2f} us")


if __name__ == "__main__":
    main()
