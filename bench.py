"""Benchmark of the streaming denoising hot path on B200.

Workload (the PI0.5 action-chunk latency config): PI0.5 action expert, one
robot stream per GPU, 18 Gemma-300M layers (width 1024, 8x256 heads, 1 KV
head, GeGLU 4096), scale/shift/gate adaRMS from the timestep MLP, 818 cached
context tokens held as int8 per-token KV, 50 action tokens, 10 Euler steps.
One "step" of this benchmark = one full 10-step action chunk, replayed as a
single CUDA graph of the engine's kernels.

Multi-GPU (torchrun): every rank serves its own independent stream (weak
scaling, no collective on the hot path); the action chunks are gathered to
rank 0 with NCCL after the timed region.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

--impl reference times the reference's PyTorch path for the same workload on
the host CPU: Reflex's own modules from its `pip install --target baseline/_ref`
copy when present, else the oracle port of
reflex/policies/pi05/modeling_pi05.py.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "p50 10-step PI0.5 action-chunk latency (ms); suffix-attn tensor-pipe % / HBM GB/s"
N_CTX = 818
CAPACITY = 1024


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="rfx", choices=["rfx", "reference"])
    ap.add_argument("--layers", type=int, default=18)
    ap.add_argument("--no-graph", action="store_true")
    ap.add_argument("--cpu-sample-chunks", type=int, default=2)
    ap.add_argument("--workload", default="chunk", choices=["chunk", "frame", "pi0-long", "vision"],
                    help="chunk: one 10-step chunk (the headline); frame: streaming frame update + chunk; "
                         "pi0-long: one PI0 chunk over a 6344-token context; vision: the SigLIP tower + projector "
                         "over one 3-camera frame")
    ap.add_argument("--engine", default="fused", choices=["fused", "per-op"],
                    help="fused: the persistent chunk executor (one launch per chunk); per-op: one launch per op")
    ap.add_argument("--streams-per-gpu", type=int, default=1,
                    help="independent robot streams served per GPU, batched along B (multi-stream sweep)")
    ap.add_argument("--multistream", type=int, default=64,
                    help="after the headline: serve this many independent streams sharded over the ranks "
                         "(streams.shard_range) and report chunks/s and the timed NCCL gather in a 'multistream' "
                         "sub-record (0: skip)")
    return ap.parse_args()


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def workload_config(args, world):
    return {
        "workload": f"PI0.5 10-step action chunk, {args.streams_per_gpu} stream(s)/GPU, "
                    "18x(1024, 8x256 MQA, GeGLU 4096), 818-token int8 KV context per stream, 50 action tokens",
        "model": "pi05-action-expert (gemma-300m shape), random-init",
        "layers": args.layers, "context_tokens": N_CTX, "suffix_tokens": 50, "euler_steps": 10,
        "streams_per_gpu": args.streams_per_gpu, "global_batch": world * args.streams_per_gpu, "kv": "int8 symmetric per-token/per-head",
        "adarms": "scale/shift/gate", "parallelism": f"dp{world} (independent streams)",
        "engine": "persistent chunk executor" if args.engine == "fused" and args.streams_per_gpu * 50 <= 64
                  else "one launch per op",
        "l2": "no flush: each chunk streams 6.2 GB of weights + 0.47 GB of fp32 modulation weights (>> 126 MB L2)",
    }


# ---------------------------------------------------------------- clocks ---
class ClockSampler:
    """Samples SM clocks and throttle reasons every 100 ms during the timed
    region (one `nvidia-smi -lms` process, ended when the region ends)."""

    def __init__(self, index: int):
        self.index, self.rows, self.proc = index, [], None
        self._t = threading.Thread(target=self._read, daemon=True)

    def _read(self):
        for line in self.proc.stdout:
            f = [x.strip() for x in line.strip().split(",")]
            if len(f) >= 7:
                self.rows.append(f)

    def __enter__(self):
        q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._t.start()
            time.sleep(0.3)  # first sample lands before the timed launches start
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self._t.join(timeout=5)

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[0]) for r in self.rows if r[0].replace(".", "").isdigit()]
        mx = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows for i in range(4) if r[3 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.rows)}


def sustained_tflops():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["bf16_tflops_sustained"])
    except Exception:
        return 1400.0


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


# ------------------------------------------------------------- CPU legs ---
def cpu_chunk_ms(layers: int, chunks: int):
    """The reference's PyTorch path of the same workload on the host CPU (the
    oracle port: reflex/policies/pi05/modeling_pi05.py:1181-1241,1403-1419 over
    the fp32 restatement of its modules), all host threads."""
    from oracle import quant as oq
    from oracle.model import Context, sample_chunk
    from reflex_b200 import synthetic
    from reflex_b200.config import pi05_config

    torch.set_num_threads(os.cpu_count() or 1)
    cfg = pi05_config(num_layers=layers, adarms="ssg")
    wts = synthetic.expert_weights(cfg, seed=0)
    ks, vs = synthetic.context_kv(cfg, N_CTX, seed=1)
    kd, vd = [], []
    for l in range(layers):
        q, s = oq.quant_i8_sym(ks[l].numpy())
        kd.append(torch.from_numpy(oq.dequant_i8_sym(q, s)))
        q, s = oq.quant_i8_sym(vs[l].numpy())
        vd.append(torch.from_numpy(oq.dequant_i8_sym(q, s)))
    ctx = Context(kd, vd, torch.ones(1, N_CTX, dtype=torch.bool))
    x0 = synthetic.noise(cfg, seed=2)
    times = []
    with torch.no_grad():
        sample_chunk(cfg, wts, ctx, x0)  # warm-up
        for _ in range(chunks):
            t0 = time.perf_counter()
            sample_chunk(cfg, wts, ctx, x0)
            times.append((time.perf_counter() - t0) * 1e3)
    return statistics.median(times), torch.get_num_threads(), times


REF_DIR = os.path.join(ROOT, "baseline", "_ref")


def reference_chunks_ms(layers: int, chunks: int, warmup: int):
    """Reflex's own PyTorch modules on the host CPU: the action expert built
    from its PI05ModelLayer / AdaRMSNorm (in-tree, gate form) / suffix embedder
    / QKVLinear / MergedColumnLinear / StreamingAttention with the uint8
    quantized 818-token context in its caches, driven through the Euler loop
    of sample_actions (reflex/policies/pi05/modeling_pi05.py:1181-1241,
    1403-1419), fp32, all host threads.  The package is the `pip install
    --target baseline/_ref` copy of the reference, imported through the
    oracle's harness (stub modules for the absent lerobot)."""
    import contextlib

    from oracle import reference_harness as H
    from reflex_b200 import synthetic
    from reflex_b200.config import pi05_config

    torch.set_num_threads(os.cpu_count() or 1)
    with contextlib.redirect_stdout(sys.stderr):  # the reference prints banners; stdout carries one JSON line
        R = H.import_reference(REF_DIR)
        cfg = pi05_config(num_layers=layers, adarms="gate")
        wts = synthetic.expert_weights(cfg, seed=0)
        ks, vs = synthetic.context_kv(cfg, N_CTX, seed=1)
        ctx = [H.quantized_context(R, ks[l], vs[l]) for l in range(layers)]
        model = H.build_reference_model(R, cfg, wts, "pi05")
        H.install_context(R, model, "pi05", ctx)
        x0, st = synthetic.noise(cfg, seed=2), synthetic.state(cfg, seed=3)
        times = []
        with torch.no_grad():
            for i in range(warmup + chunks):
                t0 = time.perf_counter()
                H.run_reference_chunk(R, model, cfg, x0, st, N_CTX)
                if i >= warmup:
                    times.append((time.perf_counter() - t0) * 1e3)
    return statistics.median(times), torch.get_num_threads(), times


def run_reference(args):
    """The reference arm: rank 0 alone times the reference's CPU path of the
    workload (its own modules from baseline/_ref when that install exists,
    else the oracle port); the other ranks exit without work."""
    rank, world, _ = dist_env()
    if rank != 0:
        return
    steps = max(1, args.steps)
    if os.path.isdir(os.path.join(REF_DIR, "reflex")):
        med, cores, times = reference_chunks_ms(args.layers, steps, min(max(args.warmup, 0), 2))
        kind, dtype = "reference", "f32"
        sample = (f"{len(times)} full 10-step chunks of the workload through Reflex's own PyTorch modules "
                  "(baseline/_ref install; in-tree gate AdaRMSNorm, its uint8 KV cache; fp32 on the host CPU)")
    else:
        med, cores, times = cpu_chunk_ms(args.layers, steps)
        kind, dtype = "port", "f32"
        sample = f"{len(times)} full chunks of the workload on the host CPU (fp32 torch oracle port)"
    line = {
        "impl": "reference", "metric": METRIC, "value": round(med, 3), "unit": "ms", "n_gpus": args.gpus,
        "steps": len(times), "warmup": args.warmup, "ms_per_step": round(statistics.mean(times), 3),
        "higher_is_better": False, "scaling": "weak", "vs_baseline": None, "dtype": dtype, "data": "synthetic",
        "config": workload_config(args, world),
        "cpu_baseline": {"value": round(med, 3), "unit": "ms", "cores": cores, "kind": kind, "sample": sample},
        "e2e": {"value": round(med, 3), "unit": "ms", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------- GPU leg ---
def build_engine(args, device):
    from reflex_b200 import synthetic
    from reflex_b200.config import pi05_config
    from reflex_b200.expert import ActionExpertEngine

    cfg = pi05_config(num_layers=args.layers, adarms="ssg", quant_mode="i8_sym")
    wts = synthetic.expert_weights(cfg, seed=0, device=device)
    B = args.streams_per_gpu
    fused = args.engine == "fused" and B * cfg.suffix_len <= 64
    # int8 symmetric KV keeps fp32 per-token scales (absmax / 127)
    eng = ActionExpertEngine(cfg, wts, batch=B, capacity=CAPACITY, n_ctx=N_CTX, device=device,
                             scale_dtype=torch.float32, fused=fused)
    del wts
    ks, vs = synthetic.context_kv(cfg, N_CTX, B=B, seed=1, device=device)
    for l in range(cfg.num_layers):
        eng.load_context(l, ks[l], vs[l])
    torch.cuda.synchronize()
    return cfg, eng


def chunk_kernel_roofline(eng, hbm_peak, reps=3):
    """Times the persistent chunk executor alone (counter clear + one launch)
    with CUDA events on the launching stream; returns per-launch duration and
    achieved HBM GB/s over its algorithmic bytes."""
    import ctypes

    from reflex_b200 import _lib as L
    from reflex_b200 import kernels as K

    cfg = eng.cfg
    # per Euler step: every layer's bf16 weights once, each stream's int8 K+V context and fp32 scales
    # (PI0 adds its action-time MLP: [W, 2W] + [W, W] bf16)
    per_step = cfg.num_layers * 17301504 * 2 + eng.B * cfg.num_layers * eng.n_ctx * (256 + 4) * 2
    if cfg.variant == "pi0":
        per_step += 3 * cfg.width * cfg.width * 2
    bytes_per = cfg.num_steps * per_step
    st = torch.cuda.current_stream()
    L.call("rfx_chunk_run", eng.chunk, K._stream())
    durs = []
    for _ in range(reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        L.call("rfx_chunk_run", eng.chunk, K._stream())
        e1.record(st)
        torch.cuda.synchronize()
        durs.append(e0.elapsed_time(e1))
    avg_ms = statistics.median(durs)
    achieved = bytes_per / (avg_ms * 1e-3) / 1e9
    traffic = None  # DRAM bytes per launch from the committed ncu capture of this kernel and workload
    capture = {("pi05", N_CTX): "chunk_kernel_pi05_818ctx.md", ("pi0", PI0_LONG_CTX): "chunk_kernel_pi0_6344ctx.md"}
    source = capture.get((cfg.variant, eng.n_ctx))
    try:
        if source is None or eng.B != 1 or cfg.num_layers != 18:
            raise OSError("no capture of this workload")
        with open(os.path.join(ROOT, "profiles", source)) as f:
            for line in f:
                if line.startswith("traffic_bytes_per_launch:"):
                    traffic = int(line.split(":")[1])
    except OSError:
        pass
    del ctypes
    return {"kernel": "chunk_kernel (persistent executor of the whole 10-step chunk, 1 CTA per SM)",
            "bound": "hbm", "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
            "frac": round(achieved / hbm_peak, 4), "traffic": traffic,
            "traffic_source": (f"ncu dram__bytes_read.sum + dram__bytes_write.sum of one launch (non-cooperative, "
                               f"profile --noncoop), profiles/{source}"
                               if traffic is not None else "not captured for this workload"),
            "bytes_per_launch": bytes_per, "avg_launch_us": round(avg_ms * 1e3, 2)}


def kernel_roofline(eng, hbm_peak, reps=3):
    """Times the gate/up GEMM launches of one Euler step back to back (18
    different weights, so nothing stays in L2) with CUDA events on the launching
    stream; returns per-launch duration and achieved HBM GB/s."""
    from reflex_b200 import kernels as K

    gu = [d for kind, d, tag in eng.ops if tag is not None and tag[0] == "gu" and tag[1] == 0]
    cfg = eng.cfg
    # algorithmic bytes of one launch: packed gate/up weight + normed input rows + GeGLU output
    T = eng.T
    bytes_per = (2 * cfg.mlp_dim * cfg.width * 2) + T * cfg.width * 2 + T * cfg.mlp_dim * 2
    st = torch.cuda.current_stream()
    for d in gu:
        K.Plan.run_direct(d)
    durs = []
    for _ in range(reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda._sleep(4_000_000)  # keeps the GPU busy while the host enqueues the launches
        e0.record(st)
        for d in gu:
            K.Plan.run_direct(d)
        e1.record(st)
        torch.cuda.synchronize()
        durs.append(e0.elapsed_time(e1) / len(gu))
    avg_ms = statistics.median(durs)
    achieved = bytes_per / (avg_ms * 1e-3) / 1e9
    traffic = None  # DRAM bytes per launch from the committed ncu capture of this kernel and shape
    try:
        with open(os.path.join(ROOT, "profiles", "linear_gate_up_pi05_b1.md")) as f:
            for line in f:
                if line.startswith("traffic_bytes_per_launch:"):
                    traffic = int(line.split(":")[1])
    except OSError:
        pass
    return {"kernel": "linear_kernel<64,LOAD,GEGLU> (gate/up projection + GELU-tanh(gate)*up)",
            "bound": "hbm", "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
            "frac": round(achieved / hbm_peak, 4), "traffic": traffic,
            "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum, profiles/linear_gate_up_pi05_b1.md",
            "bytes_per_launch": bytes_per, "avg_launch_us": round(avg_ms * 1e3, 2)}


def multistream_record(args, rank, world, device, pg, hbm_peak, tflops_peak):
    """The multi-stream configuration: `args.multistream` independent robot
    streams (each with its own 818-token int8 KV ring, 50-token suffix and
    x0) sharded data-parallel over the ranks with streams.shard_range and
    batched along B on each GPU (one CUDA graph per chunk), no collective on
    the hot path.  Device-timed per chunk with CUDA events, max over ranks;
    then the final NCCL gather of the [streams, 50, 32] action chunks, timed
    on its own.  The per-GPU roofline is the slower of the chunk's GEMM +
    attention FLOPs at the measured sustained bf16 rate and its algorithmic
    bytes at the measured HBM bandwidth."""
    from reflex_b200 import synthetic
    from reflex_b200.config import pi05_config
    from reflex_b200.expert import ActionExpertEngine
    from reflex_b200.streams import gather_chunks, shard_range

    total = args.multistream
    first, n = shard_range(total, rank, world)
    cfg = pi05_config(num_layers=args.layers, adarms="ssg", quant_mode="i8_sym")
    wts = synthetic.expert_weights(cfg, seed=0, device=device)
    eng = ActionExpertEngine(cfg, wts, batch=n, capacity=CAPACITY, n_ctx=N_CTX, device=device,
                             scale_dtype=torch.float32, fused=n * cfg.suffix_len <= 64)
    del wts
    ks, vs = synthetic.context_kv(cfg, N_CTX, B=n, seed=100 + first, device=device)
    for l in range(cfg.num_layers):
        eng.load_context(l, ks[l], vs[l])
    del ks, vs
    x0 = synthetic.noise(cfg, B=n, seed=200 + first, device=device)
    eng.set_inputs(x0)
    eng.capture()
    st = torch.cuda.current_stream()
    for _ in range(3):
        eng.set_inputs(x0)
        eng.launch_chunk()
    torch.cuda.synchronize()
    reps = max(3, min(args.steps, 10))
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(reps + 1)]
    if pg:
        pg.barrier()
    torch.cuda.synchronize()
    evs[0].record(st)
    for i in range(reps):
        eng.set_inputs(x0)
        eng.launch_chunk()
        evs[i + 1].record(st)
    torch.cuda.synchronize()
    per = statistics.median([evs[i].elapsed_time(evs[i + 1]) for i in range(reps)])
    gather_ms = None
    if pg:
        t = torch.tensor([per], device=device)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        per = t.item()
        gt = []
        for i in range(6):
            pg.barrier()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(st)
            out = gather_chunks(eng.x, total, pg)
            e1.record(st)
            torch.cuda.synchronize()
            if i > 0:
                gt.append(e0.elapsed_time(e1))
        assert out.shape[0] == total
        t = torch.tensor([statistics.median(gt)], device=device)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        gather_ms = round(t.item(), 4)
    launches = eng.num_launches
    eng.plan = None
    del eng
    torch.cuda.empty_cache()
    # per GPU and chunk: GEMM FLOPs of n*50 tokens through 18 layers, attention of n*8*50 query rows over
    # 868 keys, 10 steps; bytes: weights once per step, each stream's int8 K+V + fp32 scales per step,
    # and the fp32 modulation weights once per chunk
    flops = 10 * n * (2 * 50 * 17301504 * args.layers + args.layers * 2 * 2 * 400 * (N_CTX + 50) * 256)
    nbytes = 10 * (args.layers * 17301504 * 2 + n * args.layers * N_CTX * (256 + 4) * 2) + \
        (2 * args.layers + 1) * 3 * 1024 * 1024 * 4
    t_flops = flops / (tflops_peak * 1e12) * 1e3
    t_bytes = nbytes / (hbm_peak * 1e9) * 1e3
    return {
        "workload": f"{total} independent PI0.5 streams (818-token int8 KV ring, 50-token suffix each), "
                    f"{n} per GPU on {world} GPU(s), batched along B, one CUDA graph per chunk",
        "streams_total": total, "streams_per_gpu": n, "chunk_ms_p50": round(per, 4),
        "chunks_per_s": round(total * 1e3 / per, 2), "gather_ms": gather_ms,
        "gather_bytes": total * 50 * 32 * 4,
        "engine": "persistent chunk executor" if n * 50 <= 64 else "one launch per op",
        "gpu_launches_per_chunk": launches,
        "roofline": {"bound": "tensor" if t_flops >= t_bytes else "hbm", "flops_per_gpu_chunk": flops,
                     "bytes_per_gpu_chunk": nbytes, "floor_ms": round(max(t_flops, t_bytes), 4),
                     "frac": round(max(t_flops, t_bytes) / per, 4),
                     "peaks": f"{tflops_peak} TFLOP/s bf16 sustained, {hbm_peak} GB/s (MEASURED_PEAKS.json)"},
    }


def run_gpu(args):
    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    pg = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=device)
        pg = dist
    hbm_peak, _, peak_kind = peaks()
    from reflex_b200 import kernels as K
    from reflex_b200 import synthetic

    cfg, eng = build_engine(args, device)
    B = args.streams_per_gpu
    x0 = synthetic.noise(cfg, B=B, seed=2 + rank, device=device)
    eng.set_inputs(x0)
    if not args.no_graph:
        eng.capture()
    launches = eng.num_launches
    st = torch.cuda.current_stream()

    def one_chunk():
        eng.set_inputs(x0)
        eng.launch_chunk()

    for _ in range(max(3, args.warmup)):
        one_chunk()
    torch.cuda.synchronize()
    status = K.device_status()
    if status:
        raise RuntimeError(f"device status {status} after warm-up")

    # ---- device-timed region
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
    if pg:
        pg.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        t_wall = time.perf_counter()
        evs[0].record(st)
        for i in range(args.steps):
            one_chunk()
            evs[i + 1].record(st)
        torch.cuda.synchronize()
        wall = time.perf_counter() - t_wall
    per = [evs[i].elapsed_time(evs[i + 1]) for i in range(args.steps)]
    total_ms = evs[0].elapsed_time(evs[-1])
    p50 = statistics.median(per)
    if pg:
        t = torch.tensor([p50, total_ms], device=device)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        p50, total_ms = t[0].item(), t[1].item()
        pg.barrier()

    # ---- end to end through the public API with host buffers
    x_host = synthetic.noise(cfg, B=B, seed=2 + rank).pin_memory()
    out_host = torch.empty_like(x_host).pin_memory()
    e2e = []
    for i in range(args.steps + 3):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        eng.set_inputs(x_host.to(device, non_blocking=True))
        eng.launch_chunk()
        out_host.copy_(eng.x, non_blocking=True)
        e1.record(st)
        e1.synchronize()
        if i >= 3:
            e2e.append(e0.elapsed_time(e1))
    e2e_p50 = statistics.median(e2e)
    if pg:
        t = torch.tensor([e2e_p50], device=device)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        e2e_p50 = t.item()
        # final gather of every stream's action chunk (not on the hot path)
        from reflex_b200.streams import gather_chunks
        gathered = gather_chunks(eng.x, world * B, pg)
        assert gathered.shape[0] == world * B

    roof = chunk_kernel_roofline(eng, hbm_peak) if eng.fused else kernel_roofline(eng, hbm_peak)
    roof["peak_kind"] = f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs, burst copy)"
    status = K.device_status()
    multi = None
    if args.multistream > 0:
        eng.plan = None
        del eng
        torch.cuda.empty_cache()
        multi = multistream_record(args, rank, world, device, pg, hbm_peak, sustained_tflops())
        status = status or K.device_status()

    cpu = None
    if rank == 0 and world == 1:
        med, cores, times = cpu_chunk_ms(args.layers, args.cpu_sample_chunks)
        cpu = {"value": round(med, 3), "unit": "ms", "cores": cores, "kind": "port",
               "sample": f"{len(times)} full chunks of the same workload (fp32 torch oracle port), median"}

    if rank == 0:
        # weights once per step, each stream's int8 K+V context and fp32 scales per step, and the fp32
        # scale/shift/gate modulation weights once per chunk
        bytes_chunk = 10 * (cfg.num_layers * 17301504 * 2 + B * cfg.num_layers * N_CTX * (256 + 4) * 2) + \
            (2 * cfg.num_layers + 1) * 3 * 1024 * 1024 * 4
        line = {
            "metric": METRIC, "value": round(p50, 4), "unit": "ms", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(total_ms / args.steps, 4), "higher_is_better": False,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic: seeded random-init weights, N(0,1) context K/V quantized to int8, x0 ~ N(0,1)",
            "config": workload_config(args, world),
            "chunks_per_s": round(world * B * 1e3 / p50, 2),
            "chunk_roofline": {"algorithmic_bytes": bytes_chunk,
                               "achieved_GBps": round(bytes_chunk / (p50 * 1e-3) / 1e9, 1),
                               "peak_GBps": hbm_peak, "frac": round(bytes_chunk / (p50 * 1e-3) / 1e9 / hbm_peak, 4)},
            "roofline": roof,
            "cpu_baseline": cpu,
            "e2e": {"value": round(e2e_p50, 4), "unit": "ms", "h2d_bytes_per_step": x_host.numel() * 4,
                    "d2h_bytes_per_step": out_host.numel() * 4},
            "gpu_launches": launches * args.steps,
            "multistream": multi,
            "clocks": clk.summary(),
            "graph": not args.no_graph,
            "device_status": status,
            "wall_s_timed": round(wall, 3),
        }
        print(json.dumps(line), flush=True)
    if pg:
        pg.barrier()
        pg.destroy_process_group()


def cpu_frame_ms(layers: int):
    """The oracle port of one control tick with a frame update on the host CPU,
    all host threads: the new 768-token frame through the prefix layers
    (reflex/policies/pi05/modeling_pi05.py:1282-1333 with the full prefix
    attention of :1379-1401) over the pinned prefix + the surviving frame, its
    K/V quantized into the context, then one 10-step PI0.5 chunk over the
    1584-token context."""
    from oracle import quant as oq
    from oracle.model import Context, prefix_frame, sample_chunk
    from reflex_b200 import synthetic
    from reflex_b200.config import pi05_config, vlm_config

    torch.set_num_threads(os.cpu_count() or 1)
    pinned, flen = 48, 768
    vcfg = vlm_config(num_layers=layers)
    cfg = pi05_config(num_layers=layers, adarms="ssg")
    pw = synthetic.prefix_weights(vcfg, seed=10)
    ew = synthetic.expert_weights(cfg, seed=0)
    ks, vs = synthetic.context_kv(cfg, pinned + 2 * flen, seed=1)

    def deq(x):
        q, sc = oq.quant_i8_sym(x.numpy())
        return torch.from_numpy(oq.dequant_i8_sym(q, sc))

    old = [(deq(ks[l][:, :, :pinned + flen]), deq(vs[l][:, :, :pinned + flen])) for l in range(layers)]
    emb = synthetic.frame_embeddings(vcfg, flen, seed=20).float()
    x0 = synthetic.noise(cfg, seed=2)
    t0 = time.perf_counter()
    with torch.no_grad():
        ctx = Context([k for k, _ in old], [v for _, v in old], torch.ones(1, pinned + flen, dtype=torch.bool))
        pos = (pinned + flen + torch.arange(flen))[None]
        _, kvs = prefix_frame(vcfg, pw, emb, ctx, pos)
        full = Context([torch.cat([old[l][0], deq(kvs[l][0])], 2) for l in range(layers)],
                       [torch.cat([old[l][1], deq(kvs[l][1])], 2) for l in range(layers)],
                       torch.ones(1, pinned + 2 * flen, dtype=torch.bool))
        sample_chunk(cfg, ew, full, x0)
    return (time.perf_counter() - t0) * 1e3, torch.get_num_threads()


def frame_gu_roofline(pre, bf16_peak, peak_kind):
    """The frame update's dominant kernel: one prefix layer's gate/up projection
    (768 tokens x 32768 rows x 2048), timed alone with CUDA events on the
    launching stream; achieved TFLOP/s against the measured bf16 burst peak."""
    from reflex_b200 import kernels as K

    layer = [d for kind, d, _ in pre.ops(0) if kind != "barrier"]
    gu = layer[5]  # norm, qkv, attn, o, norm2, gate/up, down, quant
    for _ in range(2):
        K.Plan.run_direct(gu)
    torch.cuda.synchronize()
    st = torch.cuda.current_stream()
    durs = []
    for _ in range(5):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda._sleep(2_000_000)
        e0.record(st)
        K.Plan.run_direct(gu)
        e1.record(st)
        torch.cuda.synchronize()
        durs.append(e0.elapsed_time(e1))
    ms = statistics.median(durs)
    flops = 2.0 * gu.T * gu.O * gu.K
    achieved = flops / (ms * 1e-3) / 1e12
    traffic = None
    try:
        with open(os.path.join(ROOT, "profiles", "linear_gate_up_frame768.md")) as f:
            for line in f:
                if line.startswith("traffic_bytes_per_launch:"):
                    traffic = int(line.split(":")[1])
    except OSError:
        pass
    return {"kernel": "linear_tiles_kernel<256,GEGLU> (prefix gate/up projection, 768 tokens)", "bound": "tensor",
            "achieved": round(achieved, 1), "peak": bf16_peak, "unit": "TFLOP/s", "frac": round(achieved / bf16_peak, 4),
            "traffic": traffic, "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum, "
                                                  "profiles/linear_gate_up_frame768.md",
            "flops_per_launch": flops, "avg_launch_us": round(ms * 1e3, 2),
            "peak_kind": f"{peak_kind} (MEASURED_PEAKS.json bf16_tflops, burst)"}


def run_frame(args):
    """Streaming frame update + one chunk per control tick: a new frame of
    3 cameras x 256 patch embeddings through the 18 prefix layers (Gemma-2B
    shapes) over a pinned 48-token instruction prefix and a 2-frame window,
    evicting the oldest frame and quantize-appending the new one into the
    rings, then one 10-step PI0.5 chunk over the updated 1584-token context;
    both in one CUDA graph (one per ring slot the frame replaces)."""
    from reflex_b200 import kernels as K
    from reflex_b200 import synthetic
    from reflex_b200.config import pi05_config, vlm_config
    from reflex_b200.expert import ActionExpertEngine
    from reflex_b200.prefix import PrefixEngine

    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    pinned, flen, win = 48, 768, 2
    n_ctx = pinned + win * flen
    cfg = pi05_config(num_layers=args.layers, adarms="ssg", quant_mode="i8_sym")
    wts = synthetic.expert_weights(cfg, seed=0, device=device)
    eng = ActionExpertEngine(cfg, wts, batch=1, capacity=n_ctx, n_ctx=n_ctx, device=device,
                             scale_dtype=torch.float32, fused=True)
    del wts
    vcfg = vlm_config(num_layers=args.layers)
    pw = synthetic.prefix_weights(vcfg, seed=10, device=device)
    pre = PrefixEngine(vcfg, pw, eng.rings, pinned=pinned, frame_len=flen, window_frames=win)
    del pw
    ks, vs = synthetic.context_kv(cfg, n_ctx, seed=1, device=device)
    for l in range(cfg.num_layers):
        eng.load_context(l, ks[l], vs[l])
    del ks, vs
    plans = []
    for slot in range(win):
        plan = K.Plan()
        for kind, desc, _ in pre.ops(slot) + eng.ops:
            plan.add(desc, eng._kind(kind))
        plans.append(plan)
    x0 = synthetic.noise(cfg, seed=2, device=device)
    frames = [synthetic.frame_embeddings(vcfg, flen, seed=20 + i, device=device) for i in range(2)]
    stream = torch.cuda.Stream(device=device)
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        for plan in plans:
            pre.set_frame(frames[0])
            eng.set_inputs(x0)
            plan.run()
            plan.capture(stream)
    torch.cuda.current_stream().wait_stream(stream)
    st = torch.cuda.current_stream()

    def tick(i, frame, x):
        pre.set_frame(frame)
        eng.set_inputs(x)
        plans[i % win].replay()

    for i in range(max(3, args.warmup)):
        tick(i, frames[i % 2], x0)
    torch.cuda.synchronize()
    status = K.device_status()
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
    torch.cuda.synchronize()
    with ClockSampler(0) as clk:
        evs[0].record(st)
        for i in range(args.steps):
            tick(i, frames[i % 2], x0)
            evs[i + 1].record(st)
        torch.cuda.synchronize()
    per = [evs[i].elapsed_time(evs[i + 1]) for i in range(args.steps)]
    p50 = statistics.median(per)
    # end to end: the frame and x0 from pinned host memory, actions back
    fh = frames[0].cpu().pin_memory()
    xh = x0.cpu().pin_memory()
    out = torch.empty_like(xh).pin_memory()
    e2e = []
    for i in range(args.steps + 3):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        tick(i, fh.to(device, non_blocking=True), xh.to(device, non_blocking=True))
        out.copy_(eng.x, non_blocking=True)
        e1.record(st)
        e1.synchronize()
        if i >= 3:
            e2e.append(e0.elapsed_time(e1))
    prefix_bytes = args.layers * (2560 * 2048 + 2048 * 2048 + 32768 * 2048 + 2048 * 16384) * 2
    prefix_flops = 2.0 * flen * prefix_bytes / 2
    _, bf16_peak, peak_kind = peaks()
    roof = frame_gu_roofline(pre, bf16_peak, peak_kind)
    cpu_ms, cores = cpu_frame_ms(args.layers)
    line = {
        "metric": "p50 streaming frame update + 10-step PI0.5 chunk latency (ms)", "value": round(p50, 4),
        "unit": "ms", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(evs[0].elapsed_time(evs[-1]) / args.steps, 4), "higher_is_better": False,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: seeded random-init prefix and expert weights, N(0,1)/sqrt(2048) frame embeddings",
        "config": {"workload": "frame update: 3 cameras x 256 tokens through 18 Gemma-2B-shape prefix layers over "
                               "a pinned 48-token prefix + 2-frame window (1584 tokens), evict + int8 "
                               "quantize-append, then one 10-step PI0.5 chunk; one CUDA graph",
                   "layers": args.layers, "frame_tokens": flen, "pinned": pinned, "window_frames": win,
                   "context_tokens": n_ctx, "engine": "per-op prefix layers + persistent chunk executor"},
        "prefix_weight_bytes": prefix_bytes, "prefix_gflop": round(prefix_flops / 1e9, 1),
        "e2e": {"value": round(statistics.median(e2e), 4), "unit": "ms",
                "h2d_bytes_per_step": fh.numel() * 2 + xh.numel() * 4, "d2h_bytes_per_step": out.numel() * 4},
        "gpu_launches": sum(p.num_launches for p in plans) // win * args.steps,
        "roofline": roof,
        "cpu_baseline": {"value": round(cpu_ms, 3), "unit": "ms", "cores": cores, "kind": "port",
                         "sample": "1 control tick of the same workload: frame through the prefix layers + "
                                   "one chunk (fp32 torch oracle port)"},
        "clocks": clk.summary(), "device_status": status,
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------- long-context PI0 leg ---
PI0_LONG_CTX = 200 + 8 * 3 * 256  # instruction prefix + 8 frames x 3 cameras x 256 patches


def cpu_pi0_long_ms(layers: int, chunks: int):
    """The oracle port of one PI0 chunk (reflex/policies/pi0/modeling_pi0.py:
    740-845, 144-206) over the same 6344-token int8 context, all host threads."""
    from oracle import quant as oq
    from oracle.model import Context, sample_chunk
    from reflex_b200 import synthetic
    from reflex_b200.config import pi0_config

    torch.set_num_threads(os.cpu_count() or 1)
    cfg = pi0_config(num_layers=layers)
    wts = synthetic.expert_weights(cfg, seed=0)
    ks, vs = synthetic.context_kv(cfg, PI0_LONG_CTX, seed=1)
    kd, vd = [], []
    for l in range(layers):
        q, s = oq.quant_i8_sym(ks[l].numpy())
        kd.append(torch.from_numpy(oq.dequant_i8_sym(q, s)))
        q, s = oq.quant_i8_sym(vs[l].numpy())
        vd.append(torch.from_numpy(oq.dequant_i8_sym(q, s)))
    ctx = Context(kd, vd, torch.ones(1, PI0_LONG_CTX, dtype=torch.bool))
    x0, st = synthetic.noise(cfg, seed=2), synthetic.state(cfg, seed=3)
    times = []
    with torch.no_grad():
        for _ in range(chunks):
            t0 = time.perf_counter()
            sample_chunk(cfg, wts, ctx, x0, st)
            times.append((time.perf_counter() - t0) * 1e3)
    return statistics.median(times), torch.get_num_threads(), times


def run_pi0_long(args):
    """One PI0 chunk (1 state token + 50 action tokens, [action, time] MLP, plain
    RMSNorm, 18 layers, 10 Euler steps) over a 200-token prefix + 8 frames x 3
    cameras x 256 tokens of int8 KV: one chunk is one CUDA graph of the time
    embedding and the persistent chunk executor (--engine per-op: one launch
    per op)."""
    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    from reflex_b200 import kernels as K
    from reflex_b200 import synthetic
    from reflex_b200.config import pi0_config
    from reflex_b200.expert import ActionExpertEngine

    hbm_peak, _, peak_kind = peaks()
    cfg = pi0_config(num_layers=args.layers)
    wts = synthetic.expert_weights(cfg, seed=0, device=device)
    cap = (PI0_LONG_CTX + 63) // 64 * 64
    fused = args.engine == "fused"
    eng = ActionExpertEngine(cfg, wts, batch=1, capacity=cap, n_ctx=PI0_LONG_CTX, device=device,
                             scale_dtype=torch.float32, fused=fused)
    del wts
    ks, vs = synthetic.context_kv(cfg, PI0_LONG_CTX, B=1, seed=1, device=device)
    for l in range(cfg.num_layers):
        eng.load_context(l, ks[l], vs[l])
    del ks, vs
    x0 = synthetic.noise(cfg, seed=2, device=device)
    st0 = synthetic.state(cfg, seed=3, device=device)
    eng.set_inputs(x0, st0)
    eng.capture()
    stream = torch.cuda.current_stream()
    for _ in range(max(3, args.warmup)):
        eng.set_inputs(x0, st0)
        eng.launch_chunk()
    torch.cuda.synchronize()
    if K.device_status():
        raise RuntimeError("device status after warm-up")
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        evs[0].record(stream)
        for i in range(args.steps):
            eng.set_inputs(x0, st0)
            eng.launch_chunk()
            evs[i + 1].record(stream)
        torch.cuda.synchronize()
    per = [evs[i].elapsed_time(evs[i + 1]) for i in range(args.steps)]
    p50 = statistics.median(per)
    x_host = synthetic.noise(cfg, seed=2).pin_memory()
    s_host = synthetic.state(cfg, seed=3).pin_memory()
    out_host = torch.empty_like(x_host).pin_memory()
    e2e = []
    for i in range(args.steps + 2):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        eng.set_inputs(x_host.to(device, non_blocking=True), s_host.to(device, non_blocking=True))
        eng.launch_chunk()
        out_host.copy_(eng.x, non_blocking=True)
        e1.record(stream)
        e1.synchronize()
        if i >= 2:
            e2e.append(e0.elapsed_time(e1))
    roof = chunk_kernel_roofline(eng, hbm_peak) if fused else kernel_roofline(eng, hbm_peak)
    roof["peak_kind"] = f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs, burst copy)"
    cpu = None
    if rank == 0:
        med, cores, times = cpu_pi0_long_ms(args.layers, 1)
        cpu = {"value": round(med, 3), "unit": "ms", "cores": cores, "kind": "port",
               "sample": f"{len(times)} full PI0 chunk of the same workload (fp32 torch oracle port)"}
    # per step: the expert's bf16 weights, the int8 K+V context with fp32 scales
    bytes_chunk = 10 * (cfg.num_layers * 17301504 * 2 + cfg.num_layers * PI0_LONG_CTX * (256 + 4) * 2
                        + 3 * cfg.width * cfg.width * 2)
    if rank == 0:
        line = {
            "metric": "p50 10-step PI0 action-chunk latency over a 6344-token context (ms)", "value": round(p50, 4),
            "unit": "ms", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(statistics.mean(per), 4), "higher_is_better": False, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic: seeded random-init weights, N(0,1) context K/V quantized to int8, x0 and state ~ N(0,1)",
            "config": {"workload": "PI0 10-step action chunk: 1 state + 50 action tokens, 18x(1024, 8x256 MQA, GeGLU "
                                   "4096), plain RMSNorm, 200-token prefix + 8 frames x 3 cameras x 256 int8 KV "
                                   "(6344 tokens); one CUDA graph", "layers": cfg.num_layers,
                       "context_tokens": PI0_LONG_CTX, "suffix_tokens": cfg.suffix_len,
                       "engine": "persistent chunk executor" if fused else "one launch per op",
                       "l2": "no flush: each chunk streams 6.2 GB of weights + 0.6 GB of KV per step (>> 126 MB L2)"},
            "chunk_roofline": {"algorithmic_bytes": bytes_chunk,
                               "achieved_GBps": round(bytes_chunk / (p50 * 1e-3) / 1e9, 1), "peak_GBps": hbm_peak,
                               "frac": round(bytes_chunk / (p50 * 1e-3) / 1e9 / hbm_peak, 4)},
            "roofline": roof, "cpu_baseline": cpu,
            "e2e": {"value": round(statistics.median(e2e), 4), "unit": "ms",
                    "h2d_bytes_per_step": (x_host.numel() + s_host.numel()) * 4,
                    "d2h_bytes_per_step": out_host.numel() * 4},
            "gpu_launches": eng.num_launches * args.steps, "clocks": clk.summary(),
            "device_status": K.device_status(),
        }
        print(json.dumps(line), flush=True)


def cpu_vision_ms(images: int, reps: int):
    """The oracle restatement of the SigLIP tower + projector (transformers'
    SiglipVisionModel as the reference's image embedder calls it,
    reflex/policies/pi05/modeling_pi05.py:141-158) over the same images, fp32,
    all host threads."""
    from oracle import vision as ov
    from reflex_b200 import synthetic
    from reflex_b200.config import VisionConfig

    torch.set_num_threads(os.cpu_count() or 1)
    cfg = VisionConfig()
    w = synthetic.vision_weights(cfg, seed=30)
    img = synthetic.images(cfg, B=images, seed=31)
    times = []
    with torch.no_grad():
        for _ in range(reps):
            t0 = time.perf_counter()
            ov.image_features(cfg, w, img)
            times.append((time.perf_counter() - t0) * 1e3)
    return statistics.median(times), torch.get_num_threads(), times


def run_vision(args):
    """The image embedder of one control tick: three 224 x 224 camera images
    through the 27-layer SigLIP-So400m/14 tower and the PaliGemma projector
    (768 token rows), one CUDA graph per call."""
    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    from reflex_b200 import kernels as K
    from reflex_b200 import synthetic
    from reflex_b200.config import VisionConfig
    from reflex_b200.vision import VisionTower

    _, tf_peak, peak_kind = peaks()
    cfg = VisionConfig()
    cams = 3
    tower = VisionTower(cfg, synthetic.vision_weights(cfg, seed=30), max_images=cams, device=device)
    img = synthetic.images(cfg, B=cams, seed=31).to(device)
    stream = torch.cuda.current_stream()
    for _ in range(max(3, args.warmup)):
        tower.get_image_features(img)
    torch.cuda.synchronize()
    if K.device_status():
        raise RuntimeError("device status after warm-up")
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
    with ClockSampler(local) as clk:
        evs[0].record(stream)
        for i in range(args.steps):
            tower.launch(cams)
            evs[i + 1].record(stream)
        torch.cuda.synchronize()
    per = [evs[i].elapsed_time(evs[i + 1]) for i in range(args.steps)]
    p50 = statistics.median(per)
    img_host = synthetic.images(cfg, B=cams, seed=31).pin_memory()
    out_host = torch.empty(cams, cfg.tokens, cfg.proj_dim, dtype=torch.bfloat16).pin_memory()
    e2e = []
    for i in range(args.steps + 2):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        out = tower.get_image_features(img_host)
        out_host.copy_(out, non_blocking=True)
        e1.record(stream)
        e1.synchronize()
        if i >= 2:
            e2e.append(e0.elapsed_time(e1))
    flops = tower.flops(cams)
    achieved = flops / (p50 * 1e-3) / 1e12
    cpu = None
    if rank == 0:
        med, cores, times = cpu_vision_ms(cams, 2)
        cpu = {"value": round(med, 3), "unit": "ms", "cores": cores, "kind": "port",
               "sample": f"{len(times)} full calls of the same workload (fp32 torch restatement of the tower)"}
    if rank == 0:
        line = {
            "metric": "p50 latency of the image embedder for one 3-camera frame (ms)", "value": round(p50, 4),
            "unit": "ms", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(statistics.mean(per), 4), "higher_is_better": False, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic: seeded random-init SigLIP-So400m/14 + projector weights, uniform [-1, 1] images",
            "config": {"workload": "SigLIP-So400m/14 vision tower (27 x [LayerNorm, 16 x 72-dim attention, GELU MLP "
                                   "4304], width 1152) + 1152->2048 projector over 3 cameras x 224 x 224 "
                                   "(768 token rows); one CUDA graph", "layers": cfg.num_layers, "images": cams,
                       "l2": "no flush: each call streams 0.8 GB of bf16 weights (>> 126 MB L2)"},
            "roofline": {"kernel": "whole tower (GEMMs + attention)", "bound": "tensor",
                         "achieved": round(achieved, 1), "peak": tf_peak, "unit": "TFLOP/s",
                         "frac": round(achieved / tf_peak, 4), "traffic": None,
                         "flops_per_call": flops, "weight_bytes": tower.weight_bytes(),
                         "peak_kind": f"{peak_kind} (MEASURED_PEAKS.json bf16_tflops, burst cuBLAS)"},
            "cpu_baseline": cpu,
            "e2e": {"value": round(statistics.median(e2e), 4), "unit": "ms",
                    "h2d_bytes_per_step": img_host.numel() * 4, "d2h_bytes_per_step": out_host.numel() * 2},
            "gpu_launches": tower._plan(cams).num_launches * args.steps, "clocks": clk.summary(),
            "device_status": K.device_status(),
        }
        print(json.dumps(line), flush=True)


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
        return
    if args.workload == "pi0-long":
        return run_pi0_long(args)
    if args.workload == "frame":
        run_frame(args)
        return
    if args.workload == "vision":
        return run_vision(args)
    run_gpu(args)


if __name__ == "__main__":
    main()
