"""Prefill benchmark of the B200 decider engine.

One step = one full 2B int8-compute decide forward (24 layers: 6 x [3 Gated
DeltaNet + 1 gated GQA], hidden 2048, LoRA rank 32, vocab 248320) over a
512-token prompt plus the pointer-head readout of one noul question, weights
random-initialised N(0, 0.02^2) with norms 1 (synthetic data, seed 0).

value  : prefill tokens/s with the ids already resident (device time of the
         forward kernels, CUDA events on the engine stream);
e2e    : the same through the public C ABI call (dg_logits: host ids in,
         host logits out, copies inside the timed region);
roofline: the dominant kernel, the tcgen05 INT8 projection: every one of its
         launches in the timed steps is bracketed by CUDA events on the engine
         stream; achieved = sum of 2*M*N*K over the launches / their summed time;
cpu_baseline: the oracle (C++ restatement of the reference CPU path) on one
         4-layer block of the same model over a token sample, extrapolated to
         24 layers.

Multi-GPU (torchrun): every rank owns a replica and its own request (weak
scaling, no collective on the data path); time = max over ranks.
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

ROOT = os.path.dirname(os.path.abspath(__file__))
for p in (ROOT, os.path.join(ROOT, "decider-engine_b200"), os.path.join(ROOT, "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)

import numpy as np  # noqa: E402

METRIC = "prefill tok/s at 2B INT8 (1/2/4/8 B200)"
TOKENS = 512
# DRAM bytes (read + write) per gemm_i8_g64 launch, averaged over the 32
# projection launches of a 4-layer forward (the 24-layer model repeats the
# same 4-layer pattern): one ncu capture, profiles/gemm_i8_g64_swiglu_512x12288x2048.md.
GEMM_TRAFFIC_BYTES_PER_LAUNCH = 20.62e6


def cfg2(layers=24):
    from model_util import cfg2_config
    return cfg2_config(layers)


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            m = json.load(f)
        return m["hbm_gbs"], m["bf16_tflops"], "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled during the timed region."""

    def __init__(self, device):
        self.device, self.rows, self.proc = device, [], None

    def __enter__(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.device), f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) >= 8:
                self.rows.append(parts)

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows for i in range(4) if r[4 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.rows)}


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    pg = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        import torch
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device(f"cuda:{local}"))
        pg = dist
    return world, rank, local, pg


def max_over_ranks(v, dist, device):
    if dist is None:
        return v
    import torch
    t = torch.tensor([v], dtype=torch.float64, device=f"cuda:{device}")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(dist, device):
    import torch
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize(device)


class CpuSample:
    """The oracle on one 4-layer block (3 DeltaNet + 1 attention) of the 2B
    model: `time(tokens)` returns seconds for the full 24-layer forward of
    that many tokens (6 blocks)."""

    def __init__(self, threads=None):
        from model_util import random_tensors
        from oracle import oracle as O
        O.build()
        self.threads = threads or os.cpu_count()
        O.set_threads(self.threads)
        c = cfg2(4)
        c["vocab_size"] = 1024  # embedding rows are gathered, not computed
        t = random_tensors(c, rank=32, pointer_dim=0, seed=0, std=0.02, norm_jitter=0.0)
        self.model = O.OracleModel(c, t, "int8-compute", 32, 2.0)
        self.ids = np.random.default_rng(0).integers(0, 1024, 4096)
        self.model.forward(self.ids[:8])

    def time(self, tokens):
        t0 = time.perf_counter()
        self.model.forward(self.ids[:tokens])
        return (time.perf_counter() - t0) * 6.0


def workload_config(args, world):
    """The `config` object both arms report."""
    return {"workload": f"cfg2: 2B decider forward ({args.layers} layers, vocab {args.vocab}, LoRA r32) "
                        "over a 512-token prompt + pointer head, int8-compute",
            "tokens_per_step": TOKENS, "parallelism": f"dp{world}",
            "l2": "not flushed: each step streams 1.4 GB of int8 weights, > 126 MB L2"}


def run_reference(args, world, rank, local, dist):
    if rank != 0:
        return
    tokens = args.cpu_tokens
    cs = CpuSample()
    times = []
    for i in range(args.warmup + args.steps):
        s = cs.time(tokens)
        if i >= args.warmup:
            times.append(s)
    sec = sum(times) / len(times)
    value = tokens / sec
    sample = f"oracle port, one 4-layer block x {tokens} tokens per step, x6 for 24 layers"
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": sec * 1000 * TOKENS / tokens,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "int8-compute (i8 x i8 -> i32 groups, f32 promotion)", "data": "synthetic",
        "config": workload_config(args, world),
        "note": "the reference's CPU algorithm (oracle restatement) on rank 0's host cores; the Rust crate "
                "cannot be built here",
        "cpu_baseline": {"value": value, "unit": "tok/s", "cores": cs.threads, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def run_ours(args, world, rank, local, dist):
    import torch

    import decider_gpu
    from decider_gpu import GpuModel
    torch.cuda.set_device(local)
    L = decider_gpu.load()
    cfg = cfg2(args.layers)
    cfg["vocab_size"] = args.vocab
    t0 = time.time()
    model = GpuModel(cfg, "int8-compute", 32, 2.0, 256, local, TOKENS)
    model.fill_synthetic(seed=0, stddev=0.02)
    model.finalize()
    assert model.fast_path
    model.set_exact(args.exact)
    setup_s = time.time() - t0
    rng = np.random.default_rng(1000 + rank)
    ids = rng.integers(0, cfg["vocab_size"], TOKENS).astype(np.uint32)
    positions = np.array([TOKENS - 3, TOKENS - 2], np.uint64)
    logits = np.zeros(2, np.float32)
    h_ids = torch.from_numpy(ids).pin_memory()
    h_pos = torch.from_numpy(positions.astype(np.int64)).pin_memory()
    h_out = torch.zeros(2, dtype=torch.float32).pin_memory()

    def step():
        decider_gpu._lib.check(L.dg_logits(model.h, None, h_ids.data_ptr(), TOKENS, h_pos.data_ptr(), 2,
                                           h_out.data_ptr()))

    # ---- roofline source: the tcgen05 projection launches of the first 4-layer
    # block (3 DeltaNet + 1 attention layer; the model repeats that block) in
    # every timed step, bracketed by CUDA events on the engine stream (the
    # launching stream). A pair of event nodes costs the forward graph a few
    # microseconds, so events around all ~100 projections of a step would
    # slow the measured step by ~10 %; the one-block sample keeps it near 2 %.
    # Switched on before the warm-up, so that the forward's CUDA graph (eager
    # first run, captured second) is built with the timing nodes before the
    # timed region starts.
    sample_layers = min(4, args.layers)
    model.gemm_timing_layers(0, sample_layers)
    for _ in range(args.warmup):  # W >= 3: eager, captured, then replayed runs
        step()
    stream = torch.cuda.ExternalStream(L.dg_engine_stream(model.h), device=local)
    g0_ms, g0_ops, g0_n = model.gemm_time()
    a0_ops, a0_n = model.gemm_time_all()
    # ---- e2e: through the public call, host buffers, copies inside the region
    barrier(dist, local)
    n0 = decider_gpu.launch_count()
    fwd_ms = []
    with ClockSampler(local) as clocks:
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            step()
            fwd_ms.append(float(L.dg_engine_last_forward_ms(model.h)))
        e1.record(stream)
        e1.synchronize()
    launches = decider_gpu.launch_count() - n0
    barrier(dist, local)
    e2e_ms = e0.elapsed_time(e1) / args.steps
    dev_ms = sum(fwd_ms) / len(fwd_ms)
    e2e_ms = max_over_ranks(e2e_ms, dist, local)
    dev_ms = max_over_ranks(dev_ms, dist, local)
    value = world * TOKENS / (dev_ms / 1000.0)
    e2e = world * TOKENS / (e2e_ms / 1000.0)
    # ---- roofline: the dominant kernel, gemm_i8_g64 (all projection launches)
    g_ms, g_ops, g_n = model.gemm_time()
    g_ms, g_ops, g_n = g_ms - g0_ms, g_ops - g0_ops, g_n - g0_n
    a_ops, a_n = model.gemm_time_all()
    a_ops, a_n = a_ops - a0_ops, a_n - a0_n
    model.gemm_timing(False)
    # ---- p50 latency (BASELINE metric): wall time of single warm dg_logits
    # calls (host ids in, host logits out), after the timed region.
    for _ in range(3):
        step()
    lat = []
    for _ in range(args.latency_calls):
        t1 = time.perf_counter()
        step()
        lat.append((time.perf_counter() - t1) * 1000.0)
    lat.sort()
    p50 = max_over_ranks(lat[len(lat) // 2], dist, local) if lat else None
    p99 = max_over_ranks(lat[min(len(lat) - 1, (99 * len(lat)) // 100)], dist, local) if lat else None
    gemm_ms_per_launch = g_ms / max(g_n, 1)
    # Projection time of a whole step, at the sampled launches' ops rate.
    gemm_step_ms = (g_ms / g_ops) * a_ops / args.steps if g_ops > 0 else 0.0
    gemm_share = gemm_step_ms / dev_ms if dev_ms > 0 else None
    hbm, bf16, src = peaks()
    int8_peak = 2.0 * bf16
    achieved = g_ops / (g_ms / 1000.0) / 1e12 if g_ms > 0 else 0.0
    if rank != 0:
        return
    cpu = None
    if world == 1 and not args.no_cpu:
        cs = CpuSample()
        sec = cs.time(args.cpu_tokens)
        cpu = {"value": args.cpu_tokens / sec, "unit": "tok/s", "cores": cs.threads, "kind": "port",
               "sample": f"oracle port, one 4-layer block of the 2B model x {args.cpu_tokens} tokens, x6 for 24 layers"}
    line = {
        "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": dev_ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "int8-compute (i8 x i8 -> i32 groups, f32 promotion)",
        "promotion": "reference-order" if args.exact else "fma", "data": "synthetic",
        "config": dict(workload_config(args, world), setup_s=round(setup_s, 1)),
        "e2e": {"value": e2e, "unit": "tok/s", "h2d_bytes_per_step": TOKENS * 4 + 16,
                "d2h_bytes_per_step": 8, "ms_per_step": e2e_ms},
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": int8_peak, "unit": "TOP/s",
                     "frac": achieved / int8_peak, "traffic": GEMM_TRAFFIC_BYTES_PER_LAUNCH,
                     "kernel": f"gemm_i8_g64_kernel, the projection launches of layers 0-{sample_layers - 1} in "
                               "every timed step (achieved = sum 2*M*N*K / sum event time)",
                     "launches": int(g_n), "launches_per_step": int(a_n) // max(args.steps, 1),
                     "ms_per_launch": gemm_ms_per_launch, "share_of_step": gemm_share,
                     "peak_source": f"2 x {src} bf16 dense ({bf16} TF/s): int8 dense is twice bf16"},
        "latency": {"p50_ms": p50, "p99_ms": p99, "calls": len(lat),
                    "what": "wall time of one warm dg_logits call per request (512 ids in, 2 logits out), "
                            "max over ranks"},
        "gpu_launches": int(launches),
        "clocks": clocks.summary(),
    }
    if cpu:
        line["cpu_baseline"] = cpu
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--latency-calls", type=int, default=100, help="warm dg_logits calls timed for p50/p99")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-tokens", type=int, default=256)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--exact", action="store_true",
                    help="reference-order FP32 promotion instead of fused multiply-add")
    ap.add_argument("--layers", type=int, default=24,
                    help="fewer layers (multiple of 4) for small ncu captures; the bench line is 24")
    ap.add_argument("--vocab", type=int, default=248320,
                    help="smaller embedding table for small ncu captures; the bench line is 248320")
    args = ap.parse_args()
    if args.layers % 4 or args.layers <= 0:
        ap.error("--layers must be a positive multiple of 4")
    world, rank, local, dist = dist_setup()
    try:
        if args.impl == "reference":
            run_reference(args, world, rank, local, dist)
        else:
            run_ours(args, world, rank, local, dist)
    finally:
        if dist is not None:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
