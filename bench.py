"""Prefill benchmark of the B200 decider engine.

Default line (the request-sharded throughput batch): one
step = the first 256 requests of the seeded 8192-request draw (bound length
L ~ U[128, 4096], 1-4 questions of 64 tokens; a request with several
questions prefills its (L - 64)-token state once and runs its questions
together after it), on the 2B int8-compute decider (24 layers: 6 x [3 Gated
DeltaNet + 1 gated GQA], hidden 2048, LoRA rank 32, vocab 248320), weights
random-initialised N(0, 0.02^2) with norms 1 (synthetic data, seed 0).
Under torchrun the requests are sharded over the ranks by
decider_gpu.sharding.shard_requests (longest processing time first): strong
scaling, no collective on the data path, time = max over ranks.
`--workload cfg2` measures config 2 (one 512-token prompt + one noul
question per step); cfg1, cfg3 and cfg4 the other configs.

value  : prefill tokens/s from device time, ids already resident: config 5
         (and 4) the span of each dg_logits_batch call on the device (CUDA
         events from before its first kernel to the end of its last lane;
         host gaps between requests included), config 2 the forward kernels;
lanes  : config 5 deals each rank's requests to --lanes engines sharing one
         copy of the weights (dg_engine_set_lanes), each driven from its own
         host thread, so their latency-bound kernels overlap on the GPU;
e2e    : the same through the public C ABI call (dg_logits_batch / dg_logits:
         host ids in, host logits out, copies inside the timed region);
roofline: the dominant kernel, the tcgen05 INT8 projection: its launches in
         the timed steps are bracketed by CUDA events on the engine stream;
         achieved = sum of 2*M*N*K over the launches / their summed time;
cpu_baseline: the oracle (C++ restatement of the reference CPU path, -O3)
         running the whole 24-layer forward over a short prompt (--cpu-tokens)
         on every host thread, the same step the reference arm times.
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
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            # The first sample must fall inside the timed region, however short.
            t0 = time.time()
            while not self.rows and time.time() - t0 < 3.0:
                time.sleep(0.01)
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


class CpuForward:
    """The oracle (oracle/: the reference's CPU algorithm restated in C++,
    built -O3 like the reference's release profile) on the full 2B model:
    `time()` returns the seconds of one whole 24-layer int8-compute forward
    over `tokens` ids plus the pointer-head readout of one noul question, with
    every host thread. A 512-token step takes minutes on a CPU, so the CPU
    timings run the same model over a shorter prompt. Only `tokens` embedding
    rows are gathered, so a 4096-row table stands in for the 248320-row one."""

    def __init__(self, tokens, layers=24, threads=None):
        from model_util import random_tensors
        from oracle import oracle as O
        O.build()
        self.threads = threads or os.cpu_count()
        O.set_threads(self.threads)
        c = cfg2(layers)
        c["vocab_size"] = 4096
        t = random_tensors(c, rank=32, pointer_dim=256, seed=0, std=0.02, norm_jitter=0.0, bias_std=0.0, f32=True)
        self.model = O.OracleModel(c, t, "int8-compute", 32, 2.0)
        del t
        self.tokens = tokens
        self.ids = np.random.default_rng(0).integers(0, 4096, tokens)
        self.pos = [tokens - 3, tokens - 2]

    def time(self):
        t0 = time.perf_counter()
        hidden = self.model.forward(self.ids)
        self.model.head_logits(hidden, self.pos)
        return time.perf_counter() - t0

    def describe(self):
        return (f"oracle port (-O3, {self.threads} threads): the whole 24-layer 2B int8-compute forward over "
                f"{self.tokens} tokens + pointer head per step (measured, not extrapolated)")


def workload_config(args, world):
    """The `config` object both arms report."""
    return {"workload": f"cfg2: 2B decider forward ({args.layers} layers, vocab {args.vocab}, LoRA r32) "
                        "over a 512-token prompt + pointer head, int8-compute",
            "tokens_per_step": TOKENS, "parallelism": f"dp{world}",
            "l2": "not flushed: each step streams 1.4 GB of int8 weights, > 126 MB L2"}


def run_reference(args, world, rank, local, dist):
    """The reference arm: the reference's CPU algorithm (the oracle port) on
    rank 0's host cores, each step one whole 24-layer forward over the first
    --cpu-tokens tokens (a bounded sample: the 512-token step takes minutes
    on a CPU). ms_per_step is the measured step; config.tokens_per_step says
    what ran."""
    if rank != 0:
        return
    cf = CpuForward(args.cpu_tokens)
    times = []
    for i in range(args.warmup + args.steps):
        s = cf.time()
        if i >= args.warmup:
            times.append(s)
    sec = sum(times) / len(times)
    value = cf.tokens / sec
    config = dict(workload_config(args, world), tokens_per_step=cf.tokens,
                  workload=f"cfg2 sample: 2B decider forward (24 layers, LoRA r32) over the first {cf.tokens} "
                           "tokens of a prompt + pointer head, int8-compute")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": sec * 1000,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "int8-compute (i8 x i8 -> i32 groups, f32 promotion)", "data": "synthetic",
        "config": config,
        "extrapolated": {"ms_per_512_token_step": sec * 1000 * TOKENS / cf.tokens,
                         "how": "linear in tokens from the measured step; drops attention's quadratic term, "
                                "which favours the CPU"},
        "note": "the reference's CPU algorithm (oracle restatement) on rank 0's host cores; the Rust crate "
                "cannot be built here",
        "cpu_baseline": {"value": value, "unit": "tok/s", "cores": cf.threads, "kind": "port",
                         "sample": cf.describe()},
        "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def _cpu_forward_baseline(args, note=""):
    """cpu_baseline of the GPU arms: the reference arm's step (CpuForward), one
    warm-up and two timed runs."""
    cf = CpuForward(args.cpu_tokens)
    cf.time()
    sec = (cf.time() + cf.time()) / 2
    return {"value": cf.tokens / sec, "unit": "tok/s", "cores": cf.threads, "kind": "port",
            "sample": cf.describe() + note}


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
    i8_loop, i8_loop_ms = decider_gpu.measure_i8_peak(local)
    cpu = None
    if world == 1 and not args.no_cpu:
        cpu = _cpu_forward_baseline(args)
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
                     "peak_source": f"2 x {src} bf16 dense ({bf16} TF/s): int8 dense is twice bf16",
                     "i8_loop_peak": i8_loop, "frac_of_i8_loop": achieved / i8_loop if i8_loop else None,
                     "i8_loop": "dg_measure_i8_peak: one CTA per SM issuing back-to-back tcgen05.mma.kind::i8 "
                                f"128x256x32 from shared memory ({i8_loop_ms:.1f} ms launch), measured after "
                                "the timed region"},
        "latency": {"p50_ms": p50, "p99_ms": p99, "calls": len(lat),
                    "what": "wall time of one warm dg_logits call per request (512 ids in, 2 logits out), "
                            "max over ranks"},
        "gpu_launches": int(launches),
        "clocks": clocks.summary(),
    }
    if cpu:
        line["cpu_baseline"] = cpu
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ other configs
# The default line is config 5 (run_batch). `--workload cfg1|cfg2|cfg3|cfg4` measures the
# other BASELINE configs with the same contract (device-time value, e2e
# through the public call with host buffers, roofline of the dominant kernel,
# CPU baseline on rank 0 at N=1).

CFG1 = (512, 6144, 2048)  # M tokens, N outputs, K inputs
CFG3 = (64, 4096, 16, 128)  # sequences, tokens, heads, head dim
# Algorithmic bytes of one config-3 call: q, k, v read, o written (4 x 512 B),
# g and beta read (8 B) per token and head, the state read and written.
CFG3_BYTES = 64 * 16 * 4096 * (4 * 128 * 4 + 8) + 2 * 64 * 16 * 128 * 128 * 4


def _line(args, world, metric, value, unit, ms, config, dtype="int8-compute (i8 x i8 -> i32 groups, f32 promotion)",
          **extra):
    d = {"metric": metric, "value": value, "unit": unit, "n_gpus": world, "steps": args.steps,
         "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
         "vs_baseline": None, "dtype": dtype, "promotion": "reference-order" if args.exact else "fma",
         "data": "synthetic", "config": config}
    d.update(extra)
    return d


def _cfg1_inputs():
    M, N, K = CFG1
    rng = np.random.default_rng(0)
    x = rng.standard_normal((M, K)).astype(np.float32)
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    return x, w


def _cfg1_config(world):
    M, N, K = CFG1
    return {"workload": f"cfg1: one group-64 INT8 linear, M={M} tokens x N={N} x K={K}, X ~ N(0,1), "
                        "W ~ N(0,0.02^2), no LoRA", "parallelism": f"dp{world}",
            "l2": "flushed before every call (256 MB write): X and W fit in the 126 MB L2"}


def _cpu_cfg1(rows=512):
    from oracle import oracle as O
    O.build()
    threads = os.cpu_count()
    O.set_threads(threads)
    x, w = _cfg1_inputs()
    wq, ws = O.quantize_weights(w)
    O.linear_int8_prequant(x[:4], wq, ws)
    t0 = time.perf_counter()
    O.linear_int8_prequant(x[:rows], wq, ws)
    sec = time.perf_counter() - t0
    M, N, K = CFG1
    return (2.0 * rows * N * K / sec / 1e12, "TOP/s", threads,
            f"oracle linear_int8 (scalar x86 path), {rows} of the {M} rows, weights quantised beforehand")


def run_cfg1(args, world, rank, local, dist):
    import torch

    import decider_gpu
    from decider_gpu import Linear
    torch.cuda.set_device(local)
    L = decider_gpu.load()
    M, N, K = CFG1
    x, w = _cfg1_inputs()
    lin = Linear(w, device=local)
    lin.set_exact(args.exact)
    dev = f"cuda:{local}"
    xd = torch.from_numpy(x).to(dev)
    yd = torch.empty((M, N), dtype=torch.float32, device=dev)
    stream = torch.cuda.ExternalStream(lin.stream(), device=local)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    torch.cuda.synchronize(local)

    def flush_l2():
        with torch.cuda.stream(stream):
            flush.zero_()

    for _ in range(args.warmup):
        flush_l2()
        lin.forward_device(xd.data_ptr(), M, yd.data_ptr())
    barrier(dist, local)
    n0 = decider_gpu.launch_count()
    tot, gem = [], []
    with ClockSampler(local) as clocks:
        for _ in range(args.steps):
            flush_l2()
            lin.forward_device(xd.data_ptr(), M, yd.data_ptr())
            t, g = lin.last_times()
            tot.append(t)
            gem.append(g)
    launches = decider_gpu.launch_count() - n0
    barrier(dist, local)
    # e2e: dg_linear_forward with pinned host X in and Y out (copies inside).
    hx = torch.from_numpy(x).pin_memory()
    hy = torch.empty((M, N), dtype=torch.float32).pin_memory()
    e2e_ms = []
    for i in range(args.warmup + args.steps):
        flush_l2()
        torch.cuda.synchronize(local)
        t0 = time.perf_counter()
        decider_gpu._lib.check(L.dg_linear_forward(lin.h, hx.data_ptr(), M, hy.data_ptr()))
        if i >= args.warmup:
            e2e_ms.append((time.perf_counter() - t0) * 1000.0)
    ops = 2.0 * M * N * K
    dev_ms = max_over_ranks(sum(tot) / len(tot), dist, local)
    gemm_ms = max_over_ranks(sum(gem) / len(gem), dist, local)
    e2e = max_over_ranks(sum(e2e_ms) / len(e2e_ms), dist, local)
    if rank != 0:
        return
    _, bf16, src = peaks()
    peak = 2.0 * bf16
    achieved = ops / (gemm_ms / 1000.0) / 1e12
    line = _line(args, world, "INT8 GEMM TOP/s (cfg1: 512x6144x2048, group-64)",
                 world * ops / (dev_ms / 1000.0) / 1e12, "TOP/s", dev_ms, _cfg1_config(world),
                 e2e={"value": world * ops / (e2e / 1000.0) / 1e12, "unit": "TOP/s",
                      "h2d_bytes_per_step": M * K * 4, "d2h_bytes_per_step": M * N * 4, "ms_per_step": e2e},
                 roofline={"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TOP/s",
                           "frac": achieved / peak, "traffic": None,
                           "kernel": "gemm_i8_g64_kernel alone (events around its launch on the handle's stream); "
                                     "value also counts the activation quantiser",
                           "ms_per_launch": gemm_ms, "share_of_step": gemm_ms / dev_ms,
                           "peak_source": f"2 x {src} bf16 dense ({bf16} TF/s): int8 dense is twice bf16"},
                 gpu_launches=int(launches), clocks=clocks.summary())
    if world == 1 and not args.no_cpu:
        v, u, c, smp = _cpu_cfg1()
        line["cpu_baseline"] = {"value": v, "unit": u, "cores": c, "kind": "port", "sample": smp}
    print(json.dumps(line), flush=True)


def _cfg3_config(world):
    B, T, H, D = CFG3
    return {"workload": f"cfg3: gated delta rule, {B} sequences x {T} tokens x {H} heads, dk = dv = {D}, "
                        "chunk 64, zero initial state; q, k L2-normalised N(0,1), v ~ N(0,1), "
                        "beta = sigmoid(N(0,1)), g = -softplus(N(0,1))",
            "parallelism": f"dp{world}", "l2": "not flushed: 8.8 GB of inputs and outputs per step, > 126 MB L2"}


def _cpu_cfg3():
    from concurrent.futures import ThreadPoolExecutor

    from oracle import oracle as O
    O.build()
    B, T, H, D = CFG3
    threads = os.cpu_count()
    rng = np.random.default_rng(0)
    pairs = []
    for _ in range(threads):
        q = rng.standard_normal((T, D)).astype(np.float32)
        k = rng.standard_normal((T, D)).astype(np.float32)
        q = (q / np.linalg.norm(q, axis=1, keepdims=True) / np.sqrt(np.float32(D))).astype(np.float32)
        k = (k / np.linalg.norm(k, axis=1, keepdims=True)).astype(np.float32)
        v = rng.standard_normal((T, D)).astype(np.float32)
        beta = (1.0 / (1.0 + np.exp(-rng.standard_normal(T)))).astype(np.float32)
        g = (-np.log1p(np.exp(rng.standard_normal(T)))).astype(np.float32)
        pairs.append((q, k, v, g, beta))
    reps = 8
    with ThreadPoolExecutor(threads) as ex:  # the oracle call releases the GIL
        t0 = time.perf_counter()
        list(ex.map(lambda a: O.gated_delta_rule(*a), pairs * reps))
        sec = time.perf_counter() - t0
    return (reps * threads * T / H / sec, "tok/s", threads,
            f"oracle token recurrence, {reps * threads} (sequence, head) pairs x {T} tokens on {threads} threads; "
            f"a token is one token of one sequence over all {H} heads")


def run_cfg3(args, world, rank, local, dist):
    import torch

    import decider_gpu
    from decider_gpu import gated_delta_chunk_workspace_bytes, gated_delta_rule_chunked
    torch.cuda.set_device(local)
    B, T, H, D = CFG3
    dev = f"cuda:{local}"
    gen = torch.Generator(device=dev).manual_seed(rank)
    rn = lambda *shape: torch.randn(shape, generator=gen, device=dev, dtype=torch.float32)
    q, k, v = rn(B, T, H, D), rn(B, T, H, D), rn(B, T, H, D)
    q = (q / q.norm(dim=-1, keepdim=True) / np.sqrt(np.float32(D))).contiguous()
    k = (k / k.norm(dim=-1, keepdim=True)).contiguous()
    beta = torch.sigmoid(rn(B, T, H)).contiguous()
    g = (-torch.nn.functional.softplus(rn(B, T, H))).contiguous()
    state = torch.zeros((B, H, D, D), dtype=torch.float32, device=dev)
    o = torch.empty((B, T, H, D), dtype=torch.float32, device=dev)
    nbytes = gated_delta_chunk_workspace_bytes(B, T, H)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    stream = torch.cuda.Stream(device=local)
    sptr = stream.cuda_stream

    def run():
        gated_delta_rule_chunked(q.data_ptr(), k.data_ptr(), v.data_ptr(), g.data_ptr(), beta.data_ptr(), B, T, H,
                                 state.data_ptr(), o.data_ptr(), ws.data_ptr(), nbytes, sptr)

    torch.cuda.synchronize(local)
    for _ in range(args.warmup):
        with torch.cuda.stream(stream):
            state.zero_()
        run()
    barrier(dist, local)
    n0 = decider_gpu.launch_count()
    ms = []
    with ClockSampler(local) as clocks:
        for _ in range(args.steps):
            with torch.cuda.stream(stream):
                state.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            run()
            e1.record(stream)
            e1.synchronize()
            ms.append(e0.elapsed_time(e1))
    launches = decider_gpu.launch_count() - n0
    barrier(dist, local)
    # e2e: pinned host inputs copied in and outputs copied out inside the region.
    hq, hk, hv = (t.cpu().pin_memory() for t in (q, k, v))
    hg, hb = g.cpu().pin_memory(), beta.cpu().pin_memory()
    hs = torch.zeros((B, H, D, D), dtype=torch.float32).pin_memory()
    ho = torch.empty((B, T, H, D), dtype=torch.float32).pin_memory()
    hs_out = torch.empty_like(hs).pin_memory()
    e2e_ms = []
    for i in range(1 + min(args.steps, 3)):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            e0.record(stream)
            for d_, h_ in ((q, hq), (k, hk), (v, hv), (g, hg), (beta, hb), (state, hs)):
                d_.copy_(h_, non_blocking=True)
            run()
            ho.copy_(o, non_blocking=True)
            hs_out.copy_(state, non_blocking=True)
            e1.record(stream)
        e1.synchronize()
        if i:
            e2e_ms.append(e0.elapsed_time(e1))
    dev_ms = max_over_ranks(sum(ms) / len(ms), dist, local)
    e2e = max_over_ranks(sum(e2e_ms) / len(e2e_ms), dist, local)
    if rank != 0:
        return
    hbm, _, src = peaks()
    achieved = CFG3_BYTES / (dev_ms / 1000.0) / 1e9
    toks = B * T
    in_bytes = sum(t.numel() * 4 for t in (hq, hk, hv, hg, hb, hs))
    line = _line(args, world, "DeltaNet scan tok/s (cfg3: 64 x 4096 tokens x 16 heads)",
                 world * toks / (dev_ms / 1000.0), "tok/s", dev_ms, _cfg3_config(world), dtype="f32",
                 e2e={"value": world * toks / (e2e / 1000.0), "unit": "tok/s", "h2d_bytes_per_step": in_bytes,
                      "d2h_bytes_per_step": (ho.numel() + hs_out.numel()) * 4, "ms_per_step": e2e},
                 roofline={"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                           "frac": achieved / hbm, "traffic": None,
                           "kernel": "the chunked delta rule call (delta_chunk_prep, delta_chunk_scan, "
                                     "delta_chunk_out), events around the call on its stream; achieved = "
                                     f"{CFG3_BYTES / 1e9:.2f} GB algorithmic bytes per call / call time",
                           "ms_per_launch": dev_ms, "peak_source": f"{src} HBM copy bandwidth"},
                 gpu_launches=int(launches), clocks=clocks.summary(), promotion=None)
    if world == 1 and not args.no_cpu:
        v_, u, c, smp = _cpu_cfg3()
        line["cpu_baseline"] = {"value": v_, "unit": u, "cores": c, "kind": "port", "sample": smp}
    print(json.dumps(line), flush=True)


def _cfg4_requests(vocab, seed):
    """3584-token state prefix + 8 questions of 64 tokens, kinds mixed
    (noul 2 options, choice 4, score 5), option positions in each question's
    last 16 tokens."""
    rng = np.random.default_rng(seed)
    state = rng.integers(0, vocab, 3584)
    qs = []
    for i in range(8):
        n_opt = (2, 4, 5)[i % 3]
        qs.append((rng.integers(0, vocab, 64), [48 + 2 * j for j in range(n_opt)]))
    return state, qs


def _cfg5_sample(vocab, count, seed=0):
    """The first `count` requests of config 5's seeded draw: bound length
    L ~ U[128, 4096], 1-4 questions of 64 tokens; a request with one question
    is one forward of L tokens, otherwise an (L - 64)-token state and its
    questions."""
    rng = np.random.default_rng(seed)
    Ls = rng.integers(128, 4097, 8192)
    qn = rng.integers(1, 5, 8192)
    reqs, tokens = [], []
    for i in range(count):
        r = np.random.default_rng(seed * 100003 + i + 1)
        L, q = int(Ls[i]), int(qn[i])
        kinds = [(2, 4, 5)[(i + j) % 3] for j in range(q)]
        if q == 1:
            reqs.append({"questions": [(r.integers(0, vocab, L), [L - 16 + 2 * j for j in range(kinds[0])])]})
            tokens.append(L)
        else:
            qs = [(r.integers(0, vocab, 64), [48 + 2 * j for j in range(k)]) for k in kinds]
            reqs.append({"state": r.integers(0, vocab, L - 64), "questions": qs})
            tokens.append(L - 64 + 64 * q)
    return reqs, tokens, Ls[:count]


def _model_for(args, local, max_tokens):
    from decider_gpu import GpuModel
    cfg = cfg2(args.layers)
    cfg["vocab_size"] = args.vocab
    t0 = time.time()
    model = GpuModel(cfg, "int8-compute", 32, 2.0, 256, local, max_tokens)
    model.fill_synthetic(seed=0, stddev=0.02)
    model.finalize()
    assert model.fast_path
    model.set_exact(args.exact)
    return model, time.time() - t0


def run_batch(args, world, rank, local, dist, which):
    """Configs 4 and 5 through dg_logits_batch: value from the device time
    of every forward (request_ms), e2e from the wall time of the batch call
    (host ids in, host logits out), roofline from the projection launches of
    layers 0-3 in every forward."""
    import torch

    import decider_gpu
    from decider_gpu.sharding import RequestShape, request_cost, shard_requests
    torch.cuda.set_device(local)
    model, setup_s = _model_for(args, local, 4096)
    if which == "cfg4":
        state, qs = _cfg4_requests(args.vocab, 1000 + rank)
        mine = [{"state": state, "questions": qs}]
        tokens_mine = 4096
        tokens_all = world * 4096
        config = {"workload": "cfg4: 2B decider, one 3584-token state prefix then 8 questions x 64 tokens "
                              "(noul/choice(4)/score(5) mixed) continuing from its cached K/V and DeltaNet state; "
                              "one request per rank",
                  "tokens_per_step": 4096, "parallelism": f"dp{world}",
                  "l2": "not flushed: every forward streams 1.4 GB of int8 weights, > 126 MB L2"}
        scaling = "weak"
    else:
        reqs, toks, _ = _cfg5_sample(args.vocab, args.requests)
        shapes = [RequestShape(len(r.get("state", ())), tuple(len(q[0]) for q in r["questions"])) for r in reqs]
        plan = shard_requests([request_cost(s) for s in shapes], world)
        mine = [reqs[i] for i in plan[rank]]
        tokens_mine = sum(toks[i] for i in plan[rank])
        tokens_all = sum(toks)
        config = {"workload": f"cfg5: the first {args.requests} requests of the seeded 8192-request draw "
                              "(L ~ U[128,4096], 1-4 questions of 64 tokens), LPT-sharded over the ranks",
                  "tokens_per_step": tokens_all, "requests": args.requests, "parallelism": f"dp{world}",
                  "l2": "not flushed: every forward streams 1.4 GB of int8 weights, > 126 MB L2"}
        scaling = "strong"
        # Every rank derives the same plan: the share of each rank, for the report.
        shard = {"tokens_per_rank": [int(sum(toks[i] for i in p)) for p in plan],
                 "requests_per_rank": [len(p) for p in plan]}
    lanes = args.lanes if which == "cfg5" else 1
    model.set_lanes(lanes)
    model.gemm_timing_layers(0, min(4, args.layers))
    for _ in range(args.warmup):
        _, st, _, err = model.logits_batch(mine)
        assert not st.any(), err
    g0_ms, g0_ops, g0_n = model.gemm_time()
    barrier(dist, local)
    n0 = decider_gpu.launch_count()
    dev, wall, per_req = [], [], []
    with ClockSampler(local) as clocks:
        for _ in range(args.steps):
            t0 = time.perf_counter()
            _, st, ms, err = model.logits_batch(mine)
            wall.append((time.perf_counter() - t0) * 1000.0)
            assert not st.any(), err
            dev.append(model.last_batch_ms())
            per_req += [float(x) for x in ms]
    launches = decider_gpu.launch_count() - n0
    barrier(dist, local)
    g_ms, g_ops, g_n = model.gemm_time()
    g_ms, g_ops, g_n = g_ms - g0_ms, g_ops - g0_ops, g_n - g0_n
    alone = None
    if lanes > 1:
        # The projection with no other lane beside it: one untimed one-lane
        # pass over up to 32 of this rank's requests, after the timed region.
        model.set_lanes(1)
        a0 = model.gemm_time()
        _, st, _, err = model.logits_batch(mine[:32])
        assert not st.any(), err
        a1 = model.gemm_time()
        alone = ((a1[0] - a0[0]), (a1[1] - a0[1]), (a1[2] - a0[2]))
    model.gemm_timing(False)
    my_ms = sum(dev) / len(dev)
    rank_ms = [my_ms]
    if dist is not None:
        t = torch.zeros(world, dtype=torch.float64, device=f"cuda:{local}")
        t[rank] = my_ms
        dist.all_reduce(t)
        rank_ms = [float(x) for x in t.cpu()]
    dev_ms = max_over_ranks(my_ms, dist, local)
    e2e_ms = max_over_ranks(sum(wall) / len(wall), dist, local)
    per_req.sort()
    p50 = max_over_ranks(per_req[len(per_req) // 2], dist, local)
    p99 = max_over_ranks(per_req[min(len(per_req) - 1, (99 * len(per_req)) // 100)], dist, local)
    if rank != 0:
        return
    _, bf16, src = peaks()
    peak = 2.0 * bf16
    achieved = g_ops / (g_ms / 1000.0) / 1e12 if g_ms > 0 else 0.0
    i8_loop, i8_loop_ms = decider_gpu.measure_i8_peak(local)
    n_ids = sum(len(r.get("state", [])) + sum(len(q[0]) for q in r["questions"]) for r in mine)
    n_logits = sum(len(q[1]) for r in mine for q in r["questions"])
    metric = METRIC if which == "cfg5" and args.default_line else f"prefill tok/s at 2B INT8 ({which})"
    line = _line(args, world, metric, tokens_all / (dev_ms / 1000.0), "tok/s",
                 dev_ms, dict(config, setup_s=round(setup_s, 1)),
                 e2e={"value": tokens_all / (e2e_ms / 1000.0), "unit": "tok/s", "h2d_bytes_per_step": n_ids * 4,
                      "d2h_bytes_per_step": n_logits * 4, "ms_per_step": e2e_ms},
                 roofline={"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TOP/s",
                           "frac": achieved / peak, "traffic": GEMM_TRAFFIC_BYTES_PER_LAUNCH,
                           "kernel": "gemm_i8_g64_kernel, the projection launches of layers 0-3 in every forward "
                                     "the engine's own lane ran in the timed steps (achieved = sum 2*M*N*K / sum "
                                     "event time)",
                           "launches": int(g_n), "ms_per_launch": g_ms / max(g_n, 1),
                           "peak_source": f"2 x {src} bf16 dense ({bf16} TF/s): int8 dense is twice bf16",
                           "lanes": lanes,
                           "i8_loop_peak": i8_loop, "frac_of_i8_loop": achieved / i8_loop if i8_loop else None,
                           "i8_loop": "dg_measure_i8_peak: one CTA per SM issuing back-to-back "
                                      f"tcgen05.mma.kind::i8 128x256x32 ({i8_loop_ms:.1f} ms launch), after the "
                                      "timed region"},
                 latency={"p50_ms": p50, "p99_ms": p99, "requests": len(per_req),
                          "what": "device time of one request's forwards, max over ranks"},
                 gpu_launches=int(launches), clocks=clocks.summary(), scaling=scaling)
    line["config"]["tokens_rank0"] = tokens_mine
    line["config"]["lanes"] = lanes
    if alone is not None and alone[0] > 0:
        a_ach = alone[1] / (alone[0] / 1000.0) / 1e12
        line["roofline"]["alone"] = {
            "achieved": a_ach, "frac": a_ach / peak, "launches": int(alone[2]),
            "what": f"the same projection launches timed with no other lane running (one untimed one-lane pass "
                    f"over up to 32 requests after the timed region); with {lanes} lanes a projection shares "
                    "the SMs with the other lanes' kernels, so its live launch time is longer"}
    if which == "cfg5":
        tot = sum(shard["tokens_per_rank"])
        line["sharding"] = dict(shard, device_ms_per_rank=rank_ms,
                                worst_rank_token_share=max(shard["tokens_per_rank"]) / tot,
                                ideal_share=1.0 / world,
                                time_imbalance=max(rank_ms) / (sum(rank_ms) / len(rank_ms)),
                                how="LPT over a token + window^2 + per-forward cost model "
                                    "(decider_gpu.sharding.shard_requests); no collective on the data path")
    if world == 1 and not args.no_cpu:
        line["cpu_baseline"] = _cpu_forward_baseline(args, note=" (from an empty cache: a short context, which "
                                                                "favours the CPU)")
    print(json.dumps(line), flush=True)


def run_reference_workload(args, world, rank, which):
    """`--impl reference` for configs 1, 3, 4 and 5: the oracle's CPU path on
    rank 0's host cores, one bounded sample per step."""
    if rank != 0:
        return
    vals = []
    cf = None
    for i in range(args.warmup + args.steps):
        if which == "cfg1":
            v, u, c, smp = _cpu_cfg1()
            config = _cfg1_config(world)
            metric = "INT8 GEMM TOP/s (cfg1: 512x6144x2048, group-64)"
        elif which == "cfg3":
            v, u, c, smp = _cpu_cfg3()
            config = _cfg3_config(world)
            metric = "DeltaNet scan tok/s (cfg3: 64 x 4096 tokens x 16 heads)"
        else:
            if cf is None:
                cf = CpuForward(args.cpu_tokens)
            v, u, c = cf.tokens / cf.time(), "tok/s", cf.threads
            smp = cf.describe()
            config = {"workload": f"{which} sample: 2B decider forward (24 layers, LoRA r32) over {cf.tokens} tokens "
                                  "+ pointer head, int8-compute, from an empty cache",
                      "tokens_per_step": cf.tokens, "parallelism": "rank 0 host cores"}
            metric = METRIC if which == "cfg5" and args.default_line else f"prefill tok/s at 2B INT8 ({which})"
        if i >= args.warmup:
            vals.append(v)
    v = sum(vals) / len(vals)
    extra = {}
    if cf is not None:
        # Mean step time of the timed CPU forwards (the value is tokens / that time, averaged).
        extra["ms_per_step"] = 1000.0 * sum(cf.tokens / x for x in vals) / len(vals)
    print(json.dumps({
        "impl": "reference", "metric": metric, "value": v, "unit": u, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, **extra, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "data": "synthetic", "config": config,
        "note": "the reference's CPU algorithm (oracle restatement) on rank 0's host cores",
        "cpu_baseline": {"value": v, "unit": u, "cores": c, "kind": "port", "sample": smp},
        "e2e": {"value": v, "unit": u, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--latency-calls", type=int, default=100, help="warm dg_logits calls timed for p50/p99")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-tokens", type=int, default=32,
                    help="tokens of the CPU forward per step (cpu_baseline and the reference arm)")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--exact", action="store_true",
                    help="reference-order FP32 promotion instead of fused multiply-add")
    ap.add_argument("--layers", type=int, default=24,
                    help="fewer layers (multiple of 4) for small ncu captures; the bench line is 24")
    ap.add_argument("--vocab", type=int, default=248320,
                    help="smaller embedding table for small ncu captures; the bench line is 248320")
    ap.add_argument("--workload", default=None, choices=["cfg2", "cfg1", "cfg3", "cfg4", "cfg5"],
                    help="BASELINE config to measure; the default line is cfg5 (256 requests, LPT-sharded over the "
                         "ranks)")
    ap.add_argument("--requests", type=int, default=256, help="cfg5: requests taken from the seeded draw")
    ap.add_argument("--lanes", type=int, default=2,
                    help="cfg5: engines per GPU sharing one copy of the weights (dg_engine_set_lanes)")
    args = ap.parse_args()
    args.default_line = args.workload is None
    if args.workload is None:
        args.workload = "cfg5"
    if args.layers % 4 or args.layers <= 0:
        ap.error("--layers must be a positive multiple of 4")
    world, rank, local, dist = dist_setup()
    try:
        if args.impl == "reference":
            if args.workload == "cfg2":
                run_reference(args, world, rank, local, dist)
            else:
                run_reference_workload(args, world, rank, args.workload)
        elif args.workload == "cfg1":
            run_cfg1(args, world, rank, local, dist)
        elif args.workload == "cfg3":
            run_cfg3(args, world, rank, local, dist)
        elif args.workload in ("cfg4", "cfg5"):
            run_batch(args, world, rank, local, dist, args.workload)
        else:
            run_ours(args, world, rank, local, dist)
    finally:
        if dist is not None:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
