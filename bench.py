#!/usr/bin/env python
"""Benchmark of scratchtape-b200's hot path; prints ONE JSON line (rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c2|c1|c3|c5] [--impl ours|reference]

Default workload ("C2"): one byte-level-transformer MLP
layer forward + backward as six f32 GEMMs -- tokens M = 32 x 128 = 4096,
d_model 128, d_ff 512; X ~ N(0,1), W1/W2 Xavier-uniform, dY ~ N(0, 1e-2) --
run on the tcgen05 TF32 tensor cores.  A step is those six GEMMs (NN
forward, NT dX, TN dW) over one batch.  The inputs (25 MB) fit in L2, so L2
is flushed (a 160 MB write, more than the 126 MB L2) before every timed step,
outside its events.

``value``: TFLOP/s of the whole job with inputs resident in HBM, the step
replayed from a CUDA graph, timed by CUDA events per step (flush excluded),
max over ranks.  ``e2e``: the same metric through the public host-array API
(scratchtape_b200.mlp.forward_backward_host): pinned host inputs copied in,
six GEMMs, gradients copied out, every step.  ``roofline``: the TF32 GEMM
kernel's algorithmic bytes per launch over its CUDA-event duration (cold L2),
against the measured HBM copy bandwidth.  ``cpu_baseline``: the CPU oracle
(restated tensor.rs matmul, one thread like the reference) on one full step.

``--impl reference`` times that CPU restatement of the reference's path with
all host threads on the same workload (rank 0 only under torchrun).

Multi-GPU: the GEMMs of one layer do not shard (replicas only); with N ranks
each GPU runs its own replica and value is the sum over GPUs.
"""
import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "GEMM TFLOP/s & % of B200 peak per layout; kNN keys/s vs HBM; vs CPU tensor.rs"
PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
C2 = dict(m=32 * 128, d=128, dff=512)
C5 = dict(keys=1 << 27, d=256, nq=4096, k=128)
# The reference's IVF search as it quotes it (16384 queries x 8 probes over a
# 37M-key store, docs/tiers_design.md:1468; 12288 cells, README.md:76-85)
C5_IVF = dict(keys=37_000_000, nlist=12288, nprobe=8, nq=16384, clusters=12288, noise=0.5)
# dram__bytes_read.sum + dram__bytes_write.sum per k_gemm_tf32 launch of the six-launch C2 step, from one ncu
# capture: H = relu(X W1) 2.43 MB, Y = H W2 8.72 MB, dW2 = H^T dY 10.56 MB (writes stay in L2); the mean
C2_TRAFFIC_PER_LAUNCH = (2.430208e6 + 8.721408e6 + 10.557184e6) / 3
# DRAM bytes (read + write) of one k_attn_fwd + one k_attn_bwd launch at C3, from one ncu capture
C3_TRAFFIC_PER_STEP = 6.320128e6 + 10.597888e6
# DRAM bytes (read + write) of one k_mlp_step launch at C2, from one ncu capture
C2_FUSED_TRAFFIC = 4.800256e6 + 5.820416e6
# DRAM bytes of one k_knn_tmem full-pass launch, 4096 queries over 2^24 keys, from one ncu capture (the
# capture-size rule keeps it below the full 2^27): reads 1.312 GB (the 1.14 GB of codes + scales once, the
# rest L2 misses of the 16 query blocks' shared reads), writes 0.225 GB (per-block lists, candidate inserts)
C5_TRAFFIC_READ_2P24, C5_TRAFFIC_WRITE_2P24 = 1.312352512e9, 0.224658176e9


def parse_args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=None, help="timed steps (c2: 200, c5: 5)")
    p.add_argument("--warmup", type=int, default=None, help="warm-up steps (c2: 20, c5: 3)")
    p.add_argument("--config", default="all", choices=["all", "c1", "c2", "c3", "c4", "c5"],
                   help="all (default): the C5 line with c1-c4 sub-objects; cN: that config alone")
    p.add_argument("--prec", default="exact", choices=["exact", "f16"], help="C5 arithmetic")
    p.add_argument("--keys", type=int, default=C5["keys"], help="C5 total key count (all GPUs)")
    p.add_argument("--key-source", default="uniform", choices=["uniform", "rotated"],
                   help="C5 keys: uniform codes with |N(0,1)| scales (BASELINE), or Gaussian vectors rotated on the "
                        "device and run through the 2-bit quantiser (the realistic variant)")
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-ivf", action="store_true", help="C5: skip the IVF search measurement")
    p.add_argument("--no-parity", action="store_true", help="C5: skip the full-size parity check against the oracle")
    p.add_argument("--no-probes", action="store_true",
                   help="C4: skip the large-GEMM and per-GEMM probes (the launches are then the step's alone)")
    p.add_argument("--c2-path", default="fused", choices=["fused", "gemms"],
                   help="C2: the fused one-kernel step, or six separate GEMM launches")
    a = p.parse_args()
    if a.steps is None:
        a.steps = {"c5": 5, "all": 5, "c4": 24}.get(a.config, 200)
    if a.warmup is None:
        a.warmup = {"c5": 3, "all": 3, "c4": 4}.get(a.config, 20)
    return a


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return d, "measured"
    return PEAKS_FALLBACK, "fallback"


class ClockSampler:
    """Samples SM clock and throttle reasons through NVML while running."""

    REASONS = {
        "gpu_idle": 0x1, "applications_clocks_setting": 0x2, "sw_power_cap": 0x4, "hw_slowdown": 0x8,
        "sync_boost": 0x10, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40, "hw_power_brake_slowdown": 0x80,
        "display_clock_setting": 0x100,
    }

    def __init__(self, index, period=0.005):
        self.index, self.period = index, period
        self.samples, self.reasons = [], set()
        self.max_mhz = None
        self._stop = threading.Event()
        self._t = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nvml = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self.nvml = None

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self.nvml.nvmlDeviceGetClockInfo(self.h, self.nvml.NVML_CLOCK_SM))
                mask = self.nvml.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                for name, bit in self.REASONS.items():
                    if mask & bit and name != "gpu_idle":
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self.nvml is not None:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._t is not None:
            self._t.join()

    def summary(self):
        med = float(np.median(self.samples)) if self.samples else None
        return {"sm_mhz": med, "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons), "samples": len(self.samples)}


def dist_setup():
    # NCCL's own log lines (e.g. its version banner) go to stderr, so stdout
    # carries only the one JSON line
    os.environ.setdefault("NCCL_DEBUG_FILE", "/dev/stderr")
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


_PG = {"up": False}


def dist_init():
    """(world, rank, local): the NCCL process group is set up once per process
    (one rank per GPU) and shared by every measurement of the run; with one
    rank there is none."""
    import torch
    import torch.distributed as dist
    world, rank, local = dist_setup()
    if world > 1:
        torch.cuda.set_device(local)
        if not _PG["up"]:
            import datetime
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                    device_id=torch.device("cuda", local))
            _PG["up"] = True
    else:
        torch.cuda.set_device(0)
    return world, rank, local


def dist_close():
    if _PG["up"]:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()
        _PG["up"] = False


def mlp_inputs(torch, device, seed=0):
    """C2 synthetic inputs; seeded torch generator."""
    m, d, dff = C2["m"], C2["d"], C2["dff"]
    g = torch.Generator(device=device)
    g.manual_seed(seed + 1)
    x = torch.randn((m, d), generator=g, device=device)
    lim1 = (6.0 / (d + dff)) ** 0.5
    w1 = (torch.rand((d, dff), generator=g, device=device) * 2 - 1) * lim1
    w2 = (torch.rand((dff, d), generator=g, device=device) * 2 - 1) * lim1
    dy = torch.randn((m, d), generator=g, device=device) * 0.1
    return x, w1, w2, dy


def c2_flops():
    return 6 * 2 * C2["m"] * C2["d"] * C2["dff"]


def c2_bytes():
    """The C2 step's algorithmic bytes, the per-step figure of the north star's
    measurement table: six GEMMs, each reading its two f32 operands and
    writing its f32 result (M.d + d.F + M.F elements)."""
    return 6 * 4 * (C2["m"] * C2["d"] + C2["d"] * C2["dff"] + C2["m"] * C2["dff"])


def c2_unique_bytes():
    """What the fused step must move at least: X, dY, W1, W2 in; H, dH, Y, dX,
    dW1, dW2 out (f32)."""
    m, d, f = C2["m"], C2["d"], C2["dff"]
    return 4 * (2 * m * d + 2 * d * f + 2 * m * f + 2 * m * d + 2 * d * f)


def cpu_step_c2(x, w1, w2, dy, threads):
    """One C2 step on the CPU oracle: the tape's six matmuls (NT/TN through
    explicit transposes, src/tape.rs:505-510), ReLU and its mask."""
    import oracle
    pre = oracle.matmul_layout(x, w1, threads=threads)
    h = np.maximum(pre, np.float32(0))
    oracle.matmul_layout(h, w2, threads=threads)
    dh = oracle.matmul_layout(dy, oracle.transpose(w2), threads=threads)
    dh = np.where(pre > 0, dh, np.float32(0)).astype(np.float32)
    oracle.matmul_layout(oracle.transpose(h), dy, threads=threads)
    oracle.matmul_layout(dh, oracle.transpose(w1), threads=threads)
    oracle.matmul_layout(oracle.transpose(x), dh, threads=threads)


def host_c2_inputs(seed=0):
    rng = np.random.default_rng(seed + 1)
    m, d, dff = C2["m"], C2["d"], C2["dff"]
    lim = (6.0 / (d + dff)) ** 0.5
    x = rng.standard_normal((m, d)).astype(np.float32)
    w1 = rng.uniform(-lim, lim, (d, dff)).astype(np.float32)
    w2 = rng.uniform(-lim, lim, (dff, d)).astype(np.float32)
    dy = (rng.standard_normal((m, d)) * 0.1).astype(np.float32)
    return x, w1, w2, dy


def cpu_baseline_c2():
    x, w1, w2, dy = host_c2_inputs()
    times = []
    t_end = time.perf_counter() + 20.0
    while len(times) < 3 and (not times or time.perf_counter() < t_end):
        t0 = time.perf_counter()
        cpu_step_c2(x, w1, w2, dy, threads=1)
        times.append(time.perf_counter() - t0)
    t = float(np.median(times))
    return {"value": c2_flops() / t / 1e12, "unit": "TFLOP/s", "cores": 1, "kind": "port",
            "sample": "%d full C2 steps (6 GEMMs, tape transposes, ReLU mask) on the oracle's restated "
                      "tensor.rs matmul, 1 thread as the reference runs; median" % len(times),
            "ms_per_step": t * 1e3}


def run_reference(args):
    world, rank, _ = dist_setup()
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    x, w1, w2, dy = host_c2_inputs()
    for _ in range(args.warmup):
        cpu_step_c2(x, w1, w2, dy, threads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        cpu_step_c2(x, w1, w2, dy, threads)
    el = time.perf_counter() - t0
    v = c2_flops() * args.steps / el / 1e12
    line = {
        "impl": "reference", "metric": METRIC, "value": v, "unit": "TFLOP/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": el / args.steps * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "C2 MLP layer fwd+bwd GEMMs, M=4096 (32x128), d_model 128, d_ff 512, f32",
                   "global_batch": 32, "seq_len": 128, "parallelism": "replicas only (CPU, rank 0)"},
        "cpu_baseline": {"value": v, "unit": "TFLOP/s", "cores": threads, "kind": "port",
                         "sample": "full C2 steps on the oracle's restated tensor.rs matmul (row-parallel over %d "
                                   "threads; the reference itself is single threaded)" % threads},
        "e2e": {"value": v, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_ours(args):
    import torch
    import torch.distributed as dist
    world, rank, local = dist_init()
    device = torch.device("cuda", torch.cuda.current_device())
    import scratchtape_b200 as st
    from scratchtape_b200 import mlp

    peaks, peak_src = load_peaks()
    h = st.handle()
    m, d, dff = C2["m"], C2["d"], C2["dff"]
    bufs = mlp.MlpBuffers.allocate(m, d, dff, device)
    x, w1, w2, dy = mlp_inputs(torch, device, seed=rank)
    bufs.x.copy_(x)
    bufs.w1.copy_(w1)
    bufs.w2.copy_(w2)
    bufs.dy.copy_(dy)
    # a write larger than the 126 MB L2 evicts every operand before each timed step
    flush = torch.empty(160 * 1000 * 1000 // 4, dtype=torch.float32, device=device)

    fused = mlp.fused_fits(m, d, dff) and args.c2_path == "fused"
    stream = torch.cuda.Stream(device)
    sides = mlp.StepStreams(device)
    step = (lambda: mlp.forward_backward_fused(bufs)) if fused else \
        (lambda: mlp.forward_backward(bufs, streams=sides))

    # eager warm-up: grows scratch, sets kernel attributes, counts launches
    n0 = h.launches
    mlp.forward_backward_fused(bufs) if fused else mlp.forward_backward(bufs)
    torch.cuda.synchronize()
    launches_per_step = h.launches - n0

    def capture(fn):
        with torch.cuda.stream(stream):
            fn()  # warm on the capture streams
        torch.cuda.synchronize()
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr, stream=stream):
            fn()
        torch.cuda.synchronize()
        return gr

    graph = capture(step)

    def barrier():
        if world > 1:
            dist.barrier()

    for _ in range(args.warmup):
        flush.zero_()
        graph.replay()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    sampler = ClockSampler(local if world > 1 else torch.cuda.current_device())
    barrier()
    torch.cuda.synchronize()
    with sampler:
        for i in range(args.steps):
            flush.zero_()
            starts[i].record()
            graph.replay()
            ends[i].record()
        torch.cuda.synchronize()
    barrier()
    step_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    total_ms = float(sum(step_ms))
    if world > 1:
        t = torch.tensor([total_ms], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms = float(t.item())
    value = c2_flops() * args.steps * world / (total_ms / 1e3) / 1e12

    def replay_ms(gr, reps=20):
        ts = []
        for _ in range(reps):
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            gr.replay()
            e1.record()
            ts.append((e0, e1))
        torch.cuda.synchronize()
        return float(np.mean([a.elapsed_time(b) for a, b in ts]))

    # per-launch roofline, cold L2, algorithmic bytes (the six GEMMs' f32
    # operands and results) / duration: of the fused kernel and its reduction
    # together, or of each of the six GEMMs alone
    per_bytes = mlp.gemm_bytes(m, d, dff)
    bytes_total = float(c2_bytes())
    gemm_ms = []
    if fused:
        fused_ms = replay_ms(graph)
        achieved = bytes_total / (fused_ms / 1e3) / 1e9
        six = capture(lambda: mlp.forward_backward(bufs, streams=sides))
        six_ms = replay_ms(six)
        del six
    else:
        for (a_, b_, o_, mm_, kk_, nn_, epi), nb in zip(mlp.gemm_list(bufs), per_bytes):
            # one GEMM (and its split-k reduce) per graph: no host gaps
            gg = capture(lambda: st.matmul_with(a_, b_, o_, 1, mm_, kk_, nn_, epi, st.TF32))
            gemm_ms.append(replay_ms(gg))
            del gg
        achieved = bytes_total / (sum(gemm_ms) / 1e3) / 1e9
    hbm = float(peaks["hbm_gbs"])

    # e2e through the host-array APIs, pinned host buffers in and out every step:
    # (1) forward_backward_host, one blocking call per step; (2) HostStream,
    # consecutive steps pipelined (uploads, GEMMs and downloads on their own
    # streams), with the L2 flush enqueued on the compute stream before every
    # step, inside the timed region
    hx, hw1, hw2, hdy = (t.cpu().pin_memory() for t in (x, w1, w2, dy))
    outs = tuple(torch.empty(t.shape, dtype=torch.float32, pin_memory=True) for t in (bufs.y, bufs.dx, bufs.dw1,
                                                                                      bufs.dw2))
    for _ in range(max(3, args.warmup // 4)):
        mlp.forward_backward_host(hx, hw1, hw2, hdy, bufs, outs, streams=sides, fused=fused)
    e2e_steps = max(10, min(args.steps, 200))
    e_ms = []
    for _ in range(e2e_steps):
        flush.zero_()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        mlp.forward_backward_host(hx, hw1, hw2, hdy, bufs, outs, streams=sides, fused=fused)
        e1.record()
        e1.synchronize()
        e_ms.append(e0.elapsed_time(e1))
    call_total = float(sum(e_ms))

    pipe = mlp.HostStream(m, d, dff, device, fused=fused)
    pouts = [tuple(torch.empty_like(t).pin_memory() for t in outs) for _ in range(len(pipe.bufs))]

    def pipe_run(steps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record(pipe.up)
        ticket = None
        for i in range(steps):
            with torch.cuda.stream(pipe.comp):
                flush.zero_()
            ticket = pipe.submit((hx, hw1, hw2, hdy), pouts[i % len(pouts)])
        pipe.down.wait_event(ticket)
        e1.record(pipe.down)
        e1.synchronize()
        return e0.elapsed_time(e1)

    pipe_run(max(3, args.warmup // 4))
    barrier()
    e_total = pipe_run(e2e_steps)
    pipe.close()
    if world > 1:
        t = torch.tensor([e_total, call_total], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e_total, call_total = float(t[0].item()), float(t[1].item())
    e2e_value = c2_flops() * e2e_steps * world / (e_total / 1e3) / 1e12
    call_value = c2_flops() * e2e_steps * world / (call_total / 1e3) / 1e12
    h2d = sum(t.numel() * 4 for t in (hx, hw1, hw2, hdy))
    d2h = sum(t.numel() * 4 for t in outs)

    if rank == 0:
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            cpu = cpu_baseline_c2()
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": total_ms / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "tf32", "data": "synthetic",
            "config": {"workload": "C2 MLP layer fwd+bwd GEMMs (BASELINE configs[1]): M=4096 (batch 32 x seq 128), "
                                   "d_model 128, d_ff 512, f32 in/out, TF32 tensor cores; NN fwd, NT dX/dH, TN dW",
                       "global_batch": 32 * world, "seq_len": 128,
                       "parallelism": "replicas only" if world > 1 else "single GPU",
                       "l2": "flushed (a 160 MB write, more than the 126 MB L2) before every timed step: outside "
                             "the events of the device-timed steps, inside the timed region of the pipelined e2e",
                       "graph": "step replayed from one CUDA graph",
                       "step": "fused: the six GEMMs in one tcgen05 kernel (k_mlp_step) with fixed-order "
                               "in-kernel reductions of the per-block partials; H and dH written out too"
                               if fused else "six GEMM launches on three streams"},
            "roofline": ({"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                          "frac": achieved / hbm, "traffic": C2_FUSED_TRAFFIC, "peak_source": peak_src,
                          "traffic_note": "DRAM read+write (dram__bytes_read.sum + dram__bytes_write.sum) of one "
                                          "k_mlp_step launch at the C2 shape, from one ncu --set full capture "
                                          "(one launch, --clock-control none); algorithmic bytes: the six GEMMs' "
                                          "f32 operands and results, 6 x 10.75 MB",
                          "unique_io_bytes": c2_unique_bytes(),
                          "unique_io_frac": c2_unique_bytes() / (fused_ms / 1e3) / 1e9 / hbm,
                          "kernel": "k_mlp_step (one cooperative launch, reductions inside)",
                          "step_us": round(fused_ms * 1e3, 2), "algorithmic_bytes": bytes_total,
                          "per_gemm_bytes": per_bytes,
                          "six_gemm_step_us": round(six_ms * 1e3, 2),
                          "tensor_frac_of_bf16_peak": c2_flops() / (fused_ms / 1e3) / 1e12 /
                          float(peaks["bf16_tflops"])} if fused else
                         {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                          "traffic": C2_TRAFFIC_PER_LAUNCH, "peak_source": peak_src,
                          "traffic_note": "mean DRAM read+write per k_gemm_tf32 launch over the three launches of "
                                          "one ncu capture (H, Y, dW2); algorithmic bytes: the six GEMMs' f32 "
                                          "operands and results, 6 x 10.75 MB (per_gemm_bytes adds the mask read)",
                          "kernel": "k_gemm_tf32 (+k_splitk_reduce)",
                          "per_gemm_us": [round(t * 1e3, 2) for t in gemm_ms],
                          "per_gemm_bytes": per_bytes,
                          "tensor_frac_of_bf16_peak": c2_flops() / (sum(gemm_ms) / 1e3) / 1e12 /
                          float(peaks["bf16_tflops"])}),
            "e2e": {"value": e2e_value, "unit": "TFLOP/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "ms_per_step": e_total / e2e_steps, "steps": e2e_steps,
                    "api": "scratchtape_b200.mlp.HostStream.submit (pinned host arrays; consecutive steps "
                           "pipelined; L2 flushed on the compute stream before every step, inside the timed region)",
                    "blocking_call": {"value": call_value, "unit": "TFLOP/s", "ms_per_step": call_total / e2e_steps,
                                      "api": "scratchtape_b200.mlp.forward_backward_host, one blocking call per "
                                             "step, L2 flushed outside its events"}},
            "gpu_launches": launches_per_step * args.steps,
            "clocks": sampler.summary(),
        }
        if cpu is not None:
            line["cpu_baseline"] = cpu
        return line
    if world > 1:
        del graph
    return None


# ---------------------------------------------------------------------------
# C5: kNN memory scoring, 4096 f32 queries (dim 256) against 2^27 2-bit keys,
# top-128 per query.
# ---------------------------------------------------------------------------
C5_METRIC_UNIT = "keys/s"
C5_DTYPE = {"exact": "f16 query (times a per-query power of two) x 2-bit codes expanded to f16 in TMEM, f32 "
                     "accumulate (tcgen05 kind::f16) as a bounded filter; kept pairs rescored exactly in f64",
            "f16": "f16 query x f16 dequantised keys, f32 accumulate (tcgen05 kind::f16)"}
C5_KERNEL = {"exact": "k_knn_tmem (+k_knn_merge)", "f16": "k_knn_scan (+k_knn_merge)"}
C5_PEAK_NOTE = {"exact": "bf16 dense, sustained; the scan runs tcgen05 kind::f16 with the keys as the TMEM A operand, "
                         "one pass per (query, key) product plus one K = 16 filter MMA per 256 dims",
                "f16": "bf16 dense, sustained; the scan runs tcgen05 kind::f16 on f16 key tiles in shared memory"}


def c5_queries(n, d, seed=0):
    rng = np.random.default_rng(seed + 1)
    return rng.standard_normal((n, d)).astype(np.float32)


def cpu_baseline_c5(prec, threads, sample_q=64, sample_keys=1 << 20):
    """The oracle's brute force (f64, all given threads) on a sample: sample_q
    queries against sample_keys synthetic keys; scaled to keys/s for a
    4096-query batch."""
    import oracle
    rng = np.random.default_rng(7)
    codes = rng.integers(0, 256, (sample_keys, C5["d"] // 4), dtype=np.uint8)
    scales = np.abs(rng.standard_normal(sample_keys)).astype(np.float32)
    q = c5_queries(sample_q, C5["d"])
    t0 = time.perf_counter()
    oracle.knn_topk(codes, scales, q, C5["k"], mode="dot", prec=prec, threads=threads)
    el = time.perf_counter() - t0
    return el, sample_keys * sample_q / C5["nq"] / el


def run_reference_c5(args):
    world, rank, _ = dist_setup()
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    for _ in range(args.warmup):
        cpu_baseline_c5(args.prec, threads, sample_q=8, sample_keys=1 << 16)
    vals = []
    for _ in range(args.steps):
        _, v = cpu_baseline_c5(args.prec, threads, sample_q=32, sample_keys=1 << 18)
        vals.append(v)
    v = float(np.median(vals))
    sample = ("per step 32 queries x 2^18 synthetic 2-bit keys, dim 256, top-128 by exact f64 dot product "
              "(oracle brute force, %d threads); keys/s scaled to a 4096-query batch" % threads)
    line = {
        "impl": "reference", "metric": METRIC, "value": v, "unit": C5_METRIC_UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": C5["keys"] / v * 1e3,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f64", "data": "synthetic",
        "config": {"workload": "C5 kNN scoring: 4096 f32 queries x 2^27 2-bit keys, dim 256, top-128 (sampled)",
                   "parallelism": "CPU, rank 0"},
        "cpu_baseline": {"value": v, "unit": C5_METRIC_UNIT, "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": v, "unit": C5_METRIC_UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def c5_parity_check(d, n_total, out_s, out_i, q_host, device, nq_check=4):
    """The full-size parity spot check: the first `nq_check` queries' top-128
    from the timed scan against the oracle's exact f64 brute force over ALL
    n_total synthetic keys (codes regenerated on the host from the same
    counter-based generator, scales regenerated on the device by the same
    kernel in 2^24-key chunks and copied back).  Bar, as the kNN parity
    tests: indices identical outside tie bands, every returned key's exact
    score within 2 tau of the oracle's score at that rank, every returned
    score within tau of its key's exact score; tau = 2^-20 * sum|q| * 1.5 *
    max scale.  Rank 0 only."""
    import torch
    import oracle
    import scratchtape_b200.knn as K
    t0 = time.perf_counter()
    scales = np.empty(n_total, np.float32)
    chunk = 1 << 24
    for a in range(0, n_total, chunk):
        b = min(n_total, a + chunk)
        _, sc = K.synth_keys(b - a, d, seed=1, first_key=a, device=device)
        scales[a:b] = sc.cpu().numpy()
        del sc
    torch.cuda.empty_cache()
    q = np.ascontiguousarray(q_host[:nq_check])
    threads = os.cpu_count() or 1
    ws, wi = oracle.knn_topk_synth(1, 0, n_total, d, scales, q, C5["k"], threads=threads)
    gs = out_s[:nq_check].cpu().numpy().astype(np.float64)
    gi = out_i[:nq_check].cpu().numpy()
    tau = 2.0 ** -20 * np.abs(q).astype(np.float64).sum(1) * 1.5 * float(scales.max())
    ok, worst, outside = True, 0.0, 0
    for r in range(nq_check):
        exact = oracle.knn_pair_dots_synth(1, 0, d, scales, q, np.full(gi.shape[1], r), gi[r])
        ok &= bool(np.all(np.abs(exact - ws[r]) <= 2 * tau[r] + 1e-30))
        ok &= bool(np.all(np.abs(gs[r] - exact) <= tau[r] + 1e-6 * np.abs(exact)))
        gap_prev = np.r_[np.inf, ws[r][:-1] - ws[r][1:]]
        gap_next = np.r_[ws[r][:-1] - ws[r][1:], np.inf]
        tied = (gap_prev <= 2 * tau[r]) | (gap_next <= 2 * tau[r])
        outside += int(np.sum(gi[r][~tied] != wi[r][~tied]))
        worst = max(worst, float(np.max(np.abs(gs[r] - exact) / tau[r])))
    ok &= outside == 0
    return {"ok": bool(ok), "queries": nq_check, "keys": n_total,
            "ids_differing_outside_tie_bands": outside, "max_score_err_over_tau": worst,
            "oracle_s": time.perf_counter() - t0,
            "how": "oracle brute force (exact f64) over all %d keys for the first %d queries, codes regenerated on "
                   "the host, scales by the device generator; %d threads" % (n_total, nq_check, threads)}


def run_ours_c5(args):
    import torch
    import torch.distributed as dist
    world, rank, local = dist_init()
    device = torch.device("cuda", torch.cuda.current_device())
    import scratchtape_b200 as st
    import scratchtape_b200.knn as K
    from scratchtape_b200 import shard

    peaks, peak_src = load_peaks()
    h = st.handle()
    d, nq, k = C5["d"], C5["nq"], C5["k"]
    n_total = args.keys
    first, last = shard.shard_range(n_total, world, rank)
    n_local = last - first
    if args.key_source == "uniform":
        codes, scales = K.synth_keys(n_local, d, seed=1, first_key=first, device=device)
    else:
        codes, scales = c5_rotated_keys(n_local, d, first, device)
    qh = c5_queries(nq, d)
    q = torch.from_numpy(qh).to(device)
    out_s = torch.empty((nq, k), dtype=torch.float32, device=device)
    out_i = torch.empty((nq, k), dtype=torch.int64, device=device)
    comm = shard.NcclComm() if world > 1 else None

    def step(q_dev):
        # one public call: local scan of this rank's shard; with several ranks
        # the NCCL all-gather of the local best-128 lists, merge and decode
        # inside st_knn_search_sharded
        if comm is not None:
            shard.knn_search_sharded(codes, scales, q_dev, first, k=k, mode="dot", prec=args.prec, comm=comm,
                                     out=(out_s, out_i))
        else:
            K.search(codes, scales, q_dev, k=k, mode="dot", prec=args.prec, out=(out_s, out_i))

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(*vals):
        if world == 1:
            return vals
        t = torch.tensor(vals, device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return tuple(float(x) for x in t.tolist())

    n0 = h.launches
    step(q)
    torch.cuda.synchronize()
    launches_per_step = h.launches - n0
    for _ in range(max(0, args.warmup - 1)):
        step(q)
    torch.cuda.synchronize()

    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    sampler = ClockSampler(local if world > 1 else torch.cuda.current_device(), period=0.05)
    barrier()
    torch.cuda.synchronize()
    with sampler:
        for i in range(args.steps):
            ev[i][0].record()
            step(q)
            ev[i][1].record()
        torch.cuda.synchronize()
    barrier()
    total_ms, = max_over_ranks(float(sum(a.elapsed_time(b) for a, b in ev)))
    ms_per_step = total_ms / args.steps
    value = n_total / (ms_per_step / 1e3)

    # where a step's time goes: the same work as separate library calls with
    # events between them -- the local scan, the all-gather (NCCL), the merge
    # of the world's lists and the decode
    lists = torch.empty((nq, K.KMAX), dtype=torch.int64, device=device)
    gathered = torch.empty((world, nq, K.KMAX), dtype=torch.int64, device=device)
    merged = torch.empty((nq, K.KMAX), dtype=torch.int64, device=device)
    split_steps = 3
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(5)] for _ in range(split_steps)]
    barrier()
    for i in range(split_steps):
        e = evs[i]
        e[0].record()
        K.topk_keys(codes, scales, q, mode="dot", prec=args.prec, index_base=first, out=lists)
        e[1].record()
        if world > 1:
            shard.gather_lists(lists, out=gathered)
        e[2].record()
        if world > 1:
            K.merge_keys(gathered, nq, out=merged)
        e[3].record()
        K.decode(merged if world > 1 else lists, q, k, mode="dot", prec=args.prec, out=(out_s, out_i))
        e[4].record()
    torch.cuda.synchronize()
    parts = [float(np.mean([e[j].elapsed_time(e[j + 1]) for e in evs])) for j in range(4)]
    alone_ms, gather_ms, merge_ms, decode_ms = max_over_ranks(*parts)
    # at N > 1 the timed step's local scan also takes the seed thresholds' maximum over
    # the ranks (inside st_knn_search_sharded); its share is the step less the rest
    scan_ms = max(0.0, ms_per_step - gather_ms - merge_ms - decode_ms) if world > 1 else alone_ms
    split = {"scan_ms": scan_ms, "allgather_ms": gather_ms, "merge_ms": merge_ms, "decode_ms": decode_ms,
             "allgather_bytes_per_rank": nq * K.KMAX * 8,
             "limiter": "the local scan (%s): %.1f %% of a step" % (C5_KERNEL[args.prec].split(" ")[0],
                        100.0 * scan_ms / max(1e-9, scan_ms + gather_ms + merge_ms + decode_ms)),
             "how": ("the all-gather, merge and decode as separate calls (torch all_gather_into_tensor, merge_keys, "
                     "decode) with CUDA events between them, mean of %d, max over ranks; scan_ms: the timed step "
                     "(whose local scan shares the sampling stages' seeds across the ranks) less those; "
                     "scan_ms_unshared: the local scan alone, seeds from this rank's keys only" % split_steps)
                    if world > 1 else
                    "the same step as separate calls (topk_keys, merge_keys, decode) with CUDA events between "
                    "them, mean of %d" % split_steps}
    if world > 1:
        split["scan_ms_unshared"] = alone_ms

    # e2e through the public API: host queries in, host results out, every step
    hq = torch.from_numpy(qh).pin_memory()
    hs = torch.empty((nq, k), dtype=torch.float32).pin_memory()
    hi = torch.empty((nq, k), dtype=torch.int64).pin_memory()
    q2 = torch.empty_like(q)
    e_ms = []
    e2e_steps = max(2, min(args.steps, 5))
    barrier()
    for _ in range(e2e_steps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        q2.copy_(hq, non_blocking=True)
        step(q2)
        hs.copy_(out_s, non_blocking=True)
        hi.copy_(out_i, non_blocking=True)
        e1.record()
        e1.synchronize()
        e_ms.append(e0.elapsed_time(e1))
    e_total, = max_over_ranks(float(sum(e_ms)))
    e2e_value = n_total / (e_total / e2e_steps / 1e3)

    # the host link under the job's own concurrency: every rank copies 64 MiB from pinned
    # host memory to its GPU and back at the same moment (after a barrier), one
    # direction at a time and both at once; GB/s per rank, min and max over ranks --
    # what bounds the e2e lines of the configs whose inputs are copied every step
    link_n = 64 << 20
    hbuf = torch.empty(link_n, dtype=torch.uint8).pin_memory()
    hbuf2 = torch.empty(link_n, dtype=torch.uint8).pin_memory()
    dbuf = torch.empty(link_n, dtype=torch.uint8, device=device)
    dbuf2 = torch.empty(link_n, dtype=torch.uint8, device=device)
    s_up, s_down = torch.cuda.Stream(), torch.cuda.Stream()

    def link_gbs(up, down, reps=3):
        best = float("inf")
        for _ in range(reps):
            barrier()
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            if up:
                with torch.cuda.stream(s_up):
                    dbuf.copy_(hbuf, non_blocking=True)
            if down:
                with torch.cuda.stream(s_down):
                    hbuf2.copy_(dbuf2, non_blocking=True)
            torch.cuda.synchronize()
            best = min(best, time.perf_counter() - t0)
        return link_n / best / 1e9

    link = {}
    for name, up, down in (("h2d", True, False), ("d2h", False, True), ("both_each_way", True, True)):
        v = link_gbs(up, down)
        neg_min, v_max = max_over_ranks(-v, v)
        link[name + "_gbs_min_max"] = [-neg_min, v_max]
    link["how"] = ("64 MiB pinned <-> device copies, all %d ranks at once after a barrier, wall clock around "
                   "the copies (best of 3); both_each_way: the two directions on two streams together" % world)
    del hbuf, hbuf2, dbuf, dbuf2

    # the small pass: 32 queries over the same keys, where the scan would be
    # HBM-bound if it ran at the tensor pipe's full rate (the ridge is ~33
    # queries per pass at 68 B/key); reported against the HBM roofline
    q32 = q[:32].contiguous()
    keys32 = torch.empty((32, K.KMAX), dtype=torch.int64, device=device)
    K.topk_keys(codes, scales, q32, mode="dot", prec=args.prec, index_base=first, out=keys32)
    ev32 = []
    for _ in range(3):
        a32, b32 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a32.record()
        K.topk_keys(codes, scales, q32, mode="dot", prec=args.prec, index_base=first, out=keys32)
        b32.record()
        ev32.append((a32, b32))
    torch.cuda.synchronize()
    ms32, = max_over_ranks(float(np.median([a.elapsed_time(b) for a, b in ev32])))
    bytes32 = n_local * (d / 4 + 4) + 32 * d * 4
    small_pass = {"queries": 32, "scan_ms": ms32, "keys_per_s": n_total / (ms32 / 1e3),
                  "hbm_gbs": bytes32 / (ms32 / 1e3) / 1e9, "hbm_frac": bytes32 / (ms32 / 1e3) / 1e9 /
                  float(peaks["hbm_gbs"]),
                  "note": "the narrow scan (k_knn_narrow: 128 keys per MMA in TMEM, queries as 4 int8 limbs, "
                          "exact integer products), seeded by 1-in-1024 and 1-in-16 tile sample passes, + a "
                          "two-stage k_knn_merge; bytes = codes + scales + queries of one full pass"}

    ivf_pass = None
    if world == 1 and not args.no_ivf:
        ivf_pass = c5_ivf_pass(device, d)

    parity = None
    if args.key_source == "uniform" and not args.no_parity:
        # out_s / out_i hold the last step's results (every rank has the merged list)
        barrier()
        if rank == 0:
            del codes
            torch.cuda.empty_cache()
            parity = c5_parity_check(d, n_total, out_s, out_i, qh, device)
        barrier()
    if comm is not None:
        torch.cuda.synchronize()
        comm.close()

    flops_alg = 2.0 * d * nq * n_local  # per scan launch on this rank
    achieved = flops_alg / (scan_ms / 1e3) / 1e12
    peak = float(peaks.get("bf16_tflops_sustained", peaks["bf16_tflops"]))
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": C5_METRIC_UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": C5_DTYPE[args.prec], "data": "synthetic",
            "config": {"workload": "C5 kNN scoring (BASELINE configs[4]): 4096 f32 queries x 2^27 keys, dim 256, "
                                   "2-bit codes {-3,-1,1,3} x per-key scale, exact dot-product scores, top-128 per "
                                   "query; keys sharded evenly over GPUs (strong scaling), local top-128 "
                                   "all-gathered over NCCL and merged",
                       "keys": n_total, "keys_per_rank": n_local, "queries": nq, "dim": d, "k": k, "prec": args.prec,
                       "key_source": "uniform codes, |N(0,1)| scales" if args.key_source == "uniform" else
                                     "N(0,1) vectors rotated on the device (TF32 GEMM) and 2-bit quantised",
                       "parallelism": "key-sharded x%d (st_knn_search_sharded: scan, ncclAllGather, merge)" % world
                                      if world > 1 else "single GPU (st_knn_search)",
                       "l2": "inputs (%.1f GB of codes + scales) far larger than L2; no flush needed"
                             % (n_total * (d / 4 + 4) / 1e9)},
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                         "frac": achieved / peak,
                         "traffic": (C5_TRAFFIC_READ_2P24 * n_local / float(1 << 24) + C5_TRAFFIC_WRITE_2P24
                                     if args.prec == "exact" else None),
                         "traffic_note": "DRAM read + write of one k_knn_tmem full pass from an ncu capture at "
                                         "2^24 keys x 4096 queries (1.312 GB read, 0.225 GB written), reads "
                                         "scaled by this rank's keys / 2^24, writes (lists, candidate inserts) "
                                         "as captured; algorithmic bytes (codes + scales + queries): %.3g"
                                         % (n_local * (d / 4 + 4) + nq * d * 4),
                         "peak_source": peak_src + " (" + C5_PEAK_NOTE[args.prec] + ")",
                         "kernel": C5_KERNEL[args.prec],
                         "scan_ms": scan_ms, "algorithmic_tflop_per_scan": flops_alg / 1e12,
                         "hbm_gbs": n_local * (d / 4 + 4) / (scan_ms / 1e3) / 1e9,
                         "small_pass": small_pass, "ivf_pass": ivf_pass},
            "time_split": split,
            "host_link": link,
            "parity": parity,
            "e2e": {"value": e2e_value, "unit": C5_METRIC_UNIT, "h2d_bytes_per_step": int(hq.numel() * 4),
                    "d2h_bytes_per_step": int(hs.numel() * 4 + hi.numel() * 8), "ms_per_step": e_total / e2e_steps,
                    "steps": e2e_steps,
                    "api": ("st_knn_search_sharded (shard.knn_search_sharded with an NcclComm)" if world > 1 else
                            "st_knn_search (knn.search)") + " with the keys resident in HBM; pinned host queries "
                           "in, host scores/ids out, every step"},
            "gpu_launches": launches_per_step * args.steps,
            "clocks": sampler.summary(),
        }
        if world == 1 and not args.no_cpu_baseline:
            threads = os.cpu_count() or 1
            el, v = cpu_baseline_c5(args.prec if args.prec == "exact" else "f16", threads)
            line["cpu_baseline"] = {"value": v, "unit": C5_METRIC_UNIT, "cores": threads, "kind": "port",
                                    "sample": "64 queries x 2^20 synthetic keys, exact f64 brute force top-128 "
                                              "(oracle, %d threads), %.1f s; keys/s scaled to a 4096-query batch"
                                              % (threads, el)}
        return line
    return None


# ---------------------------------------------------------------------------
# C3: batched causal attention, f16 storage / f32 accumulation: batch 32,
# 4 heads, head_dim 64, seq 128; forward + backward.
# ---------------------------------------------------------------------------
C3 = dict(b=32, h=4, t=128, d=64)


def c3_flops():
    """Causal count, as BASELINE states it: fwd 2 GEMMs, bwd 4, over the
    t(t+1)/2 visible pairs of each head."""
    bh, t, d = C3["b"] * C3["h"], C3["t"], C3["d"]
    pairs = t * (t + 1) // 2
    return 6 * 2 * bh * pairs * d


def c3_bytes():
    bh, t, d = C3["b"] * C3["h"], C3["t"], C3["d"]
    tile = bh * t * d * 2
    return {"fwd": 4 * tile + bh * t * 4, "bwd": 8 * tile + bh * t * 4}


def c5_ivf_pass(device, d, reps=3):
    """KnnStore::search_ivf at the reference's quoted shape: 16384 queries x 8
    probes over 37M 2-bit keys in 12288 k-means cells (the reference's figure
    is for 4-bit keys).  Keys and queries are seeded clustered synthetics --
    a mixture of 12288 N(0,1) centres plus N(0, 0.5^2) noise, quantised on
    the device -- so the cells are populated as trained hidden states would
    populate them.  ``wall_ms`` is the public call with host queries in and
    host (distance, value) lists out, probe + host unit tables + scan +
    merge + decode, the queries in pinned host memory; ``scan_ms`` the scan +
    merge launch alone (CUDA events)."""
    import torch
    import scratchtape_b200.knn as K
    cfg = C5_IVF
    n, nlist, nprobe, nq = cfg["keys"], cfg["nlist"], cfg["nprobe"], cfg["nq"]
    g = torch.Generator(device=device)
    g.manual_seed(4242)
    centers = torch.randn((cfg["clusters"], d), generator=g, device=device)
    st = K.KnnStore(d, device=device)
    codes = torch.empty((n, d // 4), dtype=torch.uint8, device=device)
    scales = torch.empty(n, dtype=torch.float32, device=device)
    norms = torch.empty(n, dtype=torch.float32, device=device)
    for a in range(0, n, 1 << 22):
        b = min(n, a + (1 << 22))
        idx = torch.randint(0, cfg["clusters"], (b - a,), generator=g, device=device)
        x = centers[idx] + cfg["noise"] * torch.randn((b - a, d), generator=g, device=device)
        c, s_, nm = K.quantize(x)
        codes[a:b].copy_(c)
        scales[a:b].copy_(s_)
        norms[a:b].copy_(nm)
        del x, c, s_, nm
    st.codes, st.scales, st.norms = codes, scales, norms
    st.vals = (torch.arange(n, device=device) & 0xffff).to(torch.int32)
    torch.cuda.synchronize(device)
    t0 = time.perf_counter()
    st.build_ivf(nlist, iters=6)
    torch.cuda.synchronize(device)
    build_s = time.perf_counter() - t0
    qidx = torch.randint(0, cfg["clusters"], (nq,), generator=g, device=device)
    qh = (centers[qidx] + cfg["noise"] * torch.randn((nq, d), generator=g, device=device)).cpu().pin_memory()
    st.search_ivf(qh, nprobe=nprobe, mode="l2")
    torch.cuda.synchronize(device)
    walls = []
    for _ in range(reps):
        t0 = time.perf_counter()
        sc, vals = st.search_ivf(qh, nprobe=nprobe, mode="l2")
        sc.cpu(), vals.cpu()
        walls.append((time.perf_counter() - t0) * 1e3)
    q = qh.to(device)
    iv = st.ivf
    probes = K.probe_cells(q, iv["cent"], iv["cnorm"], nprobe).cpu().numpy()
    uq, ul, uk, n_lists = K.ivf_units_native(probes, iv["starts"],
                                             n_sms=torch.cuda.get_device_properties(device).multi_processor_count)
    out = torch.empty((nq, K.KMAX), dtype=torch.int64, device=device)
    K.scan_units(st.codes, st.scales, q, uq, ul, uk, n_lists, mode="l2", out=out)
    evs = []
    for _ in range(reps):
        a_, b_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a_.record()
        K.scan_units(st.codes, st.scales, q, uq, ul, uk, n_lists, mode="l2", out=out)
        b_.record()
        evs.append((a_, b_))
    torch.cuda.synchronize(device)
    scan_ms = float(np.median([a_.elapsed_time(b_) for a_, b_ in evs]))
    # the reference's own numerics (f16 keys and queries, f32 accumulate): one tensor pass instead of two
    st.search_ivf(qh, nprobe=nprobe, mode="l2", prec="f16")
    torch.cuda.synchronize(device)
    walls16 = []
    for _ in range(reps):
        t0 = time.perf_counter()
        sc, vals = st.search_ivf(qh, nprobe=nprobe, mode="l2", prec="f16")
        sc.cpu(), vals.cpu()
        walls16.append((time.perf_counter() - t0) * 1e3)
    sizes = np.diff(iv["starts"])
    pairs = int(sizes[probes.astype(np.int64)].sum())  # (query, key) scores one call needs
    wall_ms = float(np.median(walls))
    return {"queries": nq, "nprobe": nprobe, "keys": n, "cells": nlist, "mode": "l2", "prec": "exact",
            "wall_ms": wall_ms, "queries_per_s": nq / (wall_ms / 1e3), "scan_ms": scan_ms,
            "wall_ms_f16": float(np.median(walls16)),
            "scored_pairs": pairs, "pairs_per_s_scan": pairs / (scan_ms / 1e3), "units": int(uq.shape[0]),
            "lists_per_query": int(n_lists),
            "cell_keys_min_mean_max": [int(sizes.min()), float(sizes.mean()), int(sizes.max())],
            "build_ivf_s": build_s,
            "reference": "2.05 s per call for 16384 queries x 8 probes over 37M 4-bit keys (RX 9060 XT, Vulkan; "
                         "docs/tiers_design.md:1468); not run here",
            "data": "seeded clustered synthetic keys: %d N(0,1) centres + N(0, %.1f^2) noise, 2-bit quantised on "
                    "the device; queries drawn the same way" % (cfg["clusters"], cfg["noise"])}


def c5_rotated_keys(n, d, first, device, chunk=1 << 22):
    """The realistic C5 keys: N(0,1) vectors, rotated by a random orthogonal
    matrix (keys.random_rotation, tier_eval.rs:1282-1297) with the TF32 GEMM,
    then the 2-bit quantiser -- chunk by chunk on the device."""
    import torch
    import scratchtape_b200.knn as K
    from scratchtape_b200.keys import Whitener, build_keys, random_rotation, rotate_whitener
    from scratchtape_b200.matmul import TF32
    wh = Whitener(np.zeros(d, np.float32), rotate_whitener(np.eye(d, dtype=np.float32), random_rotation(d, 17)),
                  device=device)
    codes = torch.empty((n, d // 4), dtype=torch.uint8, device=device)
    scales = torch.empty(n, dtype=torch.float32, device=device)
    g = torch.Generator(device=device)
    for a in range(0, n, chunk):
        b = min(n, a + chunk)
        g.manual_seed(1000003 + first + a)
        x = torch.randn((b - a, d), generator=g, device=device)
        c, s, _ = build_keys(x, wh, TF32)
        codes[a:b].copy_(c)
        scales[a:b].copy_(s)
    torch.cuda.synchronize(device)
    return codes, scales


def c3_host_inputs(bh, seed=0):
    rng = np.random.default_rng(seed + 3)
    t, d = C3["t"], C3["d"]
    q, k, v = ((rng.standard_normal((bh, t, d)) / 8.0).astype(np.float16) for _ in range(3))
    dout = rng.standard_normal((bh, t, d)).astype(np.float16)
    return q, k, v, dout


def cpu_attn_sample(heads, threads=None):
    import oracle
    q, k, v, dout = (x.astype(np.float32) for x in c3_host_inputs(heads))
    t0 = time.perf_counter()
    oracle.attention_fwd(q, k, v, 0.125)
    oracle.attention_bwd(q, k, v, dout, 0.125)
    return time.perf_counter() - t0


def run_reference_c3(args):
    world, rank, _ = dist_setup()
    if rank != 0:
        return
    heads = 16
    for _ in range(args.warmup):
        cpu_attn_sample(2)
    ts = [cpu_attn_sample(heads) for _ in range(args.steps)]
    el = float(np.median(ts)) * (C3["b"] * C3["h"]) / heads
    v = c3_flops() / el / 1e12
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": "TFLOP/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": el * 1e3, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "C3 causal attention fwd+bwd, B32 H4 T128 D64 (sampled: 16 heads per step)",
                       "parallelism": "CPU, rank 0"},
            "cpu_baseline": {"value": v, "unit": "TFLOP/s", "cores": 1, "kind": "port",
                             "sample": "16 heads of fwd+bwd on the oracle's restated tape attention (f32, 1 thread), "
                                       "scaled to 128 heads"},
            "e2e": {"value": v, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_ours_c3(args):
    import torch
    import torch.distributed as dist
    world, rank, local = dist_init()
    device = torch.device("cuda", torch.cuda.current_device())
    import scratchtape_b200 as st
    from scratchtape_b200.attention import attention_bwd, attention_fwd
    peaks, peak_src = load_peaks()
    h = st.handle()
    bh_all, t, d = C3["b"] * C3["h"], C3["t"], C3["d"]
    from scratchtape_b200.shard import shard_range
    lo, hi = shard_range(bh_all, world, rank)
    bh = hi - lo
    hq, hk, hv, hdo = (torch.from_numpy(x[lo:hi]).pin_memory() for x in c3_host_inputs(bh_all))
    q, k, v, dout = (x.to(device) for x in (hq, hk, hv, hdo))
    o = torch.empty_like(q)
    lse = torch.empty((bh, t), dtype=torch.float32, device=device)
    dq, dk, dv = torch.empty_like(q), torch.empty_like(q), torch.empty_like(q)
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=device)
    scale = 1.0 / 8.0

    def step():
        attention_fwd(q, k, v, scale, True, out=(o, lse))
        attention_bwd(q, k, v, o, dout, lse, scale, True, out=(dq, dk, dv))

    n0 = h.launches
    step()
    torch.cuda.synchronize()
    launches_per_step = h.launches - n0
    stream = torch.cuda.Stream(device)

    def capture(fn):
        with torch.cuda.stream(stream):
            fn()  # warm on the capture stream
        torch.cuda.synchronize()
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr, stream=stream):
            fn()
        torch.cuda.synchronize()
        return gr

    # the step (forward then backward) replayed from one CUDA graph, as C2 and C4 are
    graph = capture(step)
    graph_fwd = capture(lambda: attention_fwd(q, k, v, scale, True, out=(o, lse)))
    graph_bwd = capture(lambda: attention_bwd(q, k, v, o, dout, lse, scale, True, out=(dq, dk, dv)))
    for _ in range(args.warmup):
        flush.zero_()
        graph.replay()
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            dist.barrier()

    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(args.steps)]
    sampler = ClockSampler(local if world > 1 else torch.cuda.current_device())
    barrier()
    torch.cuda.synchronize()
    with sampler:
        for i in range(args.steps):
            flush.zero_()
            ev[i][0].record()
            graph.replay()
            ev[i][1].record()
        torch.cuda.synchronize()
    barrier()
    total_ms = float(sum(a.elapsed_time(b) for a, b in ev))

    def replay_ms(gr, reps=20):
        ts = []
        for _ in range(reps):
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            gr.replay()
            e1.record()
            ts.append((e0, e1))
        torch.cuda.synchronize()
        return float(np.mean([a.elapsed_time(b) for a, b in ts]))

    fwd_ms, bwd_ms = replay_ms(graph_fwd), replay_ms(graph_bwd)
    # the same step launched eagerly (two launches from the host per step), for comparison
    eager = []
    for _ in range(20):
        flush.zero_()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        step()
        e1.record()
        eager.append((e0, e1))
    torch.cuda.synchronize()
    eager_ms = float(np.mean([a.elapsed_time(b) for a, b in eager]))
    if world > 1:
        tt = torch.tensor([total_ms, fwd_ms, bwd_ms, eager_ms], device=device, dtype=torch.float64)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        total_ms, fwd_ms, bwd_ms, eager_ms = (float(x) for x in tt.tolist())
    del graph, graph_fwd, graph_bwd
    value = c3_flops() * args.steps / (total_ms / 1e3) / 1e12

    # e2e through the public API with pinned host tensors copied in and out every
    # step: (1) one blocking fwd + bwd per step; (2) attention.HostStream,
    # consecutive steps pipelined, L2 flushed on its compute stream before every
    # step inside the timed region
    outs = [torch.empty(x.shape, dtype=x.dtype).pin_memory() for x in (q, q, q, q)]
    e_ms = []
    e2e_steps = max(10, min(args.steps, 100))
    barrier()
    for _ in range(e2e_steps):
        flush.zero_()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for src, dst in zip((hq, hk, hv, hdo), (q, k, v, dout)):
            dst.copy_(src, non_blocking=True)
        step()
        for src, dst in zip((o, dq, dk, dv), outs):
            dst.copy_(src, non_blocking=True)
        e1.record()
        e1.synchronize()
        e_ms.append(e0.elapsed_time(e1))
    call_total = float(sum(e_ms))

    from scratchtape_b200.attention import HostStream
    pipe = HostStream(bh, t, scale, True, device)
    pouts = [tuple(torch.empty_like(x).pin_memory() for x in outs) for _ in range(len(pipe.sets))]

    def pipe_run(steps):
        p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        p0.record(pipe.pipe.up)
        ticket = None
        for i in range(steps):
            with torch.cuda.stream(pipe.pipe.comp):
                flush.zero_()
            ticket = pipe.submit((hq, hk, hv, hdo), pouts[i % len(pouts)])
        pipe.pipe.down.wait_event(ticket)
        p1.record(pipe.pipe.down)
        p1.synchronize()
        return p0.elapsed_time(p1)

    pipe_run(3)
    barrier()
    e_total = pipe_run(e2e_steps)
    pipe.close()
    if world > 1:
        tt = torch.tensor([e_total, call_total], device=device, dtype=torch.float64)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        e_total, call_total = float(tt[0].item()), float(tt[1].item())
    call_value = c3_flops() * e2e_steps / (call_total / 1e3) / 1e12
    e2e_value = c3_flops() * e2e_steps / (e_total / 1e3) / 1e12
    by = c3_bytes()
    frac_b = bh / bh_all
    step_ms = total_ms / args.steps
    achieved = (by["fwd"] + by["bwd"]) * frac_b / (step_ms / 1e3) / 1e9
    hbm = float(peaks["hbm_gbs"])
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": total_ms / args.steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f16 storage / f32 accumulate", "data": "synthetic",
            "config": {"workload": "C3 batched causal attention (BASELINE configs[2]): batch 32, 4 heads, head_dim 64, "
                                   "seq 128, Q/K/V ~ N(0,1)/8 in f16, fwd + bwd (dQ, dK, dV); flops counted over the "
                                   "causal pairs", "global_batch": 32, "seq_len": 128,
                       "parallelism": "heads sharded x%d (no collective)" % world if world > 1 else "single GPU",
                       "l2": "flushed (256 MiB write) before every timed step, outside its events",
                       "graph": "forward + backward replayed from one CUDA graph per step"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                         "traffic": C3_TRAFFIC_PER_STEP * frac_b, "peak_source": peak_src,
                         "traffic_note": "DRAM read+write of one k_attn_fwd + one k_attn_bwd launch from one ncu "
                                         "capture (cold caches), per step like achieved",
                         "kernel": "k_attn_fwd + k_attn_bwd",
                         "step_us": step_ms * 1e3, "fwd_us": fwd_ms * 1e3, "bwd_us": bwd_ms * 1e3,
                         "split_note": "fwd_us / bwd_us: each kernel alone, replayed from a graph of its own after "
                                       "an L2 flush (each includes one launch's fixed cost)",
                         "eager_step_us": eager_ms * 1e3,
                         "bytes": {k2: int(v2 * frac_b) for k2, v2 in by.items()},
                         "tensor_frac_of_bf16_peak": c3_flops() * frac_b / (step_ms / 1e3) / 1e12 /
                         float(peaks["bf16_tflops"])},
            "e2e": {"value": e2e_value, "unit": "TFLOP/s", "h2d_bytes_per_step": int(4 * q.numel() * 2),
                    "d2h_bytes_per_step": int(4 * q.numel() * 2), "ms_per_step": e_total / e2e_steps,
                    "steps": e2e_steps, "api": "scratchtape_b200.attention.HostStream.submit (pinned host f16 "
                                               "tensors copied in and out every step; consecutive steps pipelined; "
                                               "L2 flushed on the compute stream before every step, inside the "
                                               "timed region)",
                    "blocking_call": {"value": call_value, "unit": "TFLOP/s", "ms_per_step": call_total / e2e_steps,
                                      "api": "attention_fwd + attention_bwd with copies, one blocking step at a "
                                             "time, L2 flushed outside its events"}},
            "gpu_launches": launches_per_step * args.steps,
            "clocks": sampler.summary(),
        }
        if world == 1 and not args.no_cpu_baseline:
            el = cpu_attn_sample(16) * bh_all / 16
            line["cpu_baseline"] = {"value": c3_flops() / el / 1e12, "unit": "TFLOP/s", "cores": 1, "kind": "port",
                                    "sample": "16 heads of fwd+bwd on the oracle's restated tape attention (f32, 1 "
                                              "thread, as the reference), scaled to 128 heads"}
        return line
    return None


# ---------------------------------------------------------------------------
# C4: full byte-level transformer training step: vocab
# 256, d 256, 4 layers, 4 heads, d_ff 1024, seq 128, batch 64 per GPU,
# pre-LN, learned positions, tied embeddings, CE + Adam; data parallel with
# local-SGD averaging every 8 steps.
# ---------------------------------------------------------------------------
def c4_batch(cfg, seed, step):
    rng = np.random.default_rng(seed * 1000003 + step)
    ids = rng.integers(0, 256, cfg.batch * cfg.t + 1, dtype=np.int32)
    return ids[:-1].copy(), ids[1:].copy()


def cpu_tape_step_c4(cfg):
    """One whole training step of the C4 model on the CPU oracle at batch 1
    (t = 128 tokens), one thread as the reference runs: the embedding; per
    layer the oracle's bitwise block forward (LayerNorm, QKV projection, causal
    softmax attention, output projection + residual, LayerNorm, ReLU FFN +
    residual: src/nn.rs:627-712 on the restated tensor.rs matmul); the final
    LayerNorm, the tied head and the cross-entropy; the backward -- every
    linear's dX and dW GEMM with the tape's explicit transposes
    (src/tape.rs:505-510), the attention backward (restated softmax backward),
    the LayerNorm backwards, the embedding scatter -- and Adam over all
    parameters (src/optim.rs:42-57).  The backward runs on stand-in values of
    the forward's shapes (the arithmetic per element is the same).  Returns
    (seconds of the batch-proportional part, seconds of Adam)."""
    import oracle
    rows, d, f, hh, t = cfg.t, cfg.d, cfg.dff, cfg.heads, cfg.t
    dk = d // hh
    rng = np.random.default_rng(0)
    r = lambda *sh: rng.standard_normal(sh).astype(np.float32) * 0.05
    blocks = [oracle.block_init(oracle.Rng(11 + i), d, hh, f) for i in range(cfg.layers)]
    tok, pos = r(cfg.vocab, d), r(t, d)
    ids = rng.integers(0, cfg.vocab, rows)
    tg = rng.integers(0, cfg.vocab, rows)
    w = {"qkv": r(d, 3 * d), "o": r(d, d), "f1": r(d, f), "f2": r(f, d)}
    acts = {"ln": r(rows, d), "qkv": r(rows, 3 * d), "hid": r(rows, f), "dx": r(rows, d), "att": r(hh, t, dk)}

    def mm_nt(a, b):  # a . b^T through an explicit transpose, as the tape
        return oracle.matmul_layout(a, oracle.transpose(b), threads=1)

    def mm_tn(a, b):
        return oracle.matmul_layout(oracle.transpose(a), b, threads=1)

    def ln_bwd(x, dy):
        mu = x.mean(1, keepdims=True, dtype=np.float32)
        xc = x - mu
        rstd = 1.0 / np.sqrt((xc * xc).mean(1, keepdims=True, dtype=np.float32) + np.float32(1e-5))
        xh = xc * rstd
        return (rstd * (dy - dy.mean(1, keepdims=True) - xh * (dy * xh).mean(1, keepdims=True))).astype(np.float32)

    t0 = time.perf_counter()
    x = tok[ids] + pos
    for p in blocks:
        x = oracle.block_forward(p, x, 1, t, d, hh, f)
    xf = oracle.layernorm_fwd(x, np.ones(d, np.float32), np.zeros(d, np.float32))
    logits = oracle.matmul_layout(xf, oracle.transpose(tok), threads=1)
    z = logits - logits.max(1, keepdims=True)
    pr = np.exp(z)
    pr /= pr.sum(1, keepdims=True)
    dlog = pr.copy()
    dlog[np.arange(rows), tg] -= 1.0
    dlog = (dlog / rows).astype(np.float32)
    mm_tn(dlog, xf)                                   # d tok (head)
    dx = ln_bwd(x, oracle.matmul_layout(dlog, tok, threads=1))
    for _ in range(cfg.layers):
        mm_tn(acts["hid"], dx)                         # dW2
        dh = mm_nt(dx, w["f2"]) * (acts["hid"] > 0)    # dH, ReLU mask
        mm_tn(acts["ln"], dh)                          # dW1
        d1 = ln_bwd(acts["ln"], mm_nt(dh, w["f1"])) + dx
        mm_tn(acts["ln"], d1)                          # dWo
        dm = mm_nt(d1, w["o"])
        a = acts["att"]
        oracle.attention_bwd(a, a, a, dm.reshape(t, hh, dk).transpose(1, 0, 2), 1.0 / dk ** 0.5)
        mm_tn(acts["ln"], acts["qkv"])                 # dWqkv
        dx = ln_bwd(acts["ln"], mm_nt(acts["qkv"], w["qkv"])) + d1
    np.add.at(np.zeros_like(tok), ids, dx)            # embedding backward
    t_rows = time.perf_counter() - t0
    n = sum(b.size for b in blocks) + tok.size + pos.size + 2 * d
    pp, gg, m1, v1 = (r(n) for _ in range(4))
    t0 = time.perf_counter()
    oracle.adam(pp, gg, m1, v1, 1, 1e-3)
    return t_rows, time.perf_counter() - t0


def cpu_baseline_c4(cfg):
    """Seconds of one C4 step on the CPU: cpu_tape_step_c4 at batch 1 with its
    batch-proportional part x batch (64) plus Adam once (median of 3)."""
    ts = [cpu_tape_step_c4(cfg) for _ in range(3)]
    rows = float(np.median([a for a, _ in ts]))
    adam = float(np.median([b for _, b in ts]))
    return rows * cfg.batch + adam


C4_CPU_SAMPLE = ("one whole C4 training step on the CPU oracle at batch 1 (128 tokens), 1 thread as the reference "
                 "runs: embedding, 4 blocks' bitwise forward (LN, QKV, causal softmax attention, projections, FFN), "
                 "final LN, tied head, cross-entropy, the backward's GEMMs (tape transposes), attention and "
                 "LayerNorm backwards, embedding scatter, then Adam over all parameters; the batch-proportional "
                 "part x64 plus Adam once, median of 3")


def run_reference_c4(args):
    world, rank, _ = dist_setup()
    if rank != 0:
        return
    cfg = _lm_config()
    for _ in range(max(1, args.warmup // 4)):
        cpu_baseline_c4(cfg)
    ts = [cpu_baseline_c4(cfg) for _ in range(max(1, min(args.steps, 3)))]
    el = float(np.median(ts))
    v = cfg.flops_per_step() / el / 1e12
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": "TFLOP/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": el * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "C4 training step (sampled at batch 1, x64; Adam once)",
                       "parallelism": "CPU, rank 0"},
            "cpu_baseline": {"value": v, "unit": "TFLOP/s", "cores": 1, "kind": "port", "sample": C4_CPU_SAMPLE},
            "e2e": {"value": v, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def _lm_config():
    """LmConfig without importing the package (the reference arm must not load the library)."""
    class Cfg:
        vocab, d, layers, heads, dff, t, batch = 256, 256, 4, 4, 1024, 128, 64

        def flops_per_step(self):
            rows = self.batch * self.t
            lin = 2 * rows * (self.d * 3 * self.d + self.d * self.d + 2 * self.d * self.dff)
            head = 2 * rows * self.d * self.vocab
            attn = 4 * self.batch * self.heads * (self.t * (self.t + 1) // 2) * (self.d // self.heads)
            return 3 * (self.layers * (lin + attn) + head)
    return Cfg()


def large_gemm_probe(torch, device, peaks):
    """Throughput of the tensor-core GEMM at large M, per layout: bf16 operands
    (ST_PREC_F16, kind::f16, f32 out) at 16384 x 4096 x 4096 and TF32 at
    8192^3 -- the "large-M GEMM" share of the north star's GEMM target, beside
    the C4 step whose own GEMMs are d_model 256 wide.  CUDA events over 10
    back-to-back launches after 3 warm-up launches; operands 160-512 MB (> L2)."""
    import scratchtape_b200 as st
    peak = float(peaks["bf16_tflops"])
    res = {}
    for name, dt, (m, k, n) in (("bf16", torch.bfloat16, (16384, 4096, 4096)), ("tf32", torch.float32, (8192, 8192, 8192))):
        for ta, tb in ((False, False), (False, True), (True, False)):
            a = torch.randn((k, m) if ta else (m, k), device=device).to(dt)
            b = torch.randn((n, k) if tb else (k, n), device=device).to(dt)
            out = torch.empty((m, n), device=device)
            for _ in range(3):
                st.mm(a, b, ta=ta, tb=tb, out=out)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(10):
                st.mm(a, b, ta=ta, tb=tb, out=out)
            e1.record()
            e1.synchronize()
            tf = 2.0 * m * n * k / (e0.elapsed_time(e1) / 10 / 1e3) / 1e12
            res["%s_%s" % (name, "NN" if not (ta or tb) else ("NT" if tb else "TN"))] = {
                "shape": [m, k, n], "tflops": tf, "frac_of_bf16_peak": tf / peak}
            del a, b, out
    res["peak_source"] = "MEASURED_PEAKS.json bf16_tflops (burst, cuBLAS bf16 8192^3)"
    return res


def c4_gemm_breakdown(torch, device, peaks, cfg):
    """Each TF32 GEMM shape of the C4 step at M = batch x seq = 8192 tokens (the
    layer's QKV, output, FFN-in and FFN-out projections, forward NN, input-gradient
    NT and weight-gradient TN) timed alone with CUDA events (10 back-to-back
    launches replayed from one CUDA graph, as the step's are, after 3 eager
    ones; operands resident), against the TF32 dense peak measured here (cuBLAS
    through torch.matmul with TF32 allowed, 8192^3, best of 10) and against the
    HBM time of its f32 operands and result: the bound of a GEMM is the larger
    of flops / TF32 peak and bytes / HBM."""
    import scratchtape_b200 as st
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = True
    x = torch.randn((8192, 8192), device=device)
    y = torch.randn((8192, 8192), device=device)
    for _ in range(3):
        torch.matmul(x, y)
    best = float("inf")
    for _ in range(10):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        torch.matmul(x, y)
        e1.record()
        e1.synchronize()
        best = min(best, e0.elapsed_time(e1))
    torch.backends.cuda.matmul.allow_tf32 = prev
    del x, y
    tf32_peak = 2.0 * 8192 ** 3 / (best / 1e3) / 1e12
    hbm = float(peaks["hbm_gbs"]) * 1e9
    m, d, f = cfg.batch * cfg.t, cfg.d, cfg.dff
    shapes = [("qkv", d, 3 * d), ("out_proj", d, d), ("ffn_in", d, f), ("ffn_out", f, d)]
    rows = []
    for name, k, n in shapes:
        for lay, (mm, kk, nn, ta, tb) in (("fwd NN", (m, k, n, False, False)), ("dX NT", (m, n, k, False, True)),
                                          ("dW TN", (k, m, n, True, False))):
            a = torch.randn((kk, mm) if ta else (mm, kk), device=device)
            b = torch.randn((nn, kk) if tb else (kk, nn), device=device)
            out = torch.empty((mm, nn), device=device)
            side = torch.cuda.Stream(device)
            side.wait_stream(torch.cuda.current_stream(device))
            with torch.cuda.stream(side):
                for _ in range(3):
                    st.mm(a, b, ta=ta, tb=tb, out=out)
            torch.cuda.current_stream(device).wait_stream(side)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=side):
                for _ in range(10):
                    st.mm(a, b, ta=ta, tb=tb, out=out)
            graph.replay()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            graph.replay()
            e1.record()
            e1.synchronize()
            del graph
            us = e0.elapsed_time(e1) / 10 * 1e3
            flops = 2.0 * mm * nn * kk
            byts = 4.0 * (mm * kk + kk * nn + mm * nn)
            bound_us = max(flops / (tf32_peak * 1e12), byts / hbm) * 1e6
            rows.append({"gemm": "%s %s" % (name, lay), "m_k_n": [mm, kk, nn], "us": us,
                         "tflops": flops / (us / 1e6) / 1e12, "frac_of_tf32_peak": flops / (us / 1e6) / 1e12 / tf32_peak,
                         "bound": "hbm" if byts / hbm > flops / (tf32_peak * 1e12) else "tensor",
                         "bound_us": bound_us, "frac_of_bound": bound_us / us})
            del a, b, out
    return {"tf32_peak_tflops": tf32_peak, "tf32_peak_how": "cuBLAS TF32 8192^3 via torch.matmul, best of 10",
            "hbm_gbs": float(peaks["hbm_gbs"]), "gemms": rows}


def run_ours_c4(args):
    import torch
    import torch.distributed as dist
    world, rank, local = dist_init()
    group = dist.group.WORLD if world > 1 else None
    device = torch.device("cuda", torch.cuda.current_device())
    import scratchtape_b200 as st
    from scratchtape_b200.lm import LmConfig, TinyLM
    peaks, peak_src = load_peaks()
    h = st.handle()
    cfg = LmConfig()
    model = TinyLM(cfg, device, seed=0)  # same init on every rank
    n_steps = args.warmup + args.steps
    host = [c4_batch(cfg, rank, i) for i in range(n_steps + 8)]
    ids_d = [torch.from_numpy(a).to(device) for a, _ in host]
    tg_d = [torch.from_numpy(b).to(device) for _, b in host]

    n0 = h.launches
    model.train_step(ids_d[0], tg_d[0], group)
    torch.cuda.synchronize()
    launches_per_step = h.launches - n0
    # the whole step (forward, backward, Adam) replays from one CUDA graph;
    # the local-SGD average runs between replays every sync_every steps
    ids_buf, tg_buf = torch.empty_like(ids_d[0]), torch.empty_like(tg_d[0])
    ids_buf.copy_(ids_d[1])
    tg_buf.copy_(tg_d[1])
    graph = model.capture_step(ids_buf, tg_buf)

    from scratchtape_b200 import shard
    comm = shard.NcclComm() if world > 1 else None
    if comm is not None:
        # NCCL sets up a new communicator's connections on its first collective:
        # do that with a same-size all-reduce now, outside the timed steps
        shard.average_params(torch.zeros_like(model.params), comm=comm)
        torch.cuda.synchronize()
    avg_ev = []

    def one_step(i, timed=False):
        ids_buf.copy_(ids_d[i])
        tg_buf.copy_(tg_d[i])
        graph.replay()
        model.step_count += 1
        if comm is not None and model.step_count % cfg.sync_every == 0:
            # local SGD: the model average over the ranks, st_avg_params (NCCL all-reduce + divide)
            if timed:
                a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a0.record()
            shard.average_params(model.params, comm=comm)
            if timed:
                a1.record()
                avg_ev.append((a0, a1))
        return model.loss

    for i in range(2, args.warmup):
        one_step(i)
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            dist.barrier()

    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    sampler = ClockSampler(local if world > 1 else torch.cuda.current_device())
    losses = []
    barrier()
    torch.cuda.synchronize()
    with sampler:
        for i in range(args.steps):
            ev[i][0].record()
            loss = one_step(args.warmup + i, timed=True)
            ev[i][1].record()
            losses.append(loss.clone())
        torch.cuda.synchronize()
    barrier()
    total_ms = float(sum(a.elapsed_time(b) for a, b in ev))
    avg_ms = float(sum(a.elapsed_time(b) for a, b in avg_ev))
    if world > 1:
        tt = torch.tensor([total_ms, avg_ms], device=device, dtype=torch.float64)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        total_ms, avg_ms = (float(x) for x in tt.tolist())
    ms = total_ms / args.steps
    value = cfg.flops_per_step() * world / (ms / 1e3) / 1e12
    tokens_s = cfg.batch * cfg.t * world / (ms / 1e3)

    # e2e: host bytes in, loss out, every step, through TinyLM.train_step
    hids = [torch.from_numpy(a).pin_memory() for a, _ in host[:8]]
    htg = [torch.from_numpy(b).pin_memory() for _, b in host[:8]]
    hloss = torch.empty(1, dtype=torch.float32).pin_memory()
    e2e_steps = 8
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(e2e_steps):
        ids_buf.copy_(hids[i], non_blocking=True)
        tg_buf.copy_(htg[i], non_blocking=True)
        graph.replay()
        model.step_count += 1
        if comm is not None and model.step_count % cfg.sync_every == 0:
            shard.average_params(model.params, comm=comm)
        hloss.copy_(model.loss, non_blocking=True)
    e1.record()
    e1.synchronize()
    e_ms = e0.elapsed_time(e1)
    if world > 1:
        tt = torch.tensor([e_ms], device=device, dtype=torch.float64)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        e_ms = float(tt.item())
    e2e_value = cfg.flops_per_step() * world * e2e_steps / (e_ms / 1e3) / 1e12
    if comm is not None:
        torch.cuda.synchronize()
        comm.close()
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "tf32 GEMMs, f16-operand attention, f32 elsewhere", "data": "synthetic",
            "config": {"workload": "C4 byte-level transformer training step (BASELINE configs[3]): vocab 256, d 256, "
                                   "4 layers, 4 heads, d_ff 1024, seq 128, batch 64 per GPU, pre-LN, learned "
                                   "positions, tied embeddings, CE + Adam, local-SGD average every 8 steps",
                       "global_batch": cfg.batch * world, "seq_len": cfg.t,
                       "parallelism": "dp%d local SGD (NCCL all-reduce every %d steps)" % (world, cfg.sync_every)
                       if world > 1 else "single GPU",
                       "tokens_per_s": tokens_s, "gemm_flops_per_step": cfg.flops_per_step(),
                       "local_sgd": {"averages_in_timed_steps": len(avg_ev), "average_ms_total": avg_ms,
                                     "share_of_step_time": avg_ms / total_ms if total_ms else 0.0,
                                     "bytes_per_average": model.n_params * 4,
                                     "api": "st_avg_params (ncclAllReduce sum + divide, on the step's stream)"}
                       if world > 1 else None,
                       "loss_first_last": [float(losses[0].item()), float(losses[-1].item())],
                       "l2": "activations (~160 MB) exceed L2; no flush"},
            "roofline": {"bound": "tensor", "achieved": cfg.flops_per_step() / (ms / 1e3) / 1e12,
                         "peak": float(peaks.get("bf16_tflops_sustained", peaks["bf16_tflops"])), "unit": "TFLOP/s",
                         "frac": cfg.flops_per_step() / (ms / 1e3) / 1e12 /
                         float(peaks.get("bf16_tflops_sustained", peaks["bf16_tflops"])),
                         "traffic": None, "peak_source": peak_src + " (bf16 dense, sustained; TF32 peak is lower)",
                         "kernel": "whole step (TF32 GEMMs dominate)"},
            "e2e": {"value": e2e_value, "unit": "TFLOP/s", "h2d_bytes_per_step": int(2 * 4 * cfg.batch * cfg.t),
                    "d2h_bytes_per_step": 4, "ms_per_step": e_ms / e2e_steps, "steps": e2e_steps,
                    "api": "scratchtape_b200.lm.TinyLM.capture_step graph replay (pinned host bytes in, loss out)"},
            "gpu_launches": launches_per_step * args.steps,
            "clocks": sampler.summary(),
            "large_gemm": None if args.no_probes else large_gemm_probe(torch, device, peaks),
        }
        if world == 1:
            line["gemm_breakdown"] = None if args.no_probes else c4_gemm_breakdown(torch, device, peaks, cfg)
        if world == 1 and not args.no_cpu_baseline:
            el = cpu_baseline_c4(cfg)
            line["cpu_baseline"] = {"value": cfg.flops_per_step() / el / 1e12, "unit": "TFLOP/s", "cores": 1,
                                    "kind": "port", "sample": C4_CPU_SAMPLE, "ms_per_step": el * 1e3}
        return line
    return None


# ---------------------------------------------------------------------------
# C1: single f32 GEMMs of Tensor::matmul, 256 x 256 x 256, in the NN, NT and TN
# layouts the tape's backward emits.  A step is the three
# layouts once.
# ---------------------------------------------------------------------------
C1_N = 256


def c1_host(seed=0):
    rng = np.random.default_rng(seed + 1)
    return [(rng.uniform(-1, 1, (C1_N, C1_N)).astype(np.float32), rng.uniform(-1, 1, (C1_N, C1_N)).astype(np.float32))
            for _ in range(3)]


def c1_flops():
    return 3 * 2 * C1_N ** 3


def cpu_c1(threads, reps=3):
    import oracle
    mats = c1_host()
    ts = []
    for _ in range(reps):
        t0 = time.perf_counter()
        for (a, b), (ta, tb) in zip(mats, ((False, False), (False, True), (True, False))):
            # the tape's NT/TN go through an explicit transpose (src/tape.rs:505-510)
            aa = oracle.transpose(a) if ta else a
            bb = oracle.transpose(b) if tb else b
            oracle.matmul_layout(aa, bb, threads=threads)
        ts.append(time.perf_counter() - t0)
    return float(np.median(ts))


def run_reference_c1(args):
    world, rank, _ = dist_setup()
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    cpu_c1(threads, reps=max(1, args.warmup))
    el = cpu_c1(threads, reps=max(3, min(args.steps, 21)))
    v = c1_flops() / el / 1e12
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": "TFLOP/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": el * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "C1 256^3 f32 GEMM x {NN, NT, TN} (tape transposes included)",
                       "parallelism": "CPU, rank 0"},
            "cpu_baseline": {"value": v, "unit": "TFLOP/s", "cores": threads, "kind": "port",
                             "sample": "the three layouts on the oracle's restated tensor.rs matmul, row-parallel over "
                                       "%d threads, median" % threads},
            "e2e": {"value": v, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_ours_c1(args):
    import torch
    import torch.distributed as dist
    world, rank, local = dist_init()
    device = torch.device("cuda", torch.cuda.current_device())
    import scratchtape_b200 as st
    peaks, peak_src = load_peaks()
    h = st.handle()
    mats = c1_host(seed=rank)
    layouts = ((False, False), (False, True), (True, False))
    dev = [(torch.from_numpy(a).to(device), torch.from_numpy(b).to(device)) for a, b in mats]
    outs = [torch.empty((C1_N, C1_N), dtype=torch.float32, device=device) for _ in range(3)]
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=device)

    # the three GEMMs are independent: NN on the current stream, NT and TN on
    # two side streams, each stream with its own handle (own split-k scratch)
    from scratchtape_b200.matmul import MatRef, matmul_with
    from scratchtape_b200.mlp import StepStreams
    sides = StepStreams(device)
    refs = [(MatRef(a, trans=ta), MatRef(b, trans=tb), MatRef(o)) for (a, b), (ta, tb), o in zip(dev, layouts, outs)]

    def step():
        main = torch.cuda.current_stream()
        fork = torch.cuda.Event()
        fork.record(main)
        for s_ in (sides.s1, sides.s2):
            s_.wait_event(fork)
        matmul_with(*refs[0], 1, C1_N, C1_N, C1_N, None, st.TF32)
        for r_, s_, h_ in ((refs[1], sides.s1, sides.h1), (refs[2], sides.s2, sides.h2)):
            with torch.cuda.stream(s_):
                matmul_with(*r_, 1, C1_N, C1_N, C1_N, None, st.TF32, h_)
        for s_ in (sides.s1, sides.s2):
            join = torch.cuda.Event()
            join.record(s_)
            main.wait_event(join)

    def launches():
        return h.launches + sides.h1.launches + sides.h2.launches

    n0 = launches()
    step()
    torch.cuda.synchronize()
    launches_per_step = launches() - n0
    graph = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream(device)
    with torch.cuda.stream(s):
        step()
    torch.cuda.synchronize()
    with torch.cuda.graph(graph, stream=s):
        step()
    for _ in range(args.warmup):
        flush.zero_()
        graph.replay()
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            dist.barrier()

    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    sampler = ClockSampler(local if world > 1 else torch.cuda.current_device())
    barrier()
    torch.cuda.synchronize()
    with sampler:
        for i in range(args.steps):
            flush.zero_()
            ev[i][0].record()
            graph.replay()
            ev[i][1].record()
        torch.cuda.synchronize()
    barrier()
    total_ms = float(sum(a.elapsed_time(b) for a, b in ev))
    # the same three GEMMs as ONE persistent grouped launch (st_gemm_group, the
    # scheduler for tiny shapes): no dependencies, so every tile of all three
    # starts at once
    from scratchtape_b200.matmul import matmul_group
    gsteps = max(20, min(args.steps, 200))
    gr2 = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        matmul_group([(a_, b_, o_, C1_N, C1_N, C1_N, None, ()) for a_, b_, o_ in refs])
    torch.cuda.synchronize()
    with torch.cuda.graph(gr2, stream=s):
        matmul_group([(a_, b_, o_, C1_N, C1_N, C1_N, None, ()) for a_, b_, o_ in refs])
    gev = []
    for i in range(gsteps + 3):
        flush.zero_()
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        g0.record()
        gr2.replay()
        g1.record()
        if i >= 3:
            gev.append((g0, g1))
    torch.cuda.synchronize()
    grouped_ms = float(np.mean([a.elapsed_time(b) for a, b in gev]))
    del gr2
    if world > 1:
        tt = torch.tensor([total_ms, grouped_ms], device=device, dtype=torch.float64)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        total_ms, grouped_ms = (float(x) for x in tt.tolist())
    ms = total_ms / args.steps
    value = c1_flops() * world / (ms / 1e3) / 1e12
    # e2e: the host-array drop-in (gpu_matmul -> st_matmul_host), copies in and out per GEMM
    for _ in range(3):
        for (a, b), (ta, tb) in zip(mats, layouts):
            st.gpu_matmul(a, b, st.TF32, ta=ta, tb=tb)
    e_steps = 20
    barrier()
    t0 = time.perf_counter()
    for _ in range(e_steps):
        for (a, b), (ta, tb) in zip(mats, layouts):
            st.gpu_matmul(a, b, st.TF32, ta=ta, tb=tb)
    e_s = time.perf_counter() - t0
    if world > 1:
        tt = torch.tensor([e_s], device=device, dtype=torch.float64)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        e_s = float(tt.item())
    e2e_value = c1_flops() * world * e_steps / e_s / 1e12
    byts = 3 * 3 * C1_N * C1_N * 4
    achieved = byts / (ms / 1e3) / 1e9
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "tf32", "data": "synthetic",
            "config": {"workload": "C1 Tensor::matmul 256^3 f32 (BASELINE configs[0]) in the NN, NT and TN layouts, "
                                   "TF32 tcgen05; NT/TN by descriptor (no transpose copy)",
                       "parallelism": "replicas only" if world > 1 else "single GPU",
                       "l2": "flushed (256 MiB write) before every timed step, outside its events",
                       "graph": "the three GEMMs replayed from one CUDA graph, on three streams (they are "
                                "independent)"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": float(peaks["hbm_gbs"]), "unit": "GB/s",
                         "frac": achieved / float(peaks["hbm_gbs"]), "traffic": None, "peak_source": peak_src,
                         "kernel": "k_gemm_tf32 (+k_splitk_reduce)", "us_per_gemm": ms * 1e3 / 3,
                         "grouped_step_us": grouped_ms * 1e3,
                         "grouped_tflops": c1_flops() / (grouped_ms / 1e3) / 1e12,
                         "grouped_note": "the three GEMMs in one st_gemm_group launch (k_gemm_group), graph "
                                         "replay, L2 flushed before each, mean of %d" % gsteps},
            "e2e": {"value": e2e_value, "unit": "TFLOP/s", "h2d_bytes_per_step": int(3 * 2 * C1_N * C1_N * 4),
                    "d2h_bytes_per_step": int(3 * C1_N * C1_N * 4), "ms_per_step": e_s / e_steps * 1e3,
                    "steps": e_steps, "timing": "host wall clock (each call copies in, multiplies, copies out, syncs)",
                    "api": "scratchtape_b200.gpu_matmul -> st_matmul_host (the NdArray::matmul drop-in)"},
            "gpu_launches": launches_per_step * args.steps,
            "clocks": sampler.summary(),
        }
        if world == 1 and not args.no_cpu_baseline:
            el = cpu_c1(1)
            line["cpu_baseline"] = {"value": c1_flops() / el / 1e12, "unit": "TFLOP/s", "cores": 1, "kind": "port",
                                    "sample": "the three layouts on the oracle's restated tensor.rs matmul (tape "
                                              "transposes included), 1 thread as the reference runs, median of 3"}
        return line
    return None


# (sub-object, measurement, timed steps, warm-up steps): the configs that ride
# along in the default line, each with its own roofline, cpu_baseline and e2e
SUBS = (("c2", "run_ours", 200, 20), ("c1", "run_ours_c1", 200, 20), ("c3", "run_ours_c3", 200, 20),
        ("c4", "run_ours_c4", 24, 4))


def run_all(args):
    """The default line: BASELINE configs[4] (C5, the 2-bit kNN scan over
    2^27 keys, key-sharded across the ranks with an NCCL all-gather and merge)
    as the headline, and configs[0]-[3] measured in the same run (every rank
    takes part in each) as the sub-objects c1-c4."""
    import copy
    import torch
    a5 = copy.copy(args)
    a5.config = "c5"
    line = run_ours_c5(a5)
    torch.cuda.empty_cache()
    for name, fn, steps, warm in SUBS:
        a = copy.copy(args)
        a.config, a.steps, a.warmup = name, steps, warm
        sub = globals()[fn](a)
        torch.cuda.empty_cache()
        if line is not None and sub is not None:
            sub.pop("metric", None)
            line[name] = sub
    return line


REFERENCE = {"all": "run_reference_c5", "c5": "run_reference_c5", "c1": "run_reference_c1",
             "c2": "run_reference", "c3": "run_reference_c3", "c4": "run_reference_c4"}
OURS = {"all": "run_all", "c5": "run_ours_c5", "c1": "run_ours_c1", "c2": "run_ours", "c3": "run_ours_c3",
        "c4": "run_ours_c4"}


def main():
    args = parse_args()
    if args.impl == "reference":
        globals()[REFERENCE[args.config]](args)  # rank 0 prints its line; other ranks exit at once
        return
    line = globals()[OURS[args.config]](args)
    if line is not None:
        print(json.dumps(line), flush=True)
    dist_close()


if __name__ == "__main__":
    main()
