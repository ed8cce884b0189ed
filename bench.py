"""Benchmark of the quantized-matmul hot path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--no-sub]
                    [--workload llama70b-megatron|llama70b|gemma-q8-sweep|q4-gemv|llama70b-gate|prefill|
                                gemma-decode] [--batch B]

Workloads (synthetic, seeded, weights ~N(0, 0.02)
quantised by this library's bit-exact device quantisers, x ~ N(0, 1)):
  gemma-q8-sweep: the seven Gemma-3-1B projections
      (K->N) 1152->1024 q, 1152->256 k, 1152->256 v, 1024->1152 o,
      1152->6912 gate, 1152->6912 up, 6912->1152 down, Q8_0, each at batch 1
      and batch 8. One step = those 14 GEMVs. 26 distinct weight sets (one per
      Gemma-3-1B layer, 741 MB > L2) are used round-robin, so weights stream
      from HBM every step.
  q4-gemv: Q4_0 [6912 x 1152] x f32 [1152], batch 1, 64 weight
      copies rotated (287 MB > L2).
  llama70b-megatron (default, configs[4]): Q4_0 gate/up 8192->28672, down
      28672->8192, Q8_0 lm_head 8192->128256, batch 1 and 32 (1.5 GB of
      weights per batch) -- the configuration BASELINE defines at 1/2/4/8
      GPUs -- with gate and up fused (SwiGLU epilogue) feeding down directly:
      with N GPUs one all-reduce per FFN and one all-gather for lm_head.
      Bytes are counted as the reference's four GEMVs. The default run (no
      --workload) prints its line with one sub-record per other configuration
      under "workloads" (one GPU): llama70b, gemma-q8-sweep, q4-gemv, prefill,
      gemma-decode at batch 1, 16 and 64, each timed in the same run with its
      own roofline, e2e and CPU baseline; with N GPUs the llama70b record.
  llama70b (configs[4] as written): the same four projections as separate
      GEMVs; with N GPUs gate/up/lm_head column-parallel with an all-gather
      each, down row-parallel with an all-reduce.
  llama70b-gate (one projection of configs[4]): Q4_0 8192->28672, batch 1,
      two weight copies (264 MB > L2); the small case for streaming-kernel
      profiles.
  gemma-decode: one full Gemma-3-1B decode step (random init,
      26 layers, Q4_0 linears, tied Q8_0 lm_head) at position 511 of a
      512-entry KV cache, batch --batch (1, 16, 64); one CUDA graph replay
      per step; metric "decode tokens/s" = batch / step time, roofline over
      the step's weight + KV bytes. N > 1: independent replicas ("weak").
  prefill: Q4_0 [11008 x 4096] x f32 [512 x 4096], one call per
      step on the tensor-core GEMM, six weight copies rotated (152 MB > L2);
      metric "prefill GEMM TFLOP/s" = 2*M*N*K / time, roofline bound "tensor"
      against the measured dense bf16/f16 peak.

Small decode shapes (all of gemma-q8-sweep and q4-gemv) run as one resident
GEMV launch per call; larger ones as an activation-prep launch plus the
streaming GEMV. gpu_launches is counted by the library while one step is
captured.

Metric: the reference's own bandwidth formula (quantize.rs:399-404),
    GB/s = sum over GEMVs of (M*K*4 + N*(K/32)*block_bytes + M*N*4) / time.
With N GPUs the projections are tensor-parallel through the library's own
NCCL communicator (include/qmm_tp.h: column-parallel q/k/v/gate/up/lm_head
joined by an all-gather, row-parallel o/down by an all-reduce; the process
group is gloo, for barriers and the timing max only), total work fixed
("strong" scaling); value is the whole-job rate.

`--impl reference` times the reference's CPU path (the C++ restatement in
oracle/, AVX2+FMA with OpenMP over all host cores; the Rust original cannot be
built here) on the same workload, on rank 0 only.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

Q4_0, Q4_1, Q8_0 = 2, 3, 8
BB = {Q4_0: 18, Q4_1: 20, Q8_0: 34}

WORKLOADS = {
    "gemma-q8-sweep": dict(
        config_index=1,
        projections=[("q", 1152, 1024, Q8_0, "col"), ("k", 1152, 256, Q8_0, "col"), ("v", 1152, 256, Q8_0, "col"),
                     ("o", 1024, 1152, Q8_0, "row"), ("gate", 1152, 6912, Q8_0, "col"),
                     ("up", 1152, 6912, Q8_0, "col"), ("down", 6912, 1152, Q8_0, "row")],
        batches=[1, 8], copies=26, model="Gemma-3-1B projections (26 layers)"),
    "q4-gemv": dict(
        config_index=0, projections=[("ffn_up", 1152, 6912, Q4_0, "col")], batches=[1], copies=64,
        model="Gemma-3-1B FFN up, Q4_0"),
    "llama70b": dict(
        config_index=4,
        projections=[("gate", 8192, 28672, Q4_0, "col"), ("up", 8192, 28672, Q4_0, "col"),
                     ("down", 28672, 8192, Q4_0, "row"), ("lm_head", 8192, 128256, Q8_0, "col")],
        batches=[1, 32], copies=1, model="Llama-3-70B layer set"),
    # the same layer set with Megatron pairing: gate/up column shards fused
    # (SwiGLU epilogue) feed the row-parallel down directly, so N > 1 needs no
    # all-gather between them; bytes are counted as the four reference GEMVs
    "llama70b-megatron": dict(
        config_index=4,
        projections=[("gate+up", 8192, 28672, Q4_0, "gated"), ("down", 28672, 8192, Q4_0, "row_h"),
                     ("lm_head", 8192, 128256, Q8_0, "col")],
        batches=[1, 32], copies=1, model="Llama-3-70B layer set, Megatron-paired FFN (gate/up -> SwiGLU -> down)"),
    "llama70b-gate": dict(
        config_index=4, projections=[("gate", 8192, 28672, Q4_0, "col")], batches=[1], copies=2,
        model="Llama-3-70B FFN gate, Q4_0"),
    "gemma-decode": dict(
        config_index=3, projections=[], batches=[1], copies=1, metric="decode",
        model="Gemma-3-1B architecture, random init: 26 layers, hidden 1152, 4 Q / 1 KV heads of 256, GeGLU 6912, "
              "vocab 262144 tied; linears Q4_0, lm_head Q8_0; KV context 512"),
    # the same decode step sharded over the N GPUs through the library's NCCL
    # communicator: FFN Megatron-paired, lm_head by vocabulary rows, attention
    # replicated (strong scaling: N ranks, one batch)
    "gemma-decode-tp": dict(
        config_index=3, projections=[], batches=[1], copies=1, metric="decode",
        model="Gemma-3-1B architecture as gemma-decode, tensor-parallel over the GPUs"),
    "prefill": dict(
        config_index=2, projections=[("ffn", 4096, 11008, Q4_0, "col")], batches=[512], copies=6,
        model="Llama-7B FFN, Q4_0, 512-token prefill", metric="flops"),
}


def metric_info(wl):
    """(metric, unit, divisor) of a workload: HBM bytes for the GEMV workloads,
    2*M*N*K flops for the prefill GEMM."""
    if wl.get("metric") == "flops":
        return "prefill GEMM TFLOP/s", "TFLOP/s", 1e12
    if wl.get("metric") == "decode":
        return "decode tokens/s", "tokens/s", 1.0
    return "quant GEMV HBM GB/s", "GB/s", 1e9


def work(wl, m, k, n, dt):
    """Algorithmic work of one call in the workload's unit."""
    if wl.get("metric") == "flops":
        return 2.0 * m * k * n
    return alg_bytes(m, k, n, dt)


def alg_bytes(m, k, n, dt):
    return m * k * 4 + n * (k // 32) * BB[dt] + m * n * 4


def gemvs_of(kind):
    """Reference GEMVs one projection stands for (a fused gate/up is two)."""
    return 2 if kind == "gated" else 1


def reference_gemvs(wl):
    """The workload as the reference's independent GEMVs (a fused gate/up pair
    as its gate and up matmuls): what the CPU baseline times."""
    out = []
    for name, k, n, dt, kind in wl["projections"]:
        if kind == "gated":
            out += [("gate", k, n, dt, "col"), ("up", k, n, dt, "col")]
        else:
            out.append((name, k, n, dt, "row" if kind == "row_h" else kind))
    return out


def host_cores():
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def load_peaks(tensor=False):
    """HBM GB/s, or dense bf16/f16 TFLOP/s (burst: the kernel is timed alone),
    from MEASURED_PEAKS.json; else the pool's earlier measurement."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["bf16_tflops"] if tensor else p["hbm_gbs"]), "measured"
    except Exception:
        return (1590.0 if tensor else 6650.0), "fallback"


def profiled_traffic(workload):
    """Per-launch DRAM bytes of the workload's dominant kernel from the committed
    ncu summary (profiles/<kernel>_<workload>.md, line
    'traffic_bytes_per_launch: <n>')."""
    import glob
    for path in sorted(glob.glob(os.path.join(ROOT, "profiles", f"*_{workload}.md"))):
        try:
            for line in open(path):
                if line.strip().startswith("traffic_bytes_per_launch:"):
                    return float(line.split(":", 1)[1])
        except OSError:
            pass
    return None


# ---- clocks ----------------------------------------------------------------------------
class ClockSampler:
    """Samples SM clock and throttle reasons with NVML while running."""

    REASONS = {0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown", 0x4: "sw_power_cap",
               0x80: "hw_power_brake_slowdown"}

    def __init__(self, device_index, period=0.005):
        self.samples = []
        self.reasons = set()
        self.period = period
        self._stop = threading.Event()
        self._h = None
        self.max_mhz = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self._nv = None
        self._t = threading.Thread(target=self._run, daemon=True)

    def _run(self):
        while not self._stop.is_set():
            if self._h is not None:
                try:
                    self.samples.append(self._nv.nvmlDeviceGetClockInfo(self._h, self._nv.NVML_CLOCK_SM))
                    r = self._nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                    for bit, name in self.REASONS.items():
                        if r & bit:
                            self.reasons.add(name)
                except Exception:
                    pass
            time.sleep(self.period)

    def __enter__(self):
        self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        self._t.join(timeout=2)

    def summary(self):
        med = statistics.median(self.samples) if self.samples else None
        return {"sm_mhz": med, "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons),
                "samples": len(self.samples)}


MIN_TIMED_S = 0.25  # every timed region is repeated until the repetitions cover this (>= 20 clock samples)


def timed_regions(enqueue, stream, dev, steps, world, sampler, sync=None):
    """Times `steps` steps with CUDA events on `stream` (enqueue(steps) issues
    them), barrier + synchronize on both sides, max over ranks; the K-step
    region is repeated until the repetitions cover MIN_TIMED_S (at least
    once), and the median repetition is reported. Returns (ms of the median
    region, every region's ms, clock samples taken during the regions).
    `sync` replaces the device synchronize (the tensor-parallel runs wait
    through the communicator, with a time limit)."""
    import torch
    import torch.distributed as dist

    sync = sync or (lambda: torch.cuda.synchronize(dev))

    def barrier():
        if world > 1:
            dist.barrier()

    def one():
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        sync()
        with torch.cuda.stream(stream):
            e0.record(stream)
            enqueue(steps)
            e1.record(stream)
        sync()
        barrier()
        ms = e0.elapsed_time(e1)
        if world > 1:  # the same number of collectives on every rank (host tensors: gloo)
            t = torch.tensor([ms])
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    n_before = len(sampler.samples)
    regions = [one()]
    reps = max(1, int(MIN_TIMED_S * 1e3 / max(regions[0], 1e-3) + 0.999))
    for _ in range(reps - 1):
        regions.append(one())
    n_timed = len(sampler.samples) - n_before
    return statistics.median(regions), regions, n_timed


# ---- our implementation -----------------------------------------------------------------
def run_ours(args, rank, world, local_rank):
    """One GEMV / GEMM workload (args.workload); returns rank 0's JSON record
    (None on other ranks)."""
    import numpy as np
    import torch
    import torch.distributed as dist

    from machinelearning_b200 import _lib
    from machinelearning_b200._lib import SILU
    from machinelearning_b200.fused import fuse_gate_up
    from machinelearning_b200.linear import QuantWeight
    from machinelearning_b200.tp import TpComm

    L = _lib.lib()
    wl = WORKLOADS[args.workload]
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    stream = torch.cuda.Stream(dev)
    sp = ctypes.c_void_p(stream.cuda_stream)
    copies = args.copies or wl["copies"]
    # N > 1: the library's own NCCL communicator (include/qmm_tp.h), non-blocking, bounded waits
    comm = TpComm.from_group(local_rank, timeout_s=120.0) if world > 1 else None

    # ---- weights: this rank's shard of every projection, `copies` layers --------------
    # column-parallel (col, gated): rows [r*N/W, (r+1)*N/W); row-parallel (row,
    # row_h): blocks [r*nb/W, (r+1)*nb/W) of every row
    problems = []  # (name, k_local, n_local, dt, kind, k_full, n_full)
    for name, k, n, dt, kind in wl["projections"]:
        if kind in ("col", "gated"):
            assert n % world == 0 and (kind == "col" or (n // world) % 32 == 0), f"{name}: N={n} over {world}"
            problems.append((name, k, n // world, dt, kind, k, n))
        else:
            assert (k // 32) % world == 0, f"{name}: K={k} blocks not divisible by {world}"
            problems.append((name, k // world, n, dt, kind, k, n))
    if comm is not None and args.join == "peer":
        # joins over peer memory: buffers for the largest joined output
        # (column: [batch][N]; row: every rank's [batch][N] partial)
        cap = max(4 * b * (n if kind in ("col", "gated") else world * n)
                  for b in wl["batches"] for (_, kl, n_l, dt, kind, k, n) in problems)
        enable_peer_or_nccl(comm, cap, args)

    gen = torch.Generator(device=dev)

    def make_weight(seed, dt, nl, kl):
        gen.manual_seed(seed)
        wf = torch.randn(nl * kl, generator=gen, device=dev, dtype=torch.float32) * 0.02
        qb = torch.empty(nl * (kl // 32) * BB[dt], dtype=torch.uint8, device=dev)
        _lib.check(L.qmm_quantize_dev(dt, 0, wf.data_ptr(), wf.numel(), qb.data_ptr(), None, sp))
        stream.synchronize()
        return QuantWeight.from_device(dt, nl, kl, qb)

    weights = []  # [copy][problem] -> QuantWeight (a gate/up pair: the fused weight)
    with torch.cuda.stream(stream):
        for c in range(copies):
            row = []
            for pi, (name, kl, nl, dt, kind, k, n) in enumerate(problems):
                seed = 1000 * c + 17 * pi + 1 + rank * 7919
                if kind == "gated":
                    g, u = make_weight(seed, dt, nl, kl), make_weight(seed + 500, dt, nl, kl)
                    row.append(fuse_gate_up(g, u))
                    g.close()
                    u.close()
                else:
                    row.append(make_weight(seed, dt, nl, kl))
            weights.append(row)
    torch.cuda.synchronize(dev)

    # ---- activations / outputs per (batch, problem) -----------------------------------
    # a row_h projection reads the preceding gated projection's hidden slice
    xs, ys = {}, {}
    for b in wl["batches"]:
        for pi, (name, kl, nl, dt, kind, k, n) in enumerate(problems):
            gen.manual_seed(50000 + 31 * pi + b)
            xs[(b, pi)] = (ys[(b, pi - 1)] if kind == "row_h" else
                           torch.randn(b, kl, generator=gen, device=dev, dtype=torch.float32))
            ys[(b, pi)] = torch.empty(b, nl * (world if kind == "col" else 1), device=dev, dtype=torch.float32)

    # the library's per-stream workspace must exist before graph capture
    need = max(L.qmm_workspace_size(dt, 0, b, nl * gemvs_of(kind), kl) for b in wl["batches"]
               for (_, kl, nl, dt, kind, *_r) in problems)
    _lib.check(L.qmm_reserve_workspace(local_rank, sp, need + (1 << 20)))

    def one_step(c):
        for b in wl["batches"]:
            for pi, (name, kl, nl, dt, kind, k, n) in enumerate(problems):
                w, x, y = weights[c][pi].handle, xs[(b, pi)].data_ptr(), ys[(b, pi)].data_ptr()
                if kind == "gated":
                    _lib.check(L.qmm_gated_forward(w, x, b, y, SILU, sp))
                elif comm is None:
                    _lib.check(L.qmm_linear_forward(w, x, b, y, 0, sp))
                elif kind == "col":
                    _lib.check(L.qmm_tp_column_forward(comm.handle, w, x, b, y, 0, sp))
                else:
                    _lib.check(L.qmm_tp_row_forward(comm.handle, w, x, b, y, 0, sp))

    launches_per_step = None  # counted by the library while one step is captured
    steps_bytes = sum(gemvs_of(kind) * alg_bytes(b, k, n, dt) for b in wl["batches"]
                      for (_, kl, nl, dt, kind, k, n) in problems)
    steps_work = sum(gemvs_of(kind) * work(wl, b, k, n, dt) for b in wl["batches"]
                     for (_, kl, nl, dt, kind, k, n) in problems)
    metric, unit, div = metric_info(wl)

    def sync():
        """Device synchronize; with a communicator, its bounded wait (a stuck
        collective aborts the communicator and raises instead of hanging)."""
        if comm is not None:
            _lib.check(comm.wait(120.0, stream))
        else:
            torch.cuda.synchronize(dev)

    # ---- CUDA graphs ---------------------------------------------------------------------------
    # A timed region of K steps runs step i on weight copy i % copies: whole
    # passes over the copies as one graph each, then one graph of the
    # remaining K % copies steps (copies 0, 1, ...), so a region is at most
    # K // copies + 1 graph launches whatever K is. With N GPUs the joins over
    # peer memory are plain kernels and are captured the same way; NCCL joins
    # (--join nccl) are enqueued directly: the library's NCCL communicator is
    # non-blocking (its launches may complete on NCCL's own thread), which
    # stream capture does not take.
    graphs = {}
    with torch.cuda.stream(stream):
        for c in range(copies):
            one_step(c)  # warm the planner/tensor-map caches outside capture
        sync()
    if comm is not None and args.join != "peer":
        n0 = L.qmm_launch_count()
        with torch.cuda.stream(stream):
            one_step(0)
        sync()
        launches_per_step = L.qmm_launch_count() - n0

        def run_steps(n):
            for i in range(n):
                one_step(i % copies)
    else:
        run_steps = None

        def capture(n):
            g = torch.cuda.CUDAGraph()
            n0 = L.qmm_launch_count()
            with torch.cuda.graph(g, stream=stream):
                for c in range(n):
                    one_step(c)
            return g, L.qmm_launch_count() - n0

        g1, launches_per_step = capture(1)
        graphs[1] = g1
        for n in {copies, args.steps % copies, args.warmup % copies}:
            if n > 1 and n not in graphs:
                graphs[n] = capture(n)[0]
    sync()

    if run_steps is None:
        def run_steps(n):
            """Exactly n steps, step i on weight copy i % copies."""
            for _ in range(n // copies):
                graphs[copies].replay()
            r = n % copies
            if r in graphs:
                graphs[r].replay()
            else:
                for _ in range(r):  # (only for counts no graph was captured for)
                    graphs[1].replay()

    # warm-up
    with torch.cuda.stream(stream):
        run_steps(args.warmup)
    sync()

    # timed regions: K steps each, events on the launching stream, max over
    # ranks, repeated to >= MIN_TIMED_S, median reported
    sampler = ClockSampler(local_rank)
    with sampler:
        with torch.cuda.stream(stream):
            run_steps(max(args.warmup, 3))  # clock soak right before the timed region
        sync()
        ms, regions, n_timed = timed_regions(run_steps, stream, dev, args.steps, world, sampler, sync)
    ms_per_step = ms / args.steps
    value = steps_work * args.steps / (ms / 1e3) / div

    # ---- end to end through the C ABI with host buffers ------------------------------------
    e2e = None if args.no_e2e else run_e2e(args, wl, problems, weights, L, sp, stream, world, dev, copies,
                                                 comm)

    # ---- CPU baseline (rank 0, N=1): the reference path restated in oracle/ -----------------
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(wl, budget_s=args.cpu_seconds)

    peak, peak_kind = load_peaks(tensor=wl.get("metric") == "flops")
    clocks = sampler.summary()
    clocks["samples_in_timed_region"] = n_timed
    # graphs that hold NCCL calls are released before the communicator goes
    graphs.clear()
    if comm is not None:
        sync()
        _lib.check(comm.close())
    line = None
    if rank == 0:
        line = {
            "metric": metric,
            "value": round(value, 1),
            "unit": unit,
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms_per_step, 5),
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": ("f32 activations rounded to f16 x Q4_0 blocks dequantised to f16 (tcgen05 MMA, f32 accumulate)"
                      if wl.get("metric") == "flops" else
                      "f32 activations x Q4_0/Q8_0 blocks (f16 tensor-core MMA, f32 accumulate)"),
            "data": "synthetic: seeded x~N(0,1); weights ~N(0,0.02) quantised on device (bit-exact reference quantiser)",
            "config": {
                "workload": args.workload,
                "baseline_config_index": wl["config_index"],
                "model": wl["model"],
                "projections": [f"{p[0]} {p[5]}->{p[6]}{' x2 (fused, SwiGLU epilogue)' if p[4] == 'gated' else ''} "
                                f"{'Q8_0' if p[3] == Q8_0 else 'Q4_0'} {p[4]}" for p in problems],
                "batches": wl["batches"],
                "parallelism": ((f"tp{world} (libqmm communicator; joins over peer memory: GEMV / GEMM epilogues "
                                 f"store into every rank's buffer over NVLink, one flag-barrier kernel per join)"
                                 if args.join == "peer" else
                                 f"tp{world} (libqmm NCCL communicator: column-parallel all-gather, row-parallel "
                                 f"all-reduce)") if world > 1 else "single"),
                "l2": f"{copies} weight copies rotated" + (" (>L2)" if copies > 1 else "; weights > L2"),
                "algorithmic_bytes_per_step": steps_bytes,
                "algorithmic_flops_per_step": sum(2 * gemvs_of(kind) * b * k * n for b in wl["batches"]
                                                  for (_, kl, nl, dt, kind, k, n) in problems),
                "graph": ("one CUDA graph per pass over the weight copies plus one for the remaining K % copies "
                          "steps (joins over peer memory captured with them); PDL between kernels"
                          if comm is None or args.join == "peer" else
                          "direct launches (non-blocking NCCL communicator; no stream capture); PDL between kernels"),
            },
            "roofline": {
                "bound": "tensor" if wl.get("metric") == "flops" else "hbm",
                "achieved": round(value / world, 1),
                "peak": peak,
                "unit": unit,
                "frac": round(value / world / peak, 4),
                "peak_kind": peak_kind,
                "traffic": profiled_traffic(args.workload),
                "note": "achieved = per-GPU algorithmic work (bytes, or 2*M*N*K flops) / timed-region duration, timed with CUDA events on the "
                        "launching stream: the GEMV launches back to back (plus, for large shapes, their activation-"
                        "prep launches and, for N>1, the collectives); the GEMV kernel is the dominant kernel "
                        "(launch shares under profiles/)",
            },
            "e2e": e2e,
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clocks,
            "timed_regions": {"count": len(regions), "ms_each": [round(r, 4) for r in regions[:8]],
                              "total_ms": round(sum(regions), 3),
                              "rule": f"K-step region repeated to >= {MIN_TIMED_S * 1e3:.0f} ms, median reported"},
        }
        if cpu is not None:
            line["cpu_baseline"] = cpu
    del weights, xs, ys
    torch.cuda.empty_cache()
    return line


def enable_peer_or_nccl(comm, nbytes, args):
    """Joins over peer memory; if their setup fails on this machine (no peer
    access, IPC refused), every rank falls back to NCCL joins together."""
    import torch
    import torch.distributed as dist
    from machinelearning_b200 import _lib
    ok = 1
    try:
        comm.enable_peer(nbytes)
    except _lib.QmmError as e:
        print(f"peer joins unavailable ({e}); joining with NCCL", file=sys.stderr, flush=True)
        ok = 0
    t = torch.tensor([ok])
    dist.all_reduce(t, op=dist.ReduceOp.MIN)
    if int(t.item()) == 0:
        args.join = "nccl"
        if ok:  # this rank's peer buffers stay unused: the forwards join through NCCL
            raise RuntimeError("a peer rank could not set up peer joins; restart with --join nccl")


def run_e2e(args, wl, problems, weights, L, sp, stream, world, dev, copies, comm):
    """Same metric through the host-buffer C-ABI entry point: every call copies
    x in from pinned host memory, runs the GEMV and copies y out (synchronous),
    as a drop-in Linear::forward with host tensors would."""
    import torch
    from machinelearning_b200 import _lib

    if world > 1 or any(p[4] in ("gated", "row_h") for p in problems):
        return e2e_staged(args, wl, problems, weights, L, sp, stream, world, dev, copies, comm)
    hx, hy = {}, {}
    h2d = d2h = 0
    for b in wl["batches"]:
        for pi, (name, kl, nl, dt, kind, k, n) in enumerate(problems):
            hx[(b, pi)] = torch.randn(b, kl).pin_memory()
            hy[(b, pi)] = torch.empty(b, nl).pin_memory()
            h2d += b * kl * 4
            d2h += b * nl * 4
    steps = max(3, min(args.steps, 200))

    def step(c):
        for b in wl["batches"]:
            for pi in range(len(problems)):
                _lib.check(L.qmm_linear_forward_host(weights[c][pi].handle, hx[(b, pi)].data_ptr(), b,
                                                     hy[(b, pi)].data_ptr(), 0, sp))

    for i in range(3):
        step(i % copies)
    t0 = time.perf_counter()
    for i in range(steps):
        step(i % copies)
    dt_s = time.perf_counter() - t0
    work_step = sum(work(wl, b, k, n, d) for b in wl["batches"] for (_, kl, nl, d, kind, k, n) in problems)
    _, unit, div = metric_info(wl)
    return {"value": round(work_step * steps / dt_s / div, 1), "unit": unit, "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h, "steps": steps, "ms_per_step": round(dt_s * 1e3 / steps, 4),
            "path": "qmm_linear_forward_host (C ABI, pinned host x/y, one synchronous call per GEMV)"}


def e2e_staged(args, wl, problems, weights, L, sp, stream, world, dev, copies, comm):
    """Pinned host x -> device -> the library's forward (the tensor-parallel C
    ABI for N > 1) -> pinned host y, every projection of every step; a
    Megatron-paired FFN copies in x and copies out down's y only. Inputs are
    copied in on the compute stream; each result is copied out on a second
    stream as soon as its kernel is done, from one of two device buffers (step
    parity), so the copies of step i overlap the compute of step i + 1 (a
    serving loop's double buffering). The timed region ends when every step's
    results are in host memory."""
    import torch
    import torch.distributed as dist
    from machinelearning_b200 import _lib
    from machinelearning_b200._lib import SILU

    hx, hy, dx, dy = {}, {}, {}, {}
    h2d = d2h = 0
    for b in wl["batches"]:
        for pi, (name, kl, nl, dt, kind, k, n) in enumerate(problems):
            out_n = nl * world if kind == "col" else nl
            for par in (0, 1):
                dy[(b, pi, par)] = torch.empty(b, out_n, device=dev)
            if kind == "row_h":
                for par in (0, 1):
                    dx[(b, pi, par)] = dy[(b, pi - 1, par)]
            else:
                hx[(b, pi)] = torch.randn(b, kl).pin_memory()
                for par in (0, 1):
                    dx[(b, pi, par)] = torch.empty(b, kl, device=dev)
                h2d += b * kl * 4
            if kind != "gated":
                hy[(b, pi)] = torch.empty(b, out_n).pin_memory()
                d2h += b * out_n * 4
    steps = max(3, min(args.steps, 100))
    cs = torch.cuda.Stream(dev)  # device -> host copies
    copied = [None, None]        # per parity: the copy stream's last event of that step

    def step(c, i):
        par = i & 1
        with torch.cuda.stream(stream):
            if copied[par] is not None:  # step i - 2's results have left these buffers
                stream.wait_event(copied[par])
            for b in wl["batches"]:
                for pi, (name, kl, nl, dt, kind, k, n) in enumerate(problems):
                    if (b, pi) in hx:
                        dx[(b, pi, par)].copy_(hx[(b, pi)], non_blocking=True)
                    w, x, y = weights[c][pi].handle, dx[(b, pi, par)].data_ptr(), dy[(b, pi, par)].data_ptr()
                    if kind == "gated":
                        _lib.check(L.qmm_gated_forward(w, x, b, y, SILU, sp))
                    elif comm is None:
                        _lib.check(L.qmm_linear_forward(w, x, b, y, 0, sp))
                    elif kind == "col":
                        _lib.check(L.qmm_tp_column_forward(comm.handle, w, x, b, y, 0, sp))
                    else:
                        _lib.check(L.qmm_tp_row_forward(comm.handle, w, x, b, y, 0, sp))
                    if (b, pi) in hy:
                        done = torch.cuda.Event()
                        done.record(stream)
                        cs.wait_event(done)
                        with torch.cuda.stream(cs):
                            hy[(b, pi)].copy_(dy[(b, pi, par)], non_blocking=True)
        ev = torch.cuda.Event()
        ev.record(cs)
        copied[par] = ev

    def drain():
        if comm is not None:
            _lib.check(comm.wait(120.0, stream))
        cs.synchronize()
        stream.synchronize()

    for i in range(3):
        step(i % copies, i)
    drain()
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    for i in range(steps):
        step(i % copies, i)
    drain()
    if world > 1:
        dist.barrier()
    dt_s = time.perf_counter() - t0
    if world > 1:
        t = torch.tensor([dt_s])
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dt_s = float(t.item())
    work_step = sum(gemvs_of(kind) * work(wl, b, k, n, d) for b in wl["batches"]
                    for (_, kl, nl, d, kind, k, n) in problems)
    _, unit, div = metric_info(wl)
    return {"value": round(work_step * steps / dt_s / div, 1), "unit": unit, "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h, "steps": steps, "ms_per_step": round(dt_s * 1e3 / steps, 4),
            "path": ("pinned host x -> the library's forward on this rank's shard (qmm_tp_* join for N > 1) -> "
                     "pinned host y on a copy stream (two device buffers: step i's copies overlap step i + 1's "
                     "compute); the region ends when every step's results are in host memory")}


# ---- CPU: the reference path restated (oracle/) -------------------------------------------
def cpu_setup(wl, max_rows_frac=1.0, layers=None):
    import numpy as np
    import oracle

    oracle.build()
    oracle.set_isa(True)
    oracle.set_threads(host_cores())
    rng = np.random.default_rng(0)
    layers = layers or min(wl["copies"], 8)
    ws = []
    for c in range(layers):
        row = []
        for name, k, n, dt, kind in reference_gemvs(wl):
            rows = max(32, int(n * max_rows_frac))
            rows = min(rows, n)
            nb = k // 32
            raw = rng.integers(0, 256, size=rows * nb * BB[dt], dtype=np.uint8).reshape(rows * nb, BB[dt])
            d = (rng.uniform(0.5, 1.5, rows * nb) * (0.06 / (127 if dt == Q8_0 else 8))).astype(np.float16)
            raw[:, 0:2] = d.view(np.uint8).reshape(-1, 2)
            row.append((raw.ravel(), rows))
        ws.append(row)
    xs = {(b, i): rng.normal(0, 1, b * p[1]).astype(np.float32)
          for b in wl["batches"] for i, p in enumerate(reference_gemvs(wl))}
    return oracle, ws, xs


def cpu_step(oracle, wl, ws, xs, c):
    bytes_done = 0
    for b in wl["batches"]:
        for i, (name, k, n, dt, kind) in enumerate(reference_gemvs(wl)):
            w, rows = ws[c][i]
            fn = oracle.matmul_f32_q8 if dt == Q8_0 else oracle.matmul_f32_q4
            fn(xs[(b, i)], w, b, k, rows)
            bytes_done += work(wl, b, k, rows, dt)
    return bytes_done


def cpu_row_fraction(wl, budget_step_s):
    """Fraction of each projection's rows one CPU step covers so that the step
    costs about `budget_step_s` (rows are independent dot products, so a row
    subset is a representative sample). Calibrated by timing a small sample."""
    probe = 0.01
    oracle, ws, xs = cpu_setup(wl, probe, layers=1)
    cpu_step(oracle, wl, ws, xs, 0)
    t0 = time.perf_counter()
    cpu_step(oracle, wl, ws, xs, 0)
    t = max(time.perf_counter() - t0, 1e-4)
    return max(0.002, min(1.0, probe * budget_step_s / t))


def cpu_baseline(wl, budget_s=10.0):
    frac = cpu_row_fraction(wl, 0.25)
    oracle, ws, xs = cpu_setup(wl, frac)
    cpu_step(oracle, wl, ws, xs, 0)
    t0 = time.perf_counter()
    done, steps = 0, 0
    while time.perf_counter() - t0 < budget_s:
        done += cpu_step(oracle, wl, ws, xs, steps % len(ws))
        steps += 1
    dt_s = time.perf_counter() - t0
    _, unit, div = metric_info(wl)
    return {"value": round(done / dt_s / div, 4), "unit": unit, "cores": oracle.threads(), "kind": "port",
            "sample": f"{steps} steps over {len(ws)} layer copies, {frac:.3f} of each projection's rows, "
                      f"{dt_s:.1f} s; AVX2+FMA restatement of the reference's CPU path, OpenMP over all cores"}


def run_reference(args, rank, world):
    if rank != 0:
        return
    wl = WORKLOADS[args.workload]
    # each step samples rows so that warmup + steps end within ~2 minutes
    per_step = min(1.0, 100.0 / max(1, args.steps + args.warmup))
    frac = cpu_row_fraction(wl, per_step)
    oracle, ws, xs = cpu_setup(wl, frac)
    for i in range(args.warmup):
        cpu_step(oracle, wl, ws, xs, i % len(ws))
    t0 = time.perf_counter()
    done = 0
    for i in range(args.steps):
        done += cpu_step(oracle, wl, ws, xs, i % len(ws))
    dt_s = time.perf_counter() - t0
    metric, unit, div = metric_info(wl)
    value = done / dt_s / div
    line = {
        "impl": "reference",
        "metric": metric,
        "value": round(value, 4),
        "unit": unit,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(dt_s * 1e3 / args.steps, 3),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "f32 activations x Q4_0/Q8_0 blocks (f32 accumulate)",
        "data": "synthetic: seeded x~N(0,1), random well-formed blocks",
        "config": {"workload": args.workload, "baseline_config_index": wl["config_index"], "model": wl["model"],
                   "batches": wl["batches"], "parallelism": "host cores"},
        "cpu_baseline": {"value": round(value, 4), "unit": unit, "cores": oracle.threads(), "kind": "port",
                         "sample": f"{frac:.4f} of each projection's rows per step, {len(ws)} layer copies; "
                                   "C++ restatement of matmul_f32_q8/_q4 (AVX2+FMA dispatch, OpenMP); "
                                   "the Rust reference cannot be built here (no cargo)"},
        "e2e": {"value": round(value, 4), "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)



# ---- gemma-decode -------------------------------------------------
DECODE_POS = 511  # the step attends over the full 512-entry KV context


def decode_bytes(cfg, batch, weights_bytes):
    """HBM bytes one decode step must move: every weight byte once, the KV
    cache read up to the position (k and v, f32), the gathered embedding rows
    and the logits written."""
    kv = cfg.n_layers * batch * cfg.n_kv_heads * (DECODE_POS + 1) * cfg.head_dim * 4 * 2
    return weights_bytes + kv + batch * (cfg.hidden // 32) * 34 + batch * cfg.vocab * 4


def decode_weight_bytes(cfg):
    """Algorithmic weight bytes of one decode step: every Q4_0 layer matrix and
    the Q8_0 lm_head once, unpadded (the GGUF bytes)."""
    H, nq, nkv, hd = cfg.hidden, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim
    per_layer = ((nq + 2 * nkv) * hd * H + H * nq * hd + 2 * cfg.ffn * H + H * cfg.ffn) // 32 * 18
    return cfg.n_layers * per_layer + cfg.vocab * (H // 32) * 34


def _decode_weights(local_rank, rank):
    from machinelearning_b200.decode import Gemma3Config, random_weights
    cfg = Gemma3Config.gemma3_1b(ctx=512)
    return cfg, random_weights(cfg, seed=1234 + rank, device=local_rank)


def run_decode(args, rank, world, local_rank, shared=None):
    """Decode tokens/s of the Gemma-3-1B step (one graph replay per step at
    position 511, batch args.batch). N > 1: one independent replica per GPU
    (gemma-decode), or one step sharded over the GPUs (gemma-decode-tp: direct
    launches, the communicator's bounded waits). shared: (cfg, weights) to
    reuse across batches. Returns rank 0's record."""
    import numpy as np
    import torch

    from machinelearning_b200 import _lib
    from machinelearning_b200.decode import Gemma3Decoder
    from machinelearning_b200.tp import TpComm
    tp = args.workload == "gemma-decode-tp" and world > 1
    # a sharded step needs the same weights on every rank
    cfg, w = shared if shared is not None else _decode_weights(local_rank, 0 if tp else rank)
    comm = TpComm.from_group(local_rank, timeout_s=120.0) if tp else None
    if comm is not None and args.join == "peer":
        enable_peer_or_nccl(comm, 4 * args.batch * max(cfg.vocab, world * cfg.hidden), args)
    model = Gemma3Decoder(cfg, w, batch=args.batch, device=local_rank, comm=comm)
    L = _lib.lib()
    dev = model.dev
    B = args.batch
    rng = np.random.default_rng(5 + (0 if tp else rank))
    model.set_tokens(rng.integers(0, cfg.vocab, B))
    model.set_position(DECODE_POS)
    n0 = L.qmm_launch_count()
    model.step(advance=False)
    model.wait(120.0)
    launches = int(L.qmm_launch_count() - n0)
    model.capture(advance=False)
    graphed = model.graph is not None
    st = model.stream

    def enqueue(n):
        for _ in range(n):
            if model.graph is not None:
                model.graph.replay()
            else:
                model._launch(False)

    def sync():
        model.wait(120.0)

    with torch.cuda.stream(st):
        enqueue(args.warmup)
    sync()
    sampler = ClockSampler(local_rank)
    with sampler:
        with torch.cuda.stream(st):
            enqueue(max(args.warmup, 3))
        sync()
        ms, regions, n_timed = timed_regions(enqueue, st, dev, args.steps, world, sampler, sync)
    ms_per_step = ms / args.steps
    # replicas: every GPU decodes its own batch; sharded: the GPUs decode one
    value = B * (1 if tp else world) * args.steps / (ms / 1e3)
    step_bytes = decode_bytes(cfg, B, decode_weight_bytes(cfg))
    achieved = step_bytes / (ms_per_step / 1e3) / 1e9

    e2e = None
    if not args.no_e2e:
        # host token ids in, host logits out, every step (pinned buffers)
        tok_h = torch.as_tensor(rng.integers(0, cfg.vocab, B).astype(np.int32)).pin_memory()
        log_h = torch.empty(B, cfg.vocab, dtype=torch.float32).pin_memory()
        k = min(args.steps, 200)

        def e2e_step():
            with torch.cuda.stream(st):
                model.tokens.copy_(tok_h, non_blocking=True)
                enqueue(1)
                log_h.copy_(model.logits, non_blocking=True)
            sync()
        for _ in range(3):
            e2e_step()
        t0 = time.perf_counter()
        for _ in range(k):
            e2e_step()
        dt_s = time.perf_counter() - t0
        if world > 1:  # the slowest rank's clock (the same collective steps on every rank)
            import torch.distributed as dist
            t = torch.tensor([dt_s])
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            dt_s = float(t.item())
        e2e = {"value": round(B * (1 if tp else world) * k / dt_s, 2), "unit": "tokens/s",
               "h2d_bytes_per_step": B * 4, "d2h_bytes_per_step": B * cfg.vocab * 4, "steps": k,
               "ms_per_step": round(dt_s * 1e3 / k, 4),
               "path": ("pinned host token ids -> the decode step (" +
                        ("graph replay" if graphed else "direct launches") +
                        ("; sharded: the communicator's wait" if tp else "") + ") -> pinned host logits, synchronous")}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = decode_cpu_baseline(cfg, w, B)
    peak, peak_kind = load_peaks()
    clocks = sampler.summary()
    clocks["samples_in_timed_region"] = n_timed
    model.close()
    if comm is not None:
        _lib.check(comm.close())
    line = None
    if rank == 0:
        line = {
            "metric": "decode tokens/s", "value": round(value, 1), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 5),
            "higher_is_better": True, "scaling": "strong" if tp else "weak", "vs_baseline": None,
            "dtype": "f32 activations and KV cache x Q4_0 linears / Q8_0 lm_head (f16 tensor-core MMA, f32 accumulate)",
            "data": "synthetic: random-init weights ~N(0,0.02) quantised on device, norm vectors ~N(0,0.1), "
                    "seeded token ids uniform in the vocabulary",
            "config": {"workload": args.workload, "baseline_config_index": 3,
                       "model": WORKLOADS["gemma-decode"]["model"],
                       "batch": B, "position": DECODE_POS, "kv_context": cfg.ctx,
                       "parallelism": (f"tp{world}: FFN Megatron-paired, lm_head vocabulary-parallel, attention "
                                       f"replicated (libqmm communicator, "
                                       f"{'joins over peer memory' if args.join == 'peer' else 'NCCL joins'})" if tp else
                                       (f"{world} replicas" if world > 1 else "single")),
                       "graph": ("one CUDA graph per step (embedding, 26 layers, final norm, lm_head)"
                                 + (", joins over peer memory captured" if tp else "")
                                 if graphed else
                                 "direct launches (sharded step with NCCL joins: the non-blocking communicator is "
                                 "not captured)"),
                       "l2": "weights 0.71 GB > L2", "bytes_per_step": step_bytes},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                         "traffic": profiled_traffic("gemma-decode"),
                         "note": "achieved = weight bytes (unpadded GGUF bytes) + KV bytes read + embedding rows + "
                                 "logits per step / step time (CUDA events on the replay stream)"},
            "e2e": e2e, "gpu_launches": launches * args.steps, "clocks": clocks,
            "timed_regions": {"count": len(regions), "ms_each": [round(r, 4) for r in regions[:8]],
                              "total_ms": round(sum(regions), 3),
                              "rule": f"K-step region repeated to >= {MIN_TIMED_S * 1e3:.0f} ms, median reported"},
        }
        if cpu is not None:
            line["cpu_baseline"] = cpu
    return line


def _decode_host_weights(w):
    """The device-quantised weights copied to the host for the CPU oracle."""
    def h(t):
        return t.cpu().numpy()
    return {"emb": h(w["emb"]), "final_norm": h(w["final_norm"]),
            "layers": [{k: h(v) for k, v in lw.items()} for lw in w["layers"]]}


def decode_cpu_time(cfg, hw, batch, steps):
    import numpy as np
    import oracle
    from oracle.decode import decode_step
    oracle.set_threads(host_cores())
    kc = [np.zeros((batch, cfg.n_kv_heads, cfg.ctx, cfg.head_dim), np.float32) for _ in range(cfg.n_layers)]
    vc = [np.zeros_like(kc[0]) for _ in range(cfg.n_layers)]
    toks = np.random.default_rng(9).integers(0, cfg.vocab, batch)
    decode_step(cfg, hw, toks, DECODE_POS, kc, vc)  # warm-up
    t0 = time.perf_counter()
    for _ in range(steps):
        decode_step(cfg, hw, toks, DECODE_POS, kc, vc)
    return (time.perf_counter() - t0) / steps


def decode_cpu_baseline(cfg, w, batch):
    import oracle
    oracle.build()
    s = decode_cpu_time(cfg, _decode_host_weights(w), batch, 2)
    return {"value": round(batch / s, 3), "unit": "tokens/s", "cores": oracle.threads(), "kind": "port",
            "sample": f"2 full decode steps at position {DECODE_POS}, batch {batch}: the oracle's numpy restatement "
                      "of the reference forward pass with the C++ matmul_f32_q4/_q8 port (AVX2+FMA, OpenMP)"}


def run_decode_reference(args, rank, world):
    """The reference's CPU decode step (oracle restatement) on the same
    device-generated weights, rank 0 only."""
    if rank != 0:
        return
    import oracle
    oracle.build()
    cfg, w = _decode_weights(int(os.environ.get("LOCAL_RANK", "0")), 0)
    hw = _decode_host_weights(w)
    del w
    steps = max(1, min(args.steps, 3))
    s = decode_cpu_time(cfg, hw, args.batch, steps)
    value = args.batch / s
    print(json.dumps({
        "impl": "reference", "metric": "decode tokens/s", "value": round(value, 4), "unit": "tokens/s",
        "n_gpus": world, "steps": steps, "warmup": 1, "ms_per_step": round(s * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32 activations and KV cache x Q4_0 / Q8_0 blocks",
        "data": "synthetic: the same random-init weights, copied to the host",
        "config": {"workload": args.workload, "baseline_config_index": 3, "batch": args.batch,
                   "position": DECODE_POS, "parallelism": "host cores"},
        "cpu_baseline": {"value": round(value, 4), "unit": "tokens/s", "cores": oracle.threads(), "kind": "port",
                         "sample": f"{steps} full decode steps at position {DECODE_POS}"},
        "e2e": {"value": round(value, 4), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)

# BASELINE configs[4], the configuration defined at 1/2/4/8 GPUs, in its
# Megatron-paired form (one all-reduce per FFN, no all-gather between gate/up
# and down); the literal form (all-gather after gate/up) is a sub-record
DEFAULT_WORKLOAD = "llama70b-megatron"
# the other BASELINE configurations, timed in the same default run (one GPU)
SUB_WORKLOADS = [("llama70b", None), ("gemma-q8-sweep", None), ("q4-gemv", None), ("prefill", None),
                 ("gemma-decode", 1),
                 ("gemma-decode", 16), ("gemma-decode", 64)]


def _init_dist(world, local_rank):
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        # the process group is the control plane only (barriers, the timing
        # max, the communicator's unique id): gloo on the host. Every byte of
        # the data path moves through the library's own NCCL communicator.
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))


def _run_one(args, rank, world, local_rank, shared_decode=None):
    if args.workload in ("gemma-decode", "gemma-decode-tp"):
        return run_decode(args, rank, world, local_rank, shared_decode)
    return run_ours(args, rank, world, local_rank)


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default=None,
                    help=f"one workload only (default: {DEFAULT_WORKLOAD}, plus one sub-record per other BASELINE "
                         "configuration on one GPU)")
    ap.add_argument("--cpu-seconds", type=float, default=8.0, help="CPU-baseline sample length")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true", help="skip the host-buffer end-to-end leg (profiling runs)")
    ap.add_argument("--no-sub", action="store_true", help="default run without the other configurations' records")
    ap.add_argument("--batch", type=int, default=1, help="gemma-decode: sequences per step (1, 16, 64)")
    ap.add_argument("--join", choices=["peer", "nccl"], default="peer",
                    help="N > 1: join tensor-parallel outputs over peer memory (default) or with NCCL collectives")
    ap.add_argument("--copies", type=int, default=None,
                    help="weight copies rotated (default: the workload's; fewer for short profiling runs)")
    args = ap.parse_args(argv)
    if args.warmup < 3:
        args.warmup = 3
    default_run = args.workload is None
    if default_run:
        args.workload = DEFAULT_WORKLOAD

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        if args.workload in ("gemma-decode", "gemma-decode-tp"):
            run_decode_reference(args, rank, world)
        else:
            run_reference(args, rank, world)
        return 0
    _init_dist(world, local_rank)
    try:
        line = _run_one(args, rank, world, local_rank)
        if default_run and not args.no_sub:
            # every other BASELINE configuration, timed in this same run (one
            # GPU); with N GPUs the literal (all-gather) form of the same layer
            # set and the decode step sharded over the GPUs at batch 1 / 16 / 64
            subs = {}
            shared = None
            for name, batch in (SUB_WORKLOADS if world == 1 else
                                [("llama70b", None), ("gemma-decode-tp", 1), ("gemma-decode-tp", 16),
                                 ("gemma-decode-tp", 64)]):
                sub = argparse.Namespace(**vars(args))
                sub.workload, sub.copies = name, None
                if batch is not None:
                    sub.batch = batch
                    if shared is None:  # sharded steps need the same weights on every rank
                        shared = _decode_weights(local_rank, rank if name == "gemma-decode" else 0)
                rec = _run_one(sub, rank, world, local_rank, shared)
                if rec is not None:
                    subs[name if batch is None else f"{name}-b{batch}"] = rec
            shared = None
            if line is not None:
                line["workloads"] = subs
        if line is not None:
            print(json.dumps(line), flush=True)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
