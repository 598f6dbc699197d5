"""Benchmark of the fused attention forward (and the bf16 GEMM) on B200.

Default workload (N=1): BASELINE config 2 -- B=4, H=32, N=4096, head_dim=128,
non-causal, bf16 Q/K/V ~ N(0,1) from a seeded counter-based generator.  With
--gpus N under torchrun every rank runs the same per-GPU workload on its own
slice of a batch of 4N (sharded by batch: weak scaling, no collective on the
data path); the box value is total FLOPs / max-over-ranks time.

One JSON line on rank 0 (see the project's benchmark contract):
  value      device-resident throughput (TFLOP/s, whole box)
  e2e        same metric through the C-ABI call with pinned host buffers:
             H2D of Q/K/V + kernel + D2H of O inside the timed region
  roofline   dominant kernel vs the measured bf16 tensor peak
  cpu_baseline  the reference's CPU attention (oracle/_ref) on a bounded
             sample, on this host's cores (rank 0, N=1 only)

--impl reference runs the reference's CPU implementation of the path (the
compiled reference code in oracle/_ref, else the oracle restatement) on all
host threads, each step a bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "attention fwd TFLOPS per GPU and per box at 1/2/4/8 B200; % of bf16 tensor peak"
GEMM_METRIC = "bf16 GEMM TFLOP/s (tcgen05 vs cuBLAS) at 8192^3"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}

# Per-GPU workloads.  "b" is the per-GPU batch.
WORKLOADS = {
    "c2": dict(name="attn_b4_h32_n4096_d128", b=4, h=32, n=4096, d=128, causal=False,
               sigma=1.0),
    "c1": dict(name="attn_b1_h8_n1024_d128", b=1, h=8, n=1024, d=128, causal=False, sigma=1.0),
    # config 3: H=64 sharded by head over N GPUs; per GPU shard of 8 heads at N=8.
    "c3": dict(name="attn_b1_h64_n16384_d128_causal_per_gpu_h8", b=1, h=8, n=16384, d=128,
               causal=True, sigma=1.0),
    # config 4: B=64 sharded by batch over 8 GPUs: 8 per GPU.
    "c4": dict(name="attn_b64_h16_n2048_d64_per_gpu_b8", b=8, h=16, n=2048, d=64, causal=False,
               sigma=0.5),
    # The GEMM path (5.GEMM): 8192^3, A and B ~ U(-1,1), B stored [K, N] as
    # the reference stores it; each rank multiplies its own pair (weak scaling).
    "gemm": dict(name="gemm_bf16_m8192_n8192_k8192_b_row_major", kind="gemm", m=8192, n=8192,
                 k=8192),
}

# dram__bytes_read.sum + dram__bytes_write.sum per launch of the dominant kernel,
# from the ncu captures in profiles/attention_fwd_d128_c2_b4h32n4096.md and
# profiles/gemm_bf16_pair_8192_b_row_major.md (None: not captured).
NCU_TRAFFIC_BYTES = {"c2": 515.99e6, "gemm": 1152.5e6}


# The JSON result line goes to the process's original stdout; everything else
# written to file descriptor 1 (library banners such as NCCL's version line)
# is sent to stderr, so stdout carries exactly one line.
_RESULT_OUT = None


def claim_stdout() -> None:
    global _RESULT_OUT
    if _RESULT_OUT is None:
        sys.stdout.flush()
        _RESULT_OUT = os.fdopen(os.dup(1), "w")
        os.dup2(2, 1)


def emit(line: dict) -> None:
    out = _RESULT_OUT if _RESULT_OUT is not None else sys.stdout
    print(json.dumps(line), file=out, flush=True)


def load_peaks() -> tuple[dict, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return json.loads(p.read_text()), "measured"
    return dict(FALLBACK_PEAKS), "fallback"


def attention_flops(w: dict) -> float:
    f = 4.0 * w["b"] * w["h"] * w["n"] * w["n"] * w["d"]
    return f / 2 if w["causal"] else f


# ---------------------------------------------------------------------------
# clocks during the timed region (NVML, sampled in a background thread)
# ---------------------------------------------------------------------------
class ClockSampler:
    def __init__(self, device_index: int, period_s: float = 0.005):
        self.samples: list[int] = []
        self.reasons: set[str] = set()
        self.max_mhz = None
        self._stop = threading.Event()
        self._period = period_s
        self._ok = False
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
            self._ok = True
        except Exception:
            self._ok = False
        self._t = threading.Thread(target=self._run, daemon=True)

    _REASONS = [("hw_slowdown", "nvmlClocksThrottleReasonHwSlowdown"),
                ("hw_thermal_slowdown", "nvmlClocksThrottleReasonHwThermalSlowdown"),
                ("sw_thermal_slowdown", "nvmlClocksThrottleReasonSwThermalSlowdown"),
                ("sw_power_cap", "nvmlClocksThrottleReasonSwPowerCap")]

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self._nv.nvmlDeviceGetClockInfo(self._h,
                                                                     self._nv.NVML_CLOCK_SM))
                mask = self._nv.nvmlDeviceGetCurrentClocksThrottleReasons(self._h)
                for name, attr in self._REASONS:
                    bit = getattr(self._nv, attr, 0)
                    if bit and (mask & bit):
                        self.reasons.add(name)
            except Exception:
                pass
            self._stop.wait(self._period)

    def __enter__(self):
        if self._ok:
            self._t.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._ok:
            self._t.join()
            self._stop.clear()
            self._period = 0.0
            self._stop.set()
            self._run_once()

    def _run_once(self):
        try:
            self.samples.append(self._nv.nvmlDeviceGetClockInfo(self._h, self._nv.NVML_CLOCK_SM))
        except Exception:
            pass

    def summary(self) -> dict:
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons),
                "samples": len(self.samples)}


# ---------------------------------------------------------------------------
# CPU side: the reference's own CPU attention on a bounded sample
# ---------------------------------------------------------------------------
def _cpu_sample_inputs(w: dict, rows: int, seed: int = 1234):
    import oracle
    rng = np.random.default_rng(seed)
    n, d = w["n"], w["d"]
    q = oracle.f32_to_bf16(rng.standard_normal((1, 1, rows, d), dtype=np.float32) * w["sigma"])
    k = oracle.f32_to_bf16(rng.standard_normal((1, 1, n, d), dtype=np.float32) * w["sigma"])
    v = oracle.f32_to_bf16(rng.standard_normal((1, 1, n, d), dtype=np.float32) * w["sigma"])
    return q, k, v


def cpu_reference_sample(w: dict, rows_per_thread: int, threads: int) -> dict:
    """Run `threads` concurrent calls of the reference CPU attention, each on
    `rows_per_thread` query rows (the last rows of a head, so causal rows see
    their full key range) against one full head of K/V.  Returns the wall time
    and the FLOPs counted the harness way (4*rows*keys*d, halved for causal)."""
    import oracle
    use_ref = oracle.ref_available()
    n, d = w["n"], w["d"]
    q, k, v = _cpu_sample_inputs(w, rows_per_thread)
    # Non-causal: rows x all keys.  Causal: the sampled rows are the LAST rows
    # of the sequence (Sq = rows, Skv = n, bottom-right aligned) -- counted as
    # rows * n * d * 4 / 2 like the harness counts a causal head.
    if use_ref:
        fn = oracle.ref().ref_attention_f32
    else:
        fn = None

    def one(_):
        out = np.zeros((1, 1, rows_per_thread, d), dtype=np.float32)
        if fn is not None:
            import ctypes
            u16 = ctypes.POINTER(ctypes.c_uint16)
            fn(q.ctypes.data_as(u16), k.ctypes.data_as(u16), v.ctypes.data_as(u16), 1, 1, 1,
               rows_per_thread, n, d, float(np.float32(1.0) / np.sqrt(np.float32(d))),
               int(w["causal"]), out.ctypes.data_as(ctypes.POINTER(ctypes.c_float)))
        else:
            out[:] = oracle.attention(q, k, v, causal=w["causal"], threads=1)
        return out

    t0 = time.perf_counter()
    with ThreadPoolExecutor(max_workers=threads) as ex:
        list(ex.map(one, range(threads)))
    dt = time.perf_counter() - t0
    flops = 4.0 * rows_per_thread * n * d * threads
    if w["causal"]:
        flops /= 2
    return {"seconds": dt, "flops": flops, "kind": "reference" if use_ref else "port"}


def gemm_cpu_sample(w: dict, rows_per_thread: int, threads: int) -> dict:
    """The oracle's double-precision GEMM loop (the reference's fp32 GEMM
    algorithm, 5.GEMM/gemm256_tma_tcgen05_bench.cu:1115-1137, restated; the
    reference has no CPU GEMM of its own) on rows_per_thread rows of C per
    thread, full N and K."""
    import oracle
    rng = np.random.default_rng(7)
    rows = rows_per_thread * threads
    a = oracle.f32_to_bf16(rng.uniform(-1.0, 1.0, (rows, w["k"])).astype(np.float32))
    b = oracle.f32_to_bf16(rng.uniform(-1.0, 1.0, (w["k"], w["n"])).astype(np.float32))
    t0 = time.perf_counter()
    oracle.gemm(a, b, False, 0, rows, threads=threads)
    dt = time.perf_counter() - t0
    return {"seconds": dt, "flops": 2.0 * rows * w["n"] * w["k"], "kind": "port"}


def host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def run_reference_arm(args, w: dict) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = host_threads()
    gemm = w.get("kind") == "gemm"
    rows = args.cpu_gemm_rows if gemm else args.cpu_rows
    sample_fn = gemm_cpu_sample if gemm else cpu_reference_sample
    for _ in range(args.warmup):
        sample_fn(w, max(1, rows // 8), threads)
    times, flops, kind = [], 0.0, "port"
    for _ in range(args.steps):
        r = sample_fn(w, rows, threads)
        times.append(r["seconds"])
        flops, kind = r["flops"], r["kind"]
    t = sum(times) / len(times)
    value = flops / t / 1e12
    if gemm:
        sample = (f"{threads} threads x {rows} rows of C x N={w['n']} x K={w['k']} per step")
        config = {"workload": w["name"], "M": w["m"], "N": w["n"], "K": w["k"], "sampled": True}
    else:
        sample = (f"{threads} threads x {rows} query rows x {w['n']} keys x d{w['d']}"
                  f"{' causal' if w['causal'] else ''} per step (1 head of K/V each)")
        config = {"workload": w["name"], "B": w["b"], "H": w["h"], "N": w["n"], "D": w["d"],
                  "causal": w["causal"], "sampled": True}
    emit({
        "impl": "reference", "metric": GEMM_METRIC if gemm else METRIC, "value": value,
        "unit": "TFLOP/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": t * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f64" if gemm else "f32",
        "data": "synthetic U(-1,1) bf16 inputs" if gemm else "synthetic N(0,sigma) bf16 inputs",
        "config": config,
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": threads, "kind": kind,
                         "sample": sample},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    })


# ---------------------------------------------------------------------------
# Rank plumbing shared by both arms (tested on CPU with gloo ranks)
# ---------------------------------------------------------------------------
def rank_index_base(rank: int, elems_per_rank: int) -> int:
    """First global element index of this rank's batch slice: rank r owns
    batches [r*B, (r+1)*B) of the global [B*world, H, N, D] tensors, so its
    generated values are those of that slice of one global tensor."""
    return rank * elems_per_rank


def max_over_ranks(value: float, world: int, device=None) -> float:
    """The slowest rank's time: all ranks call this collectively."""
    if world <= 1:
        return float(value)
    import torch
    import torch.distributed as dist
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------
def pipelined_e2e(args, inputs, out, compute, stream, world, dev, barrier, flops) -> dict:
    """The metric through the C-ABI call with host buffers: every step copies
    the inputs from pinned host memory, runs `compute(device_inputs,
    device_out)` on `stream` and copies the result back.  Steps are pipelined
    over two device buffer sets on three streams (host->device, compute,
    device->host), as a streaming caller would run them; the timed region
    spans from the first copy in to the last copy out."""
    import torch

    from benchmark_b200 import ops

    hosts = [t.cpu().pin_memory() for t in inputs]
    h_out = torch.empty(out.shape, dtype=out.dtype, pin_memory=True)
    bufs = [([torch.empty_like(t) for t in inputs], torch.empty_like(out)) for _ in range(2)]
    s_in, s_out = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    ev = lambda: torch.cuda.Event(enable_timing=False)  # noqa: E731
    computed = [ev(), ev()]
    drained = [ev(), ev()]

    def e2e_step(i: int) -> None:
        d_in, d_out = bufs[i & 1]
        loaded = ev()
        with torch.cuda.stream(s_in):
            s_in.wait_event(computed[i & 1])  # step i-2 has consumed this set
            for d, h in zip(d_in, hosts):
                d.copy_(h, non_blocking=True)
            loaded.record(s_in)
        stream.wait_event(loaded)
        stream.wait_event(drained[i & 1])  # the result of step i-2 has been copied out
        compute(d_in, d_out)
        computed[i & 1].record(stream)
        with torch.cuda.stream(s_out):
            s_out.wait_event(computed[i & 1])
            h_out.copy_(d_out, non_blocking=True)
            drained[i & 1].record(s_out)

    steps = max(2, min(args.steps, args.e2e_steps))
    for i in range(2):
        e2e_step(i)
    torch.cuda.synchronize()
    barrier()
    start = torch.cuda.Event(enable_timing=True)
    stop = torch.cuda.Event(enable_timing=True)
    start.record(s_in)
    for i in range(steps):
        e2e_step(i)
    s_in.wait_stream(s_out)
    stop.record(s_in)
    torch.cuda.synchronize()
    ops.check(stream)
    ms = max_over_ranks(start.elapsed_time(stop) / steps, world, dev)
    if not torch.equal(h_out, out.cpu()):
        raise RuntimeError("e2e output differs from the device-resident run")
    return {"value": world * flops / (ms * 1e-3) / 1e12, "unit": "TFLOP/s",
            "h2d_bytes_per_step": sum(t.numel() * t.element_size() for t in inputs),
            "d2h_bytes_per_step": out.numel() * out.element_size(), "steps": steps,
            "ms_per_step": ms, "pipelined": "2 buffer sets, H2D / compute / D2H streams"}


def run_e2e(args, w, q, k, v, o, stream, world, dev, barrier, flops) -> dict:
    from benchmark_b200 import ops

    def compute(d_in, d_out):
        ops.attention_fwd(d_in[0], d_in[1], d_in[2], out=d_out, causal=w["causal"],
                          stream=stream)

    return pipelined_e2e(args, [q, k, v], o, compute, stream, world, dev, barrier, flops)


def run_gemm_arm(args, w: dict) -> None:
    """The GEMM path: this library's tcgen05 CTA-pair kernel on C = A @ B with
    B stored [K, N], every rank on its own operands; cuBLAS on the same
    operands is reported beside it."""
    import torch
    import torch.distributed as dist

    from benchmark_b200 import _lib, ops

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    M, N, K = w["m"], w["n"], w["k"]
    a = torch.empty((M, K), dtype=torch.bfloat16, device=dev)
    b = torch.empty((K, N), dtype=torch.bfloat16, device=dev)
    c = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
    ops.fill_uniform_(a, args.seed, 10, -1.0, 1.0, index_base=rank_index_base(rank, a.numel()))
    ops.fill_uniform_(b, args.seed, 11, -1.0, 1.0, index_base=rank_index_base(rank, b.numel()))
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    flops = 2.0 * M * N * K

    def timed(impl: str) -> float:
        for _ in range(args.warmup):
            ops.gemm_bf16(a, b, out=c, b_col_major=False, impl=impl, stream=stream)
        ops.check(stream)
        barrier()
        torch.cuda.synchronize()
        start = torch.cuda.Event(enable_timing=True)
        stop = torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for _ in range(args.steps):
            ops.gemm_bf16(a, b, out=c, b_col_major=False, impl=impl, stream=stream)
        stop.record(stream)
        torch.cuda.synchronize()
        barrier()
        ops.check(stream)
        return start.elapsed_time(stop) / args.steps

    # cuBLAS is timed both before and after this kernel on the same operands
    # and the two are averaged, so a power-capped GPU's drift between the runs
    # favours neither side.
    ms_cublas_before = max_over_ranks(timed("cublas"), world, dev)
    with ClockSampler(local) as clocks:
        ms_local = timed("tcgen05")
    ms_max = max_over_ranks(ms_local, world, dev)
    ms_cublas_after = max_over_ranks(timed("cublas"), world, dev)
    ms_cublas = 0.5 * (ms_cublas_before + ms_cublas_after)
    value = world * flops / (ms_max * 1e-3) / 1e12

    def compute(d_in, d_out):
        ops.gemm_bf16(d_in[0], d_in[1], out=d_out, b_col_major=False, stream=stream)

    e2e = None if args.no_e2e else pipelined_e2e(args, [a, b], c, compute, stream, world, dev,
                                                 barrier, flops)
    peaks, peak_src = load_peaks()
    peak = float(peaks["bf16_tflops"])
    achieved = flops / (ms_local * 1e-3) / 1e12
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = host_threads()
        r = gemm_cpu_sample(w, args.cpu_gemm_rows, threads)
        cpu = {"value": r["flops"] / r["seconds"] / 1e12, "unit": "TFLOP/s", "cores": threads,
               "kind": r["kind"],
               "sample": (f"{threads} threads x {args.cpu_gemm_rows} rows of C x N={N} x K={K} "
                          f"({r['seconds']:.1f} s wall)")}
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()
    if rank != 0:
        return
    line = {
        "metric": GEMM_METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_max,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": f"synthetic: bf16 A, B ~ U(-1,1), counter-based seed {args.seed}",
        "config": {"workload": w["name"], "M": M, "N": N, "K": K, "b_layout": "[K,N]",
                   "parallelism": f"dp{world} (independent GEMM per rank)",
                   "l2": "inputs larger than L2 (256 MiB of A and B per step)"},
        "cublas_tflops": world * flops / (ms_cublas * 1e-3) / 1e12,
        "cublas_tflops_before_after": [world * flops / (ms_cublas_before * 1e-3) / 1e12,
                                       world * flops / (ms_cublas_after * 1e-3) / 1e12],
        "hbm_gbs_algorithmic": world * 2 * (M * K + K * N + M * N) / (ms_max * 1e-3) / 1e9,
        "vs_cublas": ms_cublas / ms_max,
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                     "frac": achieved / peak, "traffic": NCU_TRAFFIC_BYTES.get(args.workload),
                     "algorithmic_bytes": 2 * (M * K + K * N + M * N),
                     "kernel": "gemm_bf16_pair_kernel",
                     "peak_source": f"{peak_src} bf16_tflops (burst)"},
        "e2e": e2e,
        "gpu_launches": args.steps,
        "clocks": clocks.summary(),
        "cpu_baseline": cpu,
        "lib": _lib.LIB_PATH.name,
    }
    emit(line)


def run_gpu_arm(args, w: dict) -> None:
    import torch
    import torch.distributed as dist

    from benchmark_b200 import _lib, ops

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    B, H, N, D = w["b"], w["h"], w["n"], w["d"]
    q = torch.empty((B, H, N, D), dtype=torch.bfloat16, device=dev)
    k = torch.empty_like(q)
    v = torch.empty_like(q)
    o = torch.empty_like(q)
    per = q.numel()
    # this rank's batch slice of the global [B * world, H, N, D] tensors
    for t, tid in ((q, 0), (k, 1), (v, 2)):
        ops.fill_normal_(t, args.seed, tid, 0.0, w["sigma"],
                         index_base=rank_index_base(rank, per))
    torch.cuda.synchronize()

    stream = torch.cuda.current_stream()

    def step():
        ops.attention_fwd(q, k, v, out=o, causal=w["causal"], stream=stream)

    for _ in range(args.warmup):
        step()
    ops.check(stream)
    barrier()
    torch.cuda.synchronize()

    start = torch.cuda.Event(enable_timing=True)
    stop = torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        start.record(stream)
        for _ in range(args.steps):
            step()
        stop.record(stream)
        torch.cuda.synchronize()
    barrier()
    ops.check(stream)
    ms = start.elapsed_time(stop) / args.steps
    ms_max = max_over_ranks(ms, world, dev)
    flops = attention_flops(w)
    value = world * flops / (ms_max * 1e-3) / 1e12

    e2e = None if args.no_e2e else run_e2e(args, w, q, k, v, o, stream, world, dev, barrier,
                                           flops)

    peaks, peak_src = load_peaks()
    peak = float(peaks["bf16_tflops"])
    achieved = flops / (ms * 1e-3) / 1e12
    traffic = NCU_TRAFFIC_BYTES.get(args.workload)
    algo_bytes = 4 * q.numel() * q.element_size()  # Q, K, V read + O written once

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = host_threads()
        rows = args.cpu_baseline_rows
        r = cpu_reference_sample(w, rows, threads)
        cpu = {"value": r["flops"] / r["seconds"] / 1e12, "unit": "TFLOP/s", "cores": threads,
               "kind": r["kind"],
               "sample": (f"{threads} threads x {rows} query rows x {N} keys x d{D} "
                          f"({r['seconds']:.1f} s wall)")}

    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()
    if rank != 0:
        return
    line = {
        "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_max,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": f"synthetic: bf16 Q/K/V ~ N(0,{w['sigma']}^2), counter-based seed {args.seed}",
        "config": {"workload": w["name"], "B_per_gpu": B, "global_B": B * world, "H": H,
                   "N": N, "D": D, "causal": w["causal"],
                   "parallelism": f"dp{world} (batch-sharded heads, no collective)",
                   "l2": (f"inputs larger than L2 ({3 * q.numel() * 2 / 2**20:.0f} MiB of "
                          "Q/K/V read per step)")},
        "per_gpu_tflops": value / world,
        # algorithmic HBM rate (Q+K+V read, O written once) and exp2 rate,
        # whole box: the config-4 view of the same run
        "hbm_gbs_algorithmic": world * algo_bytes / (ms_max * 1e-3) / 1e9,
        "exp_per_s": world * (w["b"] * w["h"] * w["n"] * w["n"] / (2 if w["causal"] else 1))
        / (ms_max * 1e-3),
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                     "frac": achieved / peak, "traffic": traffic,
                     "algorithmic_bytes": algo_bytes,
                     "kernel": f"attention_fwd_kernel<{D}>",
                     "peak_source": f"{peak_src} bf16_tflops (burst)"},
        "e2e": e2e,
        "gpu_launches": args.steps,
        "clocks": clocks.summary(),
        "cpu_baseline": cpu,
        "lib": _lib.LIB_PATH.name,
    }
    emit(line)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="c2")
    ap.add_argument("--seed", type=int, default=2024)
    ap.add_argument("--e2e-steps", type=int, default=10)
    ap.add_argument("--cpu-rows", type=int, default=256,
                    help="query rows per host thread in each --impl reference step")
    ap.add_argument("--cpu-baseline-rows", type=int, default=4096,
                    help="query rows per host thread in the GPU line's cpu_baseline "
                         "(about 10 s of host work at config 2)")
    ap.add_argument("--cpu-gemm-rows", type=int, default=4,
                    help="rows of C per host thread in the CPU GEMM sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true", help="skip the host-buffer e2e leg")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    w = WORKLOADS[args.workload]
    # stdout carries exactly one JSON line: NCCL's log output goes to stderr,
    # and so does anything else a library writes to file descriptor 1 (NCCL
    # prints its version banner there under some NCCL_DEBUG settings).
    os.environ.setdefault("NCCL_DEBUG_FILE", "/dev/stderr")
    claim_stdout()
    if args.impl == "reference":
        run_reference_arm(args, w)
    elif w.get("kind") == "gemm":
        run_gemm_arm(args, w)
    else:
        run_gpu_arm(args, w)


if __name__ == "__main__":
    main()
