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
  strong     (every N) BASELINE configs 3 and 4 as fixed total problems split
             across the N ranks: config 3 (B1 H64 N16384 d128 causal) by head,
             config 4 (B64 H16 N2048 d64) by batch; box TFLOP/s and the
             slowest rank's time
  configs    (N=1) every other BASELINE config on this GPU: config 1, configs
             3 and 4 in full, and the GEMM at 8192^3 and 16384^3 with cuBLAS
             timed before and after it on the same operands

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

# BASELINE.json configs.  "b" and "h" are the per-GPU batch and heads of a
# weak-scaling workload; a "split" workload is a fixed total problem whose
# heads ("h") or batches ("b") are divided among the ranks.
WORKLOADS = {
    "c2": dict(name="attn_b4_h32_n4096_d128", b=4, h=32, n=4096, d=128, causal=False,
               sigma=1.0),
    "c1": dict(name="attn_b1_h8_n1024_d128", b=1, h=8, n=1024, d=128, causal=False, sigma=1.0),
    # config 3: B=1, H=64, N=16384 causal, split by head over the ranks
    "c3": dict(name="attn_b1_h64_n16384_d128_causal", b=1, h=64, n=16384, d=128, causal=True,
               sigma=1.0, split="h"),
    # config 4: B=64, H=16, N=2048, d=64, sigma 0.5, split by batch over the ranks
    "c4": dict(name="attn_b64_h16_n2048_d64", b=64, h=16, n=2048, d=64, causal=False,
               sigma=0.5, split="b"),
    # The GEMM path (5.GEMM): A and B ~ U(-1,1), B stored [K, N] as the
    # reference stores it; each rank multiplies its own pair (weak scaling).
    "gemm": dict(name="gemm_bf16_m8192_n8192_k8192_b_row_major", kind="gemm", m=8192, n=8192,
                 k=8192),
    "gemm16k": dict(name="gemm_bf16_m16384_n16384_k16384_b_row_major", kind="gemm", m=16384,
                    n=16384, k=16384),
}

# dram__bytes_read.sum + dram__bytes_write.sum per launch of the dominant kernel
# of each workload, from the ncu captures summarised in profiles/ (None: not
# captured).  c4 was captured on its 8-GPU shard (batch 8) and is scaled to
# the full problem by its items (the traffic grows with them: each batch
# streams its own K/V once); c3 was captured on the full 64-head problem.
NCU_TRAFFIC_BYTES = {
    "c2": 517.23e6,     # profiles/attention_fwd_d128_c2_b4h32n4096.md
    "c1": 6.37e6,       # profiles/attention_fwd_d128_c1_b1h8n1024.md
    "c3": 3.06e9,       # profiles/attention_fwd_d128_c3_causal_h64n16384_l2.md
    "c4": 8 * 107.00e6,  # profiles/attention_fwd_d64_c4_b8h16n2048.md
    "gemm": 1044.0e6,   # profiles/gemm_bf16_pair_8192_b_row_major.md (current build)
    "gemm16k": 16.35e9,  # profiles/gemm_bf16_pair_16384_b_row_major.md (current build)
}

L2_BYTES = 126 * 2**20


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


def shard(w: dict, rank: int, world: int) -> tuple[dict, int]:
    """This rank's part of workload w and the global index of its first
    element.  Weak workloads: every rank gets (b, h) of its own batch slice of
    a [b * world, h, n, d] tensor.  Split workloads: the fixed [b, h, n, d]
    problem's heads (B = 1) or batches are divided evenly among the ranks."""
    split = w.get("split")
    if split is None:
        part = dict(w)
    elif split == "h":
        if w["b"] != 1 or w["h"] % world:
            raise ValueError(f"{w['name']}: {w['h']} heads do not split over {world} ranks")
        part = dict(w, h=w["h"] // world)
    else:
        if w["b"] % world:
            raise ValueError(f"{w['name']}: batch {w['b']} does not split over {world} ranks")
        part = dict(w, b=w["b"] // world)
    per = part["b"] * part["h"] * part["n"] * part["d"]
    return part, rank_index_base(rank, per)


def l2_note(read_bytes: int, flushed: bool) -> str:
    mib = read_bytes / 2**20
    if read_bytes > L2_BYTES:
        return f"inputs larger than L2 ({mib:.0f} MiB read per step, L2 126 MiB)"
    if flushed:
        return (f"inputs fit in L2 ({mib:.1f} MiB); L2 flushed by a 256 MiB write between "
                "timed steps, each step timed alone")
    return f"inputs fit in L2 ({mib:.1f} MiB); not flushed: L2-warm figure"


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


class Ranks:
    """torch.distributed plumbing of one GPU arm process (world 1: no-ops)."""

    def __init__(self):
        import torch
        import torch.distributed as dist
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(self.local)
        self.dev = torch.device("cuda", self.local)
        if self.world > 1:
            import datetime
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                    device_id=self.dev)

    def barrier(self) -> None:
        if self.world > 1:
            import torch.distributed as dist
            dist.barrier(device_ids=[self.local])

    def max(self, value: float) -> float:
        return max_over_ranks(value, self.world, self.dev)

    def close(self) -> None:
        if self.world > 1:
            import torch.distributed as dist
            dist.barrier(device_ids=[self.local])
            dist.destroy_process_group()


def attention_inputs(part: dict, index_base: int, seed: int, dev):
    """Q, K, V (seeded, by global element index) and O for one rank's part."""
    import torch

    from benchmark_b200 import ops
    q = torch.empty((part["b"], part["h"], part["n"], part["d"]), dtype=torch.bfloat16,
                    device=dev)
    k = torch.empty_like(q)
    v = torch.empty_like(q)
    o = torch.empty_like(q)
    for t, tid in ((q, 0), (k, 1), (v, 2)):
        ops.fill_normal_(t, seed, tid, 0.0, part["sigma"], index_base=index_base)
    torch.cuda.synchronize()
    return q, k, v, o


def time_steps(step, steps: int, warmup: int, ranks: Ranks, stream, flush=None,
               clocks: ClockSampler | None = None) -> tuple[float, float]:
    """(this rank's ms per step, slowest rank's ms per step) of `step`.

    Without `flush` the steps run back to back between two events.  With it,
    `flush()` runs before every step outside the timed events (an L2 flush for
    inputs that fit in L2) and each step is timed alone."""
    import contextlib

    import torch

    from benchmark_b200 import ops
    for _ in range(warmup):
        step()
    ops.check(stream)
    ranks.barrier()
    torch.cuda.synchronize()
    ev = lambda: torch.cuda.Event(enable_timing=True)  # noqa: E731
    with clocks if clocks is not None else contextlib.nullcontext():
        if flush is None:
            start, stop = ev(), ev()
            start.record(stream)
            for _ in range(steps):
                step()
            stop.record(stream)
            torch.cuda.synchronize()
            ms = start.elapsed_time(stop) / steps
        else:
            pairs = []
            for _ in range(steps):
                flush()
                e0, e1 = ev(), ev()
                e0.record(stream)
                step()
                e1.record(stream)
                pairs.append((e0, e1))
            torch.cuda.synchronize()
            ms = sum(e0.elapsed_time(e1) for e0, e1 in pairs) / steps
    ranks.barrier()
    ops.check(stream)
    return ms, ranks.max(ms)


def l2_flusher(dev):
    import torch
    buf = torch.empty(256 * 2**20, dtype=torch.uint8, device=dev)
    return lambda: buf.fill_(1)


def attention_kernel_name(part: dict) -> str:
    """The kernel the library runs for this workload: non-causal d=64 problems
    with a unit (two Q tiles) per SM take the two-Q-tile kernel; non-causal
    d=128 problems with a unit per two SMs take the CTA-pair form of the
    one-Q-tile kernel (cta_group::2, clusters of two)."""
    units = part["b"] * part["h"] * ((part["n"] + 255) // 256)
    if part["d"] == 64 and not part["causal"] and units >= 148:
        return "attention_pair_kernel<1>"
    if part["d"] == 128 and not part["causal"] and 2 * units >= 148:
        return "attention_fwd_kernel<128> (CTA pairs, cta_group::2)"
    return f"attention_fwd_kernel<{part['d']}>"


def attention_roofline(part: dict, ms_local: float, key: str, peaks: dict, peak_src: str,
                       q_bytes: int) -> dict:
    flops = attention_flops(part)
    achieved = flops / (ms_local * 1e-3) / 1e12
    peak = float(peaks["bf16_tflops"])
    return {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
            "frac": achieved / peak, "traffic": NCU_TRAFFIC_BYTES.get(key),
            "algorithmic_bytes": 4 * q_bytes,  # Q, K, V read + O written once
            "kernel": attention_kernel_name(part),
            "peak_source": f"{peak_src} bf16_tflops (burst)"}


def measure_attention(key: str, args, ranks: Ranks, stream, peaks, peak_src, steps: int,
                      warmup: int, with_clocks: bool = False) -> dict:
    """One attention workload on every rank (its shard); whole-box numbers."""
    import torch

    from benchmark_b200 import ops
    w = WORKLOADS[key]
    part, base = shard(w, ranks.rank, ranks.world)
    q, k, v, o = attention_inputs(part, base, args.seed, ranks.dev)
    read_bytes = 3 * q.numel() * q.element_size()
    flush = l2_flusher(ranks.dev) if read_bytes <= L2_BYTES else None

    def step():
        ops.attention_fwd(q, k, v, out=o, causal=part["causal"], stream=stream)

    clocks = ClockSampler(ranks.local) if with_clocks else None
    ms, ms_max = time_steps(step, steps, warmup, ranks, stream, flush, clocks)
    box_flops = attention_flops(part) * ranks.world
    r = {"workload": w["name"], "value": box_flops / (ms_max * 1e-3) / 1e12, "unit": "TFLOP/s",
         "ms_per_step": ms_max, "rank_ms_per_step": ms, "steps": steps, "warmup": warmup,
         "gpu_launches": steps, "per_rank": {"B": part["b"], "H": part["h"]},
         "l2": l2_note(read_bytes, flush is not None),
         "hbm_gbs_algorithmic": ranks.world * 4 * q.numel() * 2 / (ms_max * 1e-3) / 1e9,
         "exp_per_s": ranks.world * part["b"] * part["h"] * part["n"] * part["n"]
         / (2 if part["causal"] else 1) / (ms_max * 1e-3),
         "roofline": attention_roofline(part, ms, key, peaks, peak_src, q.numel() * 2)}
    if clocks is not None:
        r["clocks"] = clocks.summary()
    r["_tensors"] = (q, k, v, o)
    del q, k, v, o
    torch.cuda.synchronize()
    return r


def measure_gemm(key: str, args, ranks: Ranks, stream, peaks, peak_src, steps: int,
                 warmup: int, with_clocks: bool = False) -> dict:
    """This library's tcgen05 CTA-pair GEMM on C = A @ B with B stored [K, N],
    every rank on its own operands; cuBLAS on the same operands is timed
    before and after it and the two are averaged, so a power-capped GPU's
    drift between the runs favours neither side."""
    import torch

    from benchmark_b200 import ops
    w = WORKLOADS[key]
    M, N, K = w["m"], w["n"], w["k"]
    a = torch.empty((M, K), dtype=torch.bfloat16, device=ranks.dev)
    b = torch.empty((K, N), dtype=torch.bfloat16, device=ranks.dev)
    c = torch.empty((M, N), dtype=torch.bfloat16, device=ranks.dev)
    ops.fill_uniform_(a, args.seed, 10, -1.0, 1.0,
                      index_base=rank_index_base(ranks.rank, a.numel()))
    ops.fill_uniform_(b, args.seed, 11, -1.0, 1.0,
                      index_base=rank_index_base(ranks.rank, b.numel()))
    torch.cuda.synchronize()
    flops = 2.0 * M * N * K

    def timed(impl: str, clocks=None) -> tuple[float, float]:
        def step():
            ops.gemm_bf16(a, b, out=c, b_col_major=False, impl=impl, stream=stream)
        return time_steps(step, steps, warmup, ranks, stream, None, clocks)

    _, ms_cublas_before = timed("cublas")
    clocks = ClockSampler(ranks.local) if with_clocks else None
    ms_local, ms_max = timed("tcgen05", clocks)
    _, ms_cublas_after = timed("cublas")
    ms_cublas = 0.5 * (ms_cublas_before + ms_cublas_after)
    box = lambda ms: ranks.world * flops / (ms * 1e-3) / 1e12  # noqa: E731
    achieved = flops / (ms_local * 1e-3) / 1e12
    peak = float(peaks["bf16_tflops"])
    algo = 2 * (M * K + K * N + M * N)
    r = {"workload": w["name"], "value": box(ms_max), "unit": "TFLOP/s", "ms_per_step": ms_max,
         "rank_ms_per_step": ms_local, "steps": steps, "warmup": warmup,
         "gpu_launches": steps, "M": M, "N": N, "K": K, "b_layout": "[K,N]",
         "l2": l2_note(2 * (M * K + K * N), False),
         "cublas_tflops": box(ms_cublas),
         "cublas_tflops_before_after": [box(ms_cublas_before), box(ms_cublas_after)],
         "vs_cublas": ms_cublas / ms_max,
         "hbm_gbs_algorithmic": ranks.world * algo / (ms_max * 1e-3) / 1e9,
         "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                      "frac": achieved / peak, "traffic": NCU_TRAFFIC_BYTES.get(key),
                      "algorithmic_bytes": algo, "kernel": "gemm_bf16_pair_kernel",
                      "peak_source": f"{peak_src} bf16_tflops (burst)"}}
    if clocks is not None:
        r["clocks"] = clocks.summary()
    r["_tensors"] = (a, b, c)
    return r


def public(entry: dict) -> dict:
    out = {k: v for k, v in entry.items() if not k.startswith("_")}
    out["idle_before_s"] = CONFIG_IDLE_S
    return out


def run_e2e(args, part, q, k, v, o, stream, ranks: Ranks, flops) -> dict:
    from benchmark_b200 import ops

    def compute(d_in, d_out):
        ops.attention_fwd(d_in[0], d_in[1], d_in[2], out=d_out, causal=part["causal"],
                          stream=stream)

    return pipelined_e2e(args, [q, k, v], o, compute, stream, ranks.world, ranks.dev,
                         ranks.barrier, flops)


# Idle time before each extra workload.  A B200 under its 1 kW cap lowers its
# SM clock after a few tens of ms of dense work and recovers within a fraction
# of a second of idling; without the pause each workload would inherit the
# clock the previous one left behind (with the one-Q-tile kernel, config 4
# read 458 TFLOP/s right after config 3 and 714 after the pause).
CONFIG_IDLE_S = 1.0


def strong_and_configs(args, ranks: Ranks, stream, peaks, peak_src, main_key: str) -> tuple:
    """The `strong` object (every N) and the `configs` object (N=1 only)."""
    steps = max(3, min(args.steps, args.config_steps))
    strong, configs = {}, {}
    for key in ("c3", "c4"):
        if args.no_configs:
            break
        time.sleep(CONFIG_IDLE_S)
        r = measure_attention(key, args, ranks, stream, peaks, peak_src, steps, 3,
                              with_clocks=True)
        strong[key] = {"workload": r["workload"], "value": r["value"], "unit": r["unit"],
                       "ms_per_step": r["ms_per_step"], "per_rank": r["per_rank"],
                       "split": "heads" if WORKLOADS[key]["split"] == "h" else "batch",
                       "n_gpus": ranks.world}
        if ranks.world == 1 and key != main_key:
            configs[key] = public(r)
        del r
    if ranks.world == 1 and not args.no_configs:
        for key in ("c1", "gemm", "gemm16k"):
            if key == main_key:
                continue
            fn = measure_gemm if WORKLOADS[key].get("kind") == "gemm" else measure_attention
            csteps = steps if key != "c1" else max(steps, 50)
            time.sleep(CONFIG_IDLE_S)
            configs[key] = public(fn(key, args, ranks, stream, peaks, peak_src, csteps, 3,
                                     with_clocks=True))
    return strong, configs


def run_gpu_arm(args, w: dict) -> None:
    import torch

    from benchmark_b200 import _lib

    ranks = Ranks()
    stream = torch.cuda.current_stream()
    peaks, peak_src = load_peaks()
    gemm = w.get("kind") == "gemm"
    key = args.workload
    fn = measure_gemm if gemm else measure_attention
    main = fn(key, args, ranks, stream, peaks, peak_src, args.steps, args.warmup,
              with_clocks=True)
    if gemm:
        a, b, c = main.pop("_tensors")

        def compute(d_in, d_out):
            from benchmark_b200 import ops
            ops.gemm_bf16(d_in[0], d_in[1], out=d_out, b_col_major=False, stream=stream)

        flops = 2.0 * w["m"] * w["n"] * w["k"]
        e2e = None if args.no_e2e else pipelined_e2e(args, [a, b], c, compute, stream,
                                                     ranks.world, ranks.dev, ranks.barrier,
                                                     flops)
        del a, b, c
    else:
        q, k, v, o = main.pop("_tensors")
        part, _ = shard(w, ranks.rank, ranks.world)
        e2e = None if args.no_e2e else run_e2e(args, part, q, k, v, o, stream, ranks,
                                               attention_flops(part))
        del q, k, v, o
    torch.cuda.empty_cache()

    cpu = None
    if ranks.rank == 0 and ranks.world == 1 and not args.no_cpu_baseline:
        threads = host_threads()
        if gemm:
            rows = args.cpu_gemm_rows
            r = gemm_cpu_sample(w, rows, threads)
            sample = f"{threads} threads x {rows} rows of C x N={w['n']} x K={w['k']}"
        else:
            rows = args.cpu_baseline_rows
            r = cpu_reference_sample(w, rows, threads)
            sample = f"{threads} threads x {rows} query rows x {w['n']} keys x d{w['d']}"
        cpu = {"value": r["flops"] / r["seconds"] / 1e12, "unit": "TFLOP/s", "cores": threads,
               "kind": r["kind"], "sample": f"{sample} ({r['seconds']:.1f} s wall)"}

    strong, configs = strong_and_configs(args, ranks, stream, peaks, peak_src, key)
    ranks.close()
    if ranks.rank != 0:
        return
    world = ranks.world
    if gemm:
        config = {"workload": w["name"], "M": w["m"], "N": w["n"], "K": w["k"],
                  "b_layout": "[K,N]", "parallelism": f"dp{world} (independent GEMM per rank)",
                  "l2": main["l2"]}
        data = f"synthetic: bf16 A, B ~ U(-1,1), counter-based seed {args.seed}"
        scaling = "weak"
    else:
        part, _ = shard(w, 0, world)
        split = w.get("split")
        config = {"workload": w["name"], "B_per_gpu": part["b"], "H_per_gpu": part["h"],
                  "global_B": part["b"] * world if split is None else w["b"],
                  "H": w["h"], "N": w["n"], "D": w["d"], "causal": w["causal"],
                  "parallelism": (f"dp{world} (batch-sharded heads, no collective)"
                                  if split is None else
                                  f"{'head' if split == 'h' else 'batch'}-split over {world} "
                                  "ranks, no collective"),
                  "l2": main["l2"]}
        data = (f"synthetic: bf16 Q/K/V ~ N(0,{w['sigma']}^2), counter-based seed {args.seed}")
        scaling = "weak" if split is None else "strong"
    line = {
        "metric": GEMM_METRIC if gemm else METRIC, "value": main["value"], "unit": "TFLOP/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": main["ms_per_step"], "higher_is_better": True, "scaling": scaling,
        "vs_baseline": None, "dtype": "bf16", "data": data, "config": config,
        "per_gpu_tflops": main["value"] / world,
        "hbm_gbs_algorithmic": main["hbm_gbs_algorithmic"],
    }
    for k in ("exp_per_s", "cublas_tflops", "cublas_tflops_before_after", "vs_cublas"):
        if k in main:
            line[k] = main[k]
    line.update({
        "roofline": main["roofline"], "e2e": e2e, "gpu_launches": main["gpu_launches"],
        "clocks": main.get("clocks"), "cpu_baseline": cpu, "strong": strong or None,
        "configs": configs or None, "lib": _lib.LIB_PATH.name,
    })
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
    ap.add_argument("--no-configs", action="store_true",
                    help="skip the strong-scaling and per-config objects")
    ap.add_argument("--config-steps", type=int, default=10,
                    help="timed steps of each strong/configs entry")
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
    else:
        run_gpu_arm(args, w)


if __name__ == "__main__":
    main()
