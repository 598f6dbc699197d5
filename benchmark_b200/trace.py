"""Clock-cycle trace of one CTA of the fused attention kernel.

Stands in for the reference's ATTENTION_CLOCK_TRACE build, its per-stage CSV
(0.attention/main.cu:808-1157) and the stage-rate summary of its plotter
(0.attention/plot_attention_trace.py:24-46): run `attention_fwd_trace`, decode
the per-role records, and print/write per-iteration stage durations in SM
cycles (clock64 of the CTA's SM, so all roles share one time base).

    python -m benchmark_b200.trace --b 4 --h 32 --n 4096 --d 128 --cta 7 --csv trace.csv

Softmax records (warps 0 and 4) carry warp/4 as `tile` and the CTA's global
K/V tile index as `iter`; MMA records carry the Q/O buffer as `tile`.
"""
from __future__ import annotations

import argparse
import csv
import statistics
from collections import defaultdict

import torch

from . import _lib, ops

EVENTS = {1: "tma_k", 2: "tma_v", 3: "mma_s", 4: "mma_pv_lo", 5: "mma_pv_hi", 6: "sm_wait",
          7: "sm_pf_tested", 8: "sm_ld_done", 9: "sm_max_done", 10: "sm_p_lo",
          11: "sm_pf_issued", 12: "epi_begin", 13: "epi_end", 14: "mma_wait", 15: "mma_end",
          16: "mma_go", 17: "tma_q", 18: "sm_p_computed", 19: "sm_p_stored",
          20: "sm_st_waited", 21: "sm_screened", 22: "sm_l_done"}
ROLES = {0: "tma", 1: "mma", 2: "softmax0", 3: "softmax1", 4: "epilogue"}


def run_trace(q, k, v, causal=False, cta=0, cap=16384, raise_on_timeout=True):
    """One traced launch; returns (O, records with clocks relative to the
    first).  With raise_on_timeout=False a launch whose bounded waits ran out
    still returns its records, which show where each role stopped."""
    B, Hq, Sq, D = q.shape
    Hkv, Skv = k.shape[1], k.shape[2]
    buf = torch.zeros(len(ROLES) * cap * 2, dtype=torch.int64, device=q.device)
    o = torch.empty_like(q)
    _lib.call("attention_fwd_trace", q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), B,
              Hq, Hkv, Sq, Skv, D, int(causal), -1.0, buf.data_ptr(), cap, cta,
              torch.cuda.current_stream().cuda_stream)
    try:
        ops.check()
    except _lib.B200Error as e:
        if raise_on_timeout or e.status != _lib.B200_ETIMEOUT:
            raise
        print(f"launch timed out: {e}")
    raw = buf.view(len(ROLES), cap, 2).cpu().numpy().astype("uint64")
    recs = []
    for role in range(len(ROLES)):
        for key, clk in raw[role]:
            if key == 0 and clk == 0:
                break
            recs.append({"role": ROLES[role], "event": EVENTS.get(int(key >> 32), str(key >> 32)),
                         "tile": int((key >> 24) & 0xff), "iter": int(key & 0xffffff),
                         "clock": int(clk)})
    t0 = min(r["clock"] for r in recs) if recs else 0
    for r in recs:
        r["clock"] -= t0
    return o, recs


def summarize(recs):
    """Median per-tile stage lengths (cycles) of both softmax warpgroups and
    the issuer's reaction time to each half of P."""
    at = {(r["role"], r["event"], r["tile"], r["iter"]): r["clock"] for r in recs}
    mma = {(r["event"], r["iter"]): r["clock"] for r in recs if r["role"] == "mma"}
    stages = defaultdict(list)
    for h in (0, 1):
        role = f"softmax{h}"
        iters = sorted({r["iter"] for r in recs if r["role"] == role})
        for j in iters:
            g = {e: at.get((role, e, h, j)) for e in
                 ("sm_wait", "sm_ld_done", "sm_max_done", "sm_p_lo", "sm_p_computed",
                  "sm_p_stored")}
            if None in g.values():
                continue
            p_done = g["sm_p_lo"]
            stages[f"{role}.wait_s+ld"].append(g["sm_ld_done"] - g["sm_wait"])
            stages[f"{role}.max"].append(g["sm_max_done"] - g["sm_ld_done"])
            stages[f"{role}.p_compute"].append(g["sm_p_computed"] - g["sm_max_done"])
            stages[f"{role}.prefetch+rescale"].append(g["sm_p_stored"] - g["sm_p_computed"])
            stages[f"{role}.arrive"].append(p_done - g["sm_p_stored"])
            nxt = at.get((role, "sm_wait", h, j + 1))
            if nxt is not None:
                stages[f"{role}.period"].append(nxt - g["sm_wait"])
            s_issue = mma.get(("mma_s", j))
            if s_issue is not None:
                stages[f"{role}.s_issue_to_ld_done"].append(g["sm_ld_done"] - s_issue)
            pv = mma.get(("mma_pv_hi", j))
            if pv is not None:
                stages[f"mma.{role}_p_to_pv_hi_issue"].append(pv - p_done)
    return {k: (statistics.median(v), min(v), max(v), len(v)) for k, v in sorted(stages.items())}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--b", type=int, default=4)
    ap.add_argument("--h", type=int, default=32)
    ap.add_argument("--n", type=int, default=4096)
    ap.add_argument("--d", type=int, default=128)
    ap.add_argument("--causal", action="store_true")
    ap.add_argument("--cta", type=int, default=7)
    ap.add_argument("--sigma", type=float, default=1.0)
    ap.add_argument("--csv", default=None)
    ap.add_argument("--warmup", type=int, default=3)
    a = ap.parse_args()
    q = torch.empty((a.b, a.h, a.n, a.d), dtype=torch.bfloat16, device="cuda")
    k, v = torch.empty_like(q), torch.empty_like(q)
    for t, i in ((q, 0), (k, 1), (v, 2)):
        ops.fill_normal_(t, 1, i, 0.0, a.sigma)
    for _ in range(a.warmup):
        run_trace(q, k, v, a.causal, a.cta, raise_on_timeout=False)
    _, recs = run_trace(q, k, v, a.causal, a.cta, raise_on_timeout=False)
    print(f"{len(recs)} records, CTA {a.cta}, span {max(r['clock'] for r in recs)} cycles")
    for k_, (med, lo, hi, n) in summarize(recs).items():
        print(f"{k_:32s} median {med:8.0f}  min {lo:8d}  max {hi:8d}  n {n}")
    if a.csv:
        with open(a.csv, "w", newline="") as f:
            w = csv.DictWriter(f, fieldnames=["role", "event", "tile", "iter", "clock"])
            w.writeheader()
            w.writerows(sorted(recs, key=lambda r: r["clock"]))


if __name__ == "__main__":
    main()
