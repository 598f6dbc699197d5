"""Clock-cycle trace of one CTA of the fused attention kernel.

Stands in for the reference's ATTENTION_CLOCK_TRACE build, its per-stage CSV
(0.attention/main.cu:808-1157) and the stage-rate summary of its plotter
(0.attention/plot_attention_trace.py:24-46): run `attention_fwd_trace`, decode
the per-role records, print per-tile stage durations in SM cycles (clock64 of
the CTA's SM, so all roles share one time base), and write the trace as the
reference's per-iteration CSV, which its plotter renders to SVG.

    python -m benchmark_b200.trace --b 4 --h 32 --n 4096 --d 128 --cta 7 \\
        --csv trace.csv --reference-csv trace_ref.csv

Records carry the CTA's global K/V tile index as `iter` (tile t belongs to
softmax pipe t & 1); softmax records carry the pipe as `tile`.
"""
from __future__ import annotations

import argparse
import csv
import statistics
from collections import defaultdict

EVENTS = {1: "tma_k", 2: "tma_v", 3: "tma_q", 4: "mma_s", 5: "mma_pv", 6: "mma_wait",
          7: "mma_go", 8: "mma_end", 9: "sm_wait", 10: "sm_ready", 11: "sm_ld_done",
          12: "sm_max_done", 13: "sm_p_computed", 14: "sm_published", 15: "sm_item_end",
          16: "epi_begin", 17: "epi_end"}
ROLES = {0: "tma", 1: "mma", 2: "softmax0", 3: "softmax1", 4: "epilogue", 5: "tma_v"}


def run_trace(q, k, v, causal=False, cta=0, cap=16384, raise_on_timeout=True):
    """One traced launch; returns (O, records with clocks relative to the
    first).  With raise_on_timeout=False a launch whose bounded waits ran out
    still returns its records, which show where each role stopped."""
    import torch

    from . import _lib, ops
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
    return o, decode(raw)


def decode(raw) -> list[dict]:
    """Records of a [roles, cap, 2] uint64 trace buffer, clocks relative to
    the earliest record."""
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
    return recs


def _index(recs):
    """(role, event, iter) -> clock of the first such record."""
    at = {}
    for r in recs:
        at.setdefault((r["role"], r["event"], r["iter"]), r["clock"])
    return at


def summarize(recs):
    """Median per-tile stage lengths (cycles) of both softmax pipes, their
    period, and the issuer's reaction time to a published P."""
    at = _index(recs)
    stages = defaultdict(list)
    for pipe in (0, 1):
        role = f"softmax{pipe}"
        iters = sorted({r["iter"] for r in recs if r["role"] == role and r["event"] == "sm_wait"})
        for t in iters:
            g = {e: at.get((role, e, t)) for e in
                 ("sm_wait", "sm_ready", "sm_ld_done", "sm_max_done", "sm_p_computed",
                  "sm_published")}
            if None in g.values():
                continue
            stages[f"{role}.wait_s"].append(g["sm_ready"] - g["sm_wait"])
            stages[f"{role}.ld"].append(g["sm_ld_done"] - g["sm_ready"])
            stages[f"{role}.max"].append(g["sm_max_done"] - g["sm_ld_done"])
            stages[f"{role}.p_loop"].append(g["sm_p_computed"] - g["sm_max_done"])
            stages[f"{role}.publish"].append(g["sm_published"] - g["sm_p_computed"])
            stages[f"{role}.busy"].append(g["sm_published"] - g["sm_ready"])
            nxt = at.get((role, "sm_wait", t + 2))
            if nxt is not None:
                stages[f"{role}.period"].append(nxt - g["sm_wait"])
            s_issue = at.get(("mma", "mma_s", t))
            if s_issue is not None:
                stages[f"{role}.s_issue_to_ready"].append(g["sm_ready"] - s_issue)
            pv = at.get(("mma", "mma_pv", t))
            if pv is not None:
                stages[f"mma.{role}_published_to_pv_issue"].append(pv - g["sm_published"])
    return {k: (statistics.median(v), min(v), max(v), len(v)) for k, v in sorted(stages.items())}


# ---------------------------------------------------------------------------
# The reference's per-iteration trace CSV (0.attention/main.cu:977-1016 writes
# its header; 0.attention/plot_attention_trace.py reads it)
# ---------------------------------------------------------------------------
CONSUMER_LANES = 8  # kTraceConsumerLanesPerPipe (0.attention/main.cu:80)
SYNC_COUNT = 4      # kClockTraceSyncCount (0.attention/main.cu:81)

REFERENCE_COLUMNS = (
    "mode,elapsed_ms,iter,pipe,warp_id,tma_warp_id,tma_start,tma_end,tma_cycles,mma_start,"
    "mma_end,mma_cycles,tma_issue_end,tma_issue_cycles,tma_wait_cycles,mma_issue_end,"
    "mma_issue_cycles,mma_wait_cycles,ld_start,ld_end,ld_cycles,pack_start,pack_end,pack_cycles,"
    "st_start,st_end,st_cycles,v_tma_start,v_tma_end,v_tma_cycles,v_tma_issue_end,"
    "v_tma_issue_cycles,v_tma_wait_cycles,v_tma_h0_start,v_tma_h0_end,v_tma_h0_cycles,"
    "v_tma_h0_issue_end,v_tma_h0_issue_cycles,v_tma_h0_wait_cycles,v_tma_h1_start,"
    "v_tma_h1_end,v_tma_h1_cycles,v_tma_h1_issue_end,v_tma_h1_issue_cycles,"
    "v_tma_h1_wait_cycles,pv_start,pv_end,pv_cycles,pv_issue_end,pv_issue_cycles,"
    "pv_wait_cycles,pv_warp_id,pv_h0_start,pv_h0_end,pv_h0_cycles,pv_h0_warp_id,pv_h1_start,"
    "pv_h1_end,pv_h1_cycles,pv_h1_warp_id,total_start,total_end,total_cycles").split(",")
for _w in range(CONSUMER_LANES):
    REFERENCE_COLUMNS += [f"ld_warp{_w}_start", f"ld_warp{_w}_end"]
for _kind in ("pack", "pack_detail", "st", "sum"):
    for _w in range(CONSUMER_LANES):
        REFERENCE_COLUMNS += [f"{_kind}_warp{_w}_start", f"{_kind}_warp{_w}_end"]
for _i in range(SYNC_COUNT):
    REFERENCE_COLUMNS += [f"sync{_i}_start", f"sync{_i}_end", f"sync{_i}_cycles"]
REFERENCE_COLUMNS += ["status", "cuda_error", "notes"]


def reference_rows(recs, elapsed_ms: float = 0.0, clock_offset: int = 1) -> list[dict]:
    """One row per K/V tile t of the traced CTA in the reference's columns.

    The reference's stages map onto this kernel's as follows (a stage this
    kernel does not have, or does not stamp, is written as 0, which the
    reference plotter treats as absent):
      tma    K(t) load issued -> S(t) issued (the issuer had seen K(t) land)
      mma    S(t) issued -> its softmax pipe saw S(t) complete
      ld     that moment -> the scores are in registers (tcgen05.ld done)
      pack   -> P computed (row max, exp2, bf16 pack and P stores issued)
      st     -> P published (store wait, fence, barrier arrive)
      v_tma  V(t) load issued -> PV(t) issued
      pv     PV(t) issued -> the next MMA issued after it
    `pipe` is the softmax pipe (t & 1).  Warp ids follow the plotter's lane
    model, one lane set per pipe (0.attention/plot_attention_trace.py:339-396):
    warp_id = pv_warp_id = pipe (its "QK/PV warp" lane: this kernel's MMA
    issuer, warp 13, serving that pipe), tma_warp_id = 2 + pipe (its "K/V
    TMA" lane: warps 12 and 14 here), and the traced softmax warp (warp 0 or
    4 here) as consumer lane 0 of its pipe.  Clocks are shifted by
    clock_offset so that no stamp is 0."""
    at = _index(recs)
    mma_issue = sorted((r["clock"], r["event"], r["iter"]) for r in recs
                       if r["role"] == "mma" and r["event"] in ("mma_s", "mma_pv"))
    next_issue = {}
    for (_, e0, i0), (c1, _, _) in zip(mma_issue, mma_issue[1:]):
        next_issue[(e0, i0)] = c1
    tiles = sorted({r["iter"] for r in recs if r["role"] in ("softmax0", "softmax1")
                    and r["event"] == "sm_published"})
    rows = []
    for t in tiles:
        pipe = t & 1
        role = f"softmax{pipe}"

        def g(role_, ev, it=t):
            return at.get((role_, ev, it))

        stamps = {
            "tma": (g("tma", "tma_k"), g("mma", "mma_s")),
            "mma": (g("mma", "mma_s"), g(role, "sm_ready")),
            "ld": (g(role, "sm_ready"), g(role, "sm_ld_done")),
            "pack": (g(role, "sm_ld_done"), g(role, "sm_p_computed")),
            "st": (g(role, "sm_p_computed"), g(role, "sm_published")),
            "v_tma": (g("tma_v", "tma_v"), g("mma", "mma_pv")),
            "pv": (g("mma", "mma_pv"), next_issue.get(("mma_pv", t))),
        }
        row = {c: 0 for c in REFERENCE_COLUMNS}
        row.update({"mode": "b200_two_pipe_attention_trace", "elapsed_ms": f"{elapsed_ms:.6f}",
                    "iter": t, "pipe": pipe, "warp_id": pipe, "tma_warp_id": 2 + pipe,
                    "pv_warp_id": pipe, "pv_h0_warp_id": -1, "pv_h1_warp_id": -1,
                    "status": "ok", "cuda_error": "no error",
                    "notes": "stages mapped onto the two-pipe kernel (benchmark_b200/trace.py)"})
        first = last = None
        for name, (a, b) in stamps.items():
            if a is None or b is None or b < a:
                continue
            row[f"{name}_start"] = a + clock_offset
            row[f"{name}_end"] = b + clock_offset
            row[f"{name}_cycles"] = b - a
            first = a if first is None else min(first, a)
            last = b if last is None else max(last, b)
        if row["tma_start"] == 0:  # the plotter's time base is the rows' tma_start
            continue
        for name in ("ld", "pack", "st"):
            if row[f"{name}_start"]:
                row[f"{name}_warp0_start"] = row[f"{name}_start"]
                row[f"{name}_warp0_end"] = row[f"{name}_end"]
        row["total_start"] = first + clock_offset
        row["total_end"] = last + clock_offset
        row["total_cycles"] = last - first
        rows.append(row)
    return rows


def write_reference_csv(path, recs, elapsed_ms: float = 0.0) -> int:
    rows = reference_rows(recs, elapsed_ms)
    with open(path, "w", newline="") as f:
        w = csv.DictWriter(f, fieldnames=REFERENCE_COLUMNS)
        w.writeheader()
        w.writerows(rows)
    return len(rows)


def main() -> None:
    import torch

    from . import ops
    ap = argparse.ArgumentParser()
    ap.add_argument("--b", type=int, default=4)
    ap.add_argument("--h", type=int, default=32)
    ap.add_argument("--n", type=int, default=4096)
    ap.add_argument("--d", type=int, default=128)
    ap.add_argument("--causal", action="store_true")
    ap.add_argument("--cta", type=int, default=7)
    ap.add_argument("--sigma", type=float, default=1.0)
    ap.add_argument("--csv", default=None, help="raw records (role,event,tile,iter,clock)")
    ap.add_argument("--reference-csv", default=None,
                    help="the reference's per-iteration trace CSV (its plotter's input)")
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
        print(f"{k_:40s} median {med:8.0f}  min {lo:8d}  max {hi:8d}  n {n}")
    if a.csv:
        with open(a.csv, "w", newline="") as f:
            w = csv.DictWriter(f, fieldnames=["role", "event", "tile", "iter", "clock"])
            w.writeheader()
            w.writerows(sorted(recs, key=lambda r: r["clock"]))
    if a.reference_csv:
        n = write_reference_csv(a.reference_csv, recs)
        print(f"{n} rows in the reference trace format: {a.reference_csv}")


if __name__ == "__main__":
    main()
