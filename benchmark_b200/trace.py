"""Clock-cycle trace of one CTA of the fused attention kernel.

Stands in for the reference's ATTENTION_CLOCK_TRACE build, its per-stage CSV
(0.attention/main.cu:808-1157) and the stage-rate summary of its plotter
(0.attention/plot_attention_trace.py:24-46): run `attention_fwd_trace`, decode
the per-role records, print per-tile stage durations in SM cycles (clock64 of
the CTA's SM, so all roles share one time base), and write the trace as the
reference's per-iteration CSV, which its plotter renders to SVG.

    python -m benchmark_b200.trace --b 4 --h 32 --n 4096 --d 128 --cta 7 \\
        --csv trace.csv --reference-csv trace_ref.csv

Records carry the CTA's global K/V tile index as `iter`; every softmax warp
works on every tile, and softmax records carry the warpgroup (0 or 1) of the
traced warp as `tile`.
"""
from __future__ import annotations

import argparse
import csv
import statistics
from collections import defaultdict

EVENTS = {1: "tma_k", 2: "tma_v", 3: "tma_q", 4: "mma_s", 5: "mma_pv", 6: "mma_wait",
          7: "mma_go", 8: "mma_end", 9: "sm_wait", 10: "sm_ready", 11: "sm_ld_done",
          12: "sm_max_done", 13: "sm_p_computed", 14: "sm_published", 15: "sm_item_end",
          16: "epi_begin", 17: "epi_end", 18: "sm_p_loop_done"}
ROLES = {0: "tma", 1: "mma", 2: "softmax0", 3: "softmax1", 4: "epilogue", 5: "tma_v", 6: "mma_qk"}
# The traced softmax warps: warp 0 (role softmax0) and warp 4 (role softmax1).
SOFTMAX_ROLES = ("softmax0", "softmax1")
SOFTMAX_WARP = {"softmax0": 0, "softmax1": 4}


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
    """Median per-tile stage lengths (cycles) of the two traced softmax warps
    (warp 0 of the first softmax warpgroup, warp 4 of the second; all eight
    softmax warps work on every K/V tile), their period, and the issuer's
    reaction time to a published P.

    Per tile t of a warp: wait_s (sm_wait -> sm_ready), ld (the score load),
    then for a tile whose P is computed against the running max and screened
    (the common case) p_loop (exp2, pack and P stores) and screen (P-sum
    screen and S(t+1) readiness vote), or for a first or masked tile max (the
    exact tile max) and p_loop_exact; publish (store wait, fence, arrive),
    busy (sm_ready -> published) and period (sm_wait of this tile -> sm_wait of
    the warp's next tile).  The two-Q-tile kernel (non-causal d=64) records
    the S index as the iteration and the pipe as the tile; its softmax roles
    are pipe A's warp 0 and pipe B's warp 4."""
    at = _index(recs)
    # The role's next tile (t + 1 in the one-Q-tile kernel, the pipe's next S
    # index in the two-Q-tile kernel).
    next_wait = {}
    for role in SOFTMAX_ROLES:
        waits = sorted((r["iter"], r["clock"]) for r in recs
                       if r["role"] == role and r["event"] == "sm_wait")
        for (t0, _), (_, c1) in zip(waits, waits[1:]):
            next_wait[(role, t0)] = c1
    stages = defaultdict(list)
    for role in SOFTMAX_ROLES:
        iters = sorted({r["iter"] for r in recs if r["role"] == role and r["event"] == "sm_wait"})
        for t in iters:
            g = {e: at.get((role, e, t)) for e in
                 ("sm_wait", "sm_ready", "sm_ld_done", "sm_p_computed", "sm_published")}
            if None in g.values():
                continue
            stages[f"{role}.wait_s"].append(g["sm_ready"] - g["sm_wait"])
            stages[f"{role}.ld"].append(g["sm_ld_done"] - g["sm_ready"])
            loop_done = at.get((role, "sm_p_loop_done", t))
            max_done = at.get((role, "sm_max_done", t))
            if loop_done is not None:
                stages[f"{role}.p_loop"].append(loop_done - g["sm_ld_done"])
                stages[f"{role}.screen"].append(g["sm_p_computed"] - loop_done)
            elif max_done is not None:
                stages[f"{role}.max"].append(max_done - g["sm_ld_done"])
                stages[f"{role}.p_loop_exact"].append(g["sm_p_computed"] - max_done)
            stages[f"{role}.publish"].append(g["sm_published"] - g["sm_p_computed"])
            stages[f"{role}.busy"].append(g["sm_published"] - g["sm_ready"])
            nxt = next_wait.get((role, t))
            if nxt is not None:
                stages[f"{role}.period"].append(nxt - g["sm_wait"])
            s_issue = at.get(("mma_qk", "mma_s", t))
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
      tma    K(t) load issued -> S(t) issued (the S issuer had seen K(t) land)
      mma    S(t) issued -> softmax warp 0 saw S(t) complete
      ld     that moment -> the scores are in registers (tcgen05.ld done)
      pack   -> P computed (exp2, bf16 pack, P stores issued, screen)
      st     -> P published (store wait, fence, barrier arrive)
      v_tma  V(t) load issued -> PV(t) issued
      pv     PV(t) issued -> the PV issuer's next record (its MMAs accepted)
    The kernel has one pipe: its eight softmax warps all work on every tile
    (16 rows each), so every row has pipe 0.  Warp ids follow the plotter's
    lane model (0.attention/plot_attention_trace.py:339-396): warp_id =
    pv_warp_id = 0 (its "QK/PV warp" lane: this kernel's MMA issuers, warps
    15 and 13), tma_warp_id = 2 (its "K/V TMA" lane: warps 12 and 14 here), and
    the two traced softmax warps, 0 and 4, as consumer lanes 0 and 4 of the
    eight.  Clocks are shifted by clock_offset so that no stamp is 0."""
    at = _index(recs)
    pv_warp = sorted((r["clock"], r["event"], r["iter"]) for r in recs if r["role"] == "mma")
    pv_issued = {}  # PV(t) issued -> the PV issuer's next record (its 8 MMAs accepted)
    for (_, e0, i0), (c1, _, _) in zip(pv_warp, pv_warp[1:]):
        if e0 == "mma_pv":
            pv_issued[i0] = c1
    lead = SOFTMAX_ROLES[0]
    tiles = sorted({r["iter"] for r in recs if r["role"] == lead and r["event"] == "sm_published"})
    rows = []
    for t in tiles:
        def g(role_, ev, it=t):
            return at.get((role_, ev, it))

        def consumer(role_):
            return {"ld": (g(role_, "sm_ready"), g(role_, "sm_ld_done")),
                    "pack": (g(role_, "sm_ld_done"), g(role_, "sm_p_computed")),
                    "st": (g(role_, "sm_p_computed"), g(role_, "sm_published"))}

        stamps = {
            "tma": (g("tma", "tma_k"), g("mma_qk", "mma_s")),
            "mma": (g("mma_qk", "mma_s"), g(lead, "sm_ready")),
            **consumer(lead),
            "v_tma": (g("tma_v", "tma_v"), g("mma", "mma_pv")),
            "pv": (g("mma", "mma_pv"), pv_issued.get(t)),
        }
        row = {c: 0 for c in REFERENCE_COLUMNS}
        row.update({"mode": "b200_attention_trace", "elapsed_ms": f"{elapsed_ms:.6f}",
                    "iter": t, "pipe": 0, "warp_id": 0, "tma_warp_id": 2,
                    "pv_warp_id": 0, "pv_h0_warp_id": -1, "pv_h1_warp_id": -1,
                    "status": "ok", "cuda_error": "no error",
                    "notes": "stages mapped onto the one-pipe kernel (benchmark_b200/trace.py)"})
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
        for role in SOFTMAX_ROLES:
            lane = SOFTMAX_WARP[role]
            for name, (a, b) in consumer(role).items():
                if a is None or b is None or b < a:
                    continue
                row[f"{name}_warp{lane}_start"] = a + clock_offset
                row[f"{name}_warp{lane}_end"] = b + clock_offset
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
