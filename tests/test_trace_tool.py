"""CPU checks of the clock-trace decoder (benchmark_b200/trace.py): record
layout, per-tile stage arithmetic on synthetic records, and the reference's
per-iteration trace CSV, rendered by the reference's own plotter
(0.attention/plot_attention_trace.py) where the reference checkout is present."""
import csv
import os
import re
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

from benchmark_b200 import trace

ROOT = Path(__file__).resolve().parents[1]


def _recs(tiles=8):
    """A synthetic trace: one tile every 2000 cycles, both traced softmax
    warps on every tile (warp 4 30 cycles behind warp 0), the first tile
    taking the exact-max path and the rest the screened path."""
    recs = []
    for t in range(tiles):
        base = 2000 * t + 1000
        recs.append({"role": "tma", "event": "tma_k", "tile": 0, "iter": t, "clock": base - 900})
        recs.append({"role": "tma_v", "event": "tma_v", "tile": 0, "iter": t, "clock": base - 800})
        recs.append({"role": "mma_qk", "event": "mma_s", "tile": 0, "iter": t, "clock": base - 600})
        recs.append({"role": "mma", "event": "mma_pv", "tile": 0, "iter": t, "clock": base + 1300})
        recs.append({"role": "mma", "event": "mma_wait", "tile": 4, "iter": 0, "clock": base + 1400})
        mid = ("sm_max_done", 250) if t == 0 else ("sm_p_loop_done", 950)
        for wg, lag in ((0, 0), (1, 30)):
            for ev, dt in (("sm_wait", -100), ("sm_ready", 0), ("sm_ld_done", 150), mid,
                           ("sm_p_computed", 1050), ("sm_published", 1250)):
                recs.append({"role": f"softmax{wg}", "event": ev, "tile": wg, "iter": t,
                             "clock": base + dt + lag})
    return recs


def test_summarize_stage_lengths():
    st = trace.summarize(_recs())
    assert st["softmax0.wait_s"][0] == 100
    assert st["softmax0.ld"][0] == 150
    assert st["softmax0.p_loop"][0] == 800 and st["softmax0.p_loop"][3] == 7
    assert st["softmax0.screen"][0] == 100
    assert st["softmax0.max"] == (100, 100, 100, 1)  # the first tile only
    assert st["softmax0.p_loop_exact"][0] == 800
    assert st["softmax0.publish"][0] == 200
    assert st["softmax1.busy"][0] == 1250
    assert st["softmax0.period"][0] == 2000 and st["softmax0.period"][3] == 7
    assert st["softmax1.s_issue_to_ready"][0] == 630
    assert st["mma.softmax0_published_to_pv_issue"][0] == 50
    assert st["mma.softmax1_published_to_pv_issue"][0] == 20


def _kernel_event_count():
    """Number of members of the kernel's clock-trace event enum (values 1..n)."""
    src = (Path(trace.__file__).parent / "csrc" / "attention_kernel.cuh").read_text()
    body = re.search(r"enum : uint32_t \{\s*(kEvTmaK = 1,[^}]*)\}", src).group(1)
    return len([m for m in body.replace("\n", " ").split(",") if m.strip()])


def test_event_and_role_tables_cover_the_kernel_enums():
    # One name per event the kernel's Tracer writes (1..n) and per role.
    assert sorted(trace.EVENTS) == list(range(1, _kernel_event_count() + 1))
    src = (Path(trace.__file__).parent / "csrc" / "attention_kernel.cuh").read_text()
    roles = int(re.search(r"constexpr int kTraceRoles = (\d+);", src).group(1))
    assert sorted(trace.ROLES) == list(range(roles))
    assert len(set(trace.EVENTS.values())) == len(trace.EVENTS)


def test_record_key_layout():
    # (event << 32 | tile << 24 | iter), as Tracer::operator() packs it
    key = np.uint64((7 << 32) | (3 << 24) | 12345)
    raw = np.zeros((len(trace.ROLES), 4, 2), dtype=np.uint64)
    raw[1, 0] = (key, np.uint64(500))
    raw[2, 0] = (np.uint64((9 << 32) | (1 << 24) | 2), np.uint64(400))
    recs = trace.decode(raw)
    assert {(r["role"], r["event"], r["tile"], r["iter"], r["clock"]) for r in recs} == {
        ("mma", "mma_go", 3, 12345, 100), ("softmax0", "sm_wait", 1, 2, 0)}


def test_reference_csv_columns_and_stages(tmp_path):
    path = tmp_path / "trace_ref.csv"
    n = trace.write_reference_csv(path, _recs(), elapsed_ms=0.5)
    assert n == 8
    with open(path, newline="") as f:
        rows = list(csv.DictReader(f))
    assert list(rows[0].keys()) == trace.REFERENCE_COLUMNS
    r3 = rows[3]
    assert int(r3["iter"]) == 3 and int(r3["pipe"]) == 0
    assert int(r3["ld_cycles"]) == 150 and int(r3["pack_cycles"]) == 900
    assert int(r3["st_cycles"]) == 200 and int(r3["mma_cycles"]) == 600
    assert int(r3["tma_cycles"]) == 300 and int(r3["v_tma_cycles"]) == 2100
    assert int(r3["pv_cycles"]) == 100  # PV(3) issued -> the PV issuer's next wait
    assert int(r3["ld_warp0_start"]) == int(r3["ld_start"])  # warp 0 is consumer lane 0
    assert int(r3["ld_warp4_start"]) == int(r3["ld_start"]) + 30  # warp 4 is lane 4
    assert int(r3["st_warp4_end"]) == int(r3["st_end"]) + 30
    assert int(r3["ld_warp1_start"]) == 0  # untraced lanes stay empty
    assert int(r3["warp_id"]) == 0 and int(r3["tma_warp_id"]) == 2
    assert all(int(r["tma_start"]) > 0 for r in rows)


def _reference_plotter():
    cand = os.environ.get("B200_REFERENCE_ROOT")
    root = Path(cand) if cand else ROOT.parent / "reference"
    p = root / "0.attention" / "plot_attention_trace.py"
    return p if p.exists() else None


def test_reference_plotter_renders_our_trace(tmp_path):
    plotter = _reference_plotter()
    if plotter is None:
        pytest.skip("reference checkout not present")
    path = tmp_path / "trace_ref.csv"
    trace.write_reference_csv(path, _recs(), elapsed_ms=0.5)
    svg, summary = tmp_path / "trace.svg", tmp_path / "summary.csv"
    r = subprocess.run([sys.executable, str(plotter), "--trace", str(path), "--iter-start", "2",
                        "--num-iters", "4", "--clock-mhz", "1965", "--summary-csv", str(summary),
                        "--svg", str(svg)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    text = svg.read_text()
    assert text.lstrip().startswith("<svg") or "<svg" in text[:500]
    assert summary.read_text().count("\n") > 4
