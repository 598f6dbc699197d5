"""CPU checks of the clock-trace decoder (benchmark_b200/trace.py): record
layout and per-tile stage arithmetic on synthetic records."""
import re
from pathlib import Path

import numpy as np

from benchmark_b200 import trace


def _recs():
    recs = []
    for j in range(3):
        base = 1000 * j
        for h, off in ((0, 0), (1, 10)):
            role = f"softmax{h}"
            for ev, dt in (("sm_wait", 0), ("sm_ld_done", 50), ("sm_max_done", 150),
                           ("sm_p_computed", 700), ("sm_p_stored", 800), ("sm_p_lo", 820)):
                recs.append({"role": role, "event": ev, "tile": h, "iter": j,
                             "clock": base + off + dt})
        recs.append({"role": "mma", "event": "mma_s", "tile": 0, "iter": j, "clock": base - 300})
        recs.append({"role": "mma", "event": "mma_pv_hi", "tile": 0, "iter": j,
                     "clock": base + 900})
    return recs


def test_summarize_stage_lengths():
    st = trace.summarize(_recs())
    assert st["softmax0.wait_s+ld"][0] == 50
    assert st["softmax0.max"][0] == 100
    assert st["softmax0.p_compute"][0] == 550
    assert st["softmax0.prefetch+rescale"][0] == 100
    assert st["softmax0.arrive"][0] == 20
    assert st["softmax0.period"][0] == 1000 and st["softmax0.period"][3] == 2
    assert st["softmax1.s_issue_to_ld_done"][0] == 360
    assert st["mma.softmax0_p_to_pv_hi_issue"][0] == 80


def _kernel_event_count():
    """Number of members of the kernel's clock-trace event enum (values 1..n)."""
    src = (Path(trace.__file__).parent / "csrc" / "attention_kernel.cuh").read_text()
    body = re.search(r"enum : uint32_t \{\s*(kEvTmaK = 1,[^}]*)\}", src).group(1)
    return len([m for m in body.replace("\n", " ").split(",") if m.strip()])


def test_event_and_role_tables_cover_the_kernel_enums():
    # One name per event the kernel's Tracer writes (1..n) and roles 0..4.
    assert sorted(trace.EVENTS) == list(range(1, _kernel_event_count() + 1))
    assert sorted(trace.ROLES) == [0, 1, 2, 3, 4]
    assert len(set(trace.EVENTS.values())) == len(trace.EVENTS)


def test_record_key_layout():
    # (event << 32 | tile << 24 | iter), as Tracer::operator() packs it
    key = np.uint64((7 << 32) | (3 << 24) | 12345)
    assert int(key >> np.uint64(32)) == 7
    assert int((key >> np.uint64(24)) & np.uint64(0xff)) == 3
    assert int(key & np.uint64(0xffffff)) == 12345
