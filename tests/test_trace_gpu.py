"""GPU checks of attention_fwd_trace (the clock-trace build): the traced
kernels compute the same bytes as attention_fwd, every role records, and the
decoder's stage summary and reference-format rows come out of a real trace,
for the one-Q-tile kernel on CTA pairs (non-causal d=128, 128 Q-tile pairs)
and on one CTA per Q tile (causal d=128), and the two-Q-tile kernel
(non-causal d=64)."""
import pytest
import torch

from attn_util import normal_inputs
from benchmark_b200 import ops, trace

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("B,H,N,D,causal", [
    (2, 8, 2048, 128, False),   # one-Q-tile kernel on CTA pairs (CTA 3's pair leader issues)
    (1, 4, 2048, 128, True),    # one-Q-tile kernel, causal, one CTA per Q tile
    (8, 16, 2048, 64, False),   # two-Q-tile kernel (1024 units)
])
def test_trace_matches_and_records(B, H, N, D, causal):
    q, k, v = normal_inputs(B, H, H, N, N, D, seed=51, sigma=0.5 if D == 64 else 1.0)
    ref = ops.attention_fwd(q, k, v, causal=causal)
    ops.check()
    o, recs = trace.run_trace(q, k, v, causal=causal, cta=3)
    assert torch.equal(o, ref), "traced build computes different bytes"
    roles = {r["role"] for r in recs}
    assert {"tma", "tma_v", "mma", "mma_qk", "softmax0", "softmax1"} <= roles, roles
    st = trace.summarize(recs)
    for key in ("softmax0.period", "softmax0.busy", "softmax1.period",
                "mma.softmax0_published_to_pv_issue"):
        assert key in st and st[key][0] > 0, key
    rows = trace.reference_rows(recs)
    assert rows and all(int(r["tma_start"]) > 0 for r in rows)
