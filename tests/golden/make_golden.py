"""Generate tests/golden/*.json from the REFERENCE's own CPU code.

Runs oracle/_ref (the reference's build_real_attention_reference and pattern
fillers from 0.attention/main.cu, and the GEMM validation fills from
5.GEMM/gemm256_tma_tcgen05_bench.cu, compiled in place -- see oracle/Makefile)
on the reference's validation suites plus a few extra general-shape cases, and
records FNV-1a 64-bit fingerprints of the inputs and of the fp32 outputs, with
a few sample values for diagnostics.  The oracle restatement must reproduce
every fingerprint bit for bit (tests/test_oracle.py).

Run in a checkout where the reference is present:
    make -C oracle all ref REF=<reference root>
    python tests/golden/make_golden.py
"""
from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
import oracle  # noqa: E402

HERE = Path(__file__).resolve().parent

# (label, B, Hq, Hkv, Sq, Skv, D, causal, pattern)
CASES = [
    # Fused validation suite, 0.attention/main.cu:1942-1947 (B=H=1, Sq=128, D=128).
    ("fused_real_attention_constant_k1", 1, 1, 1, 128, 128, 128, False, "constant"),
    ("fused_real_attention_rank1_k4", 1, 1, 1, 128, 512, 128, False, "rank1"),
    ("fused_real_attention_random_k4", 1, 1, 1, 128, 512, 128, False, "random"),
    ("fused_real_attention_random_k8", 1, 1, 1, 128, 1024, 128, False, "random"),
    # Scalar validation suite, 0.attention/main.cu:1998-2005.
    ("real_attention_constant_square", 1, 1, 1, 128, 128, 128, False, "constant"),
    ("real_attention_rank1_multi_k", 1, 1, 1, 128, 256, 128, False, "rank1"),
    ("real_attention_causal_k_longer", 1, 1, 1, 128, 384, 128, True, "rank1"),
    ("real_attention_random_tail", 1, 1, 1, 77, 193, 128, False, "random"),
    ("real_attention_b2_h4", 2, 4, 4, 128, 256, 128, False, "random"),
    ("real_attention_gqa", 1, 8, 2, 64, 128, 128, False, "random"),
    # Extra general shapes (the reference function is shape-generic).
    ("extra_onehot_k2", 1, 2, 2, 128, 256, 128, False, "onehot"),
    ("extra_d64_causal_tail", 1, 2, 1, 200, 300, 64, True, "random"),
    ("extra_d64_b2_gqa", 2, 4, 2, 96, 160, 64, False, "rank1"),
    ("extra_causal_sq_gt_skv", 1, 4, 2, 300, 100, 128, True, "random"),
    ("extra_causal_square_3tiles", 1, 2, 2, 384, 384, 128, True, "random"),
]


def main() -> None:
    if not oracle.ref_available():
        raise SystemExit("oracle/_ref not built: make -C oracle ref REF=<reference root>")
    cases = []
    for label, B, Hq, Hkv, Sq, Skv, D, causal, pattern in CASES:
        q = oracle.fill_pattern(pattern, "q", B, Hq, Sq, D, use_reference=True)
        k = oracle.fill_pattern(pattern, "k", B, Hkv, Skv, D, use_reference=True)
        v = oracle.fill_pattern(pattern, "v", B, Hkv, Skv, D, use_reference=True)
        out = oracle.attention(q, k, v, causal=causal, use_reference=True)
        flat = out.reshape(-1)
        cases.append({
            "label": label, "B": B, "Hq": Hq, "Hkv": Hkv, "Sq": Sq, "Skv": Skv, "D": D,
            "causal": causal, "pattern": pattern,
            "fnv_q": f"{oracle.fnv1a64(q):016x}", "fnv_k": f"{oracle.fnv1a64(k):016x}",
            "fnv_v": f"{oracle.fnv1a64(v):016x}",
            "fnv_out_f32": f"{oracle.fnv1a64(out):016x}",
            "fnv_out_bf16": f"{oracle.fnv1a64(oracle.f32_to_bf16(out)):016x}",
            "first": [float(x) for x in flat[:8]],
            "sum": float(np.sum(flat, dtype=np.float64)),
        })
        print(label, cases[-1]["fnv_out_f32"])
    (HERE / "attention_reference.json").write_text(json.dumps(
        {"source": "oracle/_ref built from the reference's 0.attention/main.cu",
         "cases": cases}, indent=1) + "\n")

    gemm = []
    for pattern in ("pattern", "ones"):
        for size in (256, 512):
            a = oracle.gemm_fill("a", pattern, size, size, use_reference=True)
            b = oracle.gemm_fill("b", pattern, size, size, use_reference=True)
            gemm.append({"pattern": pattern, "size": size, "fnv_a": f"{oracle.fnv1a64(a):016x}",
                         "fnv_b": f"{oracle.fnv1a64(b):016x}"})
    (HERE / "gemm_reference_fills.json").write_text(json.dumps(
        {"source": "oracle/_ref built from the reference's 5.GEMM/gemm256_tma_tcgen05_bench.cu",
         "fills": gemm}, indent=1) + "\n")


if __name__ == "__main__":
    main()
