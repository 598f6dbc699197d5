"""CPU tests: the oracle restatement is pinned bit for bit to the reference.

tests/golden/*.json hold FNV-1a fingerprints of the reference's own CPU
attention and fills (made by tests/golden/make_golden.py from oracle/_ref).
"""
import json
from pathlib import Path

import numpy as np
import pytest

import oracle

GOLDEN = Path(__file__).resolve().parent / "golden"
ATTN = json.loads((GOLDEN / "attention_reference.json").read_text())["cases"]
FILLS = json.loads((GOLDEN / "gemm_reference_fills.json").read_text())["fills"]


def _inputs(c):
    q = oracle.fill_pattern(c["pattern"], "q", c["B"], c["Hq"], c["Sq"], c["D"])
    k = oracle.fill_pattern(c["pattern"], "k", c["B"], c["Hkv"], c["Skv"], c["D"])
    v = oracle.fill_pattern(c["pattern"], "v", c["B"], c["Hkv"], c["Skv"], c["D"])
    return q, k, v


@pytest.mark.parametrize("case", ATTN, ids=[c["label"] for c in ATTN])
def test_pattern_fills_match_reference(case):
    q, k, v = _inputs(case)
    assert f"{oracle.fnv1a64(q):016x}" == case["fnv_q"]
    assert f"{oracle.fnv1a64(k):016x}" == case["fnv_k"]
    assert f"{oracle.fnv1a64(v):016x}" == case["fnv_v"]


@pytest.mark.parametrize("case", ATTN, ids=[c["label"] for c in ATTN])
@pytest.mark.parametrize("threads", [1, 3])
def test_attention_bit_exact_vs_reference_golden(case, threads):
    q, k, v = _inputs(case)
    out = oracle.attention(q, k, v, causal=case["causal"], threads=threads)
    assert f"{oracle.fnv1a64(out):016x}" == case["fnv_out_f32"], case["label"]
    assert f"{oracle.fnv1a64(oracle.f32_to_bf16(out)):016x}" == case["fnv_out_bf16"]
    np.testing.assert_array_equal(out.reshape(-1)[:8], np.float32(case["first"]))


def test_rows_variant_matches_full():
    c = next(x for x in ATTN if x["label"] == "extra_causal_sq_gt_skv")
    q, k, v = _inputs(c)
    full = oracle.attention(q, k, v, causal=True)
    part = oracle.attention_rows(q, k, v, b=0, h_begin=1, h_end=3, q_begin=150, q_end=260,
                                 causal=True)
    np.testing.assert_array_equal(part, full[0, 1:3, 150:260])


def test_fully_masked_rows_are_zero():
    # Sq > Skv with bottom-right causal: the first Sq-Skv rows see no key.
    c = next(x for x in ATTN if x["label"] == "extra_causal_sq_gt_skv")
    q, k, v = _inputs(c)
    out = oracle.attention(q, k, v, causal=True)
    assert not out[:, :, : c["Sq"] - c["Skv"]].any()
    assert out[:, :, c["Sq"] - c["Skv"]:].any()


@pytest.mark.skipif(not oracle.ref_available(), reason="oracle/_ref not built here")
def test_restatement_equals_reference_on_normal_inputs():
    rng = np.random.default_rng(7)
    q = oracle.f32_to_bf16(rng.standard_normal((1, 2, 96, 64), dtype=np.float32))
    k = oracle.f32_to_bf16(rng.standard_normal((1, 1, 150, 64), dtype=np.float32))
    v = oracle.f32_to_bf16(rng.standard_normal((1, 1, 150, 64), dtype=np.float32))
    for causal in (False, True):
        a = oracle.attention(q, k, v, causal=causal)
        b = oracle.attention(q, k, v, causal=causal, use_reference=True)
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


@pytest.mark.parametrize("fill", FILLS, ids=[f"{f['pattern']}_{f['size']}" for f in FILLS])
def test_gemm_fills_match_reference(fill):
    a = oracle.gemm_fill("a", fill["pattern"], fill["size"], fill["size"])
    b = oracle.gemm_fill("b", fill["pattern"], fill["size"], fill["size"])
    assert f"{oracle.fnv1a64(a):016x}" == fill["fnv_a"]
    assert f"{oracle.fnv1a64(b):016x}" == fill["fnv_b"]


@pytest.mark.parametrize("b_col_major", [True, False])
def test_gemm_oracle_exact_on_validation_patterns(b_col_major):
    # The reference's validation values are small multiples of 2^-9 whose
    # products and sums are exact in double, so any summation order gives the
    # same answer: an integer matmul is an independent exact check.
    n = 256
    a = oracle.gemm_fill("a", "pattern", n, n)
    b = oracle.gemm_fill("b", "pattern", n, n)  # [K, N]
    bm = np.ascontiguousarray(b.T) if b_col_major else b
    got = oracle.gemm(a, bm, b_col_major)
    ai = np.rint(oracle.bf16_to_f32(a).astype(np.float64) * 512).astype(np.int64)
    bi = np.rint(oracle.bf16_to_f32(b).astype(np.float64) * 512).astype(np.int64)
    exact = (ai @ bi).astype(np.float64) / (512.0 * 512.0)
    np.testing.assert_array_equal(got, exact)
    ones = oracle.gemm(oracle.gemm_fill("a", "ones", 64, 96),
                       oracle.gemm_fill("b", "ones", 64, 96) if b_col_major else
                       oracle.gemm_fill("b", "ones", 96, 64), b_col_major)
    assert (ones == 96.0).all()


def test_compare_semantics_match_harness():
    # Fails only where abs AND rel both exceed (0.attention/main.cu:1563).
    exp = np.array([1.0, 1e-3, 0.0], dtype=np.float32)
    got = np.array([1.07, 1e-3 + 0.07, 0.05], dtype=np.float32)
    r = oracle.compare(got, exp, 6e-2, 8e-2)
    assert r["bad_count"] == 1  # element 1: abs 0.07 > 0.06 and rel huge
