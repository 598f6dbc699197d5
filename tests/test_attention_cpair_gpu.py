"""GPU parity tests of the CTA-pair form of the d=128 kernel (cta_group::2:
non-causal head_dim-128 problems with a pair of Q tiles for every two SMs
and no K/V split run on clusters of two CTAs that share each K/V tile's
shared-memory copy; benchmark_b200/csrc/attention_kernel.cuh, kPair).
Ragged Q and K/V tails, an odd Q-tile count (the pair's second CTA then
has no rows), GQA, the lazy-rescale paths, clipped stores, determinism.
Each shape is sized so that its Q-tile pairs fill the SMs two by two."""
import ctypes

import numpy as np
import pytest
import torch

import oracle
from attn_util import (HARNESS_ABS, HARNESS_REL, MEAN_ABS, gate, normal_inputs, to_host_bits,
                       to_host_f32)
from benchmark_b200 import ops

pytestmark = pytest.mark.gpu


def _units(B, Hq, Sq):
    return B * Hq * (((Sq + 127) // 128 + 1) // 2)


def _sms():
    return torch.cuda.get_device_properties(0).multi_processor_count


@pytest.mark.parametrize("B,Hq,Hkv,Sq,Skv", [
    (2, 40, 8, 300, 1000),    # GQA 5:1, 3 Q tiles (a pair and a lone tile), 104-key K/V tail
    (1, 150, 150, 256, 2048),  # one pair per head
    (3, 50, 25, 129, 130),    # one row past a tile; two keys past a tile
    (1, 80, 16, 1100, 700),   # 9 Q tiles (odd), Sq > Skv
])
def test_cpairs_vs_oracle(B, Hq, Hkv, Sq, Skv):
    assert 2 * _units(B, Hq, Sq) >= _sms()
    q, k, v = normal_inputs(B, Hq, Hkv, Sq, Skv, 128, seed=61)
    outs = []
    for _ in range(2):
        o = ops.attention_fwd(q, k, v)
        ops.check()
        outs.append(to_host_bits(o))
    assert np.array_equal(outs[0], outs[1]), "output not deterministic across repeats"
    ref = oracle.attention(to_host_bits(q), to_host_bits(k), to_host_bits(v))
    gate(oracle.bf16_to_f32(outs[0]), ref, f"cpairs B{B} Hq{Hq} Hkv{Hkv} Sq{Sq} Skv{Skv}")


@pytest.mark.parametrize("slope", [0.05, 0.004, -0.05])
def test_cpairs_rescale_paths(slope):
    """Scores climbing along the keys (about 100 or 8 log2 units per tile)
    raise each row's max on (nearly) every tile, so the screen, the exact-max
    recompute and the O rescale run on most tiles in both CTAs of a pair;
    falling scores never raise it.  A 32-key tail tile."""
    B, H, Sq, Skv, D = 1, 150, 256, 4000, 128
    assert 2 * _units(B, H, Sq) >= _sms()
    q = torch.ones((B, H, Sq, D), dtype=torch.bfloat16, device="cuda")
    ramp = (torch.arange(Skv, device="cuda", dtype=torch.float32) * slope).view(1, 1, Skv, 1)
    k = (torch.ones((B, H, Skv, D), device="cuda") * ramp).to(torch.bfloat16).contiguous()
    _, _, v = normal_inputs(B, H, H, 1, Skv, D, seed=63)
    o = ops.attention_fwd(q, k, v)
    ops.check()
    ref = oracle.attention(to_host_bits(q), to_host_bits(k), to_host_bits(v))
    gate(to_host_f32(o), ref, f"cpairs rescale slope {slope}")


def test_cpairs_large_random_scores():
    """N(0,1) inputs scaled up so that the max moves by more than 2^8 at
    random tiles and rows (the same peaked-softmax bound as the d=64 pair
    test: harness rule, mean gate, max |dO| <= 4e-2)."""
    B, H, S, D = 1, 148, 512, 128
    q, k, v = normal_inputs(B, H, H, S, S, D, seed=65)
    q = (q.float() * 3.0).to(torch.bfloat16).contiguous()
    ramp = torch.linspace(0.0, 3.0, S, device="cuda").view(1, 1, S, 1)
    k = (k.float() * (1.0 + ramp)).to(torch.bfloat16).contiguous()
    o = ops.attention_fwd(q, k, v)
    ops.check()
    ref = oracle.attention(to_host_bits(q), to_host_bits(k), to_host_bits(v))
    got = to_host_f32(o)
    r = oracle.compare(got, ref, HARNESS_ABS, HARNESS_REL)
    assert np.isfinite(got).all() and r["ok"], r
    assert r["max_abs"] <= 4e-2 and r["mean_abs"] <= MEAN_ABS, r


def test_cpairs_match_scalar_kernel():
    """A medium problem (B2 H24 N2560, 20 Q tiles per head) against the
    CUDA-core scalar kernel in full."""
    q, k, v = normal_inputs(2, 24, 24, 2560, 2560, 128, seed=67)
    o = ops.attention_fwd(q, k, v)
    s = ops.attention_fwd(q, k, v, scalar=True)
    ops.check()
    diff = (o.float() - s.float()).abs()
    assert diff.max().item() <= 2e-2 and diff.mean().item() <= 2e-3, (diff.max(), diff.mean())


def test_cpairs_store_clipped_at_tensor_edge():
    """3 Q tiles per head: every second pair's second CTA has no rows and
    stores nothing; the ragged tile's store clips.  A guard region after O
    stays intact."""
    B, H, S, D = 1, 100, 300, 128
    assert 2 * _units(B, H, S) >= _sms()
    q, k, v = normal_inputs(B, H, H, S, 500, D, seed=69)
    n = B * H * S * D
    buf = torch.full((n + 8192,), 7.0, dtype=torch.bfloat16, device="cuda")
    o = buf[:n].view(B, H, S, D)
    ops.attention_fwd(q, k, v, out=o)
    ops.check()
    assert (buf[n:] == 7.0).all()
    ref = oracle.attention_rows(to_host_bits(q), to_host_bits(k), to_host_bits(v), 0, 97, 100, 0,
                                S)
    gate(to_host_f32(o)[0, 97:100], ref, "cpairs last heads")


def test_cpairs_noalloc_matches():
    """attention_fwd_noalloc with one split takes the same path."""
    from benchmark_b200 import _lib
    q, k, v = normal_inputs(1, 150, 150, 256, 1024, 128, seed=71)
    ref = ops.attention_fwd(q, k, v)
    ops.check()
    o = torch.full_like(q, float("nan"))
    st = _lib.lib().attention_fwd_noalloc(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), 1, 150, 150, 256, 1024, 128, 0,
        ctypes.c_float(-1.0), 1, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == _lib.B200_OK, _lib.last_error()
    ops.check()
    assert torch.equal(o, ref)
