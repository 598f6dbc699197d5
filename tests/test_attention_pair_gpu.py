"""GPU parity tests of the two-Q-tile kernel for head_dim 64 (non-causal
problems with at least one work unit per SM run on it;
benchmark_b200/csrc/attention_pair_kernel.cuh): ragged Q and K/V tails,
units with a single Q tile, GQA, the lazy-rescale paths, determinism.  Each
shape is sized so that its units (Q-tile pairs) reach the SM count."""
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
    (2, 40, 8, 300, 1000),    # GQA 5:1, 3 Q tiles (a pair and a single), 104-key K/V tail
    (1, 160, 160, 256, 2048),  # one pair per head
    (3, 50, 25, 129, 130),    # one row past a tile; two keys past a tile
])
def test_pairs_vs_oracle(B, Hq, Hkv, Sq, Skv):
    assert _units(B, Hq, Sq) >= _sms()
    q, k, v = normal_inputs(B, Hq, Hkv, Sq, Skv, 64, seed=41, sigma=0.5)
    outs = []
    for _ in range(2):
        o = ops.attention_fwd(q, k, v)
        ops.check()
        outs.append(to_host_bits(o))
    assert np.array_equal(outs[0], outs[1]), "output not deterministic across repeats"
    ref = oracle.attention(to_host_bits(q), to_host_bits(k), to_host_bits(v))
    gate(oracle.bf16_to_f32(outs[0]), ref, f"pairs B{B} Hq{Hq} Hkv{Hkv} Sq{Sq} Skv{Skv}")


@pytest.mark.parametrize("slope", [0.05, 0.004, -0.05])
def test_pairs_rescale_paths(slope):
    """Scores climbing along the keys (about 100 or 8 log2 units per tile)
    raise each row's max on (nearly) every tile, so the screen, the exact-max
    recompute and the O rescale run on most tiles; falling scores never
    raise it.  The K/V length leaves a 32-key tail tile."""
    B, H, Sq, Skv, D = 1, 150, 256, 4000, 64
    assert _units(B, H, Sq) >= _sms()
    q = torch.ones((B, H, Sq, D), dtype=torch.bfloat16, device="cuda")
    ramp = (torch.arange(Skv, device="cuda", dtype=torch.float32) * slope).view(1, 1, Skv, 1)
    k = (torch.ones((B, H, Skv, D), device="cuda") * ramp * 2.0).to(torch.bfloat16).contiguous()
    _, _, v = normal_inputs(B, H, H, 1, Skv, D, seed=43)
    o = ops.attention_fwd(q, k, v)
    ops.check()
    ref = oracle.attention(to_host_bits(q), to_host_bits(k), to_host_bits(v))
    gate(to_host_f32(o), ref, f"pairs rescale slope {slope}")


def test_pairs_large_random_scores():
    """N(0,1) inputs scaled up so that the max moves by more than 2^8 at
    random tiles and rows.  The softmax is then so peaked that a row's output
    is one or two V rows weighted by P values rounded to bf16, and over these
    75,776 rows the largest |dO| reaches ~0.028 for both attention kernels
    (the one-Q-tile kernel gives the same 0.0276 on this input): the harness
    rule and the mean gate apply, and the max is bounded at 4e-2."""
    B, H, S, D = 1, 148, 512, 64
    q, k, v = normal_inputs(B, H, H, S, S, D, seed=45)
    q = (q.float() * 4.0).to(torch.bfloat16).contiguous()
    ramp = torch.linspace(0.0, 3.0, S, device="cuda").view(1, 1, S, 1)
    k = (k.float() * (1.0 + ramp)).to(torch.bfloat16).contiguous()
    o = ops.attention_fwd(q, k, v)
    ops.check()
    ref = oracle.attention(to_host_bits(q), to_host_bits(k), to_host_bits(v))
    got = to_host_f32(o)
    r = oracle.compare(got, ref, HARNESS_ABS, HARNESS_REL)
    assert np.isfinite(got).all() and r["ok"], r
    assert r["max_abs"] <= 4e-2 and r["mean_abs"] <= MEAN_ABS, r


def test_pairs_match_scalar_kernel_config4_shard():
    """Config 4's 8-GPU shard (B8 H16 N2048, sigma 0.5) against the CUDA-core
    scalar kernel in full."""
    q, k, v = normal_inputs(8, 16, 16, 2048, 2048, 64, seed=47, sigma=0.5)
    o = ops.attention_fwd(q, k, v)
    s = ops.attention_fwd(q, k, v, scalar=True)
    ops.check()
    diff = (o.float() - s.float()).abs()
    assert diff.max().item() <= 2e-2 and diff.mean().item() <= 2e-3, (diff.max(), diff.mean())


def test_pairs_noalloc_matches():
    """attention_fwd_noalloc takes the same path (no scratch is needed)."""
    import ctypes

    from benchmark_b200 import _lib
    q, k, v = normal_inputs(1, 160, 160, 256, 1024, 64, seed=49)
    ref = ops.attention_fwd(q, k, v)
    ops.check()
    o = torch.full_like(q, float("nan"))
    st = _lib.lib().attention_fwd_noalloc(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), 1, 160, 160, 256, 1024, 64, 0,
        ctypes.c_float(-1.0), 0, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == _lib.B200_OK, _lib.last_error()
    ops.check()
    assert torch.equal(o, ref)
