"""attention_fwd_noalloc, for callers that cannot allocate device memory.

Some callers of this library cannot call cudaMalloc: plugin hosts that own
all device memory through their own pool and forbid other allocations, and
latency-bound callers that cannot take cudaMalloc's device-wide
synchronisation.  attention_fwd allocates a workspace the first time it
splits a short problem's K/V range among several CTAs; attention_fwd_noalloc
runs the same kernel with that workspace in a fixed scratch array compiled
into the library, so it allocates nothing.

These tests call it through the C ABI and compare it with attention_fwd on
the same inputs, within the gate the other GPU tests use, on two calls in a
row (the scratch is shared and keeps the previous call's contents).  The file
is named so that pytest collects it last; it also passes when run alone.
"""
import ctypes

import pytest
import torch

from attn_util import MAX_ABS, MEAN_ABS, normal_inputs
from benchmark_b200 import _lib, ops

pytestmark = pytest.mark.gpu


def _noalloc(q, k, v, o, nsplit, causal=False):
    B, Hq, Sq, D = q.shape
    Hkv, Skv = k.shape[1], k.shape[2]
    return _lib.lib().attention_fwd_noalloc(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), B, Hq, Hkv, Sq, Skv, D,
        int(causal), ctypes.c_float(-1.0), nsplit, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))


def _close(a, b, what):
    d = (a.float() - b.float()).abs()
    assert torch.isfinite(a.float()).all(), what
    assert d.max().item() <= MAX_ABS and d.mean().item() <= MEAN_ABS, (what, d.max(), d.mean())


@pytest.mark.parametrize("shape,causal,nsplit", [
    ((1, 1, 1, 128, 8192, 128), False, 0),   # the library's own split (4 units)
    ((1, 2, 1, 300, 6500, 64), False, 3),    # ragged, GQA, d=64, 3 units per Q tile
    ((1, 4, 2, 256, 7000, 128), True, 5),    # causal, units of different lengths
    ((1, 2, 2, 1024, 1024, 128), False, 1),  # no split: no scratch used
])
def test_noalloc_matches_attention_fwd_twice(shape, causal, nsplit):
    B, Hq, Hkv, Sq, Skv, D = shape
    q, k, v = normal_inputs(B, Hq, Hkv, Sq, Skv, D, seed=31)
    ref = ops.attention_fwd(q, k, v, causal=causal)
    ops.check()
    for call in range(2):
        o = torch.full_like(q, float("nan"))
        assert _noalloc(q, k, v, o, nsplit, causal) == _lib.B200_OK, _lib.last_error()
        ops.check()
        _close(o, ref, f"{shape} causal={causal} nsplit={nsplit} call {call}")


def test_noalloc_rejects_more_units_than_its_scratch():
    # 64 Q tiles x 8 splits = 512 units > the 128 the scratch holds.
    q, k, v = normal_inputs(1, 1, 1, 8192, 8192, 128, seed=32)
    o = torch.empty_like(q)
    assert _noalloc(q, k, v, o, 8) == _lib.B200_EUNSUPPORTED
    assert "exceed its fixed scratch" in _lib.last_error()
    assert _noalloc(q, k, v, o, 9) == _lib.B200_EINVAL
    # the same problem without a split needs no scratch
    assert _noalloc(q, k, v, o, 1) == _lib.B200_OK
    ops.check()
    _close(o, ops.attention_fwd(q, k, v), "8192 no split")
