"""GPU test of the softmax's FMA-pipe exp2 (exp2_fma_x2) against float64 2**x.

The polynomial is a degree-3 minimax fit of 2^r on [-0.5, 0.5]
(benchmark_b200/csrc/fit_exp2_poly.py: relative error 7.486e-5 with fp32
coefficients and fp32 Horner steps); range reduction and the exponent add are
exact, so the bound holds over the whole clamped range [-125, 126].  Below
-125 the polynomial returns 2^-125 (the clamp keeps its exponent field out of
the subnormal range), above 126 it returns 2^126; MUFU ex2.approx.ftz is
checked beside it.
"""
import numpy as np
import pytest
import torch

from benchmark_b200 import _lib

pytestmark = pytest.mark.gpu

FIT_BOUND = 7.486e-5          # printed by fit_exp2_poly.py
POLY_REL_TOL = FIT_BOUND + 4e-7  # plus a few fp32 ulps of the final rounding
MUFU_REL_TOL = 2.0 ** -21        # ex2.approx: about 2 ulp of fp32


def _run(x: np.ndarray):
    xd = torch.from_numpy(x.astype(np.float32)).cuda()
    yf = torch.empty_like(xd)
    ym = torch.empty_like(xd)
    _lib.call("b200_selftest_exp2", xd.data_ptr(), yf.data_ptr(), ym.data_ptr(), xd.numel(),
              None)
    torch.cuda.synchronize()
    return yf.cpu().numpy().astype(np.float64), ym.cpu().numpy().astype(np.float64)


def test_fma_exp2_relative_error_in_range():
    # dense grid over the softmax's range (x <= 0 after the max shift, up to
    # the lazy-rescale bound 8) and the rest of the clamped range
    x = np.concatenate([
        np.linspace(-125.0, 10.0, 1 << 22, dtype=np.float32),
        np.linspace(-1.0, 1.0, 1 << 20, dtype=np.float32),
        np.linspace(10.0, 126.0, 1 << 16, dtype=np.float32),
        np.arange(-125, 127, dtype=np.float32),           # integer points
        np.arange(-125, 126, dtype=np.float32) + 0.5,     # rounding ties
    ])
    yf, ym = _run(x)
    ref = np.exp2(x.astype(np.float64))
    rel = np.abs(yf - ref) / ref
    worst = int(np.argmax(rel))
    assert rel.max() <= POLY_REL_TOL, (float(rel.max()), float(x[worst]))
    # MUFU on the normal range (ftz flushes results below 2^-126)
    normal = x >= -125.0
    rel_m = np.abs(ym[normal] - ref[normal]) / ref[normal]
    assert rel_m.max() <= MUFU_REL_TOL, float(rel_m.max())


def test_fma_exp2_outside_clamp():
    x = np.array([-127.0, -150.0, -1e30, -np.inf, 127.0, 200.0, np.inf], dtype=np.float32)
    yf, ym = _run(x)
    tiny = np.exp2(-125.0)
    # below the range the polynomial stays at 2^-125 (relative to the row's
    # largest term, >= 2^-8 in the softmax, that is below 2^-117), MUFU flushes to 0
    assert np.all(np.abs(yf[:4] - tiny) <= tiny * POLY_REL_TOL), yf[:4]
    assert np.all(ym[:4] == 0.0), ym[:4]
    assert np.all(np.abs(yf[4:] - np.exp2(126.0)) <= np.exp2(126.0) * POLY_REL_TOL), yf[4:]


def test_fma_exp2_odd_length():
    x = np.linspace(-20.0, 0.0, 1001, dtype=np.float32)
    yf, _ = _run(x)
    ref = np.exp2(x.astype(np.float64))
    assert np.max(np.abs(yf - ref) / ref) <= POLY_REL_TOL
