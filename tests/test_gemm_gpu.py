"""GPU parity tests of the tcgen05 GEMM (through the C ABI).

Small shapes against the CPU oracle (the reference's double-precision loop,
5.GEMM/gemm256_tma_tcgen05_bench.cu:1115-1137, restated in oracle/gemm_ref.cpp)
with the reference's tolerance (fail only where abs > 2e-2 AND rel > 2e-2,
:1113-1127) and BASELINE's relative Frobenius error <= 1e-2; full size against
cuBLAS and the fp32 CUDA-core reference GEMM.
"""
import numpy as np
import pytest
import torch

import oracle
from benchmark_b200 import ops

pytestmark = pytest.mark.gpu

FROB = 1e-2


def to_dev(a):
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16).cuda()


def bits(t):
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def rel_frob(got, ref):
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    return float(np.linalg.norm(got - ref) / max(np.linalg.norm(ref), 1e-30))


def harness_ok(got, ref, abs_tol=2e-2, rel_tol=2e-2):
    d = np.abs(np.asarray(got, np.float64) - ref)
    r = d / np.maximum(np.abs(ref), 1e-12)
    return int(((d > abs_tol) & (r > rel_tol)).sum())


@pytest.mark.parametrize("size", [256, 512])
@pytest.mark.parametrize("pattern", ["pattern", "ones"])
@pytest.mark.parametrize("b_col_major", [False, True])
def test_reference_validation_cases(size, pattern, b_col_major):
    """The reference's --validate cases (5.GEMM/README.md:52-57)."""
    a = oracle.gemm_fill("a", pattern, size, size)
    b = oracle.gemm_fill("b", pattern, size, size)  # [K, N]
    bm = np.ascontiguousarray(b.T) if b_col_major else b
    ref = oracle.gemm(a, bm, b_col_major)
    c = ops.gemm_bf16(to_dev(a), to_dev(bm), b_col_major=b_col_major)
    ops.check()
    got = c.float().cpu().numpy()
    assert harness_ok(got, ref) == 0
    assert rel_frob(got, ref) <= FROB


@pytest.mark.parametrize("M,N,K", [(300, 264, 200), (1, 8, 8), (129, 520, 72), (128, 256, 64),
                                   (1000, 1000, 4096), (77, 8, 1032)])
@pytest.mark.parametrize("b_col_major", [False, True])
def test_ragged_uniform_vs_oracle(M, N, K, b_col_major):
    g = torch.Generator().manual_seed(M * 31 + N * 7 + K)
    a = (torch.rand(M, K, generator=g) * 2 - 1).to(torch.bfloat16)
    b = (torch.rand(K, N, generator=g) * 2 - 1).to(torch.bfloat16)
    bm = b.t().contiguous() if b_col_major else b
    c = ops.gemm_bf16(a.cuda(), bm.cuda(), b_col_major=b_col_major)
    ops.check()
    ref = oracle.gemm(bits(a), bits(bm), b_col_major)
    got = c.float().cpu().numpy()
    assert np.isfinite(got).all()
    assert rel_frob(got, ref) <= FROB, rel_frob(got, ref)
    # bf16 output rounding bounds the element error: |C| * 2^-8 + accumulation noise
    assert np.all(np.abs(got - ref) <= 8e-3 * np.abs(ref) + 2e-2 * np.sqrt(K / 64.0))


def test_output_guard_untouched():
    M, N, K = 200, 264, 128
    a = torch.randn(M, K).to(torch.bfloat16).cuda()
    b = torch.randn(N, K).to(torch.bfloat16).cuda()
    buf = torch.full((M * N + 4096,), 3.0, dtype=torch.bfloat16, device="cuda")
    c = buf[: M * N].view(M, N)
    ops.gemm_bf16(a, b, out=c, b_col_major=True)
    ops.check()
    assert (buf[M * N:] == 3.0).all()


@pytest.mark.parametrize("b_col_major", [True, False])
def test_full_size_8192_vs_cublas_and_fp32(b_col_major):
    """BASELINE's GEMM config: 8192^3, A and B ~ U(-1,1) from a seed."""
    n = 8192
    a = torch.empty((n, n), dtype=torch.bfloat16, device="cuda")
    b = torch.empty_like(a)
    ops.fill_uniform_(a, 5, 10, -1.0, 1.0)
    ops.fill_uniform_(b, 5, 11, -1.0, 1.0)
    c1 = ops.gemm_bf16(a, b, b_col_major=b_col_major)
    c2 = ops.gemm_bf16(a, b, b_col_major=b_col_major)
    cb = ops.gemm_bf16(a, b, b_col_major=b_col_major, impl="cublas")
    ref = ops.gemm_f32_reference(a, b, b_col_major=b_col_major)
    ops.check()
    assert torch.equal(c1, c2), "not deterministic"
    d = (c1.float() - ref)
    assert (d.norm() / ref.norm()).item() <= FROB
    assert ((c1.float() - cb.float()).norm() / cb.float().norm()).item() <= FROB
    # oracle rows (double precision) on a sample
    ah, bh = bits(a), bits(b)
    rows = oracle.gemm(ah, bh, b_col_major, row_begin=4093, row_end=4097)
    assert rel_frob(c1[4093:4097].float().cpu().numpy(), rows) <= FROB


def test_cublas_comparator_matches_oracle():
    M, N, K = 192, 256, 320
    a = torch.randn(M, K).to(torch.bfloat16)
    b = torch.randn(N, K).to(torch.bfloat16)
    c = ops.gemm_bf16(a.cuda(), b.cuda(), b_col_major=True, impl="cublas")
    ops.check()
    ref = oracle.gemm(bits(a), bits(b), True)
    assert rel_frob(c.float().cpu().numpy(), ref) <= FROB


@pytest.mark.parametrize("mode,dtype,tol", [(0, torch.float16, 2e-3), (1, torch.bfloat16, 1e-2),
                                            (2, torch.float32, 2e-3), (3, torch.float32, 1e-6)])
def test_cublas_modes_match_oracle(mode, dtype, tol):
    """gemm_cublas_mode: column-major C = A B in 6.cuBLAS's four modes, against
    the oracle's double-precision loop on the same (rounded) inputs."""
    from benchmark_b200 import _lib
    M, N, K = 192, 160, 256
    g = torch.Generator().manual_seed(5 + mode)
    a_rm = (torch.rand(M, K, generator=g) * 2 - 1).to(dtype)  # row-major [M,K]
    b_rm = (torch.rand(K, N, generator=g) * 2 - 1).to(dtype)  # row-major [K,N]
    # column-major storage = transposed row-major buffers
    a_cm = a_rm.t().contiguous().cuda()
    b_cm = b_rm.t().contiguous().cuda()
    c_cm = torch.empty((N, M), dtype=dtype, device="cuda")
    _lib.call("gemm_cublas_mode", a_cm.data_ptr(), b_cm.data_ptr(), c_cm.data_ptr(), M, N, K,
              mode, torch.cuda.current_stream().cuda_stream)
    ops.check()
    got = c_cm.t().float().cpu().numpy()
    ref = a_rm.double().numpy() @ b_rm.double().numpy()
    assert rel_frob(got, ref) <= tol, rel_frob(got, ref)


def test_cublas_pattern_fill():
    from benchmark_b200 import _lib
    t = torch.empty(1000, dtype=torch.float32, device="cuda")
    _lib.call("b200_fill_cublas_pattern", t.data_ptr(), t.numel(), 3, 1e-3,
              torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    i = np.arange(1000)
    want = ((i % 251) - 125).astype(np.float32) * np.float32(1e-3)
    assert np.array_equal(t.cpu().numpy(), want)
