"""CPU oracle -- TEST INFRASTRUCTURE ONLY.

ctypes bindings for the C++ restatement of the reference's CPU arithmetic
(oracle/attention_ref.cpp, oracle/gemm_ref.cpp) and, where it was built, the
reference's own CPU attention compiled in place (oracle/_ref, see
oracle/ref_shim.cu).  Only tests/, __graft_entry__.smoke() and the CPU-baseline
leg of bench.py may import this package; the product library never does.

Parity of the restatement is pinned against the reference: tests/golden holds
FNV-1a fingerprints of the reference's own outputs (made by
tests/golden/make_golden.py from oracle/_ref), and tests/test_oracle.py
requires bit-identical results.
"""
from __future__ import annotations

import ctypes
import os
import shutil
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "_build" / "liboracle.so"
REF_PATH = HERE / "_ref" / "libref_attention.so"
REF_GEMM_PATH = HERE / "_ref" / "libref_gemm.so"

_u16p = ctypes.POINTER(ctypes.c_uint16)
_f32p = ctypes.POINTER(ctypes.c_float)
_f64p = ctypes.POINTER(ctypes.c_double)
_lib = None
_ref = None
_ref_gemm = None


def build(reference_root: str | None = None) -> None:
    """Compile the restatement (and, given the reference root, oracle/_ref)."""
    make = shutil.which("make")
    if make is None:
        raise RuntimeError("make not found")
    targets = ["all"] + (["ref", f"REF={reference_root}"] if reference_root else [])
    subprocess.run([make, "-s", "-C", str(HERE), *targets], check=True)


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        L = ctypes.CDLL(str(LIB_PATH))
        i = ctypes.c_int
        L.oracle_attention_f32.argtypes = [_u16p, _u16p, _u16p, i, i, i, i, i, i,
                                           ctypes.c_float, i, _f32p, i]
        L.oracle_attention_f32.restype = None
        L.oracle_attention_rows_f32.argtypes = [_u16p, _u16p, _u16p, i, i, i, i, i, i,
                                                ctypes.c_float, i, i, i, i, i, i, _f32p, i]
        L.oracle_attention_rows_f32.restype = None
        L.oracle_fill_pattern_bf16.argtypes = [_u16p, ctypes.c_char_p, ctypes.c_char, i, i, i, i]
        L.oracle_fill_pattern_bf16.restype = None
        L.oracle_f32_to_bf16.argtypes = [ctypes.c_float]
        L.oracle_f32_to_bf16.restype = ctypes.c_uint16
        L.oracle_gemm_f64.argtypes = [_u16p, _u16p, i, i, i, i, i, i, _f64p, i]
        L.oracle_gemm_f64.restype = None
        L.oracle_gemm_fill_bf16.argtypes = [_u16p, ctypes.c_char, ctypes.c_char_p, i, i]
        L.oracle_gemm_fill_bf16.restype = None
        L.oracle_fnv1a64.argtypes = [ctypes.c_void_p, ctypes.c_size_t]
        L.oracle_fnv1a64.restype = ctypes.c_uint64
        _lib = L
    return _lib


def ref_available() -> bool:
    return REF_PATH.exists()


def _load_ref_lib(path: Path) -> ctypes.CDLL:
    """Load an oracle/_ref library.  Those link libcuda.so.1 for the reference's
    unused GPU paths; on a machine without a driver the CUDA toolkit's link
    stub satisfies that dependency (no CUDA call is ever made)."""
    try:
        return ctypes.CDLL(str(path))
    except OSError as e:
        if "libcuda" not in str(e):
            raise
        cuda_home = os.environ.get("CUDA_HOME") or str(
            Path(shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc").resolve().parent.parent)
        ctypes.CDLL(str(Path(cuda_home) / "lib64" / "stubs" / "libcuda.so"),
                    mode=ctypes.RTLD_GLOBAL)
        return ctypes.CDLL(str(path))


def ref_gemm() -> ctypes.CDLL:
    """The reference's own GEMM validation fills (oracle/_ref/libref_gemm.so)."""
    global _ref_gemm
    if _ref_gemm is None:
        R = _load_ref_lib(REF_GEMM_PATH)
        R.ref_gemm_fill_bf16.argtypes = [_u16p, ctypes.c_char, ctypes.c_char_p, ctypes.c_int,
                                         ctypes.c_int]
        R.ref_gemm_fill_bf16.restype = None
        _ref_gemm = R
    return _ref_gemm


def ref() -> ctypes.CDLL:
    """The reference's own CPU attention (oracle/_ref/libref_attention.so)."""
    global _ref
    if _ref is None:
        R = _load_ref_lib(REF_PATH)
        i = ctypes.c_int
        R.ref_attention_f32.argtypes = [_u16p, _u16p, _u16p, i, i, i, i, i, i, ctypes.c_float,
                                        i, _f32p]
        R.ref_attention_f32.restype = None
        R.ref_fill_pattern_bf16.argtypes = [_u16p, ctypes.c_char_p, ctypes.c_char, i, i, i, i]
        R.ref_fill_pattern_bf16.restype = None
        R.ref_fnv1a64.argtypes = [ctypes.c_void_p, ctypes.c_size_t]
        R.ref_fnv1a64.restype = ctypes.c_uint64
        _ref = R
    return _ref


def _p16(a: np.ndarray):
    assert a.dtype == np.uint16 and a.flags.c_contiguous
    return a.ctypes.data_as(_u16p)


def fill_pattern(pattern: str, matrix: str, B: int, H: int, S: int, D: int,
                 use_reference: bool = False) -> np.ndarray:
    """bf16 bits [B,H,S,D] of the harness pattern (0.attention/main.cu:1266-1325)."""
    out = np.empty((B, H, S, D), dtype=np.uint16)
    fn = ref().ref_fill_pattern_bf16 if use_reference else lib().oracle_fill_pattern_bf16
    fn(_p16(out), pattern.encode(), matrix.encode(), B, H, S, D)
    return out


def attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, causal: bool = False,
              softmax_scale: float = -1.0, threads: int = 0,
              use_reference: bool = False) -> np.ndarray:
    """fp32 attention of bf16-bit inputs q [B,Hq,Sq,D], k/v [B,Hkv,Skv,D]."""
    B, Hq, Sq, D = q.shape
    _, Hkv, Skv, _ = k.shape
    scale = softmax_scale if softmax_scale >= 0 else np.float32(1.0) / np.sqrt(np.float32(D))
    scale = float(np.float32(scale))
    out = np.zeros((B, Hq, Sq, D), dtype=np.float32)
    q, k, v = (np.ascontiguousarray(x) for x in (q, k, v))
    if use_reference:
        ref().ref_attention_f32(_p16(q), _p16(k), _p16(v), B, Hq, Hkv, Sq, Skv, D, scale,
                                int(causal), out.ctypes.data_as(_f32p))
    else:
        lib().oracle_attention_f32(_p16(q), _p16(k), _p16(v), B, Hq, Hkv, Sq, Skv, D, scale,
                                   int(causal), out.ctypes.data_as(_f32p), threads)
    return out


def attention_rows(q: np.ndarray, k: np.ndarray, v: np.ndarray, b: int, h_begin: int,
                   h_end: int, q_begin: int, q_end: int, causal: bool = False,
                   softmax_scale: float = -1.0, threads: int = 0) -> np.ndarray:
    """Rows [q_begin, q_end) of heads [h_begin, h_end) of batch b (fp32)."""
    B, Hq, Sq, D = q.shape
    _, Hkv, Skv, _ = k.shape
    scale = softmax_scale if softmax_scale >= 0 else np.float32(1.0) / np.sqrt(np.float32(D))
    out = np.zeros((h_end - h_begin, q_end - q_begin, D), dtype=np.float32)
    q, k, v = (np.ascontiguousarray(x) for x in (q, k, v))
    lib().oracle_attention_rows_f32(_p16(q), _p16(k), _p16(v), B, Hq, Hkv, Sq, Skv, D,
                                    float(np.float32(scale)), int(causal), b, h_begin, h_end,
                                    q_begin, q_end, out.ctypes.data_as(_f32p), threads)
    return out


def gemm(A: np.ndarray, Bm: np.ndarray, b_col_major: bool, row_begin: int = 0,
         row_end: int | None = None, threads: int = 0) -> np.ndarray:
    """Double-precision reference rows of C = A @ B (bf16-bit inputs)."""
    M, K = A.shape
    N = Bm.shape[0] if b_col_major else Bm.shape[1]
    row_end = M if row_end is None else row_end
    out = np.zeros((row_end - row_begin, N), dtype=np.float64)
    lib().oracle_gemm_f64(_p16(np.ascontiguousarray(A)), _p16(np.ascontiguousarray(Bm)), M, N,
                          K, int(b_col_major), row_begin, row_end,
                          out.ctypes.data_as(_f64p), threads)
    return out


def gemm_fill(which: str, pattern: str, rows: int, cols: int,
              use_reference: bool = False) -> np.ndarray:
    """bf16 bits of the GEMM validation fill ('a' is [M,K], 'b' is [K,N])."""
    out = np.empty((rows, cols), dtype=np.uint16)
    fn = ref_gemm().ref_gemm_fill_bf16 if use_reference else lib().oracle_gemm_fill_bf16
    fn(_p16(out), which.encode(), pattern.encode(), rows, cols)
    return out


def fnv1a64(a: np.ndarray) -> int:
    a = np.ascontiguousarray(a)
    return int(lib().oracle_fnv1a64(a.ctypes.data, a.nbytes))


def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16 bits (vectorised, same rule as
    0.attention/main.cu:1159-1165)."""
    b = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    b = b + 0x7FFF + ((b >> 16) & 1)
    return ((b >> 16) & 0xFFFF).astype(np.uint16)


def bf16_to_f32(h: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(h, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def compare(got: np.ndarray, expected: np.ndarray, abs_tol: float, rel_tol: float) -> dict:
    """The harness's compare_float (0.attention/main.cu:1552-1569): an element
    fails only when BOTH its absolute and relative error exceed the tolerance."""
    got = np.asarray(got, dtype=np.float32)
    expected = np.asarray(expected, dtype=np.float32)
    diff = np.abs(got - expected)
    rel = diff / np.maximum(np.abs(expected), np.float32(1e-6))
    bad = (diff > abs_tol) & (rel > rel_tol)
    return {"ok": not bool(bad.any()), "max_abs": float(diff.max(initial=0.0)),
            "mean_abs": float(diff.mean()) if diff.size else 0.0,
            "max_rel": float(rel.max(initial=0.0)), "bad_count": int(bad.sum())}
