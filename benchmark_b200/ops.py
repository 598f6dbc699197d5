"""torch-tensor conveniences over the C ABI.

Tensors are bf16, contiguous, on the current CUDA device; the calls run on the
current torch stream.  torch is only the device-memory and stream plumbing:
all arithmetic happens in libb200attn.so's CUDA kernels.
"""
from __future__ import annotations

import torch

from . import _lib


def _stream_ptr(stream: torch.cuda.Stream | None) -> int:
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def _check_bf16(*ts: torch.Tensor) -> None:
    for t in ts:
        if t.dtype != torch.bfloat16 or not t.is_cuda or not t.is_contiguous():
            raise ValueError("expected contiguous bf16 CUDA tensors")


def attention_fwd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                  out: torch.Tensor | None = None, causal: bool = False,
                  softmax_scale: float = -1.0, stream: torch.cuda.Stream | None = None,
                  scalar: bool = False) -> torch.Tensor:
    """q [B,Hq,Sq,D], k/v [B,Hkv,Skv,D] -> o [B,Hq,Sq,D] (bf16).

    scalar=True runs the validation-only CUDA-core kernel instead of the fused one."""
    _check_bf16(q, k, v)
    B, Hq, Sq, D = q.shape
    Bk, Hkv, Skv, Dk = k.shape
    if Bk != B or Dk != D or tuple(v.shape) != tuple(k.shape):
        raise ValueError("q/k/v shapes disagree")
    if out is None:
        out = torch.empty_like(q)
    _check_bf16(out)
    name = "attention_fwd_scalar" if scalar else "attention_fwd"
    _lib.call(name, q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), B, Hq, Hkv, Sq,
              Skv, D, int(bool(causal)), float(softmax_scale), _stream_ptr(stream))
    return out


def fill_normal_(t: torch.Tensor, seed: int, tensor_id: int, mean: float = 0.0,
                 sigma: float = 1.0, index_base: int = 0,
                 stream: torch.cuda.Stream | None = None) -> torch.Tensor:
    _check_bf16(t)
    _lib.call("b200_fill_normal_bf16", t.data_ptr(), t.numel(), seed, tensor_id, index_base,
              mean, sigma, _stream_ptr(stream))
    return t


def fill_uniform_(t: torch.Tensor, seed: int, tensor_id: int, lo: float = -1.0, hi: float = 1.0,
                  index_base: int = 0, stream: torch.cuda.Stream | None = None) -> torch.Tensor:
    _check_bf16(t)
    _lib.call("b200_fill_uniform_bf16", t.data_ptr(), t.numel(), seed, tensor_id, index_base,
              lo, hi, _stream_ptr(stream))
    return t


def check(stream: torch.cuda.Stream | None = None) -> None:
    """Synchronise and raise B200Error(B200_ETIMEOUT) if a device wait gave up."""
    _lib.call("b200_check", _stream_ptr(stream))


def gemm_bf16(a: torch.Tensor, b: torch.Tensor, out: torch.Tensor | None = None,
              b_col_major: bool = True, impl: str = "tcgen05",
              stream: torch.cuda.Stream | None = None) -> torch.Tensor:
    """C [M,N] (bf16) = A [M,K] @ B, B given as [N,K] (b_col_major) or [K,N].

    impl: "tcgen05" (this library's kernel) or "cublas" (comparator)."""
    _check_bf16(a, b)
    M, K = a.shape
    N = b.shape[0] if b_col_major else b.shape[1]
    if out is None:
        out = torch.empty((M, N), dtype=torch.bfloat16, device=a.device)
    name = {"tcgen05": "gemm_bf16", "cublas": "gemm_bf16_cublas"}[impl]
    _lib.call(name, a.data_ptr(), b.data_ptr(), out.data_ptr(), M, N, K, int(b_col_major),
              _stream_ptr(stream))
    return out


def gemm_f32_reference(a: torch.Tensor, b: torch.Tensor, b_col_major: bool = True,
                       stream: torch.cuda.Stream | None = None) -> torch.Tensor:
    _check_bf16(a, b)
    M, K = a.shape
    N = b.shape[0] if b_col_major else b.shape[1]
    out = torch.empty((M, N), dtype=torch.float32, device=a.device)
    _lib.call("gemm_f32_reference", a.data_ptr(), b.data_ptr(), out.data_ptr(), M, N, K,
              int(b_col_major), _stream_ptr(stream))
    return out
