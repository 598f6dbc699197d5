"""ctypes binding of libb200attn.so (include/b200attn.h).

The library is built in-tree by `python -m benchmark_b200.build`; there is no
fallback implementation: if the shared object is missing, every call raises.
"""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "libb200attn.so"
HEADER = PKG.parent / "include" / "b200attn.h"

STATUS_NAMES = {0: "B200_OK", 1: "B200_EINVAL", 2: "B200_EUNSUPPORTED", 3: "B200_ECUDA",
                4: "B200_ETIMEOUT"}
B200_OK, B200_EINVAL, B200_EUNSUPPORTED, B200_ECUDA, B200_ETIMEOUT = range(5)


class B200Error(RuntimeError):
    def __init__(self, status: int, message: str):
        self.status = status
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {message}")


_lib: ctypes.CDLL | None = None

_vp = ctypes.c_void_p
_i = ctypes.c_int
_f = ctypes.c_float
_u64 = ctypes.c_uint64
_u32 = ctypes.c_uint32

_PROTOTYPES = {
    "attention_fwd": [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _f, _vp],
    "attention_fwd_trace": [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _f, _vp, _i, _i,
                            _vp],
    "attention_fwd_scalar": [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _f, _vp],
    "attention_fwd_noalloc": [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _f, _i, _vp],
    "b200_fill_normal_bf16": [_vp, _u64, _u64, _u32, _u64, _f, _f, _vp],
    "b200_fill_uniform_bf16": [_vp, _u64, _u64, _u32, _u64, _f, _f, _vp],
    "b200_check": [_vp],
    "b200_selftest_wait_timeout": [_u64, _vp],
    "b200_selftest_exp2": [_vp, _vp, _vp, _u64, _vp],
    "gemm_bf16": [_vp, _vp, _vp, _i, _i, _i, _i, _vp],
    "gemm_bf16_cublas": [_vp, _vp, _vp, _i, _i, _i, _i, _vp],
    "gemm_f32_reference": [_vp, _vp, _vp, _i, _i, _i, _i, _vp],
    "gemm_cublas_mode": [_vp, _vp, _vp, _i, _i, _i, _i, _vp],
    "b200_fill_cublas_pattern": [_vp, _u64, _i, _f, _vp],
}


def header_functions() -> list[str]:
    """Names of every function declared in include/b200attn.h."""
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return re.findall(r"^\s*(?:const\s+)?[A-Za-z_][\w\s\*]*?\b([a-z_][a-z0-9_]*)\s*\(", text,
                      flags=re.M)


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(f"{LIB_PATH.name} is not built; run `python -m benchmark_b200.build` "
                              "(there is no non-CUDA fallback)")
        L = ctypes.CDLL(str(LIB_PATH))
        for name, argtypes in _PROTOTYPES.items():
            fn = getattr(L, name, None)
            if fn is None:
                continue
            fn.argtypes = argtypes
            fn.restype = ctypes.c_int
        L.b200_last_error.argtypes = []
        L.b200_last_error.restype = ctypes.c_char_p
        L.b200_version.argtypes = []
        L.b200_version.restype = ctypes.c_int
        _lib = L
    return _lib


def last_error() -> str:
    return lib().b200_last_error().decode(errors="replace")


def check(status: int) -> None:
    if status != B200_OK:
        raise B200Error(status, last_error())


def call(name: str, *args) -> None:
    check(getattr(lib(), name)(*args))
