"""CPU tests of the C-ABI library: it loads, exports every declared entry
point, and rejects bad arguments with a status code before touching CUDA."""
import ctypes

import pytest

from benchmark_b200 import _lib


def test_library_exports_every_header_symbol():
    L = _lib.lib()
    names = _lib.header_functions()
    assert "attention_fwd" in names and "b200_check" in names
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, missing


def test_version():
    assert _lib.lib().b200_version() >= 100


def _attn(q=16, k=16, v=16, o=16, B=1, Hq=1, Hkv=1, Sq=128, Skv=128, D=128, causal=0,
          scale=-1.0, name="attention_fwd"):
    return getattr(_lib.lib(), name)(q, k, v, o, B, Hq, Hkv, Sq, Skv, D, causal, scale, None)


@pytest.mark.parametrize("name", ["attention_fwd", "attention_fwd_scalar"])
def test_attention_rejects_bad_arguments(name):
    assert _attn(q=0, name=name) == _lib.B200_EINVAL
    assert "null" in _lib.last_error()
    assert _attn(k=24, name=name) == _lib.B200_EINVAL           # misaligned
    assert "aligned" in _lib.last_error()
    assert _attn(B=0, name=name) == _lib.B200_EINVAL
    assert _attn(Sq=0, name=name) == _lib.B200_EINVAL
    assert _attn(Skv=-1, name=name) == _lib.B200_EINVAL
    assert _attn(Hq=6, Hkv=4, name=name) == _lib.B200_EINVAL    # Hq % Hkv != 0
    assert _attn(D=96, name=name) == _lib.B200_EUNSUPPORTED
    assert "head_dim" in _lib.last_error()
    assert _attn(scale=float("inf"), name=name) == _lib.B200_EINVAL


def test_fill_rejects_null():
    L = _lib.lib()
    assert L.b200_fill_normal_bf16(None, 10, 1, 0, 0, 0.0, 1.0, None) == _lib.B200_EINVAL
    assert L.b200_fill_normal_bf16(None, 0, 1, 0, 0, 0.0, 1.0, None) == _lib.B200_OK


def test_gemm_rejects_bad_arguments():
    L = _lib.lib()
    if not hasattr(L, "gemm_bf16"):
        pytest.skip("gemm not built")
    assert L.gemm_bf16(None, 16, 16, 256, 256, 256, 1, None) == _lib.B200_EINVAL
    assert L.gemm_bf16(16, 16, 16, 0, 256, 256, 1, None) == _lib.B200_EINVAL
    assert L.gemm_bf16(16, 16, 16, 256, 256, 100, 1, None) == _lib.B200_EUNSUPPORTED


def test_last_error_is_thread_local():
    import threading
    L = _lib.lib()
    assert _attn(q=0) == _lib.B200_EINVAL
    seen = {}

    def other():
        seen["msg"] = L.b200_last_error()

    t = threading.Thread(target=other)
    t.start()
    t.join()
    assert seen["msg"] in (b"", None)
    assert b"null" in L.b200_last_error()
