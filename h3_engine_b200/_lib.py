"""ctypes binding of libh3b.so (the C ABI in include/h3b.h).

The library is built in-tree (``python -m h3_engine_b200.csrc.build``).  There
is no fallback: if the shared object is missing or cannot be loaded every op
raises, so a GPU run can never silently take another path.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().with_name("libh3b.so")

_c_void_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_i32 = ctypes.c_int
_f32 = ctypes.c_float

# name -> (restype, argtypes); must match include/h3b.h
SIGNATURES: dict[str, tuple] = {
    "h3b_version": (_i32, []),
    "h3b_status_string": (ctypes.c_char_p, [_i32]),
    "h3b_launch_count": (ctypes.c_longlong, []),
    "h3b_device_error": (_i32, [ctypes.POINTER(_i32), _i32]),
    "h3b_amax_bf16": (_i32, [_c_void_p, _i64, _i64, _i64, _c_void_p, _c_void_p]),
    "h3b_nvfp4_quantize": (_i32, [_c_void_p, _i64, _i64, _i64, _c_void_p, _f32, _c_void_p,
                                  _c_void_p, _c_void_p, _i32, _i64, _c_void_p]),
    "h3b_nvfp4_dequantize": (_i32, [_c_void_p, _c_void_p, _i32, _i64, _c_void_p, _i64, _i64,
                                    _c_void_p, _c_void_p]),
    "h3b_nvfp4_gemm": (_i32, [_c_void_p, _c_void_p, _c_void_p, _i64, _i64,
                              _c_void_p, _c_void_p, _c_void_p, _i64, _i64, _i64,
                              _c_void_p, _c_void_p, _i64, _c_void_p, _c_void_p, _i32, _c_void_p,
                              _i64, _c_void_p, _c_void_p]),
    "h3b_rmsnorm_stats": (_i32, [_c_void_p, _i64, _i64, _i64, _c_void_p, _f32, _c_void_p,
                                 _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p]),
    "h3b_rmsnorm_quantize": (_i32, [_c_void_p, _i64, _i64, _i64, _c_void_p, _c_void_p, _c_void_p,
                                    _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p,
                                    _c_void_p, _i64, _c_void_p, _c_void_p]),
    "h3b_qk_norm_rope": (_i32, [_c_void_p, _i64, _i64, _c_void_p, _i64, _i64, _i64, _i32, _i32,
                                _c_void_p, _c_void_p, _f32, _c_void_p, _c_void_p, _i32, _i64,
                                _c_void_p]),
    "h3b_attention_varlen": (_i32, [_c_void_p, _i64, _i64, _i64, _i64, _c_void_p, _i64, _i64,
                                    _i64, _i64, _i32, _i32, ctypes.POINTER(ctypes.c_int32), _i32,
                                    _f32, _c_void_p, _i64, _c_void_p]),
    "h3b_attention_qkv": (_i32, [_c_void_p, _i64, _c_void_p, _i64, _c_void_p, _i64, _i64, _i32,
                                 _i32, ctypes.POINTER(ctypes.c_int32), _i32, _f32, _c_void_p, _i64,
                                 _c_void_p]),
    "h3b_qk_norm_rope_out": (_i32, [_c_void_p, _i64, _c_void_p, _i64, _c_void_p, _i64, _c_void_p,
                                    _i64, _i64, _i32, _i32, _c_void_p, _c_void_p, _f32, _c_void_p,
                                    _c_void_p, _i32, _i64, _c_void_p]),
    "h3b_gate_residual": (_i32, [_c_void_p, _i64, _c_void_p, _i64, _c_void_p, _c_void_p, _i64,
                                 _i64, _i64, _c_void_p, _i64, _c_void_p]),
    "h3b_ada_modulate": (_i32, [_c_void_p, _i64, _c_void_p, _c_void_p, _c_void_p, _i64, _i64,
                                _i64, _c_void_p, _i64, _c_void_p]),
    "h3b_rmsnorm_quantize_noalloc": (_i32, [_c_void_p, _i64, _i64, _i64, _c_void_p, _f32,
                                            _c_void_p, _c_void_p, _c_void_p, _c_void_p,
                                            _c_void_p, _c_void_p, _i64, _c_void_p]),
    "h3b_selftest_bounded_wait": (_i32, [_i64, _c_void_p]),
    "h3b_peer_buffer_create": (_i32, [_i64, ctypes.POINTER(_c_void_p), _c_void_p]),
    "h3b_peer_buffer_open": (_i32, [_c_void_p, ctypes.POINTER(_c_void_p)]),
    "h3b_peer_buffer_close": (_i32, [_c_void_p]),
    "h3b_peer_buffer_destroy": (_i32, [_c_void_p]),
    "h3b_amax_exchange": (_i32, [_c_void_p, _c_void_p, _i32, _i32, _i64, _i64, _c_void_p]),
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


class H3BError(RuntimeError):
    """A libh3b call returned a non-zero h3b_status."""

    def __init__(self, what: str, status: int, message: str):
        super().__init__(f"{what} failed: status {status} ({message})")
        self.status = status


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(
                    f"{LIB_PATH} is missing: build it with `python -m h3_engine_b200.csrc.build` "
                    "(the NVFP4 path has no CPU fallback)")
            handle = ctypes.CDLL(str(LIB_PATH))
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(handle, name)
                fn.restype = res
                fn.argtypes = args
            _lib = handle
    return _lib


def status_string(status: int) -> str:
    return lib().h3b_status_string(status).decode()


def check(status: int, what: str) -> None:
    if status != 0:
        raise H3BError(what, status, status_string(status))


def launch_count() -> int:
    return int(lib().h3b_launch_count())


def device_error(clear: bool = True) -> int:
    """Synchronize the current device and return (and by default clear) its error word."""
    code = _i32(0)
    check(lib().h3b_device_error(ctypes.byref(code), 1 if clear else 0), "h3b_device_error")
    return int(code.value)
