"""CPU tests of the C ABI: the library loads, exports exactly what
include/h3b.h declares, and rejects bad arguments on the host before any
CUDA call."""
import ctypes
import re
from pathlib import Path

import pytest

from h3_engine_b200 import _lib

HEADER = Path(__file__).resolve().parent.parent / "include" / "h3b.h"


def declared_functions() -> list[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(h3b_[a-z0-9_]+)\s*\(", text)))


def test_library_loads_and_exports_header_symbols():
    lib = _lib.lib()
    names = declared_functions()
    assert names, "no declarations parsed"
    for name in names:
        assert hasattr(lib, name), f"{name} declared in h3b.h but not exported"
    # every binding in the Python layer is declared in the header
    assert set(_lib.SIGNATURES) <= set(names)
    assert set(names) <= set(_lib.SIGNATURES), "header function without a ctypes binding"


def test_status_strings():
    assert _lib.status_string(0) == "ok"
    for s in range(1, 7):
        assert _lib.status_string(s) != "unknown status"
    assert _lib.status_string(99) == "unknown status"


def test_host_validation_rejects_bad_shapes_without_gpu():
    lib = _lib.lib()
    p = ctypes.c_void_p(16 * 1024)   # never dereferenced: validation fails first
    # K not a multiple of 64
    assert lib.h3b_nvfp4_quantize(p, 4, 48, 48, p, 0.0, None, p, p, 1, 128, None) == 1
    # bad layout enum
    assert lib.h3b_nvfp4_quantize(p, 4, 64, 64, p, 0.0, None, p, p, 7, 128, None) == 1
    # swizzled layout needs Mpad % 128 == 0
    assert lib.h3b_nvfp4_quantize(p, 4, 64, 64, p, 0.0, None, p, p, 1, 100, None) == 1
    # neither amax nor a positive gs
    assert lib.h3b_nvfp4_quantize(p, 4, 64, 64, None, 0.0, None, p, p, 1, 128, None) == 1
    # misaligned input
    assert lib.h3b_nvfp4_quantize(ctypes.c_void_p(16 * 1024 + 2), 4, 64, 64, p, 0.0, None, p, p,
                                  1, 128, None) == 2
    # GEMM: K % 256, N % 128, a_rows % 128, unknown activation, bad gsb_seg
    g = lib.h3b_nvfp4_gemm
    assert g(p, p, None, 128, 128, p, p, None, 0, 256, 128, None, None, 0, None, None, 0, p, 256, None, None) == 1
    assert g(p, p, None, 128, 128, p, p, None, 0, 200, 256, None, None, 0, None, None, 0, p, 200, None, None) == 1
    assert g(p, p, None, 100, 100, p, p, None, 0, 256, 256, None, None, 0, None, None, 0, p, 256, None, None) == 1
    assert g(p, p, None, 128, 128, p, p, None, 0, 256, 256, None, None, 0, None, None, 9, p, 256, None, None) == 1
    assert g(p, p, None, 128, 128, p, p, None, 96, 256, 256, None, None, 0, None, None, 0, p, 256, None, None) == 1
    # M == 0 is a no-op that succeeds without touching memory
    assert g(p, p, None, 0, 128, p, p, None, 0, 256, 256, None, None, 0, None, None, 0, p, 256, None, None) == 0
    assert lib.h3b_nvfp4_dequantize(p, p, 1, 100, None, 4, 64, p, None) == 1


def test_attention_rejects_bad_documents():
    """Argument checks of h3b_attention_varlen that run before any CUDA call."""
    import ctypes
    from h3_engine_b200 import _lib
    lib = _lib.lib()
    p = ctypes.c_void_p(16 * 1024)

    def call(cu, kv_rows, ndocs=None):
        arr = (ctypes.c_int32 * len(cu))(*cu)
        n = len(cu) - 1 if ndocs is None else ndocs
        return lib.h3b_attention_varlen(p, kv_rows, 768, 0, 0, p, kv_rows, 768, 256, 512, 2, 128,
                                        arr, n, 0.088, p, 256, None)

    assert call(list(range(66)), 65) == 1                 # 65 documents > 64
    assert call([0, 10, 20], 21) == 1                     # cu[-1] != rows
    assert call([0, 12, 10, 20], 20) == 1                 # decreasing offsets
    assert call([1, 10, 20], 20) == 1                     # cu[0] != 0
