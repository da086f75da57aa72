"""C ABI checks that need no GPU: the library loads, exports every symbol that
include/vkb200.h declares, and reports errors through vkb_status."""
import ctypes as C
import os
import re

import numpy as np
import pytest

from vokra_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = set()
    for fn in os.listdir(os.path.join(ROOT, "include")):
        if fn.endswith(".h"):
            src = open(os.path.join(ROOT, "include", fn)).read()
            src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
            names |= set(re.findall(r"\b(vkb_[a-z0-9_]+)\s*\(", src))
    return sorted(names)


def test_header_declares_entry_points():
    d = declared_symbols()
    assert "vkb_linear" in d and "vkb_kv_attention" in d and len(d) >= 30


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    missing = [n for n in declared_symbols() if not hasattr(lib, n)]
    assert not missing, missing


def test_python_binding_covers_every_declared_symbol():
    missing = [n for n in declared_symbols() if n not in _lib.SIGNATURES]
    assert not missing, missing


def test_abi_version_and_null_handling():
    lib = _lib.load()
    assert lib.vkb_abi_version() == 1
    assert lib.vkb_context_create(0, None) == _lib.ERROR_INVALID_ARGUMENT
    assert b"null" in lib.vkb_last_error()
    assert lib.vkb_linear(None, None, 1, None, 0, None, None, 0, 0, None, C.c_float(1)) == _lib.ERROR_INVALID_ARGUMENT
    assert lib.vkb_kv_append(None, 0, None, None) == _lib.ERROR_INVALID_ARGUMENT
    assert lib.vkb_context_launch_count(None) == 0


def test_dequant_gemv_validation_matches_reference_rules_without_gpu():
    # validate_dequant_gemv (kv_quant/gpu_ops.rs:95) runs before any device work.
    lib = _lib.load()
    x = np.zeros(63, np.float32)
    b = np.zeros(4 * 2 * 34, np.uint8)
    dummy = C.c_void_p(1)
    st = lib.vkb_kv_dequant_gemv_host(dummy, _lib.KV_FP32, None, 0, 0, 0, None, 0, None)
    assert st == _lib.ERROR_INVALID_ARGUMENT and b"Fp32" in lib.vkb_last_error()
    st = lib.vkb_kv_dequant_gemv_host(dummy, _lib.KV_Q8_0, b.ctypes.data_as(C.c_void_p), b.nbytes, 4, 2,
                                      x.ctypes.data_as(C.c_void_p), x.size, None)
    assert st == _lib.ERROR_INVALID_ARGUMENT and b"x.len()" in lib.vkb_last_error()
    x = np.zeros(64, np.float32)
    st = lib.vkb_kv_dequant_gemv_host(dummy, _lib.KV_Q8_0, b.ctypes.data_as(C.c_void_p), 100, 4, 2,
                                      x.ctypes.data_as(C.c_void_p), x.size, None)
    assert st == _lib.ERROR_INVALID_ARGUMENT and b"blocks_bytes" in lib.vkb_last_error()


def test_context_create_without_gpu_is_backend_unavailable():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    lib = _lib.load()
    h = C.c_void_p()
    assert lib.vkb_context_create(0, C.byref(h)) == _lib.ERROR_BACKEND_UNAVAILABLE
