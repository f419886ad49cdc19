"""The C-ABI library loads, exports every function include/*.h declares, and rejects bad
arguments before touching a device.  CPU only: no kernel is launched here."""
import ctypes as C
import glob
import os
import re

import pytest

from lightship_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        src = open(h).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        for m in re.finditer(r"^\s*[A-Za-z_][\w\s\*]*?\b(lsc_\w+)\s*\(", src, flags=re.M):
            names.add(m.group(1))
    return sorted(names)


def test_header_declares_functions():
    names = declared_functions()
    assert "lsc_gemm_i8" in names and "lsc_compile_operator" in names
    assert len(names) >= 20


@pytest.mark.parametrize("name", declared_functions())
def test_library_exports_declared_symbol(name):
    lib = _lib.lib()
    assert hasattr(lib, name), f"{name} is declared in include/ but not exported"


def test_bindings_cover_header():
    assert set(declared_functions()) <= set(_lib.SIGNATURES), \
        set(declared_functions()) - set(_lib.SIGNATURES)


def test_version_and_status_strings():
    lib = _lib.lib()
    assert b"sm_100a" in lib.lsc_version()
    assert lib.lsc_status_string(0) == b"success"
    assert lib.lsc_status_string(15) == b"device wait timed out"
    assert lib.lsc_status_string(999) == b"unknown status"


def test_argument_validation_without_device():
    lib = _lib.lib()
    one = C.c_float(1.0)
    # K not a multiple of 16 is rejected before any device call
    st = lib.lsc_gemm_i8(C.c_void_p(16), C.c_void_p(16), 4, 4, 3, None, C.byref(one), 1.0, 0, 0,
                         C.c_void_p(16), None, None, None)
    assert st == _lib.ERROR_INVALID_ARGUMENT
    assert "multiple of 16" in _lib.last_error()
    # no output requested
    st = lib.lsc_gemm_i8(C.c_void_p(16), C.c_void_p(16), 4, 4, 16, None, C.byref(one), 1.0, 0, 0,
                         None, None, None, None)
    assert st == _lib.ERROR_INVALID_ARGUMENT
    # bad activation / rounding
    st = lib.lsc_gemm_i8(C.c_void_p(16), C.c_void_p(16), 4, 4, 16, None, C.byref(one), 1.0, 9, 0,
                         C.c_void_p(16), None, None, None)
    assert st == _lib.ERROR_INVALID_ARGUMENT
    st = lib.lsc_gemm_i8(C.c_void_p(16), C.c_void_p(16), 4, 4, 16, None, C.byref(one), 1.0, 0, 7,
                         C.c_void_p(16), None, None, None)
    assert st == _lib.ERROR_INVALID_ARGUMENT
    # misaligned operands
    st = lib.lsc_gemm_i8(C.c_void_p(17), C.c_void_p(16), 4, 4, 16, None, C.byref(one), 1.0, 0, 0,
                         C.c_void_p(16), None, None, None)
    assert st == _lib.ERROR_INVALID_ARGUMENT
    # empty problem is a no-op success
    assert lib.lsc_gemm_i8(None, None, 0, 4, 16, None, None, 1.0, 0, 0, C.c_void_p(16), None, None,
                           None) == _lib.SUCCESS
    # quantize: a non-quantized dtype is rejected
    st = lib.lsc_quantize_f32(C.c_void_p(16), C.c_void_p(16), 4, 0, 1.0, 0, 0, None)
    assert st == _lib.ERROR_UNSUPPORTED_DATATYPE
    # find_scale_zp needs a workspace
    st = lib.lsc_find_scale_zp_f32(C.c_void_p(16), 4, 9, 1, None, 0, C.c_void_p(16), C.c_void_p(16), None)
    assert st == _lib.ERROR_INVALID_ARGUMENT
    assert lib.lsc_find_scale_zp_workspace_size() >= 12


def test_backend_create_reports_missing_device():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a CUDA device is present")
    h = C.c_void_p()
    cfg = _lib.lsc_config(0, 0, 0, 0, 0)
    st = _lib.lib().lsc_backend_create(C.byref(cfg), C.byref(h))
    assert st == _lib.ERROR_BACKEND_NOT_AVAILABLE
    assert not h.value


def test_withhold_hook_argument_checks():
    """The bounded-wait test hook takes a launch count and a 1 ms .. 2 s wait limit; setting it
    launches nothing (0 cancels)."""
    lib = _lib.lib()
    assert lib.lsc_debug_withhold_copy(-1, 10_000_000) == _lib.ERROR_INVALID_ARGUMENT
    assert lib.lsc_debug_withhold_copy(1, 10) == _lib.ERROR_INVALID_ARGUMENT
    assert lib.lsc_debug_withhold_copy(1, 3_000_000_000) == _lib.ERROR_INVALID_ARGUMENT
    assert lib.lsc_debug_withhold_copy(1, 10_000_000) == _lib.SUCCESS
    assert lib.lsc_debug_withhold_copy(0, 10_000_000) == _lib.SUCCESS
