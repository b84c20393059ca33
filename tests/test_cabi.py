"""The C ABI library loads without a GPU and exports every entry point that
include/d2p_b200.h declares (no compute calls: those need a GPU)."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "d2p_b200.h")
LIB = os.path.join(ROOT, "d2p_b200", "libd2p_b200.so")


def declared():
    txt = open(HEADER).read()
    return sorted(set(re.findall(r"^D2P_API\s+[\w\s\*]+?\b(d2p_\w+)\s*\(", txt, flags=re.M)))


@pytest.fixture(scope="module")
def lib():
    if not os.path.exists(LIB):
        from d2p_b200 import _build

        _build.build_cuda_lib()
    return ctypes.CDLL(LIB)


def test_header_declares_entry_points():
    names = declared()
    for need in ("d2p_sw_forward_backward", "d2p_sw_hvp", "d2p_sw_param_jacobian", "d2p_sw_backward_full",
                 "d2p_sw_value_backward", "d2p_sw_affine_forward_backward", "d2p_sw_affine_hvp",
                 "d2p_sw_affine_param_jacobian", "d2p_sw_affine_backward_full", "d2p_sw_workspace_bytes",
                 "d2p_error_string", "d2p_version"):
        assert need in names, need


def test_library_exports_every_declared_symbol(lib):
    missing = [n for n in declared() if not hasattr(lib, n)]
    assert not missing, missing


def test_host_only_helpers(lib):
    lib.d2p_version.restype = ctypes.c_int
    assert lib.d2p_version() >= 100
    lib.d2p_error_string.restype = ctypes.c_char_p
    lib.d2p_error_string.argtypes = [ctypes.c_int]
    assert b"workspace" in lib.d2p_error_string(1002)
    assert lib.d2p_error_string(0) == b"success"
    f = lib.d2p_sw_workspace_bytes
    f.restype = ctypes.c_size_t
    f.argtypes = [ctypes.c_int] * 5
    n_fb = f(0, 0, 256, 512, 512)
    assert 0 < n_fb < (1 << 40)
    assert f(1, 0, 4, 64, 64) > 0
    assert f(0, 3, 2, 10, 12) >= f(0, 2, 2, 10, 12)
    assert f(7, 0, 1, 1, 1) == ctypes.c_size_t(-1).value
    # the reference's int32 table rule: (L1+1)*(L2+1) <= INT_MAX
    assert f(0, 0, 1, 70000, 70000) == ctypes.c_size_t(-1).value


def test_argument_validation_without_gpu(lib):
    """Invalid arguments are rejected on the host before any CUDA call."""
    fn = lib.d2p_sw_param_jacobian
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                   ctypes.c_float, ctypes.c_float, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t,
                   ctypes.c_void_p]
    assert fn(None, None, 1, 4, 4, 5, -1.0, 1.0, None, None, 0, None) == 1001   # bad param_type
    assert fn(None, None, 0, 4, 4, 0, -1.0, 1.0, None, None, 0, None) == 0      # empty batch: no-op
    fb = lib.d2p_sw_forward_backward
    fb.restype = ctypes.c_int
    fb.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_float,
                   ctypes.c_float, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                   ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]
    # workspace too small is reported before launching
    assert fb(ctypes.c_void_p(16), None, 2, 8, 8, -1.0, 1.0, None, None, None, None, None, None, None, 0,
              None) == 1002
