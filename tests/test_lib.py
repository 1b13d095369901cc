"""The C-ABI library: it loads, exports every symbol include/xcb_moe.h declares, and its host-side queries
validate shapes (no kernel launches: these run without a GPU)."""
import ctypes
import os
import re

import pytest

from xcalibur_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_symbols():
    src = open(os.path.join(ROOT, "include", "xcb_moe.h")).read()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w[\w\s\*]*?\b(xcb_\w+)\s*\(", src, re.M)))


def test_header_declares_what_the_binding_binds():
    assert header_symbols() == sorted(_lib.EXPORTS)


def test_library_exports_every_symbol():
    lib = _lib.load()
    for name in header_symbols():
        assert hasattr(lib, name), name


def _shape(E=8, Et=None, off=0, H=1024, I=512):
    return _lib.XcbMoeShape(E, Et if Et is not None else E + off, off, H, I)


def test_shape_checks():
    lib = _lib.load()
    ok = _shape()
    assert lib.xcb_moe_check_shape(ctypes.byref(ok)) == _lib.XCB_OK
    assert lib.xcb_moe_check_shape(ctypes.byref(_shape(H=1000))) == _lib.XCB_ERR_UNSUPPORTED
    assert lib.xcb_moe_check_shape(ctypes.byref(_shape(E=0))) == _lib.XCB_ERR_INVALID_ARG
    assert lib.xcb_moe_check_shape(ctypes.byref(_shape(E=8, Et=4))) == _lib.XCB_ERR_INVALID_ARG
    assert lib.xcb_moe_check_shape(ctypes.byref(_shape(E=1024))) == _lib.XCB_ERR_UNSUPPORTED
    assert lib.xcb_moe_check_shape(None) == _lib.XCB_ERR_INVALID_ARG
    assert lib.xcb_status_str(_lib.XCB_ERR_WORKSPACE) == b"workspace too small"


def test_packed_and_workspace_sizes():
    lib = _lib.load()
    s = _shape(E=256, H=7168, I=2048)
    assert lib.xcb_moe_packed_bytes(ctypes.byref(s), 0) == 2 * 256 * 256 * 9 * 7168
    assert lib.xcb_moe_packed_bytes(ctypes.byref(s), 1) == 2 * 256 * 448 * 9 * 2048
    n1 = lib.xcb_moe_workspace_bytes(ctypes.byref(s), 1, 8)
    n2 = lib.xcb_moe_workspace_bytes(ctypes.byref(s), 64, 8)
    assert 0 < n1 < n2
    offs = (ctypes.c_size_t * 6)()
    assert lib.xcb_moe_workspace_offsets(ctypes.byref(s), 64, 8, offs, 6) == 6
    assert all(o % 256 == 0 and o < n2 for o in offs)
    assert lib.xcb_moe_workspace_offsets(ctypes.byref(s), 64, 8, offs, 2) == -1


def test_forward_rejects_bad_arguments_before_launch():
    lib = _lib.load()
    s = _shape()
    w = _lib.XcbMoeWeights(s, 16, 16, 16, 16, None)
    a = _lib.XcbMoeArgs(4, 2, 0, 0, 16, None, None, None, 16, None, None)   # no routing given
    assert lib.xcb_moe_forward(ctypes.byref(w), ctypes.byref(a), 16, 1 << 30, None) == _lib.XCB_ERR_INVALID_ARG
    a = _lib.XcbMoeArgs(4, 2, 0, 0, 16, 16, 16, 16, 16, None, None)          # both given
    assert lib.xcb_moe_forward(ctypes.byref(w), ctypes.byref(a), 16, 1 << 30, None) == _lib.XCB_ERR_INVALID_ARG
    a = _lib.XcbMoeArgs(4, 2, 0, 0, 16, 16, None, None, 16, None, None)
    assert lib.xcb_moe_forward(ctypes.byref(w), ctypes.byref(a), 16, 16, None) == _lib.XCB_ERR_WORKSPACE
    a = _lib.XcbMoeArgs(4, 2, 0, 0, 18, 16, None, None, 16, None, None)      # misaligned x
    assert lib.xcb_moe_forward(ctypes.byref(w), ctypes.byref(a), 16, 1 << 30, None) == _lib.XCB_ERR_INVALID_ARG
    a = _lib.XcbMoeArgs(4, 2, _lib.XCB_FLAG_POST_NORM, 0, 16, 16, None, None, 16, None, None)  # no post_norm_w
    assert lib.xcb_moe_forward(ctypes.byref(w), ctypes.byref(a), 16, 1 << 30, None) == _lib.XCB_ERR_INVALID_ARG
    a = _lib.XcbMoeArgs(4, 2, 0, -1, 16, 16, None, None, 16, None, None)     # negative wait limit
    assert lib.xcb_moe_forward(ctypes.byref(w), ctypes.byref(a), 16, 1 << 30, None) == _lib.XCB_ERR_INVALID_ARG
    a = _lib.XcbMoeArgs(0, 2, 0, 0, 16, 16, None, None, 16, None, None)      # T = 0: nothing to do
    assert lib.xcb_moe_forward(ctypes.byref(w), ctypes.byref(a), 16, 0, None) == _lib.XCB_OK
