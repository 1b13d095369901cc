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


def _plan(shape, T, k, given, flags=0):
    """xcb_moe_plan_info: the planner of a forward call, run without a GPU."""
    lib = _lib.load()
    out = (ctypes.c_int32 * 8)()
    assert lib.xcb_moe_plan_info(ctypes.byref(shape), T, k, flags, int(given), out, 8) == 8
    keys = ("prefill", "in_kernel_routes", "job_routes", "rows", "buffers", "stages", "stage_bytes", "two_token")
    return dict(zip(keys, list(out)))


def test_plan_of_the_deepseek_decode_step():
    """Configuration 2 (one token, router logits): one launch, one-route jobs, two activation buffers and the three
    64.5 KB stages of the one-token plan."""
    p = _plan(_shape(256, H=7168, I=2048), 1, 8, False)
    assert p == {"prefill": 0, "in_kernel_routes": 1, "job_routes": 1, "rows": 1, "buffers": 2, "stages": 3,
                 "stage_bytes": 64512, "two_token": 0}


def test_plan_of_two_tokens_stages_both_rows():
    """Two tokens at the DeepSeek-V3 shape: one-token jobs keep two buffers, and the kernel instantiation that
    stages both rows at start runs (routes given, as the expert-parallel local layer passes them)."""
    p = _plan(_shape(128, Et=256, H=7168, I=2048), 2, 8, True)
    assert (p["prefill"], p["job_routes"], p["rows"], p["buffers"], p["two_token"]) == (0, 1, 1, 2, 1)


@pytest.mark.parametrize("T", [1, 8, 16, 32, 128])
def test_plan_at_the_reference_shape_keeps_two_buffers(T):
    """The reference's shape (H = I = 4096, 32 of 256 experts, given routes): the decode path with jobs as wide as
    two activation buffers allow (not 8-route jobs with one buffer and three stages)."""
    p = _plan(_shape(32, Et=256, H=4096, I=4096), T, 8, True)
    assert p["prefill"] == 0 and p["buffers"] == 2 and p["stage_bytes"] == 36864
    assert 1 <= p["job_routes"] <= 8 and p["rows"] == p["job_routes"]
    assert p["in_kernel_routes"] == int(T * 8 <= 256)


def test_plan_keeps_wide_jobs_when_experts_get_many_routes():
    """When the expected routes per expert exceed what two buffers allow, the jobs stay wide: narrower jobs would
    stream an expert's weights once per job."""
    p = _plan(_shape(256, H=7168, I=2048), 64, 8, False, flags=_lib.XCB_FLAG_DECODE_PATH)
    assert p["prefill"] == 0 and p["in_kernel_routes"] == 0 and p["job_routes"] >= 2


def test_plan_of_a_large_batch_is_the_prefill_path():
    p = _plan(_shape(256, H=7168, I=2048), 4096, 8, False)
    assert p["prefill"] == 1 and p["job_routes"] == 0


def test_plan_info_rejects_bad_arguments():
    lib = _lib.load()
    out = (ctypes.c_int32 * 8)()
    s = _shape()
    assert lib.xcb_moe_plan_info(ctypes.byref(s), 0, 8, 0, 0, out, 8) == _lib.XCB_ERR_INVALID_ARG
    assert lib.xcb_moe_plan_info(ctypes.byref(s), 4, 17, 0, 0, out, 8) == _lib.XCB_ERR_INVALID_ARG
    assert lib.xcb_moe_plan_info(ctypes.byref(_shape(E=0)), 4, 8, 0, 0, out, 8) != 8


@pytest.mark.parametrize("T,prefill", [(32, 0), (48, 0), (96, 0), (97, 1), (128, 1)])
def test_plan_path_by_routes_per_expert(T, prefill):
    """A layer holding all 256 DeepSeek-V3 experts stays on the decode path up to 3 routes per expert on average
    (96 tokens x top-8), where its weight stream beats the tensor-core path."""
    assert _plan(_shape(256, H=7168, I=2048), T, 8, False)["prefill"] == prefill


@pytest.mark.parametrize("T,prefill", [(32, 0), (48, 0), (49, 1), (64, 1)])
def test_plan_path_at_the_qwen3_shape(T, prefill):
    """128 experts (H = 2048, I = 768): 3 routes per expert is 48 tokens x top-8."""
    assert _plan(_shape(128, H=2048, I=768), T, 8, False)["prefill"] == prefill


def test_plan_shard_path_uses_the_held_routes():
    """An expert-parallel shard (32 of 256 experts held) is planned by the routes it expects to hold: 128 tokens x
    top-8 (~128 held routes) decode, 256 tokens (~256) prefill."""
    assert _plan(_shape(32, Et=256, H=4096, I=4096), 128, 8, True)["prefill"] == 0
    assert _plan(_shape(32, Et=256, H=4096, I=4096), 256, 8, True)["prefill"] == 1
