"""ctypes binding of the C-ABI library (include/xcb_moe.h).

This is the stub a maintainer of the reference would add on its side of the boundary: the reference reaches its
native code through a pybind module compiled at run time (``okc_run``, kernels/moe_w4a16_h200/moe_w4a16.py:3063-3098);
here the library is prebuilt and loaded once.  Importing this module fails loudly when the library is missing —
there is no CPU or eager fallback.
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
# the in-tree build; XCB_MOE_LIB selects another build of the same library (e.g. one compiled with other tile knobs)
LIB_PATH = os.environ.get("XCB_MOE_LIB") or os.path.join(HERE, "libxcb_moe.so")

XCB_OK = 0
XCB_ERR_INVALID_ARG = 1
XCB_ERR_UNSUPPORTED = 2
XCB_ERR_WORKSPACE = 3
XCB_ERR_CUDA = 4
XCB_ERR_DEVICE = 5
XCB_STATUS_DEVICE_TIMEOUT = 1
XCB_STATUS_BAD_EXPERT = 2
XCB_STATUS_NAN_SCALE = 4
XCB_STATUS_CAPACITY = 8
XCB_FLAG_POST_NORM = 1
XCB_FLAG_DECODE_PATH = 2
XCB_FLAG_PREFILL_PATH = 4
XCB_FLAG_PDL = 8
XCB_FLAG_DETERMINISTIC = 16
XCB_STATIC_SCRATCH_BYTES = 8 << 20

# every symbol include/xcb_moe.h declares
EXPORTS = (
    "xcb_status_str",
    "xcb_moe_check_shape",
    "xcb_moe_packed_bytes",
    "xcb_moe_pack_weights",
    "xcb_moe_workspace_bytes",
    "xcb_moe_workspace_offsets",
    "xcb_moe_plan_info",
    "xcb_moe_workspace_init",
    "xcb_moe_forward",
    "xcb_moe_route",
    "xcb_moe_experts",
    "xcb_moe_forward_static",
    "xcb_moe_static_read_status",
    "xcb_moe_read_status",
    "xcb_nvfp4_quantize",
    "xcb_hbm_probe",
    "xcb_moe_topk",
    "xcb_ep_plan",
    "xcb_ep_gather",
    "xcb_ep_p2p_bytes",
    "xcb_p2p_alloc",
    "xcb_p2p_open",
    "xcb_p2p_close",
    "xcb_p2p_free",
    "xcb_ep_p2p_dispatch",
    "xcb_ep_p2p_combine",
    "xcb_ep_combine",
)


class XcbMoeShape(ctypes.Structure):
    _fields_ = [("num_experts", ctypes.c_int32), ("total_experts", ctypes.c_int32), ("expert_offset", ctypes.c_int32),
                ("hidden", ctypes.c_int32), ("inter", ctypes.c_int32)]


class XcbMoeWeights(ctypes.Structure):
    _fields_ = [("shape", XcbMoeShape), ("gate_up", ctypes.c_void_p), ("down", ctypes.c_void_p),
                ("gate_up_gs", ctypes.c_void_p), ("down_gs", ctypes.c_void_p), ("post_norm_w", ctypes.c_void_p)]


class XcbMoeArgs(ctypes.Structure):
    _fields_ = [("tokens", ctypes.c_int32), ("top_k", ctypes.c_int32), ("flags", ctypes.c_int32),
                ("wait_limit_us", ctypes.c_int32), ("hidden_states", ctypes.c_void_p), ("router_logits", ctypes.c_void_p),
                ("topk_ids", ctypes.c_void_p), ("topk_weights", ctypes.c_void_p), ("out", ctypes.c_void_p),
                ("topk_ids_out", ctypes.c_void_p), ("topk_weights_out", ctypes.c_void_p)]


_LIB = None


def load(path: str = LIB_PATH) -> ctypes.CDLL:
    """Load the library (once).  Raises OSError if it was not built."""
    global _LIB
    if _LIB is not None:
        return _LIB
    if not os.path.exists(path):
        raise OSError(f"{path} is missing: run `python -m xcalibur_b200.build` (or __graft_entry__.build())")
    lib = ctypes.CDLL(path)
    P, I32, SZ, U64 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_size_t, ctypes.c_uint64
    sig = {
        "xcb_status_str": (ctypes.c_char_p, [ctypes.c_int]),
        "xcb_moe_check_shape": (ctypes.c_int, [ctypes.POINTER(XcbMoeShape)]),
        "xcb_moe_packed_bytes": (SZ, [ctypes.POINTER(XcbMoeShape), ctypes.c_int]),
        "xcb_moe_pack_weights": (ctypes.c_int, [ctypes.POINTER(XcbMoeShape), P, P, P, P, P, P, P, P, P]),
        "xcb_moe_workspace_bytes": (SZ, [ctypes.POINTER(XcbMoeShape), I32, I32]),
        "xcb_moe_workspace_offsets": (ctypes.c_int, [ctypes.POINTER(XcbMoeShape), I32, I32,
                                                      ctypes.POINTER(ctypes.c_size_t), ctypes.c_int]),
        "xcb_moe_plan_info": (ctypes.c_int, [ctypes.POINTER(XcbMoeShape), I32, I32, I32, I32,
                                              ctypes.POINTER(ctypes.c_int32), I32]),
        "xcb_moe_workspace_init": (ctypes.c_int, [P, SZ, I32, I32, P]),
        "xcb_moe_forward": (ctypes.c_int, [ctypes.POINTER(XcbMoeWeights), ctypes.POINTER(XcbMoeArgs), P, SZ, P]),
        "xcb_moe_route": (ctypes.c_int, [ctypes.POINTER(XcbMoeWeights), ctypes.POINTER(XcbMoeArgs), P, SZ, P]),
        "xcb_moe_experts": (ctypes.c_int, [ctypes.POINTER(XcbMoeWeights), ctypes.POINTER(XcbMoeArgs), P, SZ, P]),
        "xcb_moe_forward_static": (ctypes.c_int, [ctypes.POINTER(XcbMoeWeights), ctypes.POINTER(XcbMoeArgs), P]),
        "xcb_moe_read_status": (ctypes.c_int, [P, ctypes.POINTER(I32), P]),
        "xcb_moe_static_read_status": (ctypes.c_int, [ctypes.POINTER(I32), P]),
        "xcb_nvfp4_quantize": (ctypes.c_int, [P, I32, I32, I32, P, P, P, P, P]),
        "xcb_hbm_probe": (ctypes.c_int, [P, SZ, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                         P, ctypes.c_int, P, P, P]),
        "xcb_moe_topk": (ctypes.c_int, [P, I32, I32, I32, P, P, P]),
        "xcb_ep_plan": (ctypes.c_int, [P, I32, I32, I32, I32, P, P, P, P, P]),
        "xcb_ep_p2p_bytes": (SZ, [I32, I32, I32, I32]),
        "xcb_p2p_alloc": (ctypes.c_int, [SZ, ctypes.POINTER(ctypes.c_void_p), P]),
        "xcb_p2p_open": (ctypes.c_int, [P, ctypes.POINTER(ctypes.c_void_p)]),
        "xcb_p2p_close": (ctypes.c_int, [P]),
        "xcb_p2p_free": (ctypes.c_int, [P]),
        "xcb_ep_p2p_dispatch": (ctypes.c_int, [P, P, I32, I32, I32, I32, I32, I32, I32, P, P, U64, P]),
        "xcb_ep_p2p_combine": (ctypes.c_int, [P, I32, I32, I32, I32, I32, I32, P, P, P, U64, P]),
        "xcb_ep_gather": (ctypes.c_int, [P, P, P, I32, I32, I32, I32, P, P, P, P, P, P]),
        "xcb_ep_combine": (ctypes.c_int, [P, P, P, I32, I32, I32, P, P]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _LIB = lib
    return lib


class XcbError(RuntimeError):
    def __init__(self, code: int, what: str):
        self.code = code
        msg = load().xcb_status_str(code).decode()
        super().__init__(f"{what}: {msg} (code {code})")


def check(code: int, what: str):
    if code != XCB_OK:
        raise XcbError(code, what)
