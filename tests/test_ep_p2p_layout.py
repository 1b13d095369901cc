"""Host-side checks of the NVLink peer exchange (no GPU): the Python layout mirror equals the library's, and the
entry points reject bad arguments before any launch."""
import ctypes

import pytest

from xcalibur_b200 import _lib
from xcalibur_b200.ep import p2p_layout


@pytest.mark.parametrize("G,T,H,k", [(2, 32, 7168, 8), (8, 32, 7168, 8), (4, 7, 1024, 2), (32, 1, 64, 16)])
def test_layout_mirror_matches_library(G, T, H, k):
    lib = _lib.load()
    x, ids, wts, part, flag, total = p2p_layout(G, T, H, k)
    assert lib.xcb_ep_p2p_bytes(G, T, H, k) == total
    assert x == 0 and x < ids < wts < part < flag < total
    assert all(o % 256 == 0 for o in (ids, wts, part, flag))
    assert ids >= G * T * H * 2 and wts - ids >= G * T * k * 4 and part - wts >= G * T * k * 4
    assert flag - part >= G * T * H * 2


def test_bad_arguments_are_rejected_on_the_host():
    lib = _lib.load()
    assert lib.xcb_ep_p2p_bytes(0, 1, 64, 8) == 0
    assert lib.xcb_ep_p2p_bytes(33, 1, 64, 8) == 0
    fake = ctypes.c_void_p(16)
    # T = 0, T > T_max, H not a multiple of 8, rank outside [0, G), null peers; E beyond 512 (dispatch only)
    for args in [(0, 4, 64, 8, 2, 0, fake), (5, 4, 64, 8, 2, 0, fake), (1, 4, 60, 8, 2, 0, fake),
                 (1, 4, 64, 8, 2, 2, fake), (1, 4, 64, 8, 2, 0, None)]:
        T, Tm, H, k, G, rank, peers = args
        assert lib.xcb_ep_p2p_dispatch(fake, fake, T, Tm, H, 256, k, G, rank, peers, fake, 0, None) == \
            _lib.XCB_ERR_INVALID_ARG
        assert lib.xcb_ep_p2p_combine(fake, T, Tm, H, k, G, rank, peers, fake, fake, 0, None) == \
            _lib.XCB_ERR_INVALID_ARG
    assert lib.xcb_ep_p2p_dispatch(fake, fake, 1, 4, 64, 513, 8, 2, 0, fake, fake, 0, None) == _lib.XCB_ERR_INVALID_ARG
    assert lib.xcb_p2p_alloc(0, ctypes.byref(ctypes.c_void_p()), None) == _lib.XCB_ERR_INVALID_ARG
    assert lib.xcb_p2p_open(None, ctypes.byref(ctypes.c_void_p())) == _lib.XCB_ERR_INVALID_ARG
