"""The allocation-free entry point ``xcb_moe_forward_static``, called through the C-ABI.

Some callers cannot allocate device memory: host frameworks that own every device byte through their own
allocator and forbid plugins to call cudaMalloc, and latency-critical decode loops where cudaMalloc/cudaFree would
stall or synchronise the device.  For them the library keeps one fixed scratch array per GPU.  This test checks
that the entry point gives the same output as ``xcb_moe_forward`` with a caller workspace and as the CPU oracle, on
calls in a row (each reuses the scratch the one before left behind), through both the single-launch decode kernel
and the router + tensor-core path, that device-side errors of these calls can be read back with
``xcb_moe_static_read_status``, and that it refuses a call too large for the array.
The file name sorts last so a run that stops at the first failure has run every other test first.
"""
import ctypes

import numpy as np
import pytest
import torch

from oracle import moe_ref
from tests._util import ATOL, RTOL, assert_close_bf16

pytestmark = pytest.mark.gpu


def _layer(dev, seed, E=8, H=1024, I=512):
    from xcalibur_b200 import PreparedMoE

    rng = np.random.default_rng(seed)
    w = moe_ref.make_weights(rng, E, H, I)
    layer = PreparedMoE(*[torch.from_numpy(np.ascontiguousarray(a)).to(dev) for a in w])
    layer.np_weights = w
    return layer, rng


def _read_static_status(lib):
    v = ctypes.c_int32(0)
    rc = lib.xcb_moe_static_read_status(ctypes.byref(v), None)
    return rc, v.value


def _inputs(rng, dev, T, H, E):
    x, logits = moe_ref.make_inputs(rng, T, H, E)
    return (torch.from_numpy(x.view(np.int16)).to(dev).view(torch.bfloat16), torch.from_numpy(logits).to(dev))


def test_static_scratch_matches_workspace_forward(cuda_device):
    from xcalibur_b200 import _lib

    lib = _lib.load()
    dev = cuda_device
    layer, rng = _layer(dev, seed=77)
    stream = torch.cuda.current_stream(dev).cuda_stream
    # calls in a row of different sizes: in-kernel routing (16 x 2, 5 x 3 routes), the router + tensor-core path
    # (64 tokens: above the decode kernel's 32), then a small call again on the scratch that path left behind
    for T, k in ((16, 2), (5, 3), (64, 2), (3, 2)):
        x, logits = _inputs(rng, dev, T, layer.H, layer.E)
        want = layer.forward(x, logits, k)
        out = torch.full((T, layer.H), float("nan"), dtype=torch.bfloat16, device=dev)
        args = _lib.XcbMoeArgs(T, k, 0, 0, x.data_ptr(), logits.data_ptr(), None, None, out.data_ptr(), None, None)
        rc = lib.xcb_moe_forward_static(ctypes.byref(layer._weights), ctypes.byref(args), stream)
        assert rc == _lib.XCB_OK, lib.xcb_status_str(rc)
        torch.cuda.synchronize(dev)
        assert torch.isfinite(out.float()).all()
        assert torch.allclose(out.float(), want.float(), rtol=RTOL, atol=ATOL)
        # and against the CPU oracle on the same inputs
        xb = x.view(torch.int16).cpu().numpy().view(np.uint16)
        ref, _, _ = moe_ref.moe_layer(xb, logits.cpu().numpy(), *layer.np_weights, k)
        assert_close_bf16(out, ref)
    assert _read_static_status(lib) == (_lib.XCB_OK, 0)


def test_static_scratch_status_is_readable(cuda_device):
    """An expert id outside the router's range is a device-side error: the call drops that route and sets
    XCB_STATUS_BAD_EXPERT in the fixed scratch, where xcb_moe_static_read_status finds it; the read clears it, and
    the next call does not wipe bits a caller has not read yet."""
    from xcalibur_b200 import _lib

    lib = _lib.load()
    dev = cuda_device
    layer, rng = _layer(dev, seed=79)
    stream = torch.cuda.current_stream(dev).cuda_stream
    _read_static_status(lib)                                   # start from a clean word
    T, k = 4, 2
    x, _ = _inputs(rng, dev, T, layer.H, layer.E)
    ids = torch.tensor([[0, 1], [2, 99], [3, 4], [5, 6]], dtype=torch.int32, device=dev)   # 99: out of range
    wts = torch.full((T, k), 0.5, dtype=torch.float32, device=dev)
    out = torch.empty((T, layer.H), dtype=torch.bfloat16, device=dev)
    args = _lib.XcbMoeArgs(T, k, 0, 0, x.data_ptr(), None, ids.data_ptr(), wts.data_ptr(), out.data_ptr(), None,
                           None)
    assert lib.xcb_moe_forward_static(ctypes.byref(layer._weights), ctypes.byref(args), stream) == _lib.XCB_OK
    good = torch.tensor([[0, 1], [2, 3], [3, 4], [5, 6]], dtype=torch.int32, device=dev)
    args2 = _lib.XcbMoeArgs(T, k, 0, 0, x.data_ptr(), None, good.data_ptr(), wts.data_ptr(), out.data_ptr(), None,
                            None)
    assert lib.xcb_moe_forward_static(ctypes.byref(layer._weights), ctypes.byref(args2), stream) == _lib.XCB_OK
    rc, bits = _read_static_status(lib)
    assert rc == _lib.XCB_ERR_DEVICE and bits & _lib.XCB_STATUS_BAD_EXPERT, (rc, bits)
    assert _read_static_status(lib) == (_lib.XCB_OK, 0)


def test_static_scratch_rejects_oversized_call(cuda_device):
    from xcalibur_b200 import _lib

    lib = _lib.load()
    layer, rng = _layer(cuda_device, seed=78)
    T, k = 4096, 8
    shape = layer.shape
    assert lib.xcb_moe_workspace_bytes(ctypes.byref(shape), T, k) > _lib.XCB_STATIC_SCRATCH_BYTES
    x = torch.zeros((T, layer.H), dtype=torch.bfloat16, device=cuda_device)
    logits = torch.zeros((T, layer.E), dtype=torch.float32, device=cuda_device)
    out = torch.zeros((T, layer.H), dtype=torch.bfloat16, device=cuda_device)
    args = _lib.XcbMoeArgs(T, k, 0, 0, x.data_ptr(), logits.data_ptr(), None, None, out.data_ptr(), None, None)
    assert lib.xcb_moe_forward_static(ctypes.byref(layer._weights), ctypes.byref(args),
                                      torch.cuda.current_stream(cuda_device).cuda_stream) == _lib.XCB_ERR_WORKSPACE
