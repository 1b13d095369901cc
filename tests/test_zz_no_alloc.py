"""The allocation-free entry point ``xcb_moe_forward_static``, called through the C-ABI.

Some callers cannot allocate device memory: host frameworks that own every device byte through their own
allocator and forbid plugins to call cudaMalloc, and latency-critical decode loops where cudaMalloc/cudaFree would
stall or synchronise the device.  For them the library keeps one fixed scratch array per GPU.  This test checks
that the entry point gives the same output as ``xcb_moe_forward`` with a caller workspace, on two calls in a row
(the second call reuses the scratch the first one left behind), and that it refuses a call too large for the array.
The file name sorts last so a run that stops at the first failure has run every other test first.
"""
import ctypes

import numpy as np
import pytest
import torch

from oracle import moe_ref
from tests._util import ATOL, RTOL

pytestmark = pytest.mark.gpu


def _layer(dev, seed, E=8, H=1024, I=512):
    from xcalibur_b200 import PreparedMoE

    rng = np.random.default_rng(seed)
    w = moe_ref.make_weights(rng, E, H, I)
    layer = PreparedMoE(*[torch.from_numpy(np.ascontiguousarray(a)).to(dev) for a in w])
    return layer, rng


def _inputs(rng, dev, T, H, E):
    x, logits = moe_ref.make_inputs(rng, T, H, E)
    return (torch.from_numpy(x.view(np.int16)).to(dev).view(torch.bfloat16), torch.from_numpy(logits).to(dev))


def test_static_scratch_matches_workspace_forward(cuda_device):
    from xcalibur_b200 import _lib

    lib = _lib.load()
    dev = cuda_device
    layer, rng = _layer(dev, seed=77)
    stream = torch.cuda.current_stream(dev).cuda_stream
    for T, k in ((16, 2), (5, 3)):                   # two calls in a row, different sizes
        x, logits = _inputs(rng, dev, T, layer.H, layer.E)
        want = layer.forward(x, logits, k)
        out = torch.full((T, layer.H), float("nan"), dtype=torch.bfloat16, device=dev)
        args = _lib.XcbMoeArgs(T, k, 0, 0, x.data_ptr(), logits.data_ptr(), None, None, out.data_ptr(), None, None)
        rc = lib.xcb_moe_forward_static(ctypes.byref(layer._weights), ctypes.byref(args), stream)
        assert rc == _lib.XCB_OK, lib.xcb_status_str(rc)
        torch.cuda.synchronize(dev)
        assert torch.isfinite(out.float()).all()
        assert torch.allclose(out.float(), want.float(), rtol=RTOL, atol=ATOL)


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
