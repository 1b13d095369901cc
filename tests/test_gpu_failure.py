"""Failure detection on one GPU without a fault: a bounded device wait is made to run out (its flag is one that
nothing will raise), and the test checks that the kernel returned, that the status word says so, and that the
workspace is usable again by the next call.  Nothing here traps, faults or hangs the GPU: every wait in these
kernels gives up after the call's ``wait_limit_us``.

The reference's spins are unbounded (the phase A -> B handoff and the grid barrier of
kernels/moe_w4a16_h200/moe_w4a16.py:1625 and :2635-2639); here every one of them is bounded."""
import numpy as np
import pytest
import torch

from oracle import moe_ref
from tests._util import assert_close_bf16, oracle_layer

pytestmark = pytest.mark.gpu


def _weights_from_np(w, dev):
    c13, s13, g13, c2, s2, g2 = w
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    return {"w13": t(c13), "w13_sf": t(s13), "w13_gs": t(g13), "w2": t(c2), "w2_sf": t(s2), "w2_gs": t(g2)}


def test_decode_grid_barrier_wait_runs_out_and_recovers(cuda_device):
    """Post-norm decode calls end in a grid barrier on a workspace counter.  With that counter pushed far below
    zero no CTA count can reach it: every CTA gives up after the 1 ms limit, XCB_STATUS_DEVICE_TIMEOUT is set, the
    kernel still runs to its end (the last CTA returns the counters to zero), and the next call on the same
    workspace is correct again."""
    from xcalibur_b200 import PreparedMoE, _lib

    dev = cuda_device
    rng = np.random.default_rng(51)
    E, H, I, T, k = 8, 1024, 512, 3, 2
    w = moe_ref.make_weights(rng, E, H, I)
    gamma = moe_ref.f32_to_bf16_bits(rng.standard_normal(H, dtype=np.float32) * np.float32(0.1))
    weights = _weights_from_np(w, dev)
    pn = torch.from_numpy(gamma.view(np.int16)).to(dev).view(torch.bfloat16)
    layer = PreparedMoE(*weights.values(), pn)
    x, logits = moe_ref.make_inputs(rng, T, H, E)
    xd = torch.from_numpy(x.view(np.int16)).to(dev).view(torch.bfloat16)
    ld = torch.from_numpy(logits).to(dev)
    ws = layer.workspace(T, k)
    ws[4:8].view(torch.int32).fill_(-(1 << 30))           # control word 1: the decode kernel's grid barrier
    layer.forward(xd, ld, k, post_norm=True, wait_limit_us=1000)
    torch.cuda.synchronize(dev)                            # the kernel returned
    assert layer.check_device_status() & _lib.XCB_STATUS_DEVICE_TIMEOUT
    assert int(ws[4:8].view(torch.int32).item()) == 0      # the last CTA reset the barrier
    out, ids, wts = layer.forward(xd, ld, k, post_norm=True, return_routing=True)
    torch.cuda.synchronize(dev)
    assert layer.check_device_status() == 0
    want = oracle_layer(xd, weights, ids.cpu().numpy(), wts.cpu().numpy(), post_norm_w=pn)
    assert_close_bf16(out, want)


def test_wait_limit_is_validated():
    """A negative limit is refused on the host before anything is launched."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from xcalibur_b200 import PreparedMoE

    rng = np.random.default_rng(52)
    w = moe_ref.make_weights(rng, 4, 256, 256)
    layer = PreparedMoE(*_weights_from_np(w, torch.device("cuda:0")).values())
    x = torch.zeros((1, 256), dtype=torch.bfloat16, device="cuda:0")
    with pytest.raises(ValueError):
        layer.forward(x, torch.zeros((1, 4), device="cuda:0"), 2, wait_limit_us=-1)
