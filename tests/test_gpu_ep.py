"""Expert parallelism on two GPUs (NVLink peer exchange and NCCL): each rank's output equals a single-GPU layer
holding every expert."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from tests._ep_gpu_worker import nccl_worker
from tests._util import assert_close_bf16

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("T,p2p,calls", [(1, True, 3), (7, True, 2), (1, False, 1), (600, True, 1)])
def test_ep_two_gpus_match_single_gpu(tmp_path, T, p2p, calls):
    """Dense exchange over NVLink peer memory (several consecutive steps), dense exchange over NCCL, planned
    exchange over NCCL."""
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world, E, H, I, k = 2, 32, 2048, 768, 8
    mp.spawn(nccl_worker, args=(world, _free_port(), E, H, I, T, k, 77, str(tmp_path), p2p, calls), nprocs=world,
             join=True)
    for r in range(world):
        with open(os.path.join(tmp_path, f"p2p_{r}.txt")) as f:
            why = f.read()
        assert not why, f"rank {r}: the peer exchange was requested but not set up: {why}"
        assert int(np.load(os.path.join(tmp_path, f"nccl_status_{r}.npy"))[0]) == 0
        got, want = np.load(os.path.join(tmp_path, f"nccl_{r}.npy"))
        assert_close_bf16(torch.from_numpy(got.view(np.int16)).view(torch.bfloat16), want)


@pytest.mark.parametrize("Tm,H,E,k,steps", [(4, 256, 64, 4, (3, 1, 4)), (32, 7168, 256, 8, (2, 32, 1, 7))])
def test_p2p_exchange_one_rank_round_trip(cuda_device, Tm, H, E, k, steps):
    """The peer-exchange kernels on one rank (its buffer is its only peer, so each kernel raises the flags it then
    waits for): the received rows equal what was sent, the received top-k rows equal the library router's on the
    same logits, the combine returns the partial rows summed over the one rank, and consecutive steps keep the
    flags in step.  At H = 7168 and T_max = 32 several blocks push to each peer, and steps of 2, 32, 1 and 7
    tokens leave some of them with no rows: the flags' targets must not depend on a step's size."""
    import ctypes

    from xcalibur_b200 import _lib
    from xcalibur_b200.ep import _DeviceBytes, p2p_layout

    lib = _lib.load()
    G = 1
    nbytes = lib.xcb_ep_p2p_bytes(G, Tm, H, k)
    own = ctypes.c_void_p()
    handle = (ctypes.c_ubyte * 64)()
    assert lib.xcb_p2p_alloc(nbytes, ctypes.byref(own), handle) == _lib.XCB_OK
    try:
        buf = torch.as_tensor(_DeviceBytes(own.value, nbytes), device=cuda_device)
        xo, io, wo, _, _, _ = p2p_layout(G, Tm, H, k)
        peers = torch.tensor([own.value], dtype=torch.int64, device=cuda_device)
        status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
        stream = torch.cuda.current_stream(cuda_device).cuda_stream
        g = torch.Generator(device=cuda_device).manual_seed(5)
        for step, T in enumerate(steps):
            x = torch.randn((T, H), generator=g, device=cuda_device).to(torch.bfloat16)
            logits = torch.randn((T, E), generator=g, device=cuda_device)
            ids = torch.empty((T, k), dtype=torch.int32, device=cuda_device)
            wts = torch.empty((T, k), dtype=torch.float32, device=cuda_device)
            assert lib.xcb_moe_topk(logits.data_ptr(), T, E, k, ids.data_ptr(), wts.data_ptr(), stream) == _lib.XCB_OK
            assert lib.xcb_ep_p2p_dispatch(x.data_ptr(), logits.data_ptr(), T, Tm, H, E, k, G, 0, peers.data_ptr(),
                                           status.data_ptr(), 0, stream) == _lib.XCB_OK
            parts = torch.randn((T, H), generator=g, device=cuda_device).to(torch.bfloat16)
            out = torch.empty((T, H), dtype=torch.bfloat16, device=cuda_device)
            torch.cuda.synchronize(cuda_device)
            xr = buf[xo:xo + T * H * 2].view(torch.bfloat16).view(T, H).clone()
            ids_r = buf[io:io + T * k * 4].view(torch.int32).view(T, k).clone()
            w_r = buf[wo:wo + T * k * 4].view(torch.float32).view(T, k).clone()
            assert lib.xcb_ep_p2p_combine(parts.data_ptr(), T, Tm, H, k, G, 0, peers.data_ptr(), out.data_ptr(),
                                          status.data_ptr(), 0, stream) == _lib.XCB_OK
            torch.cuda.synchronize(cuda_device)
            assert int(status.item()) == 0, f"step {step}: device status {int(status.item())}"
            assert torch.equal(xr, x)
            assert torch.equal(ids_r, ids)
            assert torch.equal(w_r, wts)
            assert torch.equal(out, parts)
    finally:
        torch.cuda.synchronize(cuda_device)
        lib.xcb_p2p_free(own)


def test_p2p_exchange_set_up_on_one_rank(tmp_path, cuda_device):
    """The exchange object on a one-rank process group: its set-up (mapping agreement and exact-value self-test)
    passes, two steps round-trip, and close releases it (in a child process, so no process group is left here)."""
    from tests._ep_gpu_worker import p2p_single_rank_worker

    mp.spawn(p2p_single_rank_worker, args=(_free_port(), str(tmp_path)), nprocs=1, join=True)
    with open(os.path.join(tmp_path, "p2p_single.txt")) as f:
        msg = f.read()
    assert msg == "", msg


def test_p2p_wait_for_a_silent_peer_runs_out(cuda_device):
    """Rank 0 of a two-rank exchange whose rank 1 never sends (its 'buffer' is a second local allocation that no
    kernel writes to rank 0): the dispatch's wait for rank 1's rows and the combine's wait for its partial sums give
    up after the 1 ms limit, the status word reports XCB_STATUS_DEVICE_TIMEOUT, both kernels return (the stream
    synchronises) and the combine's output is NaN rows, not a plausible result.  Nothing but the wait's own limit is
    exercised: every access stays inside the two allocations."""
    import ctypes

    from xcalibur_b200 import _lib

    lib = _lib.load()
    G, Tm, H, E, k, T = 2, 4, 256, 64, 4, 3
    nbytes = lib.xcb_ep_p2p_bytes(G, Tm, H, k)
    bufs = []
    try:
        for _ in range(G):
            p = ctypes.c_void_p()
            assert lib.xcb_p2p_alloc(nbytes, ctypes.byref(p), (ctypes.c_ubyte * 64)()) == _lib.XCB_OK
            bufs.append(p)
        peers = torch.tensor([b.value for b in bufs], dtype=torch.int64, device=cuda_device)
        status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
        stream = torch.cuda.current_stream(cuda_device).cuda_stream
        x = torch.randn((T, H), device=cuda_device).to(torch.bfloat16)
        logits = torch.randn((T, E), device=cuda_device)
        limit_ns = 1_000_000
        assert lib.xcb_ep_p2p_dispatch(x.data_ptr(), logits.data_ptr(), T, Tm, H, E, k, G, 0, peers.data_ptr(),
                                       status.data_ptr(), limit_ns, stream) == _lib.XCB_OK
        torch.cuda.synchronize(cuda_device)
        assert int(status.item()) & _lib.XCB_STATUS_DEVICE_TIMEOUT
        status.zero_()
        parts = torch.ones((G * T, H), dtype=torch.bfloat16, device=cuda_device)
        out = torch.zeros((T, H), dtype=torch.bfloat16, device=cuda_device)
        assert lib.xcb_ep_p2p_combine(parts.data_ptr(), T, Tm, H, k, G, 0, peers.data_ptr(), out.data_ptr(),
                                      status.data_ptr(), limit_ns, stream) == _lib.XCB_OK
        torch.cuda.synchronize(cuda_device)
        assert int(status.item()) & _lib.XCB_STATUS_DEVICE_TIMEOUT
        assert torch.isnan(out.float()).all()
    finally:
        torch.cuda.synchronize(cuda_device)
        for b in bufs:
            lib.xcb_p2p_free(b)
