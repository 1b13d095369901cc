"""Expert-parallel exchange protocol under gloo, world size 2 (no GPU): every rank's output equals the
single-process oracle layer on its tokens."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from oracle import moe_ref
from tests._ep_model import gloo_leave_worker, gloo_worker
from tests._util import ATOL, RTOL


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("T", [1, 7, 40])  # 40 > DENSE_MAX_TOKENS: the planned, uneven exchange
def test_ep_two_ranks_match_single_process(tmp_path, T):
    world, E, H, I, k = 2, 8, 256, 256, 4
    mp.spawn(gloo_worker, args=(world, _free_port(), E, H, I, T, k, 123, str(tmp_path)), nprocs=world, join=True)
    for r in range(world):
        got, want = np.load(os.path.join(tmp_path, f"ep_{r}.npy"))
        g, w = moe_ref.bf16_bits_to_f32(got), moe_ref.bf16_bits_to_f32(want)
        assert np.all(np.abs(g - w) <= ATOL + RTOL * np.abs(w)), f"rank {r}: max err {np.abs(g - w).max():.3g}"
    # the split sizes agree across ranks: what rank a sends to rank b is what b receives from a
    s0, s1 = (np.load(os.path.join(tmp_path, f"ep_splits_{r}.npy")) for r in range(world))
    assert s0[1] == s1[2] and s1[0] == s0[3]


@pytest.mark.parametrize("T", [3, 40])  # dense and planned exchanges
def test_rank_that_leaves_between_steps_ends_the_next_step_with_an_error(tmp_path, T):
    """Failure detection on the host: when a rank leaves after a step, the other rank's next step fails with an
    error (bounded by the group's timeout) rather than hanging."""
    world, E, H, I, k = 2, 8, 256, 256, 4
    mp.spawn(gloo_leave_worker, args=(world, _free_port(), E, H, I, T, k, 321, str(tmp_path)), nprocs=world,
             join=True)
    with open(os.path.join(tmp_path, "leave_0.txt")) as f:
        msg = f.read()
    assert msg.startswith("error after"), msg
    assert float(msg.split()[2]) < 30.0, msg
