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
        assert int(np.load(os.path.join(tmp_path, f"nccl_status_{r}.npy"))[0]) == 0
        got, want = np.load(os.path.join(tmp_path, f"nccl_{r}.npy"))
        assert_close_bf16(torch.from_numpy(got.view(np.int16)).view(torch.bfloat16), want)
