"""Worker of the two-GPU expert-parallel test (test infrastructure): one rank per GPU over NCCL."""
from __future__ import annotations

import datetime
import os

import numpy as np
import torch
import torch.distributed as dist


def nccl_worker(rank, world, port, E, H, I, T, k, seed, result_dir, p2p=True, calls=1):
    from xcalibur_b200 import PreparedMoE, synth
    from xcalibur_b200.ep import ExpertParallelMoE

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    ep = None
    try:
        w = synth.make_weights(E, H, I, seed=seed, device=dev)           # the whole layer, same on every rank
        epr = E // world
        shard = {n: t[rank * epr:(rank + 1) * epr].contiguous() for n, t in w.items()}
        ep = ExpertParallelMoE(*shard.values(), total_experts=E, top_k=k, p2p=p2p)
        full = PreparedMoE(*w.values())
        got, want = [], []
        for c in range(calls):  # consecutive calls: the peer exchange's per-step flags must advance in step
            x, logits = synth.make_inputs(T, H, E, seed=seed + 1 + rank + 100 * c, device=dev, bias_std=0.5)
            got.append(ep.forward(x, logits, k))
            want.append(full.forward(x, logits, k))
        torch.cuda.synchronize()
        st = ep.ops.device_status() | ep.ops.layer.check_device_status() | full.check_device_status()
        if ep.p2p is not None:
            st |= ep.p2p.device_status()
        np.save(os.path.join(result_dir, f"nccl_{rank}.npy"),
                np.stack([torch.cat(got).view(torch.int16).cpu().numpy().view(np.uint16),
                          torch.cat(want).view(torch.int16).cpu().numpy().view(np.uint16)]))
        np.save(os.path.join(result_dir, f"nccl_status_{rank}.npy"), np.array([st]))
        with open(os.path.join(result_dir, f"p2p_{rank}.txt"), "w") as f:  # whether the peer exchange was used
            f.write("" if (not p2p or ep.p2p is not None) else (ep.p2p_error or "not set up"))
    finally:
        if ep is not None:
            ep.close()
        dist.destroy_process_group()


def p2p_single_rank_worker(rank, port, result_dir):
    """One rank: the peer exchange's set-up (mapping agreement and self-test), two exchange steps and close."""
    from xcalibur_b200 import _lib
    from xcalibur_b200.ep import P2PExchange

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    dist.init_process_group("nccl", rank=0, world_size=1, timeout=datetime.timedelta(seconds=60))
    msg = ""
    try:
        lib = _lib.load()
        ex = P2PExchange(lib, None, 0, 1, 32, 1024, 64, 8, dev)
        stream = torch.cuda.current_stream(dev).cuda_stream
        for T in (1, 5):
            x = torch.randn((T, 1024), device=dev).to(torch.bfloat16)
            logits = torch.randn((T, 64), device=dev)
            ids = torch.empty((T, 8), dtype=torch.int32, device=dev)
            wts = torch.empty((T, 8), dtype=torch.float32, device=dev)
            lib.xcb_moe_topk(logits.data_ptr(), T, 64, 8, ids.data_ptr(), wts.data_ptr(), stream)
            ex.dispatch(x, logits)
            xr, ids_r, w_r = ex.recv(T)
            out = ex.combine(xr.clone(), T)
            torch.cuda.synchronize()
            if not (torch.equal(xr, x) and torch.equal(ids_r, ids) and torch.equal(w_r, wts) and torch.equal(out, x)):
                msg += f"T={T}: round trip differs; "
        if ex.device_status():
            msg += "device status set; "
        ex.close()
    except Exception as e:  # noqa: BLE001 - reported to the test
        msg += repr(e)
    finally:
        dist.destroy_process_group()
    with open(os.path.join(result_dir, "p2p_single.txt"), "w") as f:
        f.write(msg)
