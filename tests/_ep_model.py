"""CPU model of the per-rank steps of an expert-parallel call (test infrastructure).

``xcalibur_b200.ep.ExpertParallelMoE`` runs topk / plan / gather / local layer / combine in the C-ABI library and
moves rows with ``torch.distributed.all_to_all_single``.  This module restates those per-rank steps on the CPU with
numpy and the oracle, so the exchange protocol itself (count exchange, uneven splits, return order, rank-ordered
combine) can run under the gloo backend on a machine without GPUs."""
from __future__ import annotations

import os

import numpy as np
import torch
import torch.distributed as dist

from oracle import moe_ref


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def _from_bits(b: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(b).view(np.int16)).view(torch.bfloat16)


class CpuEpOps:
    """Same inputs and outputs as xcalibur_b200.ep.CudaEpOps, on CPU tensors."""

    def __init__(self, weights_local, lo: int):
        self.w = weights_local        # numpy reference-layout arrays of this rank's experts
        self.lo = lo

    def topk(self, logits, k):
        ids, wts = moe_ref.route_topk(logits.numpy().astype(np.float32), k)
        return torch.from_numpy(ids.astype(np.int32)), torch.from_numpy(wts.astype(np.float32))

    def plan(self, ids, epr, world):
        ids = ids.numpy()
        T = ids.shape[0]
        send_pos = np.full((max(T, 1), world), -1, np.int32)
        send_tok = np.zeros((world, max(T, 1)), np.int32)
        counts = np.zeros(world, np.int32)
        for t in range(T):
            for d in sorted(set((ids[t] // epr).tolist())):
                send_pos[t, d] = counts[d]
                send_tok[d, counts[d]] = t
                counts[d] += 1
        return torch.from_numpy(counts), torch.from_numpy(send_tok), torch.from_numpy(send_pos)

    def gather(self, x, ids, wts, counts, send_tok, total):
        rows = [int(send_tok[d, i]) for d in range(counts.numel()) for i in range(int(counts[d]))]
        idx = torch.tensor(rows, dtype=torch.long)
        return x[idx].contiguous(), ids[idx].contiguous(), wts[idx].contiguous()

    def local(self, xr, ids_r, w_r, post_norm):
        if xr.shape[0] == 0:
            return torch.empty((0, xr.shape[1]), dtype=torch.bfloat16)
        out, _ = moe_ref.moe_forward(_bits(xr), ids_r.numpy(), w_r.numpy(), *self.w, local_start=self.lo)
        return _from_bits(out)

    def combine(self, parts, counts, send_pos, T):
        base = np.concatenate([[0], np.cumsum(counts.numpy())[:-1]]).astype(np.int64)
        pf = moe_ref.bf16_bits_to_f32(_bits(parts))
        acc = np.zeros((T, parts.shape[1]), np.float32)
        sp = send_pos.numpy()
        for d in range(counts.numel()):
            ok = sp[:T, d] >= 0
            acc[ok] += pf[base[d] + sp[:T, d][ok]]
        return _from_bits(moe_ref.f32_to_bf16_bits(acc))


def gloo_worker(rank, world, port, E, H, I, T, k, seed, result_dir):
    """One rank: its shard of a seeded layer, its own tokens, the EP forward under gloo; saves its output and the
    single-process oracle output for the same tokens."""
    from xcalibur_b200.ep import ExpertParallelMoE

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(seed)
        w = moe_ref.make_weights(rng, E, H, I)                  # every rank draws the whole layer, keeps its share
        epr = E // world
        sl = slice(rank * epr, (rank + 1) * epr)
        wl = [a[sl] for a in w]
        rng_t = np.random.default_rng(seed + 1 + rank)
        x, logits = moe_ref.make_inputs(rng_t, T, H, E, bias_std=0.5)
        layer = ExpertParallelMoE(*[torch.from_numpy(np.ascontiguousarray(a)) for a in wl], total_experts=E,
                                  _ops=CpuEpOps(wl, rank * epr))
        out = layer.forward(_from_bits(x), torch.from_numpy(logits), k)
        want, _, _ = moe_ref.moe_layer(x, logits, *w, k)
        np.save(os.path.join(result_dir, f"ep_{rank}.npy"), np.stack([_bits(out), want]))
        np.save(os.path.join(result_dir, f"ep_splits_{rank}.npy"), np.array(layer.last["send"] + layer.last["recv"]))
    finally:
        dist.destroy_process_group()


def gloo_leave_worker(rank, world, port, E, H, I, T, k, seed, result_dir):
    """Rank 1 runs one step and then leaves (returns between steps, with no collective in flight); rank 0 runs a
    second step, whose first collective must end with an error once its peer is gone (the process group's short
    timeout bounds it) instead of waiting for good.  Rank 0 writes what it saw."""
    import datetime
    import time

    from xcalibur_b200.ep import ExpertParallelMoE

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
    rng = np.random.default_rng(seed)
    w = moe_ref.make_weights(rng, E, H, I)
    epr = E // world
    wl = [a[rank * epr:(rank + 1) * epr] for a in w]
    layer = ExpertParallelMoE(*[torch.from_numpy(np.ascontiguousarray(a)) for a in wl], total_experts=E,
                              _ops=CpuEpOps(wl, rank * epr))
    x, logits = moe_ref.make_inputs(np.random.default_rng(seed + 1 + rank), T, H, E)
    layer.forward(_from_bits(x), torch.from_numpy(logits), k)      # step 1 on both ranks
    if rank == 1:
        os._exit(0)                                              # leaves between steps, without a goodbye
    t0 = time.monotonic()
    try:
        layer.forward(_from_bits(x), torch.from_numpy(logits), k)  # step 2: the peer is gone
        msg = "step 2 completed without its peer"
    except Exception as e:  # noqa: BLE001 - the failure is the expected outcome
        msg = f"error after {time.monotonic() - t0:.1f} s: {type(e).__name__}"
    with open(os.path.join(result_dir, "leave_0.txt"), "w") as f:
        f.write(msg)
    # the group cannot be torn down collectively any more; end the process without running its destructor
    os._exit(0)
