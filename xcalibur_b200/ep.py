"""Expert-parallel NVFP4 MoE layer: the experts are sharded contiguously over the ranks of a torch.distributed
group, every rank routes its own tokens, and tokens travel to the ranks that hold their experts and back.

The reference models an expert-parallel rank only as a local expert range whose non-local routes it masks
(kernels/moe_w4a16_h200/moe_w4a16.py:105-110, :513-520); the cross-rank sum was its harness's job.  Here one call
is, on every rank (``forward``):

1. ``xcb_moe_topk``: top-k over all experts for this rank's tokens;
2. ``xcb_ep_plan``: a token goes once to every rank holding one of its experts (in token order); the per-rank
   counts are exchanged (all-to-all of G integers, read on the host for the split sizes);
3. ``xcb_ep_gather`` + all-to-all: the token rows with their full top-k ids and weights;
4. the local layer (``PreparedMoE`` with ``expert_offset``) on the received rows: routes to experts this rank does
   not hold contribute nothing, so each received row yields this rank's partial sum;
5. all-to-all back in the same order, then ``xcb_ep_combine``: out[t] = bf16(sum of its partials in rank order).

Small batches (at most DENSE_MAX_TOKENS tokens per rank, decode) skip the plan: every token goes to every rank with
equal splits and no host synchronisation.  On GPUs that exchange runs over NVLink peer memory (``P2PExchange``:
one buffer per rank mapped into every peer through CUDA IPC; a dispatch kernel writes this rank's rows into every
peer and waits for theirs, a combine kernel returns the partial sums and adds them in rank order), so a decode step
needs no collective library call; elsewhere it is three all-to-alls.

The transport is ``torch.distributed.all_to_all_single`` (NCCL over NVLink on GPUs).  The per-rank steps run in the
C-ABI library; ``_ops`` exists so that tests can substitute a CPU model of those steps and check the exchange
protocol itself with the gloo backend (world size 2) on machines without GPUs.
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from ._lib import check
from .moe import PreparedMoE


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def p2p_layout(G: int, T_max: int, H: int, k: int):
    """Byte offsets (x, ids, wts, part, flag) and total size of a peer-exchange buffer (mirrors the C library's)."""
    o = 0

    def take(b):
        nonlocal o
        at = o
        o = (o + b + 255) // 256 * 256
        return at

    x = take(G * T_max * H * 2)
    ids = take(G * T_max * k * 4)
    wts = take(G * T_max * k * 4)
    part = take(G * T_max * H * 2)
    flag = take((2 * G + 4) * 4)
    return x, ids, wts, part, flag, o


class _DeviceBytes:
    """A device allocation seen by torch as a uint8 tensor (zero-copy, through the CUDA array interface)."""

    def __init__(self, ptr: int, nbytes: int):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False), "version": 3,
                                         "strides": None}


class P2PUnavailable(RuntimeError):
    """The peer exchange could not be set up on every rank (mapping or self-test failed); all ranks agree on it."""


class P2PExchange:
    """This rank's end of the NVLink peer exchange of the dense (small-batch) expert-parallel step.

    Collective: every rank of ``group`` constructs it (the buffers' IPC handles are exchanged, every rank's mapping
    and a one-step self-test are checked by all ranks together) and must ``close`` it before the process group is
    destroyed.  Raises ``P2PUnavailable`` on every rank if any rank failed, after releasing what it set up."""

    def __init__(self, lib, group, rank: int, world: int, T_max: int, H: int, E: int, k: int, device,
                 timeout_ns: int = 0):
        self.lib, self.group, self.rank, self.world = lib, group, rank, world
        self.timeout_ns = int(timeout_ns)  # bound of every device wait of the exchange (0: the library's 2 s)
        self.T_max, self.H, self.E, self.k, self.device = T_max, H, E, k, device
        self.offs = p2p_layout(world, T_max, H, k)
        nbytes = int(lib.xcb_ep_p2p_bytes(world, T_max, H, k))
        if nbytes != self.offs[5]:
            raise RuntimeError("peer-exchange layout mismatch between the library and its Python mirror")
        own = ctypes.c_void_p()
        handle = (ctypes.c_ubyte * 64)()
        check(lib.xcb_p2p_alloc(nbytes, ctypes.byref(own), handle), "xcb_p2p_alloc")
        self.own = own.value
        handles = [None] * world
        dist.all_gather_object(handles, bytes(handle), group=group)
        self.opened = []
        ptrs = []
        why = ""
        try:
            for d in range(world):
                if d == rank:
                    ptrs.append(self.own)
                    continue
                h = (ctypes.c_ubyte * 64).from_buffer_copy(handles[d])
                p = ctypes.c_void_p()
                check(lib.xcb_p2p_open(h, ctypes.byref(p)), "xcb_p2p_open")
                self.opened.append(p.value)
                ptrs.append(p.value)
        except Exception as e:  # noqa: BLE001 - reported to every rank below
            why = f"rank {rank}: {e}"
        if not self._agree(not why):
            self.close()
            raise P2PUnavailable(why or "another rank could not map the peer buffers")
        self.peers = torch.tensor(ptrs, dtype=torch.int64, device=device)
        self.buf = torch.as_tensor(_DeviceBytes(self.own, nbytes), device=device)
        self.status = torch.zeros(1, dtype=torch.int32, device=device)
        why = self._self_test()
        if not self._agree(not why):
            self.close()
            raise P2PUnavailable(why or "the self-test failed on another rank")

    def _agree(self, ok: bool) -> bool:
        """True on every rank if ``ok`` is true on every rank."""
        flag = torch.tensor([1 if ok else 0], dtype=torch.int32, device=self.device)
        dist.all_reduce(flag, op=dist.ReduceOp.MIN, group=self.group)
        return bool(flag.item())

    def _logits_of(self, d: int, T: int):
        """Deterministic router logits of rank d for the self-test (identical on every rank)."""
        g = torch.Generator(device=self.device).manual_seed(7919 + d)
        return torch.randn((T, self.E), generator=g, device=self.device, dtype=torch.float32)

    def _self_test(self) -> str:
        """One exchange step with known values: every rank sends rows tagged with its rank and token and the top-k
        of logits every rank can rebuild (checked against the library's own router), and returns partial rows whose
        bf16 sum over the ranks is exact.  Returns "" or what went wrong."""
        G, H, k, r, dev = self.world, self.H, self.k, self.rank, self.device
        T = 2
        try:
            t = torch.arange(T, device=dev, dtype=torch.float32)[:, None]
            x = (r + 0.25 * t).expand(T, H).to(torch.bfloat16).contiguous()
            self.dispatch(x, self._logits_of(r, T))
            xr, ids_r, w_r = self.recv(T)
            d = torch.arange(G, device=dev, dtype=torch.float32).repeat_interleave(T)[:, None]
            tt = torch.arange(T, device=dev, dtype=torch.float32).repeat(G)[:, None]
            want_x = (d + 0.25 * tt).expand(G * T, H).to(torch.bfloat16)
            want_ids = torch.empty((G * T, k), dtype=torch.int32, device=dev)
            want_w = torch.empty((G * T, k), dtype=torch.float32, device=dev)
            stream = torch.cuda.current_stream(dev).cuda_stream
            for src in range(G):
                lg = self._logits_of(src, T)
                check(self.lib.xcb_moe_topk(lg.data_ptr(), T, self.E, k, want_ids[src * T:].data_ptr(),
                                            want_w[src * T:].data_ptr(), stream), "xcb_moe_topk")
            # the partial row every rank returns for rank d's token t is (d + 1) + 2 t, so rank r's combined row t
            # is G (r + 1 + 2 t): exact in bf16 for up to 32 ranks, and wrong if a row reached the wrong rank
            parts = ((d + 1) + 2 * tt).expand(G * T, H).to(torch.bfloat16).contiguous()
            out = self.combine(parts, T)
            want_out = (G * (r + 1 + 2 * t)).expand(T, H).to(torch.bfloat16)
            torch.cuda.synchronize(dev)
            st = self.device_status()
            if st:
                return f"rank {r}: device status {st}"
            if not (torch.equal(xr, want_x) and torch.equal(ids_r, want_ids) and torch.equal(w_r, want_w)):
                return f"rank {r}: received rows differ from what the peers sent"
            if not torch.equal(out, want_out):
                return f"rank {r}: combined partial sums differ"
            return ""
        except Exception as e:  # noqa: BLE001 - reported to every rank
            return f"rank {r}: {e}"

    def recv(self, T: int):
        """This step's received rows, in place: x bf16 [G T, H], top-k ids int32 [G T, k], weights fp32 [G T, k]."""
        G, H, k = self.world, self.H, self.k
        xo, io, wo = self.offs[0], self.offs[1], self.offs[2]
        xr = self.buf[xo:xo + G * T * H * 2].view(torch.bfloat16).view(G * T, H)
        ids = self.buf[io:io + G * T * k * 4].view(torch.int32).view(G * T, k)
        wts = self.buf[wo:wo + G * T * k * 4].view(torch.float32).view(G * T, k)
        return xr, ids, wts

    def dispatch(self, x, logits):
        """Route this rank's tokens (router logits fp32 [T, E]) and send their rows and top-k rows to every rank."""
        T = x.shape[0]
        logits = logits.to(torch.float32).contiguous()
        stream = torch.cuda.current_stream(self.device).cuda_stream
        check(self.lib.xcb_ep_p2p_dispatch(x.data_ptr(), logits.data_ptr(), T, self.T_max, self.H, self.E, self.k,
                                           self.world, self.rank, self.peers.data_ptr(), self.status.data_ptr(),
                                           self.timeout_ns, stream), "xcb_ep_p2p_dispatch")

    def combine(self, parts, T: int):
        out = torch.empty((T, self.H), dtype=torch.bfloat16, device=self.device)
        stream = torch.cuda.current_stream(self.device).cuda_stream
        check(self.lib.xcb_ep_p2p_combine(parts.data_ptr(), T, self.T_max, self.H, self.k, self.world, self.rank,
                                          self.peers.data_ptr(), out.data_ptr(), self.status.data_ptr(),
                                          self.timeout_ns, stream), "xcb_ep_p2p_combine")
        return out

    def device_status(self) -> int:
        """Status bits of the exchange kernels (XCB_STATUS_DEVICE_TIMEOUT), read and cleared (synchronises)."""
        v = int(self.status.item())
        self.status.zero_()
        return v

    def close(self):
        """Unmap the peers' buffers, wait for every rank to do the same, free this rank's (collective)."""
        if self.own is None:
            return
        torch.cuda.synchronize(self.device)
        for p in self.opened:
            self.lib.xcb_p2p_close(p)
        self.opened = []
        dist.barrier(group=self.group)
        self.buf = None
        self.lib.xcb_p2p_free(self.own)
        self.own = None


class CudaEpOps:
    """The per-rank steps of an expert-parallel call, on the GPU through the C-ABI."""

    def __init__(self, layer: PreparedMoE):
        self.layer = layer
        self.lib = layer.lib
        self.device = layer.device
        self.status = torch.zeros(1, dtype=torch.int32, device=self.device)

    def topk(self, logits: torch.Tensor, k: int):
        T, E = logits.shape
        ids = torch.empty((T, k), dtype=torch.int32, device=self.device)
        wts = torch.empty((T, k), dtype=torch.float32, device=self.device)
        logits = logits.to(torch.float32).contiguous()
        check(self.lib.xcb_moe_topk(logits.data_ptr(), T, E, k, ids.data_ptr(), wts.data_ptr(), _stream(self.device)),
              "xcb_moe_topk")
        return ids, wts

    def plan(self, ids: torch.Tensor, experts_per_rank: int, world: int):
        T, k = ids.shape
        counts = torch.empty(world, dtype=torch.int32, device=self.device)
        send_tok = torch.empty((world, max(T, 1)), dtype=torch.int32, device=self.device)
        send_pos = torch.empty((max(T, 1), world), dtype=torch.int32, device=self.device)
        check(self.lib.xcb_ep_plan(ids.data_ptr(), T, k, experts_per_rank, world, counts.data_ptr(),
                                   send_tok.data_ptr(), send_pos.data_ptr(), self.status.data_ptr(),
                                   _stream(self.device)), "xcb_ep_plan")
        return counts, send_tok, send_pos

    def gather(self, x, ids, wts, counts, send_tok, total: int):
        T, H = x.shape
        k = ids.shape[1]
        xs = torch.empty((total, H), dtype=torch.bfloat16, device=self.device)
        ids_s = torch.empty((total, k), dtype=torch.int32, device=self.device)
        w_s = torch.empty((total, k), dtype=torch.float32, device=self.device)
        if total:
            check(self.lib.xcb_ep_gather(x.data_ptr(), ids.data_ptr(), wts.data_ptr(), T, H, k, counts.numel(),
                                         counts.data_ptr(), send_tok.data_ptr(), xs.data_ptr(), ids_s.data_ptr(),
                                         w_s.data_ptr(), _stream(self.device)), "xcb_ep_gather")
        return xs, ids_s, w_s

    def local(self, xr, ids_r, w_r, post_norm: bool):
        if xr.shape[0] == 0:
            return torch.empty((0, xr.shape[1]), dtype=torch.bfloat16, device=self.device)
        return self.layer.forward(xr, None, topk_ids=ids_r, topk_weights=w_r, post_norm=post_norm)

    def combine(self, parts, counts, send_pos, T: int):
        H = parts.shape[1]
        out = torch.empty((T, H), dtype=torch.bfloat16, device=self.device)
        if T:
            check(self.lib.xcb_ep_combine(parts.data_ptr() if parts.numel() else None, counts.data_ptr(),
                                          send_pos.data_ptr(), T, H, counts.numel(), out.data_ptr(),
                                          _stream(self.device)), "xcb_ep_combine")
        return out

    def device_status(self) -> int:
        """Status bits of the plan kernel (XCB_STATUS_BAD_EXPERT), read and cleared."""
        v = int(self.status.item())
        self.status.zero_()
        return v


class ExpertParallelMoE:
    """This rank's share of an expert-parallel MoE layer.

    ``w13 .. w2_gs`` hold experts ``[rank * E / G, (rank + 1) * E / G)`` of ``total_experts = E`` (reference layout,
    ``moe_w4a16.py:72-79``); every rank of ``group`` calls ``forward`` with its own tokens, collectively."""

    def __init__(self, w13, w13_sf, w13_gs, w2, w2_sf, w2_gs, *, total_experts: int, group=None,
                 post_norm_w=None, top_k: int = 8, p2p: bool = True, _ops=None):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if total_experts % self.world:
            raise ValueError(f"{total_experts} experts do not split evenly over {self.world} ranks")
        self.E = int(total_experts)
        self.epr = self.E // self.world
        if w13.shape[0] != self.epr:
            raise ValueError(f"rank {self.rank} must hold {self.epr} experts, got {w13.shape[0]}")
        self.post_norm = post_norm_w is not None
        if _ops is None:
            layer = PreparedMoE(w13, w13_sf, w13_gs, w2, w2_sf, w2_gs, post_norm_w, total_experts=self.E,
                                expert_offset=self.rank * self.epr)
            _ops = CudaEpOps(layer)
        self.ops = _ops
        self.last = {}
        # dense steps over NVLink peer memory (GPU ranks only; collective construction)
        self.p2p = None
        self.p2p_error = None
        if p2p and isinstance(_ops, CudaEpOps) and self.world > 1:
            H = w13.shape[2] * 2
            try:
                self.p2p = P2PExchange(_ops.lib, group, self.rank, self.world, self.DENSE_MAX_TOKENS, H, self.E,
                                       top_k, _ops.device)
            except P2PUnavailable as e:  # every rank lands here together: the dense step falls back to NCCL
                self.p2p_error = str(e)

    def device_status(self) -> int:
        """Device status bits of this rank's last steps (exchange waits that timed out, expert ids out of range,
        the local layer's own bits), read and cleared.  It synchronises, so a serving loop calls it between steps
        rather than inside one; a step whose exchange timed out has NaN output rows in any case."""
        bits = 0
        if self.p2p is not None:
            bits |= self.p2p.device_status()
        if isinstance(self.ops, CudaEpOps):
            bits |= self.ops.device_status() | self.ops.layer.check_device_status()
        return bits

    def close(self):
        """Release the peer exchange (collective; before the process group is destroyed)."""
        if self.p2p is not None:
            self.p2p.close()
            self.p2p = None

    def _a2a(self, send: torch.Tensor, send_splits, recv_splits, trailing) -> torch.Tensor:
        out = torch.empty((sum(recv_splits), *trailing), dtype=send.dtype, device=send.device)
        dist.all_to_all_single(out, send, output_split_sizes=list(recv_splits), input_split_sizes=list(send_splits),
                               group=self.group)
        return out

    # Up to this many tokens per rank a call is exchanged densely: every token goes to every rank (fixed, equal
    # splits), so no counts exchange and no host synchronisation are needed; a rank holding none of a token's experts
    # returns a zero partial for it.  Small batches (decode) are latency-bound, and this halves their collectives.
    DENSE_MAX_TOKENS = 32

    def _dense_p2p(self, x, router_logits, top_k):
        """Three kernels per step: route + send (peer dispatch), the local layer on the received rows in place,
        return + sum (peer combine)."""
        T = x.shape[0]
        ex = self.p2p
        ex.dispatch(x, router_logits)
        xr, ids_r, w_r = ex.recv(T)
        parts = self.ops.local(xr, ids_r, w_r, self.post_norm)
        out = ex.combine(parts, T)
        mine = slice(self.rank * T, (self.rank + 1) * T)
        # copies: the receive buffer is rewritten by the peers' next dispatch
        self.last.update({"ids": ids_r[mine].clone(), "wts": w_r[mine].clone(), "send": [T] * self.world,
                          "recv": [T] * self.world, "recv_ids": ids_r.clone()})
        return out

    def _dense(self, x, ids, wts, top_k):
        T, H = x.shape
        G = self.world
        key = (T, G, x.device)
        if self.last.get("dense_key") != key:  # combine tables of the fixed layout: token t's row from rank d is d*T+t
            dev = x.device
            self._dense_counts = torch.full((G,), T, dtype=torch.int32, device=dev)
            self._dense_pos = torch.arange(T, dtype=torch.int32, device=dev)[:, None].expand(T, G).contiguous()
            self.last["dense_key"] = key
        xs = x.unsqueeze(0).expand(G, T, H).reshape(G * T, H).contiguous()
        meta = torch.cat([ids, wts.view(torch.int32)], dim=1).unsqueeze(0).expand(G, T, 2 * top_k)
        meta = meta.reshape(G * T, 2 * top_k).contiguous()
        xr = torch.empty_like(xs)
        mr = torch.empty_like(meta)
        dist.all_to_all_single(xr, xs, group=self.group)
        dist.all_to_all_single(mr, meta, group=self.group)
        ids_r = mr[:, :top_k].contiguous()
        w_r = mr[:, top_k:].contiguous().view(torch.float32)
        parts = self.ops.local(xr, ids_r, w_r, self.post_norm)
        back = torch.empty_like(parts)
        dist.all_to_all_single(back, parts, group=self.group)
        out = self.ops.combine(back, self._dense_counts, self._dense_pos, T)
        self.last.update({"ids": ids, "wts": wts, "send": [T] * G, "recv": [T] * G, "recv_ids": ids_r})
        return out

    def forward(self, hidden_states: torch.Tensor, router_logits: torch.Tensor, top_k: int) -> torch.Tensor:
        """One layer over this rank's tokens (collective over the group): bf16 [T, H] out.  Every rank must pass
        the same token count when it is at most DENSE_MAX_TOKENS (the dense exchange uses equal splits)."""
        x = hidden_states.contiguous()
        T, H = x.shape
        if tuple(router_logits.shape) != (T, self.E):
            raise ValueError(f"router_logits must be [T, {self.E}]")
        if 0 < T <= self.DENSE_MAX_TOKENS and self.p2p is not None and top_k == self.p2p.k:
            return self._dense_p2p(x, router_logits, top_k)
        ids, wts = self.ops.topk(router_logits, top_k)
        if 0 < T <= self.DENSE_MAX_TOKENS:
            return self._dense(x, ids, wts, top_k)
        counts, send_tok, send_pos = self.ops.plan(ids, self.epr, self.world)
        recv_counts = torch.empty_like(counts)
        dist.all_to_all_single(recv_counts, counts, group=self.group)
        send_splits = [int(v) for v in counts.cpu().tolist()]
        recv_splits = [int(v) for v in recv_counts.cpu().tolist()]
        xs, ids_s, w_s = self.ops.gather(x, ids, wts, counts, send_tok, sum(send_splits))
        xr = self._a2a(xs, send_splits, recv_splits, (H,))
        ids_r = self._a2a(ids_s, send_splits, recv_splits, (top_k,))
        w_r = self._a2a(w_s, send_splits, recv_splits, (top_k,))
        parts = self.ops.local(xr, ids_r, w_r, self.post_norm)
        back = self._a2a(parts, recv_splits, send_splits, (H,))
        out = self.ops.combine(back, counts, send_pos, T)
        self.last.update({"ids": ids, "wts": wts, "send": send_splits, "recv": recv_splits, "recv_ids": ids_r})
        return out

    __call__ = forward
