"""Host side of the B200 NVFP4 MoE layer: the reference operator's Python interface over the C-ABI library.

Two interfaces, both thin: PyTorch only supplies device memory and the current stream, every byte of work runs
in the sm_100a kernels of ``libxcb_moe.so``.

* ``moe_w4a16(hidden_states, router_logits, w13, w13_sf, w13_gs, w2, w2_sf, w2_gs, top_k, *, post_norm_w=None,
  topk_ids=None, topk_weights=None)`` — the north_star signature.  Weights are in the reference layout
  (kernels/moe_w4a16_h200/moe_w4a16.py:72-79); they are repacked on the GPU on first use and the packed copy is
  cached while the source tensors stay alive and unmodified.
* ``prepare(weights)`` / ``kernel_fn(data, state)`` — the reference's own operator contract
  (moe_w4a16.py:3292 and :3370, wrapped at :3938 / :3956): precomputed ``topk_ids``/``topk_weights``, local
  experts ``[local_start, local_start + local_count)`` and the per-route post-norm with ``post_norm_w``.

Errors follow the reference's: shape/argument problems raise before anything is launched (the reference uses
``assert`` and ``TORCH_CHECK``, moe_w4a16.py:3300-3302, :2822-2848); device-side status (a NaN block scale, an
expert id out of range, a bounded wait that expired) is read by ``check_device_status``.
"""
from __future__ import annotations

import ctypes
import weakref
from typing import Optional, TypedDict

import torch

from . import _lib, packer
from ._lib import XcbMoeArgs, XcbMoeShape, XcbMoeWeights, check


class Weights(TypedDict):
    """Reference weight dict (moe_w4a16.py:72-79)."""
    w13: torch.Tensor
    w13_sf: torch.Tensor
    w13_gs: torch.Tensor
    w2: torch.Tensor
    w2_sf: torch.Tensor
    w2_gs: torch.Tensor
    post_norm_w: torch.Tensor


class Config(TypedDict):
    """Reference per-call config (moe_w4a16.py:82-90)."""
    bs: int
    d_hidden: int
    d_expert: int
    n_experts: int
    local_start: int
    local_count: int
    top_k: int
    sharding: str


class Inputs(TypedDict):
    """Reference per-call inputs (moe_w4a16.py:93-97)."""
    hidden_states: torch.Tensor
    topk_ids: torch.Tensor
    topk_weights: torch.Tensor
    config: Config


def _u8(t: torch.Tensor) -> torch.Tensor:
    if t.dtype == torch.uint8:
        return t.contiguous()
    if t.dtype == torch.float8_e4m3fn:
        return t.contiguous().view(torch.uint8)
    raise TypeError(f"expected uint8 or float8_e4m3fn, got {t.dtype}")


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


_TABLES: dict = {}


def _xor_tables(device: torch.device) -> torch.Tensor:
    key = (device.type, device.index)
    if key not in _TABLES:
        words = packer.xor_table_words()
        _TABLES[key] = torch.tensor([w - (1 << 32) if w >= 1 << 31 else w for w in words], dtype=torch.int32,
                                    device=device)
    return _TABLES[key]


_PATH_FLAGS = {"auto": 0, "decode": _lib.XCB_FLAG_DECODE_PATH, "prefill": _lib.XCB_FLAG_PREFILL_PATH}


class PreparedMoE:
    """Packed weights of one MoE layer on one GPU plus its per-stream workspaces.

    ``w13`` uint8 [E, 2I, H/2], ``w13_sf`` E4M3 [E, 2I, H/16], ``w13_gs`` fp32 [E], ``w2`` uint8 [E, H, I/2],
    ``w2_sf`` [E, H, I/16], ``w2_gs`` [E] hold ``num_experts = E`` experts that are global experts
    ``expert_offset .. expert_offset + E - 1`` of a router with ``total_experts`` outputs.
    """

    def __init__(self, w13, w13_sf, w13_gs, w2, w2_sf, w2_gs, post_norm_w=None, *, total_experts=None,
                 expert_offset: int = 0):
        if not w13.is_cuda:
            raise ValueError("weights must be CUDA tensors (there is no CPU path)")
        self.device = w13.device
        self.lib = _lib.load()
        E, R2, H2 = w13.shape
        H, I = 2 * H2, R2 // 2
        if tuple(w2.shape) != (E, H, I // 2) or tuple(w13_sf.shape) != (E, 2 * I, H // 16) or \
                tuple(w2_sf.shape) != (E, H, I // 16) or w13_gs.numel() != E or w2_gs.numel() != E:
            raise ValueError("inconsistent NVFP4 weight shapes")
        self.E, self.H, self.I = E, H, I
        self.total_experts = int(total_experts if total_experts is not None else E + expert_offset)
        self.expert_offset = int(expert_offset)
        self.shape = XcbMoeShape(E, self.total_experts, self.expert_offset, H, I)
        check(self.lib.xcb_moe_check_shape(ctypes.byref(self.shape)), "xcb_moe_check_shape")
        with torch.cuda.device(self.device):
            nA = self.lib.xcb_moe_packed_bytes(ctypes.byref(self.shape), 0)
            nB = self.lib.xcb_moe_packed_bytes(ctypes.byref(self.shape), 1)
            self.gate_up = torch.empty(nA, dtype=torch.uint8, device=self.device)
            self.down = torch.empty(nB, dtype=torch.uint8, device=self.device)
            status = torch.zeros(1, dtype=torch.int32, device=self.device)
            check(self.lib.xcb_moe_pack_weights(ctypes.byref(self.shape), _u8(w13).data_ptr(), _u8(w13_sf).data_ptr(),
                                                _u8(w2).data_ptr(), _u8(w2_sf).data_ptr(),
                                                _xor_tables(self.device).data_ptr(), self.gate_up.data_ptr(),
                                                self.down.data_ptr(), status.data_ptr(),
                                                _stream_handle(self.device)), "xcb_moe_pack_weights")
            if int(status.item()) & _lib.XCB_STATUS_NAN_SCALE:
                raise ValueError("NaN E4M3 block scale in the weights")
        self.gate_up_gs = w13_gs.to(device=self.device, dtype=torch.float32).contiguous()
        self.down_gs = w2_gs.to(device=self.device, dtype=torch.float32).contiguous()
        self.post_norm_w = None
        if post_norm_w is not None:
            if post_norm_w.dtype != torch.bfloat16 or post_norm_w.numel() != H:
                raise ValueError("post_norm_w must be bf16 [hidden]")
            self.post_norm_w = post_norm_w.to(self.device).contiguous()
        self._weights = XcbMoeWeights(self.shape, self.gate_up.data_ptr(), self.down.data_ptr(),
                                      self.gate_up_gs.data_ptr(), self.down_gs.data_ptr(), _ptr(self.post_norm_w))
        self._ws: dict = {}

    # -------------------------------------------------------------------------------------- workspace
    def workspace(self, tokens: int, top_k: int) -> torch.Tensor:
        """The workspace of the current stream, grown (never shrunk) to hold ``tokens`` x ``top_k`` routes."""
        stream = _stream_handle(self.device)
        key = (stream, top_k)
        ws = self._ws.get(key)
        if ws is None or ws[1] < tokens:
            cap = max(tokens, 1 if ws is None else ws[1] * 2)
            nbytes = self.lib.xcb_moe_workspace_bytes(ctypes.byref(self.shape), cap, top_k)
            if nbytes == 0:
                raise ValueError("invalid workspace request")
            buf = torch.empty(nbytes, dtype=torch.uint8, device=self.device)
            check(self.lib.xcb_moe_workspace_init(buf.data_ptr(), nbytes, cap, top_k, stream), "xcb_moe_workspace_init")
            ws = (buf, cap)
            self._ws[key] = ws
        return ws[0]

    # -------------------------------------------------------------------------------------- forward
    def build_call(self, hidden_states: torch.Tensor, router_logits: Optional[torch.Tensor] = None, top_k: int = 8,
                   *, topk_ids: Optional[torch.Tensor] = None, topk_weights: Optional[torch.Tensor] = None,
                   post_norm: bool = False, out: Optional[torch.Tensor] = None, return_routing: bool = False,
                   path: str = "auto", wait_limit_us: int = 0, pdl: bool = False, deterministic: bool = False):
        """Validate one call and bind its buffers; returns a ``LayerCall`` whose ``launch()`` enqueues it.

        ``path``: "auto" (the library picks by batch size), "decode" (the streaming decode kernel) or "prefill"
        (the tensor-core grouped GEMMs).  ``wait_limit_us``: bound of every device-side wait of the call (0: the
        library's 2 s); a wait that runs out sets XCB_STATUS_DEVICE_TIMEOUT (``check_device_status``).  ``pdl``:
        launch a single-launch decode call with programmatic dependent launch (it may start while the previous
        kernel of the stream finishes, and waits for it before reading anything).  ``deterministic``: on the
        prefill path, combine the routes in a separate fixed-order pass (bit-reproducible output) instead of inside
        the down projection."""
        x = hidden_states
        if x.dtype != torch.bfloat16 or x.dim() != 2 or x.shape[1] != self.H:
            raise ValueError(f"hidden_states must be bf16 [T, {self.H}]")
        if x.device != self.device:
            raise ValueError("hidden_states is on another device than the weights")
        x = x.contiguous()
        T = x.shape[0]
        logits = ids = wts = None
        if router_logits is not None:
            if topk_ids is not None or topk_weights is not None:
                raise ValueError("give router_logits or topk_ids/topk_weights, not both")
            logits = router_logits.to(torch.float32).contiguous()
            if tuple(logits.shape) != (T, self.total_experts):
                raise ValueError(f"router_logits must be [T, {self.total_experts}]")
        else:
            if topk_ids is None or topk_weights is None:
                raise ValueError("router_logits or topk_ids + topk_weights are required")
            ids = topk_ids.to(torch.int32).contiguous()
            wts = topk_weights.to(torch.float32).contiguous()
            top_k = ids.shape[1]
            if tuple(ids.shape) != (T, top_k) or tuple(wts.shape) != (T, top_k):
                raise ValueError("topk_ids / topk_weights must be [T, top_k]")
        if post_norm and self.post_norm_w is None:
            raise ValueError("post_norm needs post_norm_w")
        if out is None:
            out = torch.empty((T, self.H), dtype=torch.bfloat16, device=self.device)
        ids_out = wts_out = None
        if return_routing:
            ids_out = torch.empty((T, top_k), dtype=torch.int32, device=self.device)
            wts_out = torch.empty((T, top_k), dtype=torch.float32, device=self.device)
        ws = self.workspace(T, top_k) if T else None
        if path not in _PATH_FLAGS:
            raise ValueError(f"path must be one of {sorted(_PATH_FLAGS)}")
        flags = (_lib.XCB_FLAG_POST_NORM if post_norm else 0) | _PATH_FLAGS[path] | (_lib.XCB_FLAG_PDL if pdl else 0)
        flags |= _lib.XCB_FLAG_DETERMINISTIC if deterministic else 0
        if wait_limit_us < 0:
            raise ValueError("wait_limit_us must be >= 0")
        args = XcbMoeArgs(T, top_k, flags, int(wait_limit_us), x.data_ptr(), _ptr(logits),
                          _ptr(ids), _ptr(wts), out.data_ptr(), _ptr(ids_out), _ptr(wts_out))
        return LayerCall(self, args, ws, (x, logits, ids, wts), out, ids_out, wts_out, return_routing)

    def forward(self, hidden_states: torch.Tensor, router_logits: Optional[torch.Tensor] = None, top_k: int = 8, *,
                topk_ids: Optional[torch.Tensor] = None, topk_weights: Optional[torch.Tensor] = None,
                post_norm: bool = False, out: Optional[torch.Tensor] = None, return_routing: bool = False,
                path: str = "auto", wait_limit_us: int = 0, pdl: bool = False, deterministic: bool = False):
        call = self.build_call(hidden_states, router_logits, top_k, topk_ids=topk_ids, topk_weights=topk_weights,
                               post_norm=post_norm, out=out, return_routing=return_routing, path=path,
                               wait_limit_us=wait_limit_us, pdl=pdl, deterministic=deterministic)
        call.launch()
        return call.result()

    __call__ = forward

    def check_device_status(self) -> int:
        """Synchronise the current stream and return (and clear) the device status bits of its workspaces."""
        bits = 0
        stream = _stream_handle(self.device)
        for (s, _k), (buf, _cap) in self._ws.items():
            if s != stream:
                continue
            v = ctypes.c_int32(0)
            rc = self.lib.xcb_moe_read_status(buf.data_ptr(), ctypes.byref(v), stream)
            if rc not in (_lib.XCB_OK, _lib.XCB_ERR_DEVICE):
                check(rc, "xcb_moe_read_status")
            bits |= v.value
        return bits


class LayerCall:
    """One bound layer call: its C-ABI argument block, workspace and the tensors it keeps alive."""

    def __init__(self, layer, args, ws, keep, out, ids_out, wts_out, return_routing):
        self.layer, self.args, self.ws, self._keep = layer, args, ws, keep
        self.out, self.ids_out, self.wts_out, self.return_routing = out, ids_out, wts_out, return_routing

    def launch(self, part: str = "forward"):
        """Enqueue on the current stream: ``forward`` (both halves), ``route`` or ``experts``."""
        if self.args.tokens == 0:
            return
        fn = {"forward": self.layer.lib.xcb_moe_forward, "route": self.layer.lib.xcb_moe_route,
              "experts": self.layer.lib.xcb_moe_experts}[part]
        check(fn(ctypes.byref(self.layer._weights), ctypes.byref(self.args), self.ws.data_ptr(), self.ws.numel(),
                 _stream_handle(self.layer.device)), f"xcb_moe_{part}")

    def result(self):
        return (self.out, self.ids_out, self.wts_out) if self.return_routing else self.out


# ------------------------------------------------------------------------------------------ north_star entry
_CACHE: "weakref.WeakKeyDictionary[torch.Tensor, tuple]" = weakref.WeakKeyDictionary()


def _prepared_for(w13, w13_sf, w13_gs, w2, w2_sf, w2_gs, post_norm_w) -> PreparedMoE:
    key_src = (w13, w13_sf, w13_gs, w2, w2_sf, w2_gs, post_norm_w)
    sig = tuple((t.data_ptr(), t._version, tuple(t.shape)) if t is not None else None for t in key_src)
    hit = _CACHE.get(w13)
    if hit is not None and hit[0] == sig:
        return hit[1]
    layer = PreparedMoE(w13, w13_sf, w13_gs, w2, w2_sf, w2_gs, post_norm_w)
    _CACHE[w13] = (sig, layer)
    return layer


def moe_w4a16(hidden_states, router_logits, w13, w13_sf, w13_gs, w2, w2_sf, w2_gs, top_k, *, post_norm_w=None,
              topk_ids=None, topk_weights=None, return_routing=False):
    """One NVFP4-weight / BF16-activation MoE layer on the GPU.

    ``y = sum_k w_k * down_e(SiLU(gate_e x) * up_e x)``; with ``post_norm_w`` each route is scaled by
    ``(1 + post_norm_w)`` and normalised by its RMS (the reference contract).  Routing comes from
    ``router_logits`` (softmax -> top-k -> renormalise, ties to the lower expert id) or, when ``router_logits``
    is None, from ``topk_ids`` / ``topk_weights``.
    """
    layer = _prepared_for(w13, w13_sf, w13_gs, w2, w2_sf, w2_gs, post_norm_w)
    return layer.forward(hidden_states, router_logits, top_k, topk_ids=topk_ids, topk_weights=topk_weights,
                         post_norm=post_norm_w is not None, return_routing=return_routing)


# ------------------------------------------------------------------------------------------ reference contract
def prepare(weights: Weights, *, local_start: int = 0, local_count: Optional[int] = None,
            n_experts: Optional[int] = None) -> dict:
    """Reference ``prepare`` (moe_w4a16.py:3292): pack the local experts once, on their GPU.

    ``weights`` holds every expert (as in the reference, which indexes ``weights["w13"][e]`` for its local
    range); experts ``[local_start, local_start + local_count)`` are packed."""
    E = weights["w13"].shape[0]
    n_experts = E if n_experts is None else n_experts
    local_count = E - local_start if local_count is None else local_count
    sl = slice(local_start, local_start + local_count)
    layer = PreparedMoE(weights["w13"][sl], weights["w13_sf"][sl], weights["w13_gs"][sl], weights["w2"][sl],
                        weights["w2_sf"][sl], weights["w2_gs"][sl], weights.get("post_norm_w"),
                        total_experts=n_experts, expert_offset=local_start)
    return {"layer": layer, "lo": local_start, "cnt": local_count}


def kernel_fn(data: Inputs, state: dict) -> torch.Tensor:
    """Reference ``kernel_fn`` (moe_w4a16.py:3370): precomputed routing, post-norm, fresh output, no host sync."""
    cfg = data["config"]
    if cfg["local_start"] != state["lo"] or cfg["local_count"] != state["cnt"]:
        raise ValueError("config local range differs from the prepared state")
    layer: PreparedMoE = state["layer"]
    return layer.forward(data["hidden_states"], None, topk_ids=data["topk_ids"], topk_weights=data["topk_weights"],
                         post_norm=layer.post_norm_w is not None)
