"""Test helpers: run the CPU oracle on the experts a batch actually uses, compare with tolerances."""
from __future__ import annotations

import numpy as np
import torch

from oracle import moe_ref

RTOL = 1e-2   # north_star tolerance for the layer output against the fp32 reference
ATOL = 1e-2


def to_np(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().numpy()


def bf16_bits(t: torch.Tensor) -> np.ndarray:
    return to_np(t.contiguous().view(torch.int16)).view(np.uint16)


def oracle_layer(x, weights: dict, ids: np.ndarray, wts: np.ndarray, *, post_norm_w=None, local_start=0,
                 local_count=None):
    """Oracle output for GPU-resident inputs, copying only the experts the routes use to the host."""
    E = weights["w13"].shape[0]
    local_count = E if local_count is None else local_count
    flat = ids.reshape(-1)
    used = np.unique(flat[(flat >= local_start) & (flat < local_start + local_count)])
    remap = np.full(max(int(flat.max()) + 1, local_start + local_count) + 1, -1, np.int64)
    remap[used] = np.arange(used.size)
    cid = np.where((flat >= local_start) & (flat < local_start + local_count), remap[np.clip(flat, 0, None)], -1)
    cid = cid.reshape(ids.shape).astype(np.int32)
    sel = torch.as_tensor(used, device=weights["w13"].device, dtype=torch.long)

    def pick(name):
        t = weights[name]
        if t.dtype == torch.float8_e4m3fn:
            t = t.view(torch.uint8)
        return to_np(t.index_select(0, sel)) if used.size else to_np(t[:0])

    if used.size == 0:
        T, H = x.shape
        return np.zeros((T, H), np.uint16)
    pn = None if post_norm_w is None else bf16_bits(post_norm_w)
    out, _ = moe_ref.moe_forward(bf16_bits(x), cid, wts, pick("w13"), pick("w13_sf"), pick("w13_gs"), pick("w2"),
                                 pick("w2_sf"), pick("w2_gs"), post_norm_w_bits=pn, local_start=0)
    return out


def assert_close_bf16(got: torch.Tensor, want_bits: np.ndarray, rtol=RTOL, atol=ATOL, frobenius=5e-3):
    g = moe_ref.bf16_bits_to_f32(bf16_bits(got))
    w = moe_ref.bf16_bits_to_f32(want_bits)
    assert np.isfinite(g).all()
    err = np.abs(g - w)
    bad = err > atol + rtol * np.abs(w)
    assert not bad.any(), f"{bad.sum()} of {bad.size} outside tolerance; max err {err.max():.3g}"
    # and in aggregate the kernel tracks the reference much more tightly than the per-element bound
    rel = np.linalg.norm(g - w) / max(np.linalg.norm(w), 1e-30)
    if frobenius is not None:
        assert rel < frobenius, f"relative Frobenius error {rel:.3g}"
    return rel
