"""CPU restatement of the NVFP4 W4A16 MoE layer — test infrastructure (see oracle/__init__.py for its status).

Layer (north_star form, no post-norm), for token t with routes s = 0..k-1, expert e = ids[t, s], weight w:

    g, u = x_t W_gate[e]^T, x_t W_up[e]^T          (fp32; W dequantised from NVFP4)
    h    = bf16(SiLU(g) * u)                          (kernels/moe_w4a16_h200/moe_w4a16.py:616-627 rounds here)
    y    = h W_down[e]^T                              (fp32, moe_w4a16.py:628-657)
    out  = bf16(sum_s w_s * y_s)

Reference-contract form (``post_norm_w`` given; moe_w4a16.py:8-33, :2715-2745, README.md:10-19):

    y_s  <- y_s * (1 + post_norm_w)                   (post_norm_w is bf16, 1 + w formed in fp32)
    out  = bf16(sum_s w_s * rsqrt(mean_n(y_s^2) + 1e-8) * y_s)

Routes whose expert is not local (outside [local_start, local_start + local_count)) contribute nothing
(moe_w4a16.py:513-520, :2669).  ``w13`` stacks gate rows 0..I-1 above up rows I..2I-1 (moe_w4a16.py:3297-3305).

Router (absent from the reference, which takes precomputed ids; defined here for the north_star signature):
rank experts by raw logit, descending, ties to the lower expert index; the route weights are the softmax over
the k selected logits, which equals softmax -> top-k -> renormalise.
"""
from __future__ import annotations

import numpy as np

from . import nvfp4


# ----------------------------------------------------------------------------------------------- bf16 helpers
def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    b = np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16
    return b.view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even float32 -> bf16 bit pattern (finite inputs)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = ((u >> 16) & 1) + 0x7FFF
    return ((u + r) >> 16).astype(np.uint16)


def bf16_round(x: np.ndarray) -> np.ndarray:
    return bf16_bits_to_f32(f32_to_bf16_bits(x))


# ----------------------------------------------------------------------------------------------- router
def route_topk(logits: np.ndarray, k: int):
    """logits float32 [T, E] -> (ids int32 [T, k], weights float32 [T, k])."""
    lg = np.asarray(logits, dtype=np.float32)
    T, E = lg.shape
    order = np.argsort(-lg, axis=1, kind="stable")[:, :k]          # stable: ties keep the lower index first
    sel = np.take_along_axis(lg, order, axis=1)
    m = sel[:, :1]
    ex = np.exp((sel - m).astype(np.float32)).astype(np.float32)
    den = np.zeros((T, 1), dtype=np.float32)
    for s in range(k):                                               # fixed summation order
        den[:, 0] += ex[:, s]
    return order.astype(np.int32), (ex / den).astype(np.float32)


def permute(ids: np.ndarray, local_start: int, local_count: int):
    """Stable expert-major permutation of the flat routes f = t*k + s (moe_w4a16.py:491-611 semantics).

    Returns (order int32 [n_local]: flat route at each permuted position, pos int32 [T*k]: permuted position of
    each flat route or -1 if its expert is not local, counts int32 [local_count], offsets int32 [local_count+1]).
    """
    flat = np.asarray(ids, dtype=np.int64).reshape(-1)
    loc = flat - local_start
    is_local = (loc >= 0) & (loc < local_count)
    f_idx = np.nonzero(is_local)[0]
    order = f_idx[np.argsort(loc[f_idx], kind="stable")]
    pos = np.full(flat.shape[0], -1, dtype=np.int32)
    pos[order] = np.arange(order.shape[0], dtype=np.int32)
    counts = np.bincount(loc[is_local], minlength=local_count).astype(np.int32)
    offsets = np.zeros(local_count + 1, dtype=np.int32)
    offsets[1:] = np.cumsum(counts)
    return order.astype(np.int32), pos, counts, offsets


# ----------------------------------------------------------------------------------------------- layer
def moe_forward(x_bf16_bits, ids, weights, w13, w13_sf, w13_gs, w2, w2_sf, w2_gs, *, post_norm_w_bits=None,
                local_start: int = 0, threads: int | None = None):
    """The layer on the CPU.  All tensors are numpy arrays in the reference layouts; x and post_norm_w are bf16
    bit patterns (uint16).  Returns the output as bf16 bits [T, H] and the fp32 pre-rounding sum."""
    import torch  # fp32 matmuls on the host cores

    if threads:
        torch.set_num_threads(threads)
    x = bf16_bits_to_f32(x_bf16_bits)
    T, H = x.shape
    k = ids.shape[1]
    E_loc = w13.shape[0]
    inter = w13.shape[1] // 2
    order, pos, counts, offsets = permute(ids, local_start, E_loc)
    tok = order // k
    wt = np.asarray(weights, dtype=np.float32).reshape(-1)
    y_all = np.zeros((order.shape[0], H), dtype=np.float32)
    gamma = None if post_norm_w_bits is None else (np.float32(1.0) + bf16_bits_to_f32(post_norm_w_bits))
    for e in range(E_loc):
        p0, p1 = offsets[e], offsets[e + 1]
        if p0 == p1:
            continue
        xe = torch.from_numpy(np.ascontiguousarray(x[tok[p0:p1]]))
        wa = torch.from_numpy(nvfp4.dequantize_fast(w13[e], w13_sf[e], w13_gs[e]))
        gu = (xe @ wa.T).numpy()
        g, u = gu[:, :inter], gu[:, inter:]
        h = bf16_round((g / (np.float32(1.0) + np.exp(-g))) * u)
        wb = torch.from_numpy(nvfp4.dequantize_fast(w2[e], w2_sf[e], w2_gs[e]))
        y = (torch.from_numpy(h) @ wb.T).numpy()
        if gamma is not None:
            y = (y * gamma[None, :]).astype(np.float32)
        y_all[p0:p1] = y
    acc = np.zeros((T, H), dtype=np.float32)
    for s in range(k):                                               # fixed order over the routes of a token
        p = pos.reshape(T, k)[:, s]
        ok = p >= 0
        ys = y_all[p[ok]]
        r = wt.reshape(T, k)[ok, s][:, None]
        if gamma is not None:
            ss = np.mean(ys.astype(np.float32) ** 2, axis=1, dtype=np.float32)
            r = (r * (np.float32(1.0) / np.sqrt(ss + np.float32(1e-8)))[:, None]).astype(np.float32)
        acc[ok] += (r * ys).astype(np.float32)
    return f32_to_bf16_bits(acc), acc


def moe_layer(x_bf16_bits, router_logits, w13, w13_sf, w13_gs, w2, w2_sf, w2_gs, top_k, **kw):
    """north_star signature: route from logits, then the layer.  Returns (out bits, ids, weights)."""
    ids, wts = route_topk(router_logits, top_k)
    out, _ = moe_forward(x_bf16_bits, ids, wts, w13, w13_sf, w13_gs, w2, w2_sf, w2_gs, **kw)
    return out, ids, wts


# ----------------------------------------------------------------------------------------------- inputs
def make_weights(rng: np.random.Generator, E: int, H: int, I: int, std: float = 0.02):
    """Seeded NVFP4 weights per the benchmark recipe: gate_up [E, 2I, H] and down [E, H, I] from N(0, std)."""
    w13 = rng.standard_normal((E, 2 * I, H), dtype=np.float32) * np.float32(std)
    w2 = rng.standard_normal((E, H, I), dtype=np.float32) * np.float32(std)
    c13, s13, g13 = nvfp4.quantize(w13)
    c2, s2, g2 = nvfp4.quantize(w2)
    return c13, s13, g13, c2, s2, g2


def make_inputs(rng: np.random.Generator, T: int, H: int, E: int, bias_std: float = 0.0):
    """BF16 N(0,1) activations and fp32 N(0,1) router logits (plus an optional per-expert N(0, bias_std) bias)."""
    x = f32_to_bf16_bits(rng.standard_normal((T, H), dtype=np.float32))
    logits = rng.standard_normal((T, E), dtype=np.float32)
    if bias_std:
        logits = (logits + rng.standard_normal((1, E), dtype=np.float32) * np.float32(bias_std)).astype(np.float32)
    return x, logits
