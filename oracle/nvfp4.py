"""NVFP4 number formats, quantiser and dequantiser on the CPU (numpy) — test infrastructure.

Formats (reference: kernels/moe_w4a16_h200/moe_w4a16.py:72-79 for the tensor layouts, :3151-3158 for the nibble
order, :3313-3318 for the e4m3 decode through torch.float8_e4m3fn; docs/cute_sassy.md:311-321 for E2M1):

* weight codes: uint8 ``[..., R, K/2]``, two E2M1 codes per byte, the LOW nibble holds the even k;
* block scales: E4M3 (fn) bytes ``[..., R, K/16]``, one per 16 consecutive k of a row;
* global scale: fp32, one per expert per tensor; ``W[r, k] = e2m1(code) * e4m3(sf[r, k // 16]) * gs``.

The quantiser follows the recipe the benchmark configurations state: ``gs = amax(W) / (6 * 448)``,
``sf = e4m3_rne(amax(block) / 6 / gs)``, ``code = e2m1_rne(w / (e4m3(sf) * gs))`` with saturation at +-6.
Every step is float32 arithmetic in a fixed order so the GPU quantiser can match it bit for bit.
"""
from __future__ import annotations

import numpy as np

E2M1_VALUES = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0, -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0],
                       dtype=np.float32)


def _e4m3_table() -> np.ndarray:
    vals = np.zeros(256, dtype=np.float32)
    for b in range(256):
        s = -1.0 if b & 0x80 else 1.0
        e = (b >> 3) & 0xF
        m = b & 7
        if e == 0xF and m == 7:
            vals[b] = np.nan
        elif e == 0:
            vals[b] = s * (m / 8.0) * 2.0 ** -6
        else:
            vals[b] = s * (1.0 + m / 8.0) * 2.0 ** (e - 7)
    return vals


E4M3_VALUES = _e4m3_table()


def e4m3_decode(b: np.ndarray) -> np.ndarray:
    return E4M3_VALUES[np.asarray(b, dtype=np.uint8)]


def e4m3_encode_rne(x: np.ndarray) -> np.ndarray:
    """float32 -> E4M3 byte, round to nearest even, saturating at +-448 (x must be finite)."""
    x = np.asarray(x, dtype=np.float32)
    sign = np.signbit(x)
    a = np.abs(x).astype(np.float64)
    pos = E4M3_VALUES[:0x7F].astype(np.float64)      # 0x00..0x7E, ascending, finite
    idx = np.searchsorted(pos, a, side="left")
    idx = np.clip(idx, 0, 0x7E)
    lo = np.clip(idx - 1, 0, 0x7E)
    # candidates lo (<= a) and idx (>= a); pick nearer, ties to even code (mantissa lsb 0)
    exact = pos[idx] == a
    dlo = a - pos[lo]
    dhi = pos[idx] - a
    pick_hi = (dhi < dlo) | ((dhi == dlo) & ((idx & 1) == 0))
    code = np.where(exact, idx, np.where(pick_hi, idx, lo))
    code = np.where(a >= 448.0, 0x7E, code)
    code = code.astype(np.uint8)
    return np.where(sign & (code != 0), code | 0x80, code).astype(np.uint8)


def e2m1_encode_rne(x: np.ndarray) -> np.ndarray:
    """float32 -> E2M1 nibble (0..15), round to nearest even on the grid, saturating at +-6."""
    x = np.asarray(x, dtype=np.float32)
    a = np.abs(x)
    # thresholds between grid points; a tie goes to the code with an even mantissa bit
    grid = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], dtype=np.float32)
    mids = (grid[:-1] + grid[1:]) / 2  # 0.25 0.75 1.25 1.75 2.5 3.5 5
    code = np.searchsorted(mids, a, side="left").astype(np.uint8)  # a <= mid -> lower code
    tie = np.isin(a, mids)
    # at a tie searchsorted(left) picked the lower code; move up when the lower code has an odd mantissa
    code = np.where(tie & ((code & 1) == 1), code + 1, code).astype(np.uint8)
    code = np.minimum(code, 7).astype(np.uint8)
    neg = np.signbit(x) & (code != 0)        # a value that rounds to zero is stored as +0
    return np.where(neg, code | 8, code).astype(np.uint8)


def quantize(w: np.ndarray):
    """Quantise fp32 ``[E, R, K]`` weights per the NVFP4 recipe.

    Returns (codes uint8 [E,R,K/2], sf uint8 [E,R,K/16] (E4M3 bytes), gs float32 [E]).
    """
    w = np.asarray(w, dtype=np.float32)
    E, R, K = w.shape
    assert K % 16 == 0
    amax = np.max(np.abs(w.reshape(E, -1)), axis=1).astype(np.float32)
    gs = (amax / np.float32(6.0 * 448.0)).astype(np.float32)
    gs = np.where(gs == 0, np.float32(1.0), gs).astype(np.float32)
    blocks = w.reshape(E, R, K // 16, 16)
    bamax = np.max(np.abs(blocks), axis=3).astype(np.float32)
    sf = e4m3_encode_rne((bamax / np.float32(6.0)) / gs[:, None, None])
    scale = (e4m3_decode(sf) * gs[:, None, None]).astype(np.float32)
    safe = np.where(scale == 0, np.float32(1.0), scale)
    q = blocks / safe[..., None]
    q = np.where(scale[..., None] == 0, np.float32(0.0), q).astype(np.float32)
    nib = e2m1_encode_rne(q).reshape(E, R, K)
    codes = (nib[..., 0::2] | (nib[..., 1::2] << 4)).astype(np.uint8)
    return codes, sf, gs


def unpack_codes(codes: np.ndarray) -> np.ndarray:
    """uint8 [..., K/2] -> nibbles [..., K] (low nibble = even k)."""
    c = np.asarray(codes, dtype=np.uint8)
    out = np.empty(c.shape[:-1] + (c.shape[-1] * 2,), dtype=np.uint8)
    out[..., 0::2] = c & 0xF
    out[..., 1::2] = c >> 4
    return out


def dequantize(codes: np.ndarray, sf: np.ndarray, gs) -> np.ndarray:
    """One tensor (or a stack): codes [..., R, K/2], sf [..., R, K/16], gs scalar or [...] -> fp32 [..., R, K].

    W = e2m1(code) * e4m3(sf) * gs, each product rounded to float32 (exact for e2m1*e4m3).
    """
    nib = unpack_codes(codes)
    vals = E2M1_VALUES[nib]
    s = e4m3_decode(sf)
    K = vals.shape[-1]
    s_full = np.repeat(s, 16, axis=-1)[..., :K]
    gs = np.asarray(gs, dtype=np.float32)
    if gs.ndim:
        gs = gs.reshape(gs.shape + (1, 1))
    return ((vals * s_full).astype(np.float32) * gs).astype(np.float32)


def dequantize_fast(codes: np.ndarray, sf: np.ndarray, gs) -> np.ndarray:
    """``dequantize`` for one tensor with torch's host threads (the same table lookups and float32 products, so the
    result is identical element for element; used for the full-size expert shapes)."""
    import torch

    c = torch.from_numpy(np.ascontiguousarray(codes, dtype=np.uint8))
    nib = torch.stack((c & 0xF, c >> 4), dim=-1).reshape(*c.shape[:-1], -1).long()
    vals = torch.from_numpy(E2M1_VALUES)[nib]
    s = torch.from_numpy(E4M3_VALUES)[torch.from_numpy(np.ascontiguousarray(sf, dtype=np.uint8)).long()]
    s = s.repeat_interleave(16, dim=-1)[..., :vals.shape[-1]]
    return ((vals * s) * torch.tensor(np.float32(gs))).numpy()
