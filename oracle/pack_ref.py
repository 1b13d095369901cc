"""CPU model of the decode-path weight layout — test infrastructure.

Builds, with numpy, the exact bytes the GPU packer (``xcb_moe_pack_weights``) must produce, from the layout and
bit map that ``xcalibur_b200.packer`` defines, and decodes packed bytes back to weight values the way the
kernel's registers see them.  The reference analogue is the host repack of
kernels/moe_w4a16_h200/moe_w4a16.py:3168-3190 plus its GF(2) word transform at :3903-3933.
"""
from __future__ import annotations

import numpy as np

from xcalibur_b200 import packer

from . import nvfp4


def packed_row_order(R: int, gate_up: bool) -> np.ndarray:
    """Original row index of each packed row (gate/up interleaved in 8-row groups for gate_up)."""
    if not gate_up:
        return np.arange(R)
    inter = R // 2
    rb = np.arange(inter // 8)[:, None]
    g = np.arange(8)[None, :]
    return np.stack((8 * rb + g, inter + 8 * rb + g), axis=1).reshape(-1)


def _scale_tables():
    code = np.zeros(256, dtype=np.uint8)
    fold = np.zeros(256, dtype=np.uint8)          # 0 none, 1 zero, 2 negative
    for b in range(256):
        if (b & 0x7F) == 0x7F:
            code[b] = 0xFF
            continue
        c, f = packer.scale_code(b)
        code[b] = c
        fold[b] = {None: 0, "zero": 1, "neg": 2}[f]
    return code, fold


SCALE_CODE, SCALE_FOLD = _scale_tables()


def canonical(codes: np.ndarray, sf: np.ndarray):
    """Fold zero and negative scales into the codes; return (codes', scale codes) for one [R, K/2] matrix."""
    R, K2 = codes.shape
    fold = SCALE_FOLD[sf]                                        # [R, K/16]
    fold_b = np.repeat(fold, 8, axis=1)[:, :K2]                  # per code byte (8 bytes per 16-k block)
    c = codes.copy()
    c = np.where(fold_b == 1, np.uint8(0), c)
    c = np.where(fold_b == 2, c ^ np.uint8(0x88), c).astype(np.uint8)
    return c, SCALE_CODE[sf]


def _apply_T(words: np.ndarray) -> np.ndarray:
    _, tabs = packer.packing_transform()
    tabs = np.asarray(tabs, dtype=np.uint32)
    w = words.astype(np.uint32)
    return (tabs[0][w & 255] ^ tabs[1][(w >> 8) & 255] ^ tabs[2][(w >> 16) & 255] ^ tabs[3][w >> 24]).astype(np.uint32)


def join_units(code_bytes: np.ndarray, scale_bytes: np.ndarray) -> np.ndarray:
    """[nb, nS*512] codes + [nb, nS*64] scales -> [nb, 9K] units: per group of gs slices, its codes then its scales."""
    nb = code_bytes.shape[0]
    nS = code_bytes.shape[1] // 512
    gs = packer.group_slices(64 * nS)
    parts = []
    for g0 in range(0, nS, gs):
        ns = gs
        parts.append(code_bytes[:, g0 * 512:(g0 + ns) * 512])
        parts.append(scale_bytes[:, g0 * 64:(g0 + ns) * 64])
    return np.concatenate(parts, axis=1).reshape(nb, -1)


def split_units(units: np.ndarray, K: int):
    """Inverse of join_units: [nb, 9K] -> ([nb, nS*512] codes, [nb, nS*64] scales)."""
    nS = K // 64
    gs = packer.group_slices(K)
    cs, ss = [], []
    off = 0
    for g0 in range(0, nS, gs):
        ns = gs
        cs.append(units[:, off:off + ns * 512])
        ss.append(units[:, off + ns * 512:off + ns * 576])
        off += ns * 576
    return np.concatenate(cs, axis=1), np.concatenate(ss, axis=1)


def pack_matrix(codes: np.ndarray, sf: np.ndarray, gate_up: bool) -> np.ndarray:
    """One expert matrix (codes [R, K/2], sf [R, K/16]) -> packed bytes [R/16 units, 9K]."""
    R, K2 = codes.shape
    K = 2 * K2
    rows = packed_row_order(R, gate_up)
    c, sc = canonical(codes[rows], sf[rows])
    nb, nS = R // 16, K // 64
    cb = c.reshape(nb, 2, 8, K2)                                 # [rb, h, g, byte]
    # byte index for (S, t, j, hi): 32S + 8t + 2j + hi
    S = np.arange(nS)[:, None, None, None]
    t = np.arange(4)[None, :, None, None]
    j = np.arange(4)[None, None, :, None]
    hi = np.arange(2)[None, None, None, :]
    bidx = (32 * S + 8 * t + 2 * j + hi)                          # [S, t, j, hi]
    r0 = cb[:, 0][:, :, bidx]                                    # [rb, g, S, t, j, hi]  rows g
    r8 = cb[:, 1][:, :, bidx]                                    # rows g + 8
    word = (r0[..., 0].astype(np.uint32) | (r8[..., 0].astype(np.uint32) << 8)
            | (r0[..., 1].astype(np.uint32) << 16) | (r8[..., 1].astype(np.uint32) << 24))  # [rb, g, S, t, j]
    word = _apply_T(word)
    word = word.transpose(0, 2, 1, 3, 4)                         # [rb, S, g, t, j] -> lane = 4g + t
    code_bytes = np.ascontiguousarray(word).view(np.uint8).reshape(nb, nS * 512)
    sb = sc.reshape(nb, 2, 8, K // 16)                           # [rb, h, g, block]
    S4 = np.arange(nS // 4)[:, None, None, None, None]
    g = np.arange(8)[None, :, None, None, None]
    tt = np.arange(4)[None, None, :, None, None]
    s4 = np.arange(4)[None, None, None, :, None]
    h = np.arange(2)[None, None, None, None, :]
    blk = 4 * (4 * S4 + s4) + tt                                 # scale block of (slice, t)
    scl = sb[:, h, g, blk]                                        # [rb, S4, g, t, s4, h]
    scale_bytes = np.ascontiguousarray(scl).reshape(nb, K)
    return join_units(code_bytes, scale_bytes)


def pack_tensor(codes: np.ndarray, sf: np.ndarray, gate_up: bool) -> np.ndarray:
    """[E, R, K/2] + [E, R, K/16] -> flat packed bytes in the decode-path layout."""
    return np.concatenate([pack_matrix(codes[e], sf[e], gate_up).reshape(-1) for e in range(codes.shape[0])])


def unpack_matrix_values(units: np.ndarray, R: int, K: int, gate_up: bool) -> np.ndarray:
    """Decode packed units back to fp32 weights (without gs) in the ORIGINAL row order, the kernel's way:
    run D on every word, read each bf16 field (value e2m1 * 2^-126), multiply by the scale code's value."""
    nb, nS = R // 16, K // 64
    code_bytes, scale_bytes = split_units(units, K)
    words = np.ascontiguousarray(code_bytes).view(np.uint32).reshape(nb, nS, 8, 4, 4)   # rb, S, g, t, j
    M = packer.FIELD_MASK
    q = words.astype(np.uint64)
    rotl = lambda v, s: ((v << s) | (v >> (32 - s))) & 0xFFFFFFFF
    u6 = (q << 6) & 0xFFFFFFFF
    regs = [q & M, (q << 4) & M, (u6 ^ rotl(q, 10)) & M, (u6 ^ rotl(q, 12)) & M]
    out = np.zeros((nb, 16, K), dtype=np.float32)
    sb = np.ascontiguousarray(scale_bytes).reshape(nb, nS // 4, 8, 4, 4, 2)          # rb, S4, g, t, s4, h
    for i, r in enumerate(regs):
        for hh in range(2):
            bits = ((r >> (16 * hh)) & 0xFFFF).astype(np.uint32) << 16
            val = (bits.astype(np.uint32)).view(np.float32) * np.float32(2.0 ** 126)   # e2m1 value
            row_h = i & 1                 # registers 0, 2 -> row g; 1, 3 -> row g + 8
            koff = 2 * (i >> 1) + hh      # registers 0, 1 -> k+0/+1; 2, 3 -> k+2/+3
            S = np.arange(nS)[:, None, None, None]
            t = np.arange(4)[None, None, :, None]
            j = np.arange(4)[None, None, None, :]
            k = 64 * S + 16 * t + 4 * j + koff                                     # [S, 1, t, j]
            g = np.arange(8)[None, :, None, None]
            sc = sb[:, :, :, :, :, row_h]                                           # rb, S4, g, t, s4
            scode = sc.reshape(nb, nS // 4, 8, 4, 4).transpose(0, 1, 4, 2, 3).reshape(nb, nS, 8, 4)  # rb,S,g,t
            sval = np.vectorize(packer.scale_code_value)(scode).astype(np.float32)
            w = val * sval[..., None]
            rows = g + 8 * row_h
            kk = np.broadcast_to(k, (nS, 8, 4, 4))
            rr = np.broadcast_to(rows, (nS, 8, 4, 4))
            for b in range(nb):
                out[b, rr, kk] = w[b]
    vals = out.reshape(R, K)
    orig = np.empty_like(vals)
    orig[packed_row_order(R, gate_up)] = vals
    return orig


def dequantize_no_gs(codes: np.ndarray, sf: np.ndarray) -> np.ndarray:
    return nvfp4.dequantize(codes, sf, np.float32(1.0))


# ------------------------------------------------------------------------------------------------ prefill layout
def wide_row_order(R: int, gate_up: bool) -> np.ndarray:
    """Original row of each wide-layout packed row: per 128-row block, gate 0-31 / up 0-31 / gate 32-63 / up 32-63
    of the block's 64 features for gate_up; identity for down."""
    if not gate_up:
        return np.arange(R)
    inter = R // 2
    b = np.arange(R // 128)[:, None, None]
    q = np.arange(4)[None, :, None]
    i = np.arange(32)[None, None, :]
    f = 64 * b + 32 * (q // 2) + i
    return (f + inter * (q % 2)).reshape(-1)


def pack_matrix_wide(codes: np.ndarray, sf: np.ndarray, gate_up: bool) -> np.ndarray:
    """One expert matrix (codes [R, K/2], sf [R, K/16]) -> prefill-layout bytes [R/128 blocks, 9K/16 * 128]."""
    R, K2 = codes.shape
    K = 2 * K2
    rows = wide_row_order(R, gate_up)
    c, sc = canonical(codes[rows], sf[rows])
    nb, ns = R // 128, K // 256
    # natural word w of a row = its code bytes 4w..4w+3 (k = 8w..8w+7), k = 256 s + 64 chunk + 32 j + 8 w'
    words = np.ascontiguousarray(c).view("<u4").reshape(nb, 128, ns, 4, 2, 4)   # b, row, s, chunk, j, w'
    words = _apply_T(words)
    code_part = np.ascontiguousarray(words.transpose(0, 2, 3, 4, 1, 5)).view(np.uint8).reshape(nb, ns, 4, 4096)
    scale_part = np.ascontiguousarray(sc.reshape(nb, 128, ns, 4, 4).transpose(0, 2, 3, 1, 4)).reshape(nb, ns, 4, 512)
    return np.concatenate([code_part, scale_part], axis=3).reshape(nb, -1)


def pack_tensor_wide(codes: np.ndarray, sf: np.ndarray, gate_up: bool) -> np.ndarray:
    """[E, R, K/2] + [E, R, K/16] -> flat packed bytes in the prefill-path layout."""
    return np.concatenate([pack_matrix_wide(codes[e], sf[e], gate_up).reshape(-1) for e in range(codes.shape[0])])


def unpack_matrix_wide_values(blocks: np.ndarray, R: int, K: int, gate_up: bool) -> np.ndarray:
    """Decode prefill-layout bytes back to fp32 weights (without gs) in the ORIGINAL row order, the way the
    kernel's dequantising threads do: run D on every word, register i half h is k = 8w + 2i + h."""
    nb, ns = R // 128, K // 256
    b = np.ascontiguousarray(blocks).reshape(nb, ns, 4, 4608)
    words = np.ascontiguousarray(b[..., :4096]).view(np.uint32).reshape(nb, ns, 4, 2, 128, 4)  # b, s, c, j, row, w'
    scodes = b[..., 4096:].reshape(nb, ns, 4, 128, 4)                                          # b, s, c, row, blk
    M = packer.FIELD_MASK
    q = words.astype(np.uint64)
    rotl = lambda v, s: ((v << s) | (v >> (32 - s))) & 0xFFFFFFFF
    u6 = (q << 6) & 0xFFFFFFFF
    regs = [q & M, (q << 4) & M, (u6 ^ rotl(q, 10)) & M, (u6 ^ rotl(q, 12)) & M]
    svals = np.array([packer.scale_code_value(v) for v in range(256)], dtype=np.float32)[scodes]  # b, s, c, row, blk
    out = np.zeros((nb, 128, ns, 4, 2, 4, 8), dtype=np.float32)      # b, row, s, c, j, w', k-in-word
    for i, r in enumerate(regs):
        for hh in range(2):
            bits = ((r >> (16 * hh)) & 0xFFFF).astype(np.uint32) << 16
            val = bits.view(np.float32) * np.float32(2.0 ** 126)   # b, s, c, j, row, w'
            out[..., 2 * i + hh] = val.transpose(0, 4, 1, 2, 3, 5)
    blk = np.array([[2 * j + w // 2 for w in range(4)] for j in range(2)])                        # j, w'
    sv = svals.transpose(0, 3, 1, 2, 4)[:, :, :, :, blk]                                          # b, row, s, c, j, w'
    vals = (out * sv[..., None]).reshape(R, K)
    orig = np.empty_like(vals)
    orig[wide_row_order(R, gate_up)] = vals
    return orig
