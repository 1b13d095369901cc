"""CPU model of both packed weight layouts — test infrastructure.

Builds, with numpy, the exact bytes the GPU packer (``xcb_moe_pack_weights``) must produce, from the layouts and
bit maps that ``xcalibur_b200.packer`` defines, and decodes packed bytes back to weight values the way the
kernels' registers see them.  The reference analogue is the host repack of
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
    """Fold zero and negative scales into the codes; return (codes', scale codes) for one [R, K/2] matrix
    (prefill-path layout only)."""
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


def pack_matrix(codes: np.ndarray, sf: np.ndarray, gate_up: bool) -> np.ndarray:
    """One expert matrix (codes [R, K/2], sf [R, K/16]) -> decode-path packed bytes [R/16 units, 9K].

    A unit is K/64 slice records of 576 bytes: ``[32 lanes][4 words]`` of codes, then ``[32 lanes][2]`` scale bytes.
    Word j of lane 4g + t in slice S = raw code bytes (row g, row g + 8, row g, row g + 8) at code byte
    32S + 8t + 2j + (0, 0, 1, 1); the lane's two scale bytes are the raw E4M3 scales of rows g and g + 8 for
    block 4S + t."""
    R, K2 = codes.shape
    K = 2 * K2
    rows = packed_row_order(R, gate_up)
    c, sc = codes[rows], sf[rows]
    nb, nS = R // 16, K // 64
    cb = c.reshape(nb, 2, 8, K2)                                 # [rb, h, g, byte]
    S = np.arange(nS)[:, None, None, None]
    t = np.arange(4)[None, :, None, None]
    j = np.arange(4)[None, None, :, None]
    hi = np.arange(2)[None, None, None, :]
    bidx = (32 * S + 8 * t + 2 * j + hi)                          # [S, t, j, hi]
    r0 = cb[:, 0][:, :, bidx]                                    # [rb, g, S, t, j, hi]  rows g
    r8 = cb[:, 1][:, :, bidx]                                    # rows g + 8
    word = (r0[..., 0].astype(np.uint32) | (r8[..., 0].astype(np.uint32) << 8)
            | (r0[..., 1].astype(np.uint32) << 16) | (r8[..., 1].astype(np.uint32) << 24))  # [rb, g, S, t, j]
    word = word.transpose(0, 2, 1, 3, 4)                         # [rb, S, g, t, j] -> lane = 4g + t
    code_bytes = np.ascontiguousarray(word).view(np.uint8).reshape(nb, nS, 512)
    sb = sc.reshape(nb, 2, 8, K // 16)                           # [rb, h, g, block]
    g = np.arange(8)[None, :, None, None]
    tt = np.arange(4)[None, None, :, None]
    S2 = np.arange(nS)[:, None, None, None]
    h = np.arange(2)[None, None, None, :]
    scl = sb[:, h, g, 4 * S2 + tt]                               # [rb, S, g, t, h]
    scale_bytes = np.ascontiguousarray(scl).reshape(nb, nS, 64)
    return np.concatenate([code_bytes, scale_bytes], axis=2).reshape(nb, 9 * K)


def pack_tensor(codes: np.ndarray, sf: np.ndarray, gate_up: bool) -> np.ndarray:
    """[E, R, K/2] + [E, R, K/16] -> flat packed bytes in the decode-path layout."""
    return np.concatenate([pack_matrix(codes[e], sf[e], gate_up).reshape(-1) for e in range(codes.shape[0])])


def unpack_matrix_values(units: np.ndarray, R: int, K: int, gate_up: bool) -> np.ndarray:
    """Decode packed units back to fp32 weights (without gs) in the ORIGINAL row order, the way the kernel's
    registers see them: each code byte -> two E2M1 values (low nibble first), times the lane's E4M3 scale."""
    nb, nS = R // 16, K // 64
    rec = np.ascontiguousarray(units).reshape(nb, nS, 576)
    words = rec[:, :, :512].copy().view(np.uint32).reshape(nb, nS, 8, 4, 4)          # rb, S, g, t, j
    scl = rec[:, :, 512:].reshape(nb, nS, 8, 4, 2)                                  # rb, S, g, t, h
    sval = nvfp4.e4m3_decode(scl)
    out = np.zeros((nb, 16, K), dtype=np.float32)
    S = np.arange(nS)[:, None, None, None]
    t = np.arange(4)[None, None, :, None]
    j = np.arange(4)[None, None, None, :]
    g = np.arange(8)[None, :, None, None]
    for b in range(4):                           # byte b of the word: register b of the step
        byte = (words >> (8 * b)) & 0xFF
        row_h = b & 1                            # bytes 0, 2 -> row g; 1, 3 -> row g + 8
        for nib in range(2):                     # low nibble -> even k
            val = nvfp4.E2M1_VALUES[(byte >> (4 * nib)) & 0xF] * sval[..., row_h][..., None]
            k = 64 * S + 16 * t + 4 * j + 2 * (b >> 1) + nib
            kk = np.broadcast_to(k, (nS, 8, 4, 4))
            rr = np.broadcast_to(g + 8 * row_h, (nS, 8, 4, 4))
            for u in range(nb):
                out[u, rr, kk] = val[u]
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
