"""Weight-layout definitions for the B200 kernels, built on the GF(2) decoder machinery (``gf2``).

Replaces the reference's host-side repack (kernels/moe_w4a16_h200/moe_w4a16.py:3168-3275 ``_pack_codes`` /
``_pack_scales`` and the GF(2) word transform at :3903-3933).  Here the host only derives the 32x32 bit map and
the layout constants; the bytes themselves are produced on the GPU by ``xcb_moe_pack_weights`` in the C-ABI
library, which reads the four 256-entry XOR tables built below.

Decode-path ("skinny") layout of one expert matrix W [R rows, K] (K % 256 == 0, R % 16 == 0).  It feeds the
hardware FP4 converter of sm_100a (``cvt.rn.f16x2.e2m1x2``: one code byte -> two f16, low nibble first) and the
m16n8k16 tensor-core step, so it is a pure byte permutation of the reference tensors (no transform, no folding):

* Rows are taken in *packed order*: for gate_up, 16-row block ``rb`` holds gate rows 8rb..8rb+7 then up rows
  8rb..8rb+7 (so one mma.sync accumulator lane owns the gate and the up value of the same intermediate
  feature); for down, rows stay in order.
* A block is one *unit* of ``9*K`` bytes: K/64 slice records of 576 bytes, each ``[32 lanes][4 steps]`` u32 of
  codes (512 bytes) followed by ``[32 lanes][2 row halves]`` scale bytes (64).  Consecutive units of one expert
  are contiguous, so the kernel streams any run of them as bulk copies of whole slices.
* Lane L = 4g + t, slice S, step j holds the word (W[g][b], W[g+8][b], W[g][b+1], W[g+8][b+1]) of code bytes
  b = 32S + 8t + 2j (low nibble = even k): the four f16x2 A-fragment registers of rows {g, g+8} at
  k = 64S + 16t + 4j + {0,1,2,3}.  All 16 k of a lane's slice share one 16-wide scale block (4S + t), so one
  scale pair serves four steps; the activation operand of that step is x[token][64S + 16t + 4j + 0..3].
* The lane's two scale bytes are the raw E4M3 scales of rows g and g + 8 for block 4S + t (converted to f16x2 by
  ``cvt.rn.f16x2.e4m3x2``).  Each f16 weight e2m1 * e4m3 is exact (at most 6 significant bits, magnitude in
  [2^-10, 2688]); the epilogue multiplies by the fp32 global scale.

Prefill-path ("wide") layout of the same matrix, stored after the decode-path bytes in the same buffer.  It feeds
the tcgen05 kernel, whose dequantising threads write one weight row each into a tensor-memory lane (the MMA's A
operand), so a word holds 8 consecutive k of ONE row:

* Rows are cut into blocks of 128 packed rows (one per TMEM lane).  For gate_up, block ``b`` holds lanes 0-31 =
  gate rows 64b..64b+31, 32-63 = the up rows of the same features, 64-95 = gate 64b+32..64b+63, 96-127 = their up
  rows; down keeps rows in order.
* A block is ``K/256`` stages of 18432 bytes (256 k each); a stage is 4 chunks of 4608 bytes (64 k); a chunk is
  its codes ``[2 halves][128 rows][4 words]`` u32 (4096 bytes; half j, word w cover k = 64c + 32j + 8w .. +7) then
  its scale codes ``[128 rows][4 blocks]`` bytes (512).  The blocks of one expert are consecutive.
* The natural word is the row's 4 code bytes at k/2 (low nibble = even k), so the decoder's register i holds
  (k + 2i, k + 2i + 1), exactly a tensor-memory column of two bf16; it is stored as ``T(word)`` with ``T = D^-1 P``:
  ``P`` sends nibble n to the bf16 fields (sign 15, exponent 8..7, mantissa 6, +16 for the high half) of register
  n // 2, half n % 2; ``D`` is the decoder the kernel runs:

      r0 = q & M;   r1 = (q << 4) & M;   r2 = ((q << 6) ^ rotl(q, 10)) & M;   r3 = ((q << 6) ^ rotl(q, 12)) & M

  with M = 0x81C081C0.  Each register then holds two bf16 values e2m1 * 2^-126.  The four shift sources are the
  minimum for this mask: the mask repeats with period 16 so no three shifts, rotations or byte permutations
  of q cover all 32 input bits (checked by ``decoder_search``).
* Scale bytes are canonicalised losslessly at pack time: a zero scale zeroes its 16 codes, a negative scale
  flips its codes' sign bits, and the magnitude is re-encoded as ``c = ((E + 9) << 3) | m`` for the value
  ``2^E (1 + m/8)``, E in [-9, 8] (the E4M3 subnormals become normal).  The kernel forms the bf16 factor
  ``(c << 4) | 0x6000`` = value * 2^74 with one integer multiply-add; the decoded weight in bf16 is
  exactly ``e2m1 * sf * 2^-52`` and the epilogue multiplies by ``gs * 2^52``.
"""
from __future__ import annotations

import itertools

from . import gf2

FIELD_MASK = 0x81C081C0
FIELD_POS = (6, 7, 8, 15)           # code bit (m, e0, e1, s) -> bf16 bit
WEIGHT_EXP_SHIFT = 52               # decoded bf16 weight = value * 2^-52
SCALE_BF16_OR = 0x6000              # (c << 4) | 0x6000 = scale * 2^74 as bf16 bits


def _field_rows(src_rows, reg_positions):
    return [src_rows[p] for p in reg_positions]


def out_positions():
    """Output field bit positions of one register: (half, field) -> bit."""
    return [FIELD_POS[b] + 16 * h for h in range(2) for b in range(4)]


def decoder_rows():
    """The kernel's decoder D as 32 GF(2) rows (output index 8*reg + 4*half + field)."""
    q = gf2.identity()
    shl4, shl6 = gf2.shift_left(4), gf2.shift_left(6)
    rot10, rot12 = gf2.rotation(10), gf2.rotation(12)
    regs = [
        [q],
        [shl4],
        [shl6, rot10],
        [shl6, rot12],
    ]
    rows = []
    for srcs in regs:
        for p in out_positions():
            acc = 0
            for s in srcs:
                acc ^= s[p]
            rows.append(acc)
    return tuple(rows)


def natural_rows():
    """The reference decode P of the natural word: nibble n = 2*reg + half, code bit b -> output 8*reg+4*half+b."""
    return tuple(1 << (4 * (2 * i + h) + b) for i in range(4) for h in range(2) for b in range(4))


def decode_word(q: int):
    """Run D on one packed word the way the kernel does; returns the four bf16x2 registers."""
    m = FIELD_MASK
    rotl = lambda v, s: ((v << s) | (v >> (32 - s))) & 0xFFFFFFFF
    u6 = (q << 6) & 0xFFFFFFFF
    return (q & m, (q << 4) & m, (u6 ^ rotl(q, 10)) & m, (u6 ^ rotl(q, 12)) & m)


def fields_from_registers(regs) -> int:
    """Pack the 32 field bits of four registers into one word in output-index order (inverse view of D)."""
    out = 0
    for i, r in enumerate(regs):
        for j, p in enumerate(out_positions()):
            out |= ((r >> p) & 1) << (8 * i + j)
    return out


_T_CACHE = None


def packing_transform():
    """T = D^-1 P (proved for all words by gf2.packing_transform) and its four XOR byte tables."""
    global _T_CACHE
    if _T_CACHE is None:
        D = decoder_rows()
        assert all(fields_from_registers(decode_word(1 << i)) == gf2.columns(D)[i] for i in range(32)), \
            "decoder_rows does not describe decode_word"
        T = gf2.packing_transform(D, natural_rows())
        _T_CACHE = (T, gf2.xor_tables(T))
    return _T_CACHE


def xor_table_words():
    """The 4 x 256 u32 tables, flattened (what the GPU packer reads)."""
    _, tabs = packing_transform()
    return [v for tab in tabs for v in tab]


def decoder_search(max_sources: int = 3) -> int:
    """Count decoders ``r_i = src & M`` whose sources (q plus ``max_sources`` shifts, rotations or byte
    permutations of q) cover all 32 input bits — a necessary condition for an invertible decoder."""
    cand = [gf2.rotation(s) for s in range(1, 32)] + [gf2.shift_left(s) for s in range(1, 32)]
    for sel in itertools.product(range(4), repeat=4):
        if sel != (0, 1, 2, 3):
            cand.append(tuple(1 << (8 * sel[i // 8] + i % 8) for i in range(32)))
    pos = out_positions()

    def cover(rows):
        c = 0
        for p in pos:
            c |= rows[p]
        return c

    base = cover(gf2.identity())
    covs = sorted({cover(r) for r in cand})
    hits = 0
    for combo in itertools.combinations(covs, max_sources):
        u = base
        for c in combo:
            u |= c
        if u == 0xFFFFFFFF:
            hits += 1
    return hits


# --------------------------------------------------------------------------------------------- scale codes
def scale_code(b: int):
    """E4M3 byte -> (canonical scale code c, fold) where fold is 'zero', 'neg' or None.  NaN -> ValueError."""
    if (b & 0x7F) == 0x7F:
        raise ValueError("NaN block scale")
    e, m = (b >> 3) & 0xF, b & 7
    if e == 0 and m == 0:
        return scale_code(0x38)[0], "zero"          # any valid code; the block's codes become 0
    fold = "neg" if b & 0x80 else None
    if e >= 1:
        return ((e + 2) << 3) | m, fold
    sub = {1: 0, 2: 8, 3: 12, 4: 16, 5: 18, 6: 20, 7: 22}
    return sub[m], fold


def scale_code_value(c: int) -> float:
    """Value encoded by a canonical scale code (before the 2^74 factor)."""
    return 2.0 ** ((c >> 3) - 9) * (1.0 + (c & 7) / 8.0)


# --------------------------------------------------------------------------------------------- sizes
def unit_bytes(K: int) -> int:
    return 9 * K


WIDE_ROWS = 128          # rows per wide-layout block (tensor-memory lanes)
WIDE_STAGE_BYTES = 18432 # 256 k x 128 rows
WIDE_CHUNK_BYTES = 4608  # 64 k x 128 rows


def wide_bytes(E: int, R: int, K: int) -> int:
    """Packed bytes of one [E, R, K] tensor in the prefill-path layout (same as the decode-path size)."""
    return E * (R // WIDE_ROWS) * (K // 256) * WIDE_STAGE_BYTES


def packed_bytes(E: int, R: int, K: int) -> int:
    """Bytes of one packed tensor buffer: the decode-path layout followed by the prefill-path layout."""
    return skinny_bytes(E, R, K) + wide_bytes(E, R, K)


def skinny_bytes(E: int, R: int, K: int) -> int:
    """Packed bytes of one [E, R, K] tensor in the decode-path layout."""
    return E * (R // 16) * unit_bytes(K)


def check_shape(H: int, I: int):
    if H % 256 or I % 256:
        raise ValueError(f"hidden ({H}) and intermediate ({I}) sizes must be multiples of 256")
