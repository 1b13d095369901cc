"""Bit-level linear algebra over GF(2) for FP4 weight decoders.

A decoder that only shifts, rotates, masks and XORs bits of a packed 32-bit word is a linear map over GF(2).
A map is held as a tuple of row masks: row ``i`` is the set of input bits whose parity is output bit ``i``.
This is the convention of the reference's ``xcalibur/gf2.py`` (``apply``, ``compose``, ``inverse``, ``rank``,
``packing_transform`` at xcalibur/gf2.py:27-97), so maps and test vectors carry over unchanged; the code
below is an independent implementation.

The packer uses one identity from that module: if ``P`` is the decode the weights are written for and ``D``
is the cheap decode the kernel runs, then packing every word with ``T = D^-1 P`` makes ``D(T(w)) == P(w)`` for
all 2^32 words.  Equality of linear maps is checked exactly on the 32 basis words.
"""
from __future__ import annotations

from typing import Callable, Iterable, Sequence

Rows = tuple


def _bits(mask: int):
    while mask:
        low = mask & -mask
        yield low.bit_length() - 1
        mask ^= low


def apply(rows: Sequence[int], word: int) -> int:
    """Image of ``word``: output bit i = parity(rows[i] & word)."""
    out = 0
    for i, r in enumerate(rows):
        out |= (bin(r & word).count("1") & 1) << i
    return out


def columns(rows: Sequence[int]) -> tuple:
    """Images of the basis words e_0..e_{n-1} (the map's columns)."""
    n = len(rows)
    cols = [0] * n
    for i, r in enumerate(rows):
        for b in _bits(r):
            if b < n:
                cols[b] |= 1 << i
    return tuple(cols)


def from_columns(cols: Sequence[int], n_out: int | None = None) -> tuple:
    """Rows of the map whose basis images are ``cols``."""
    n_out = len(cols) if n_out is None else n_out
    rows = [0] * n_out
    for j, c in enumerate(cols):
        for i in _bits(c):
            rows[i] |= 1 << j
    return tuple(rows)


def from_function(fn: Callable[[int], int], bits: int = 32) -> tuple:
    """Rows of a bit-linear function, read off its basis images (linearity is the caller's claim)."""
    return from_columns([fn(1 << j) & ((1 << bits) - 1) for j in range(bits)], bits)


def identity(bits: int = 32) -> tuple:
    return tuple(1 << i for i in range(bits))


def rotation(k: int, bits: int = 32) -> tuple:
    """Rotate left by k."""
    k %= bits
    return tuple(1 << ((i - k) % bits) for i in range(bits))


def shift_left(k: int, bits: int = 32) -> tuple:
    return tuple((1 << (i - k)) if i >= k else 0 for i in range(bits))


def compose(a: Sequence[int], b: Sequence[int]) -> tuple:
    """Rows of x -> a(b(x))."""
    out = []
    for row in a:
        acc = 0
        for j in _bits(row):
            acc ^= b[j]
        out.append(acc)
    return tuple(out)


def rank(rows: Iterable[int]) -> int:
    basis: list[int] = []
    for r in rows:
        for v in basis:
            r = min(r, r ^ v)
        if r:
            basis.append(r)
            basis.sort(reverse=True)
    return len(basis)


def inverse(rows: Sequence[int]) -> tuple:
    """Inverse of a square map by Gauss-Jordan on [rows | I]; raises ValueError if singular."""
    n = len(rows)
    aug = [(r, 1 << i) for i, r in enumerate(rows)]
    for col in range(n):
        pivot = next((k for k in range(col, n) if (aug[k][0] >> col) & 1), None)
        if pivot is None:
            raise ValueError("singular map")
        aug[col], aug[pivot] = aug[pivot], aug[col]
        pr, pi = aug[col]
        for k in range(n):
            if k != col and (aug[k][0] >> col) & 1:
                aug[k] = (aug[k][0] ^ pr, aug[k][1] ^ pi)
    return tuple(ai for _, ai in aug)


def equal(a: Sequence[int], b: Sequence[int]) -> bool:
    """Exact equality for every input word."""
    return tuple(a) == tuple(b)


def packing_transform(decoder: Sequence[int], reference: Sequence[int]) -> tuple:
    """T with decoder(T(w)) == reference(w) for all w (the lossless repacking for a new decoder)."""
    t = compose(inverse(decoder), reference)
    if compose(decoder, t) != tuple(reference):
        raise AssertionError("packing proof failed")
    if rank(t) != len(t):
        raise AssertionError("packing transform is singular")
    return t


def compatible(a_rows: Sequence[int], b_rows: Sequence[int]) -> bool:
    """Two partial decoders can be stacked if their rows stay independent."""
    return rank(tuple(a_rows) + tuple(b_rows)) == len(a_rows) + len(b_rows)


def join_all(atoms, target_rank: int):
    """Every set of pairwise-compatible atoms (name, rows) whose stacked rows reach ``target_rank``."""
    names = [a[0] for a in atoms]
    rowsets = [tuple(a[1]) for a in atoms]
    n = len(atoms)
    ok = [[i != j and compatible(rowsets[i], rowsets[j]) for j in range(n)] for i in range(n)]
    found = []

    def walk(chosen, stacked, start):
        if len(stacked) == target_rank:
            if rank(stacked) == target_rank:
                found.append(tuple(names[i] for i in chosen))
            return
        for j in range(start, n):
            if len(stacked) + len(rowsets[j]) <= target_rank and all(ok[i][j] for i in chosen):
                walk(chosen + [j], stacked + rowsets[j], j + 1)

    walk([], (), 0)
    return found


def xor_tables(t_rows: Sequence[int]) -> list:
    """The map as four 256-entry byte tables: T(w) = tab[0][w&255] ^ tab[1][(w>>8)&255] ^ ... (for the packers)."""
    cols = columns(t_rows)
    tabs = []
    for byte in range(len(cols) // 8):
        tab = []
        for v in range(256):
            acc = 0
            for b in _bits(v):
                acc ^= cols[byte * 8 + b]
            tab.append(acc)
        tabs.append(tab)
    return tabs
