"""Generate the committed golden fixtures under tests/golden/.

Two groups:

* ``ref_*``: produced by RUNNING THE REFERENCE's own Python code on the CPU (it must be importable: pass
  ``--reference <path to the xCalibur checkout>``).  They pin
  - the GF(2) machinery (xcalibur/gf2.py; vectors of tests/test_core.py:6-20 plus random maps),
  - the FP4/FP8 dequantisation bit semantics: random codes and scales are packed by the reference's
    ``_pack_codes`` / ``_pack_scales`` (kernels/moe_w4a16_h200/moe_w4a16.py:3168-3190, wrapped by its GF(2)
    transform at :3903-3933), decoded with the reference's shipped decoder ``_XC_DQ4`` (moe_w4a16.py:3475,
    restated below and checked against the reference's source text) and its e4m3 LUT (moe_w4a16.py:3315-3318),
    giving e2m1(code) * e4m3(scale) for every (row, k).
* ``ref_okc_pack.json``: digests of the reference's own ``prepare`` repacks (``_pack_codes`` with its GF(2) word
  transform, ``_pack_scales``, ``_fat_order``, ``_unit_order``, moe_w4a16.py:3168-3209, :3903-3933; the e4m3 LUT,
  :3313-3318) on seeded codes and scales of one 256-row, K = 4096 expert slice, for the gate_up row order with its
  sign fold and for the down row order.  They pin ``oracle/okc_ref.py``, which rebuilds the reference's layouts on
  the GPU box (where the reference's Python is absent) to run its prebuilt kernel.
* ``layer_c1.json``: checksums of the CPU oracle's layer output on the seeded C1 configuration (guards the
  oracle against drift; no reference needed).

Run:  python tests/golden/make_golden.py --reference /path/to/xCalibur  [--okc-only]
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))


def _rotl(v, s):
    return ((v << s) | (v >> (32 - s))) & 0xFFFFFFFF


def ref_decoder(q):
    """The reference's shipped dq4 (moe_w4a16.py:3475), restated; q is a uint64 numpy array of words."""
    M = 0x81C081C0
    return ((((q << 2) & 0xFFFFFFFF) ^ q) & M, ((q << 6) & 0xFFFFFFFF) & M, _rotl(q, 10) & M, (_rotl(q, 12) ^ q) & M)


def make_ref_fixtures(ref_root: str):
    sys.path.insert(0, ref_root)
    sys.path.insert(0, os.path.join(ref_root, "kernels", "moe_w4a16_h200"))
    import torch
    import xcalibur as xc
    import moe_w4a16 as m

    # --- the restated decoder must be the one the reference ships
    src = m._XC_DQ4
    for frag in ("((q << 2) ^ q) & 0x81C081C0u", "(q << 6) & 0x81C081C0u", "__funnelshift_l(q, q, 10) & 0x81C081C0u",
                 "(__funnelshift_l(q, q, 12) ^ q) & 0x81C081C0u"):
        assert frag in src, frag

    # --- GF(2) vectors
    P = tuple(1 << i for i in range(32))
    D = xc.compose(xc.rotation(5), P)
    T = xc.packing_transform(D, P)
    words = [0, 1, 0x12345678, 0xFFFFFFFF, 0x0F0F0F0F]
    rng = np.random.default_rng(7)
    rand_maps = []
    while len(rand_maps) < 4:
        rows = tuple(int(x) for x in rng.integers(0, 2**32, 32, dtype=np.uint64))
        if xc.rank(rows) == 32:
            rand_maps.append(rows)
    gf = {
        "words": words,
        "rot5_T": list(T),
        "rot5_apply": [xc.apply(D, xc.apply(T, w)) for w in words],
        "random_maps": [list(r) for r in rand_maps],
        "random_inverse": [list(xc.inverse(r)) for r in rand_maps],
        "random_compose": [list(xc.compose(rand_maps[i], rand_maps[i + 1])) for i in range(3)],
        "random_columns": [list(xc.columns(r)) for r in rand_maps],
        "join_atoms": [["a", [1, 2]], ["b", [4, 8]], ["c", [5, 2]], ["d", [12]]],
        "join_result": [list(j) for j in xc.join_all([("a", (1, 2)), ("b", (4, 8)), ("c", (5, 2)), ("d", (12,))], 4)],
        "xc_cols": list(m._XC_COLS),
    }
    with open(os.path.join(HERE, "ref_gf2.json"), "w") as f:
        json.dump(gf, f)

    # --- e4m3 LUT exactly as the reference builds it (value * 2^64 in bf16, moe_w4a16.py:3315-3318)
    lut = (torch.arange(256, dtype=torch.int32).to(torch.uint8).view(torch.float8_e4m3fn).float() * 2.0**64)
    lut_bits = lut.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)

    # --- dequantisation through the reference's packer + decoder, one 16-row block at K = 4096
    R, K = 16, 4096
    codes = rng.integers(0, 256, (R, K // 2), dtype=np.uint8)
    sf = rng.integers(0x01, 0x7F, (R, K // 16), dtype=np.uint8)          # subnormal and normal, positive
    sf[0, :4] = [0x00, 0x01, 0x07, 0x7E]
    rows = torch.arange(R)
    words = m._pack_codes(torch.from_numpy(codes), rows).numpy().view(np.uint32).astype(np.uint64)
    sbytes = m._pack_scales(torch.from_numpy(sf).view(torch.float8_e4m3fn), rows).numpy().view(np.uint8)
    words = words.reshape(1, 8, 8, 8, 4, 4)                                 # rb, w, c, g, t, s
    sbytes = sbytes.reshape(1, 8, 8, 4, 8, 2)                               # rb, w, g, t, c, h
    regs = ref_decoder(words)
    lutf = (lut_bits.astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    vals = np.full((R, K), np.nan, dtype=np.float64)
    reg_hj = [(0, 0), (1, 0), (0, 2), (1, 2)]                               # moe_w4a16.py:196
    w_i, c_i, g_i, t_i, s_i = np.meshgrid(np.arange(8), np.arange(8), np.arange(8), np.arange(4), np.arange(4),
                                          indexing="ij")
    for Rg, (h, j0) in enumerate(reg_hj):
        for up in range(2):
            bits = ((regs[Rg][0] >> (16 * up)) & 0xFFFF).astype(np.uint32) << 16
            e2m1_scaled = bits.view(np.float32).astype(np.float64)            # e2m1 * 2^-126
            row = 8 * h + g_i
            k = ((w_i * 8 + c_i) * 4 + t_i) * 16 + s_i * 4 + j0 + up
            scale = lutf[sbytes[0][w_i, g_i, t_i, c_i, h]]                   # e4m3 * 2^64
            vals[row, k] = e2m1_scaled * scale * 2.0**62
    assert not np.isnan(vals).any()
    np.savez_compressed(os.path.join(HERE, "ref_dequant.npz"), codes=codes, sf=sf, values=vals.astype(np.float32),
                        lut_bits=lut_bits)
    print("wrote ref_gf2.json, ref_dequant.npz")


OKC_PACK_SEED = 2024


def okc_pack_inputs():
    """Seeded codes and scale bytes of one 256-row, K = 4096 slice, for gate_up (I = 128) and for down."""
    rng = np.random.default_rng(OKC_PACK_SEED)
    c13 = rng.integers(0, 256, (256, 2048), dtype=np.uint8)
    s13 = rng.integers(0x08, 0x7F, (256, 256), dtype=np.uint8)
    c2 = rng.integers(0, 256, (256, 2048), dtype=np.uint8)
    s2 = rng.integers(0x08, 0x7F, (256, 256), dtype=np.uint8)
    return c13, s13, c2, s2


def _sha(a) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def make_okc_pack_fixture(ref_root: str):
    sys.path.insert(0, os.path.join(ref_root, "kernels", "moe_w4a16_h200"))
    import torch
    import moe_w4a16 as m

    c13, s13, c2, s2 = (torch.from_numpy(a) for a in okc_pack_inputs())
    I = 128
    rb = torch.arange(I // 8)
    g = torch.arange(8)
    rows_a = torch.stack((8 * rb[:, None] + g[None, :], I + 8 * rb[:, None] + g[None, :]), 1).reshape(-1)
    rows_b = torch.arange(256)
    out = {}
    for tag, codes, sf, rows in (("gate_up", c13 ^ 0x88, s13, rows_a), ("down", c2, s2, rows_b)):
        wds = m._pack_codes(codes, rows)
        scs = m._pack_scales(sf.view(torch.float8_e4m3fn), rows)
        out[tag] = {"words": _sha(wds.numpy()), "scales": _sha(scs.numpy()),
                    "fat": _sha(m._fat_order(wds, scs).numpy()), "unit": _sha(m._unit_order(wds, scs).numpy()),
                    "words_head": [int(v) for v in wds[:8]]}
    lut = (torch.arange(256, dtype=torch.int32).to(torch.uint8).view(torch.float8_e4m3fn).float()
           * 2.0**64).to(torch.bfloat16).view(torch.int16).to(torch.int32) & 0xFFFF
    out["lut"] = _sha((lut | (lut << 16)).to(torch.int32).numpy())
    out["seed"] = OKC_PACK_SEED
    with open(os.path.join(HERE, "ref_okc_pack.json"), "w") as f:
        json.dump(out, f, indent=1)
    print("wrote ref_okc_pack.json")


def layer_digest(out_bits, ids, wts):
    h = lambda a: hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()
    return {"out_sha256": h(out_bits), "ids_sha256": h(ids), "weights_sha256": h(wts)}


def make_layer_fixture():
    sys.path.insert(0, ROOT)
    from oracle import moe_ref

    rng = np.random.default_rng(0)
    E, H, I, T, k = 8, 1024, 512, 16, 2
    w = moe_ref.make_weights(rng, E, H, I)
    x, logits = moe_ref.make_inputs(rng, T, H, E)
    out, ids, wts = moe_ref.moe_layer(x, logits, *w, k)
    d = {"config": {"seed": 0, "E": E, "H": H, "I": I, "T": T, "top_k": k}, **layer_digest(out, ids, wts),
         "ids": ids.tolist(), "out_row0_bits": out[0, :16].tolist(),
         "weights_sha256_inputs": hashlib.sha256(w[0].tobytes() + w[1].tobytes() + x.tobytes()).hexdigest()}
    with open(os.path.join(HERE, "layer_c1.json"), "w") as f:
        json.dump(d, f, indent=1)
    print("wrote layer_c1.json")


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=None, help="path of an xCalibur checkout (for the ref_* fixtures)")
    ap.add_argument("--layer-only", action="store_true")
    ap.add_argument("--okc-only", action="store_true", help="only ref_okc_pack.json")
    a = ap.parse_args()
    if a.okc_only:
        make_okc_pack_fixture(a.reference)
        sys.exit(0)
    if not a.layer_only:
        if not a.reference:
            ap.error("--reference is required for the ref_* fixtures")
        make_ref_fixtures(a.reference)
        make_okc_pack_fixture(a.reference)
    make_layer_fixture()
