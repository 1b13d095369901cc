"""The CPU oracle: pinned against outputs of the reference's own code, and checked for its own invariants."""
import json
import os

import numpy as np
import pytest

from oracle import moe_ref, nvfp4

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def test_dequant_matches_reference_packer_and_decoder():
    d = np.load(os.path.join(GOLD, "ref_dequant.npz"))
    v = nvfp4.dequantize(d["codes"], d["sf"], np.float32(1.0))
    assert np.array_equal(v, d["values"])


def test_e4m3_table_matches_reference_lut():
    d = np.load(os.path.join(GOLD, "ref_dequant.npz"))
    lut = (d["lut_bits"].astype(np.uint32) << 16).view(np.float32)
    mine = nvfp4.E4M3_VALUES * np.float32(2.0 ** 64)
    ok = np.isnan(mine) | (lut == mine)
    assert ok.all()


def test_e2m1_rounding_ties_to_even():
    vals = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 7.0, -0.25, -0.75, -5.0, 0.3, -0.1], np.float32)
    codes = nvfp4.e2m1_encode_rne(vals)
    assert codes.tolist() == [0, 2, 2, 4, 4, 6, 6, 7, 0, 10, 14, 1, 0]


def test_e4m3_rne_roundtrip():
    b = np.arange(0x7F, dtype=np.uint8)
    assert np.array_equal(nvfp4.e4m3_encode_rne(nvfp4.e4m3_decode(b)), b)
    assert nvfp4.e4m3_encode_rne(np.float32([500.0, 448.0, 2 ** -10]))[:2].tolist() == [0x7E, 0x7E]
    assert nvfp4.e4m3_encode_rne(np.float32([2 ** -10]))[0] == 0  # tie to even (0) at half the smallest subnormal


def test_quantize_error_bound():
    rng = np.random.default_rng(3)
    w = rng.standard_normal((2, 64, 256), dtype=np.float32) * np.float32(0.02)
    c, s, g = nvfp4.quantize(w)
    wd = nvfp4.dequantize(c, s, g)
    blocks = np.abs(w).reshape(2, 64, 16, 16).max(-1)
    step = np.repeat(blocks, 16, axis=-1) / 6.0 * 2.2          # half the widest E2M1 gap, with scale rounding
    assert np.all(np.abs(wd - w) <= step + 1e-6)


def test_router_ties_to_lower_index():
    logits = np.array([[1.0, 3.0, 3.0, 0.5, 3.0, -1.0]], np.float32)
    ids, w = moe_ref.route_topk(logits, 4)
    assert ids.tolist() == [[1, 2, 4, 0]]
    assert abs(w.sum() - 1.0) < 1e-6


def test_permutation_is_stable_sort():
    rng = np.random.default_rng(1)
    ids = rng.integers(0, 6, (50, 3)).astype(np.int32)
    order, pos, counts, offsets = moe_ref.permute(ids, 1, 4)
    flat = ids.reshape(-1)
    loc = [f for f in range(flat.size) if 1 <= flat[f] < 5]
    want = sorted(loc, key=lambda f: (flat[f], f))
    assert order.tolist() == want
    assert all(pos[f] == -1 for f in range(flat.size) if f not in loc)
    assert counts.sum() == len(loc) and offsets[-1] == len(loc)


def test_layer_c1_fixture_is_stable():
    """The committed digest of the oracle's C1 output (tests/golden/layer_c1.json) still holds."""
    import sys
    sys.path.insert(0, GOLD)
    from make_golden import layer_digest

    gold = json.load(open(os.path.join(GOLD, "layer_c1.json")))
    cfg = gold["config"]
    rng = np.random.default_rng(cfg["seed"])
    w = moe_ref.make_weights(rng, cfg["E"], cfg["H"], cfg["I"])
    x, logits = moe_ref.make_inputs(rng, cfg["T"], cfg["H"], cfg["E"])
    out, ids, wts = moe_ref.moe_layer(x, logits, *w, cfg["top_k"])
    d = layer_digest(out, ids, wts)
    assert d["ids_sha256"] == gold["ids_sha256"]
    assert d["out_sha256"] == gold["out_sha256"]


def test_post_norm_form():
    """Reference-contract form: rms-normalised routes; scaling y by a constant leaves the output unchanged."""
    rng = np.random.default_rng(2)
    E, H, I, T, k = 4, 256, 256, 5, 2
    c13, s13, g13, c2, s2, g2 = moe_ref.make_weights(rng, E, H, I)
    x, logits = moe_ref.make_inputs(rng, T, H, E)
    ids, wts = moe_ref.route_topk(logits, k)
    gam = moe_ref.f32_to_bf16_bits(np.zeros(H, np.float32))
    o1, _ = moe_ref.moe_forward(x, ids, wts, c13, s13, g13, c2, s2, g2, post_norm_w_bits=gam)
    o2, _ = moe_ref.moe_forward(x, ids, wts, c13, s13, g13, c2, s2, g2 * np.float32(4.0), post_norm_w_bits=gam)
    a, b = moe_ref.bf16_bits_to_f32(o1), moe_ref.bf16_bits_to_f32(o2)
    assert np.allclose(a, b, rtol=1e-2, atol=1e-2)
    # each token's output is a convex combination of unit-rms rows: its rms is at most 1
    assert np.all(np.sqrt(np.mean(a.astype(np.float64) ** 2, axis=1)) <= 1.0 + 1e-2)


def test_nonlocal_routes_contribute_nothing():
    rng = np.random.default_rng(4)
    E, H, I, T, k = 4, 256, 256, 6, 2
    w = moe_ref.make_weights(rng, E, H, I)
    x, logits = moe_ref.make_inputs(rng, T, H, 8)
    ids, wts = moe_ref.route_topk(logits, k)
    out, _ = moe_ref.moe_forward(x, ids, wts, *w, local_start=4)         # experts 4..7 held
    for t in range(T):
        if not any(4 <= e < 8 for e in ids[t]):
            assert not moe_ref.bf16_bits_to_f32(out[t]).any()


def test_fast_dequantize_is_identical():
    rng = np.random.default_rng(5)
    c = rng.integers(0, 256, (64, 512), dtype=np.uint8)
    s = rng.integers(0, 256, (64, 64), dtype=np.uint8)
    s[(s & 0x7F) == 0x7F] = 0x38                          # no NaN scale bytes
    for gs in (np.float32(0.0123), np.float32(3.0)):
        a = nvfp4.dequantize(c, s, gs)
        b = nvfp4.dequantize_fast(c, s, gs)
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
