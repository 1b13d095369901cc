"""Both weight layouts on the CPU: decode(pack(w)) equals the oracle's dequantisation, bit for bit."""
import numpy as np
import pytest

from oracle import nvfp4, pack_ref
from xcalibur_b200 import packer


@pytest.mark.parametrize("gate_up", [False, True])
@pytest.mark.parametrize("R,K", [(32, 256), (16, 768), (48, 1024), (16, 1280), (16, 3072)])
def test_pack_roundtrip_exact(gate_up, R, K):
    rng = np.random.default_rng(R * 7 + K)
    w = rng.standard_normal((1, R, K)).astype(np.float32) * np.float32(0.02)
    codes, sf, _ = nvfp4.quantize(w)
    # edge scales: zero, subnormal, negative, max
    sf[0, 0, 0] = 0x00
    sf[0, 1, 1] = 0x80
    sf[0, 2, 0] = 0x03
    sf[0, 3, 2] = 0xB8
    sf[0, 4, 1] = 0x7E
    pk = pack_ref.pack_matrix(codes[0], sf[0], gate_up)
    assert pk.shape == (R // 16, packer.unit_bytes(K))
    vals = pack_ref.unpack_matrix_values(pk, R, K, gate_up)
    ref = pack_ref.dequantize_no_gs(codes[0], sf[0])
    assert np.array_equal(vals, ref)


@pytest.mark.parametrize("gate_up", [False, True])
@pytest.mark.parametrize("R,K", [(128, 256), (256, 768), (128, 1280), (384, 512)])
def test_pack_wide_roundtrip_exact(gate_up, R, K):
    rng = np.random.default_rng(R * 11 + K)
    w = rng.standard_normal((1, R, K)).astype(np.float32) * np.float32(0.02)
    codes, sf, _ = nvfp4.quantize(w)
    sf[0, 0, 0] = 0x00
    sf[0, 1, 1] = 0x80
    sf[0, 2, 0] = 0x03
    sf[0, 70, 2] = 0xB8
    sf[0, 127, 1] = 0x7E
    pk = pack_ref.pack_matrix_wide(codes[0], sf[0], gate_up)
    assert pk.size == packer.wide_bytes(1, R, K)
    vals = pack_ref.unpack_matrix_wide_values(pk, R, K, gate_up)
    ref = pack_ref.dequantize_no_gs(codes[0], sf[0])
    assert np.array_equal(vals, ref)


def test_wide_row_order_is_a_permutation():
    for R in (128, 512):
        order = pack_ref.wide_row_order(R, True)
        assert sorted(order.tolist()) == list(range(R))
        # lane L of block b: gate (even quarter) or up (odd quarter) of feature 64b + 32(q//2) + L%32
        assert order[32] == R // 2 and order[64] == 32 and order[127] == R // 2 + 63


def test_scale_codes_cover_every_finite_e4m3():
    seen = {}
    for b in range(256):
        if (b & 0x7F) == 0x7F:
            with pytest.raises(ValueError):
                packer.scale_code(b)
            continue
        c, fold = packer.scale_code(b)
        v = float(nvfp4.E4M3_VALUES[b])
        if fold == "zero":
            assert v == 0.0
            continue
        assert 0 <= c <= 143
        assert packer.scale_code_value(c) == abs(v)
        # the bf16 factor the kernel forms: (c << 4) | 0x6000 == |v| * 2^74
        bits = ((c << 4) | packer.SCALE_BF16_OR) << 16
        f = np.array([bits], np.uint32).view(np.float32)[0]
        assert float(f) == abs(v) * 2.0 ** 74
        seen.setdefault(c, abs(v))
    assert len(seen) == 126


def test_packed_sizes():
    assert packer.skinny_bytes(256, 4096, 7168) == 256 * 256 * 9 * 7168
    assert packer.wide_bytes(256, 4096, 7168) == packer.skinny_bytes(256, 4096, 7168)
    assert packer.packed_bytes(8, 1024, 512) == 2 * packer.skinny_bytes(8, 1024, 512)
    with pytest.raises(ValueError):
        packer.check_shape(7168, 1000)
