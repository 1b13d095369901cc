"""GPU parity: every kernel behind the C-ABI against the CPU oracle on the same seeded inputs.

Integer and byte work (quantiser codes, packed bytes, top-k ids, the expert permutation) must match bit for bit;
the layer output must match within rtol 1e-2 / atol 1e-2 (the north_star tolerance, RTOL/ATOL in tests/_util.py)."""
import ctypes

import numpy as np
import pytest
import torch

from oracle import moe_ref, nvfp4, pack_ref
from xcalibur_b200 import packer
from tests._util import assert_close_bf16, bf16_bits, oracle_layer, to_np

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev(cuda_device):
    from xcalibur_b200 import _lib

    _lib.load()
    return cuda_device


def _weights_from_np(w, dev):
    c13, s13, g13, c2, s2, g2 = w
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    return {"w13": t(c13), "w13_sf": t(s13), "w13_gs": t(g13), "w2": t(c2), "w2_sf": t(s2), "w2_gs": t(g2)}


def _routing_arrays(layer, T, k):
    """pos / order / counts / offsets as the router left them in the current stream's workspace."""
    from xcalibur_b200 import _lib

    ws = layer.workspace(T, k)
    offs = (ctypes.c_size_t * 6)()
    assert layer.lib.xcb_moe_workspace_offsets(ctypes.byref(layer.shape), T, k, offs, 6) == 6
    R, E = T * k, layer.E
    i32 = lambda o, n: to_np(ws[o:o + 4 * n].view(torch.int32))
    return {"pos": i32(offs[2], R), "order": i32(offs[3], R), "counts": i32(offs[4], E), "offsets": i32(offs[5], E + 1)}


# ------------------------------------------------------------------------------------------------ quantiser, packer
def test_quantizer_bit_exact(dev):
    from xcalibur_b200 import synth

    rng = np.random.default_rng(11)
    w = rng.standard_normal((3, 64, 512), dtype=np.float32) * np.float32(0.02)
    w[1, 5, 32:48] = 0.0                              # an all-zero block
    w[2, 7, 0] = 0.5                                  # a dominant value (other blocks get tiny scales)
    c, s, g = synth.quantize(torch.from_numpy(w).to(dev))
    c0, s0, g0 = nvfp4.quantize(w)
    assert np.array_equal(to_np(g), g0)
    assert np.array_equal(to_np(s), s0)
    assert np.array_equal(to_np(c), c0)


def test_packer_bit_exact(dev):
    from xcalibur_b200 import PreparedMoE

    rng = np.random.default_rng(12)
    E, H, I = 3, 512, 256
    c13, s13, g13, c2, s2, g2 = moe_ref.make_weights(rng, E, H, I)
    s13[0, 0, 0], s13[1, 3, 2], s13[2, 9, 5], s2[0, 1, 1], s2[2, 4, 0] = 0x00, 0x05, 0xB0, 0x80, 0x7E
    layer = PreparedMoE(*_weights_from_np((c13, s13, g13, c2, s2, g2), dev).values())
    torch.cuda.synchronize()
    gu, dn = to_np(layer.gate_up), to_np(layer.down)
    assert gu.size == 2 * packer.skinny_bytes(E, 2 * I, H) and dn.size == 2 * packer.skinny_bytes(E, H, I)
    # decode-path layout, then the prefill-path layout of the same weights
    assert np.array_equal(gu[:gu.size // 2], pack_ref.pack_tensor(c13, s13, True))
    assert np.array_equal(dn[:dn.size // 2], pack_ref.pack_tensor(c2, s2, False))
    assert np.array_equal(gu[gu.size // 2:], pack_ref.pack_tensor_wide(c13, s13, True))
    assert np.array_equal(dn[dn.size // 2:], pack_ref.pack_tensor_wide(c2, s2, False))


def test_packer_rejects_nan_scale(dev):
    from xcalibur_b200 import PreparedMoE

    rng = np.random.default_rng(13)
    w = list(moe_ref.make_weights(rng, 2, 256, 256))
    w[1][1, 2, 3] = 0x7F
    with pytest.raises(ValueError, match="NaN"):
        PreparedMoE(*_weights_from_np(w, dev).values())


# ------------------------------------------------------------------------------------------------ layer
def _c1(dev, seed=0):
    rng = np.random.default_rng(seed)
    E, H, I, T, k = 8, 1024, 512, 16, 2
    w = moe_ref.make_weights(rng, E, H, I)
    x, logits = moe_ref.make_inputs(rng, T, H, E)
    return w, x, logits, (E, H, I, T, k)


def test_c1_layer_parity(dev):
    from xcalibur_b200 import PreparedMoE

    w, x, logits, (E, H, I, T, k) = _c1(dev)
    layer = PreparedMoE(*_weights_from_np(w, dev).values())
    xd = torch.from_numpy(x.view(np.int16)).to(dev).view(torch.bfloat16)
    out, ids, wts = layer.forward(xd, torch.from_numpy(logits).to(dev), k, return_routing=True)
    torch.cuda.synchronize()
    assert layer.check_device_status() == 0
    want_out, want_ids, want_w = moe_ref.moe_layer(x, logits, *w, k)
    assert np.array_equal(to_np(ids), want_ids)                          # bit-exact top-k
    assert np.allclose(to_np(wts), want_w, rtol=1e-6, atol=1e-7)
    r = _routing_arrays(layer, T, k)                                       # bit-exact permutation
    order, pos, counts, offsets = moe_ref.permute(want_ids, 0, E)
    assert np.array_equal(r["pos"], pos) and np.array_equal(r["order"], order)
    assert np.array_equal(r["counts"], counts) and np.array_equal(r["offsets"], offsets)
    assert_close_bf16(out, want_out)


def test_repeat_calls_identical_and_graph_capture(dev):
    from xcalibur_b200 import PreparedMoE

    w, x, logits, (E, H, I, T, k) = _c1(dev, seed=5)
    layer = PreparedMoE(*_weights_from_np(w, dev).values())
    xd = torch.from_numpy(x.view(np.int16)).to(dev).view(torch.bfloat16)
    ld = torch.from_numpy(logits).to(dev)
    outs = [layer.forward(xd, ld, k).clone() for _ in range(3)]
    for o in outs[1:]:
        assert torch.equal(o, outs[0])                                    # deterministic, counters reset
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        static_out = layer.forward(xd, ld, k)                             # warm the stream's workspace
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            static_out = layer.forward(xd, ld, k)
    torch.cuda.current_stream().wait_stream(s)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    assert torch.equal(static_out, outs[0])


def test_router_ties_bit_exact(dev):
    from xcalibur_b200 import PreparedMoE

    rng = np.random.default_rng(21)
    E, H, I, T, k = 16, 256, 256, 40, 4
    w = moe_ref.make_weights(rng, E, H, I)
    x, _ = moe_ref.make_inputs(rng, T, H, E)
    logits = rng.integers(-2, 3, (T, E)).astype(np.float32)               # many exact ties
    logits[0] = 0.0
    layer = PreparedMoE(*_weights_from_np(w, dev).values())
    xd = torch.from_numpy(x.view(np.int16)).to(dev).view(torch.bfloat16)
    out, ids, wts = layer.forward(xd, torch.from_numpy(logits).to(dev), k, return_routing=True)
    want_ids, _ = moe_ref.route_topk(logits, k)
    assert np.array_equal(to_np(ids), want_ids)
    assert to_np(ids)[0].tolist() == [0, 1, 2, 3]
    assert_close_bf16(out, oracle_layer(xd, layer_src(w, dev), want_ids, to_np(wts)))


def layer_src(w, dev):
    return _weights_from_np(w, dev)


def test_reference_contract_post_norm_and_local_range(dev):
    """kernel_fn/prepare with precomputed ids, 4 of 12 experts local, post-norm (moe_w4a16.py:3292, :3370)."""
    from xcalibur_b200 import kernel_fn, prepare

    rng = np.random.default_rng(31)
    E, H, I, T, k, lo, cnt = 12, 512, 512, 24, 4, 4, 4
    w = moe_ref.make_weights(rng, E, H, I)
    x, logits = moe_ref.make_inputs(rng, T, H, E)
    ids, wts = moe_ref.route_topk(logits, k)
    gamma = moe_ref.f32_to_bf16_bits(rng.standard_normal(H, dtype=np.float32) * np.float32(0.1))
    weights = _weights_from_np(w, dev)
    weights["w13_sf"] = weights["w13_sf"].view(torch.float8_e4m3fn)     # the reference passes e4m3 tensors
    weights["w2_sf"] = weights["w2_sf"].view(torch.float8_e4m3fn)
    weights["post_norm_w"] = torch.from_numpy(gamma.view(np.int16)).to(dev).view(torch.bfloat16)
    state = prepare(weights, local_start=lo, local_count=cnt, n_experts=E)
    xd = torch.from_numpy(x.view(np.int16)).to(dev).view(torch.bfloat16)
    data = {"hidden_states": xd, "topk_ids": torch.from_numpy(ids.astype(np.int64)).to(dev),
            "topk_weights": torch.from_numpy(wts).to(dev),
            "config": {"bs": T, "d_hidden": H, "d_expert": I, "n_experts": E, "local_start": lo, "local_count": cnt,
                       "top_k": k, "sharding": "ep3"}}
    out = kernel_fn(data, state)
    torch.cuda.synchronize()
    want, _ = moe_ref.moe_forward(x, ids, wts, *w, post_norm_w_bits=gamma)  # all experts ...
    want_local = oracle_layer(xd, weights, ids, wts, post_norm_w=weights["post_norm_w"], local_start=lo,
                              local_count=cnt)
    assert_close_bf16(out, want_local)
    # tokens with no local route are exactly zero
    none_local = ~((ids >= lo) & (ids < lo + cnt)).any(axis=1)
    assert not to_np(out.float())[none_local].any()
    assert not np.array_equal(want, want_local)


def test_bad_expert_id_sets_status(dev):
    from xcalibur_b200 import PreparedMoE, _lib

    rng = np.random.default_rng(41)
    E, H, I, T, k = 4, 256, 256, 3, 2
    w = moe_ref.make_weights(rng, E, H, I)
    x, _ = moe_ref.make_inputs(rng, T, H, E)
    layer = PreparedMoE(*_weights_from_np(w, dev).values())
    xd = torch.from_numpy(x.view(np.int16)).to(dev).view(torch.bfloat16)
    ids = torch.tensor([[0, 9], [1, 2], [3, -1]], dtype=torch.int32, device=dev)
    wts = torch.full((T, k), 0.5, dtype=torch.float32, device=dev)
    out = layer.forward(xd, None, topk_ids=ids, topk_weights=wts)
    assert layer.check_device_status() == _lib.XCB_STATUS_BAD_EXPERT
    good = np.array([[0, -5], [1, 2], [3, -5]], np.int32)                # dropped routes -> never local
    assert_close_bf16(out, oracle_layer(xd, _weights_from_np(w, dev), good, to_np(wts)))
    assert layer.check_device_status() == 0


def test_zero_tokens(dev):
    from xcalibur_b200 import PreparedMoE

    rng = np.random.default_rng(42)
    w = moe_ref.make_weights(rng, 4, 256, 256)
    layer = PreparedMoE(*_weights_from_np(w, dev).values())
    out = layer.forward(torch.empty((0, 256), dtype=torch.bfloat16, device=dev),
                        torch.empty((0, 4), device=dev), 2)
    assert out.shape == (0, 256)


# ------------------------------------------------------------------------------------------------ benchmark shapes
def _synthetic(E, H, I, T, seed, dev, bias_std=0.0):
    from xcalibur_b200 import synth

    weights = synth.make_weights(E, H, I, seed=seed, device=dev)
    x, logits = synth.make_inputs(T, H, E, seed=seed + 1, device=dev, bias_std=bias_std)
    return weights, x, logits


@pytest.mark.parametrize("T", [1, 4])
def test_deepseek_decode_parity(dev, T):
    """C2 shape (H=7168, I=2048, E=256, top-8) at T = 1 and 4; the oracle runs on the experts the batch uses."""
    from xcalibur_b200 import PreparedMoE

    weights, x, logits = _synthetic(256, 7168, 2048, T, 100, dev)
    layer = PreparedMoE(*weights.values())
    out, ids, wts = layer.forward(x, logits, 8, return_routing=True)
    torch.cuda.synchronize()
    assert layer.check_device_status() == 0
    want_ids, want_w = moe_ref.route_topk(to_np(logits), 8)
    assert np.array_equal(to_np(ids), want_ids)
    assert_close_bf16(out, oracle_layer(x, weights, want_ids, want_w))


@pytest.mark.parametrize("source", ["logits", "given", "given_pdl"])
def test_deepseek_decode_two_tokens(dev, source):
    """Two tokens at the C2 shape (H=7168, I=2048, top-8): every job holds one token, so the decode kernel stages
    both token rows at start and each phase-A segment reads its token's row (the shape of the expert-parallel decode
    step's local layer at two ranks).  With 16 experts the two tokens share several, so segments of either token
    follow each other in any order; routes from the router, given, and given with PDL."""
    from xcalibur_b200 import PreparedMoE

    weights, x, logits = _synthetic(16, 7168, 2048, 2, 130, dev)
    layer = PreparedMoE(*weights.values())
    if source == "logits":
        out, ids, wts = layer.forward(x, logits, 8, return_routing=True)
        want_ids, want_w = moe_ref.route_topk(to_np(logits), 8)
        torch.cuda.synchronize()
        assert np.array_equal(to_np(ids), want_ids)
    else:
        rng = np.random.default_rng(131)
        want_ids = np.stack([rng.choice(16, 8, replace=False) for _ in range(2)]).astype(np.int32)
        want_w = rng.dirichlet(np.ones(8), size=2).astype(np.float32)
        out = layer.forward(x, None, topk_ids=torch.from_numpy(want_ids).to(dev),
                            topk_weights=torch.from_numpy(want_w).to(dev), pdl=source == "given_pdl")
    torch.cuda.synchronize()
    assert layer.check_device_status() == 0
    assert_close_bf16(out, oracle_layer(x, weights, want_ids, want_w))


def test_many_one_route_jobs_on_a_small_shard(dev):
    """At the C2 hidden size the decode path cuts one-route jobs.  A shard of 8 local experts out of 64, with 32
    tokens that all route to those 8, gives 256 jobs: the workspace's per-job counters must hold one job per route
    (a bound of routes / 8 + local experts would hold 41), and the output must match the oracle."""
    from xcalibur_b200 import PreparedMoE

    weights, x, _ = _synthetic(8, 7168, 2048, 32, 140, dev)
    layer = PreparedMoE(*weights.values(), total_experts=64, expert_offset=0)
    rng = np.random.default_rng(141)
    ids = np.stack([rng.permutation(8) for _ in range(32)]).astype(np.int32)
    wts = rng.dirichlet(np.ones(8), size=32).astype(np.float32)
    out = layer.forward(x, None, topk_ids=torch.from_numpy(ids).to(dev), topk_weights=torch.from_numpy(wts).to(dev),
                        path="decode")
    torch.cuda.synchronize()
    assert layer.check_device_status() == 0
    assert_close_bf16(out, oracle_layer(x, weights, ids, wts))


@pytest.mark.parametrize("T", [1, 8, 64, 512])
def test_qwen3_parity(dev, T):
    """C4 shape (H=2048, I=768, E=128, top-8)."""
    from xcalibur_b200 import PreparedMoE

    weights, x, logits = _synthetic(128, 2048, 768, T, 200, dev)
    layer = PreparedMoE(*weights.values())
    out, ids, wts = layer.forward(x, logits, 8, return_routing=True)
    torch.cuda.synchronize()
    want_ids, want_w = moe_ref.route_topk(to_np(logits), 8)
    assert np.array_equal(to_np(ids), want_ids)
    r = _routing_arrays(layer, T, 8)
    order, pos, _, _ = moe_ref.permute(want_ids, 0, 128)
    assert np.array_equal(r["pos"], pos) and np.array_equal(r["order"], order)
    assert_close_bf16(out, oracle_layer(x, weights, want_ids, want_w))


def test_batch_invariance_at_prefill_size(dev):
    """Size-independent property at the C3 size (T=4096, biased router): each token's output equals the output
    of a small batch holding just that token (itself checked against the oracle above)."""
    from xcalibur_b200 import PreparedMoE

    weights, x, logits = _synthetic(256, 7168, 2048, 4096, 300, dev, bias_std=0.5)
    layer = PreparedMoE(*weights.values())
    out = layer.forward(x, logits, 8)
    torch.cuda.synchronize()
    assert layer.check_device_status() == 0
    rows = torch.tensor([0, 1, 777, 2048, 4095], device=dev)
    small = layer.forward(x.index_select(0, rows), logits.index_select(0, rows), 8)
    torch.cuda.synchronize()
    assert torch.isfinite(out.float()).all()
    got = out.index_select(0, rows)
    assert torch.allclose(got.float(), small.float(), rtol=1e-2, atol=1e-2)


def test_no_local_route_gives_zero_output(dev):
    """Every route outside the held experts: the single-launch path still writes a zero output."""
    from xcalibur_b200 import kernel_fn, prepare

    rng = np.random.default_rng(51)
    E, H, I, T, k = 8, 256, 256, 3, 2
    w = _weights_from_np(moe_ref.make_weights(rng, E, H, I), dev)
    state = prepare(w, local_start=0, local_count=4, n_experts=E)
    x = torch.randn((T, H), device=dev).to(torch.bfloat16)
    ids = torch.tensor([[4, 5], [6, 7], [7, 4]], dtype=torch.int64, device=dev)
    data = {"hidden_states": x, "topk_ids": ids, "topk_weights": torch.full((T, k), 0.5, device=dev),
            "config": {"bs": T, "d_hidden": H, "d_expert": I, "n_experts": E, "local_start": 0, "local_count": 4,
                       "top_k": k, "sharding": "ep2"}}
    out = kernel_fn(data, state)
    torch.cuda.synchronize()
    assert not out.float().abs().sum().item()


def test_repeated_expert_within_a_token(dev):
    """Precomputed routing may name one expert twice for a token (T=1): both routes count."""
    from xcalibur_b200 import PreparedMoE

    rng = np.random.default_rng(52)
    E, H, I, k = 4, 512, 256, 4
    w = moe_ref.make_weights(rng, E, H, I)
    weights = _weights_from_np(w, dev)
    layer = PreparedMoE(*weights.values())
    x, _ = moe_ref.make_inputs(rng, 1, H, E)
    xd = torch.from_numpy(x.view(np.int16)).to(dev).view(torch.bfloat16)
    ids = np.array([[2, 2, 0, 2]], np.int32)
    wts = np.array([[0.4, 0.3, 0.2, 0.1]], np.float32)
    out = layer.forward(xd, None, topk_ids=torch.from_numpy(ids).to(dev), topk_weights=torch.from_numpy(wts).to(dev))
    torch.cuda.synchronize()
    assert_close_bf16(out, oracle_layer(xd, weights, ids, wts))


@pytest.mark.parametrize("T,path", [(1, "decode"), (3, "decode"), (3, "prefill")])
def test_activations_beyond_f16_range(dev, T, path):
    """Activations far outside the f16 range (|x| up to ~1e7) and tiny ones in the same rows: the decode kernel
    converts each token's row to f16 with a power-of-two scale, so the output must still match the oracle."""
    from xcalibur_b200 import PreparedMoE

    rng = np.random.default_rng(60 + T)
    E, H, I, k = 8, 1024, 512, 2
    w = moe_ref.make_weights(rng, E, H, I)
    weights = _weights_from_np(w, dev)
    layer = PreparedMoE(*weights.values())
    x, logits = moe_ref.make_inputs(rng, T, H, E)
    xf = moe_ref.bf16_bits_to_f32(x) * np.float32(3.0e6)
    xf[:, ::7] *= np.float32(1e-12)                      # tiny values beside the large ones
    xd = torch.from_numpy(xf).to(dev).to(torch.bfloat16)
    out, ids, wts = layer.forward(xd, torch.from_numpy(logits).to(dev), k, return_routing=True, path=path)
    torch.cuda.synchronize()
    assert layer.check_device_status() == 0
    ref = moe_ref.bf16_bits_to_f32(oracle_layer(xd, weights, to_np(ids), to_np(wts)))
    got = out.float().cpu().numpy()
    assert np.isfinite(got).all()
    scale = np.abs(ref).max()
    assert np.abs(got - ref).max() <= 1e-2 * scale


def test_bench_reference_arm_experts_match_library(dev):
    """bench.py's reference arm builds its experts without this repository's CUDA library (same fp32 draws,
    quantised on the host by the CPU oracle); they must equal the library-built layer byte for byte, so both arms
    time the same layer."""
    import bench
    from xcalibur_b200 import synth

    cfg = dict(E=12, H=512, I=256)
    full = synth.make_weights(cfg["E"], cfg["H"], cfg["I"], seed=99, device=dev)
    used = np.array([0, 5, 8, 11])
    host = bench.reference_arm_experts(cfg, used, seed=99, device=dev)
    for name in ("w13", "w13_sf", "w13_gs", "w2", "w2_sf", "w2_gs"):
        assert np.array_equal(host[name], to_np(full[name][torch.as_tensor(used, device=dev)])), name


@pytest.mark.parametrize("post_norm", [False, True])
def test_pdl_chained_launches_match_plain_launches(dev, post_norm):
    """Programmatic dependent launch (the reference's PDL switch, moe_w4a16.py:169, :2864-2878): a chain of decode
    calls where each call's input is the previous call's output, launched back to back with PDL, also replayed from a
    CUDA graph.  Without the post-norm the chain equals the same chain launched in plain stream order bit for bit
    (its magnitudes shrink quadratically, so that chain is three calls long).  With it, each route's sum of squares
    is an fp32 atomic sum whose order varies, so last-bit differences would compound along a chain: every link of
    the PDL chain is compared instead with a plain launch on that link's own input."""
    from xcalibur_b200 import PreparedMoE, synth

    E, H, I, T, k = 16, 1024, 512, 2, 4
    weights = synth.make_weights(E, H, I, seed=606, device=dev)
    pn = (torch.randn(H, device=dev) * 0.1).to(torch.bfloat16) if post_norm else None
    layer = PreparedMoE(*weights.values(), pn)
    x, _ = synth.make_inputs(T, H, E, seed=607, device=dev)
    logits = [synth.make_inputs(T, H, E, seed=610 + i, device=dev)[1] for i in range(6 if post_norm else 3)]

    def chain(pdl):
        h = x
        outs = []
        for lg in logits:
            h = layer.forward(h, lg, k, post_norm=post_norm, pdl=pdl)   # reads the previous kernel's output
            outs.append(h)
        return outs

    def check(outs):
        torch.cuda.synchronize()
        assert layer.check_device_status() == 0
        if not post_norm:
            for a, b in zip(plain, outs):
                assert torch.isfinite(a.float()).all() and a.float().abs().max() > 0
                assert torch.equal(a, b)
            return
        for i, (lg, o) in enumerate(zip(logits, outs)):
            ref = layer.forward(x if i == 0 else outs[i - 1].clone(), lg, k, post_norm=True)
            torch.cuda.synchronize()
            assert torch.isfinite(o.float()).all() and o.float().abs().max() > 0
            torch.testing.assert_close(o.float(), ref.float(), rtol=1e-2, atol=1e-2)

    plain = [o.clone() for o in chain(False)]
    check([o.clone() for o in chain(True)])
    s = torch.cuda.Stream(dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(s):
        chain(True)                                        # the stream's workspace exists before capture
    torch.cuda.current_stream(dev).wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        captured = chain(True)
    g.replay()
    check([o.clone() for o in captured])


@pytest.mark.parametrize("scale", [1e-7, 1e-3, 3e4])
def test_decode_keeps_relative_precision_at_any_activation_scale(dev, scale):
    """The decode kernel converts activations to f16 with a per-token power-of-two scale; rows whose largest
    magnitude is far below or above 1 must keep their relative precision (a row of 1e-7 values would otherwise sink
    into f16's subnormal range and a row of 3e4 values overflow it)."""
    from xcalibur_b200 import PreparedMoE

    rng = np.random.default_rng(71)
    E, H, I, T, k = 8, 1024, 512, 3, 2
    w = moe_ref.make_weights(rng, E, H, I)
    x = moe_ref.f32_to_bf16_bits(rng.standard_normal((T, H), dtype=np.float32) * np.float32(scale))
    logits = rng.standard_normal((T, E), dtype=np.float32)
    layer = PreparedMoE(*_weights_from_np(w, dev).values())
    xd = torch.from_numpy(x.view(np.int16)).to(dev).view(torch.bfloat16)
    out = layer.forward(xd, torch.from_numpy(logits).to(dev), k, path="decode")
    torch.cuda.synchronize()
    want, _, _ = moe_ref.moe_layer(x, logits, *w, k)
    wf = moe_ref.bf16_bits_to_f32(want)
    assert np.abs(wf).max() > 0
    assert_close_bf16(out, want, atol=1e-2 * float(np.abs(wf).max()))
