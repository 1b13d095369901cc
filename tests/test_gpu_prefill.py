"""GPU parity of the prefill path (tcgen05 grouped GEMMs) against the CPU oracle, and against the decode path.

The prefill path is what xcb_moe_forward runs for more than 256 routes or 32 tokens; these tests force it
(``path="prefill"``) on small batches too, so the oracle stays cheap, and cover ragged token tiles (counts that
are not multiples of 16, 32 or 128), experts with no tokens, experts with several token tiles, post-norm, a local
expert range, repeated calls and graph capture."""
import numpy as np
import pytest
import torch

from oracle import moe_ref
from tests._util import assert_close_bf16, oracle_layer, to_np

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev(cuda_device):
    from xcalibur_b200 import _lib

    _lib.load()
    return cuda_device


def _np_weights(w, dev):
    c13, s13, g13, c2, s2, g2 = w
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    return {"w13": t(c13), "w13_sf": t(s13), "w13_gs": t(g13), "w2": t(c2), "w2_sf": t(s2), "w2_gs": t(g2)}


def _bf16(x, dev):
    return torch.from_numpy(x.view(np.int16)).to(dev).view(torch.bfloat16)


def test_prefill_c1_parity(dev):
    """The C1 configuration (T=16, H=1024, I=512, E=8, top-2) through the prefill path."""
    from xcalibur_b200 import PreparedMoE

    rng = np.random.default_rng(0)
    E, H, I, T, k = 8, 1024, 512, 16, 2
    w = moe_ref.make_weights(rng, E, H, I)
    x, logits = moe_ref.make_inputs(rng, T, H, E)
    layer = PreparedMoE(*_np_weights(w, dev).values())
    out, ids, wts = layer.forward(_bf16(x, dev), torch.from_numpy(logits).to(dev), k, return_routing=True,
                                  path="prefill")
    torch.cuda.synchronize()
    assert layer.check_device_status() == 0
    want_out, want_ids, _ = moe_ref.moe_layer(x, logits, *w, k)
    assert np.array_equal(to_np(ids), want_ids)
    assert_close_bf16(out, want_out)


def test_prefill_ragged_tiles(dev):
    """Token counts per expert of 0, 1, 15, 17, 33, 127, 128, 129, 300: partial MMA widths, partial TMA boxes,
    several token tiles per weight block, and an expert with no tokens at all."""
    from xcalibur_b200 import PreparedMoE

    rng = np.random.default_rng(7)
    E, H, I, k = 9, 512, 256, 1
    counts = [0, 1, 15, 17, 33, 127, 128, 129, 300]
    ids = np.concatenate([np.full(c, e, np.int32) for e, c in enumerate(counts)])
    rng.shuffle(ids)
    T = ids.size
    w = moe_ref.make_weights(rng, E, H, I)
    x, _ = moe_ref.make_inputs(rng, T, H, E)
    wts = rng.uniform(0.5, 1.5, (T, k)).astype(np.float32)
    weights = _np_weights(w, dev)
    layer = PreparedMoE(*weights.values())
    xd = _bf16(x, dev)
    out = layer.forward(xd, None, topk_ids=torch.from_numpy(ids[:, None]).to(dev),
                        topk_weights=torch.from_numpy(wts).to(dev), path="prefill")
    torch.cuda.synchronize()
    assert layer.check_device_status() == 0
    assert_close_bf16(out, oracle_layer(xd, weights, ids[:, None], wts))


def test_prefill_post_norm_local_range(dev):
    """Reference contract (precomputed ids, post-norm, 5 of 12 experts local) through the prefill path."""
    from xcalibur_b200 import PreparedMoE

    rng = np.random.default_rng(31)
    E, H, I, T, k, lo, cnt = 12, 512, 512, 96, 4, 3, 5
    w = moe_ref.make_weights(rng, E, H, I)
    x, logits = moe_ref.make_inputs(rng, T, H, E)
    ids, wts = moe_ref.route_topk(logits, k)
    gamma = moe_ref.f32_to_bf16_bits(rng.standard_normal(H, dtype=np.float32) * np.float32(0.1))
    weights = _np_weights(w, dev)
    gd = torch.from_numpy(gamma.view(np.int16)).to(dev).view(torch.bfloat16)
    sl = slice(lo, lo + cnt)
    layer = PreparedMoE(weights["w13"][sl], weights["w13_sf"][sl], weights["w13_gs"][sl], weights["w2"][sl],
                        weights["w2_sf"][sl], weights["w2_gs"][sl], gd, total_experts=E, expert_offset=lo)
    xd = _bf16(x, dev)
    out = layer.forward(xd, None, topk_ids=torch.from_numpy(ids).to(dev), topk_weights=torch.from_numpy(wts).to(dev),
                        post_norm=True, path="prefill")
    torch.cuda.synchronize()
    assert layer.check_device_status() == 0
    want = oracle_layer(xd, weights, ids, wts, post_norm_w=gd, local_start=lo, local_count=cnt)
    assert_close_bf16(out, want)


def test_prefill_deepseek_shapes(dev):
    """DeepSeek-V3 expert shapes (H=7168, I=2048, 256 experts, top-8): full 28-stage reduction for gate_up,
    56 row blocks for down; 4 tokens keep the oracle to 32 experts."""
    from xcalibur_b200 import PreparedMoE, synth

    weights = synth.make_weights(256, 7168, 2048, seed=100, device=dev)
    x, logits = synth.make_inputs(4, 7168, 256, seed=101, device=dev)
    layer = PreparedMoE(*weights.values())
    out, ids, wts = layer.forward(x, logits, 8, return_routing=True, path="prefill")
    torch.cuda.synchronize()
    assert layer.check_device_status() == 0
    want_ids, want_w = moe_ref.route_topk(to_np(logits), 8)
    assert np.array_equal(to_np(ids), want_ids)
    assert_close_bf16(out, oracle_layer(x, weights, want_ids, want_w))


def test_prefill_matches_decode_path(dev):
    """Both kernels on the same 200-token batch (Qwen3-shaped experts, skewed router)."""
    from xcalibur_b200 import PreparedMoE, synth

    weights = synth.make_weights(128, 2048, 768, seed=400, device=dev)
    x, logits = synth.make_inputs(200, 2048, 128, seed=401, device=dev, bias_std=0.5)
    layer = PreparedMoE(*weights.values())
    a = layer.forward(x, logits, 8, path="prefill").clone()
    b = layer.forward(x, logits, 8, path="decode").clone()
    torch.cuda.synchronize()
    assert layer.check_device_status() == 0
    assert torch.allclose(a.float(), b.float(), rtol=1e-2, atol=1e-2)
    rel = (a.float() - b.float()).norm() / b.float().norm()
    assert rel < 5e-3


@pytest.mark.parametrize("deterministic", [True, False])
def test_prefill_repeat_and_graph_capture(dev, deterministic):
    """Repeated calls and a CUDA-graph replay: bit-identical with the fixed-order combine pass; with the combine
    fused into the down projection (fp32 reductions in a varying order) within the tolerance."""
    from xcalibur_b200 import PreparedMoE, synth

    weights = synth.make_weights(32, 1024, 512, seed=500, device=dev)
    x, logits = synth.make_inputs(333, 1024, 32, seed=501, device=dev)
    layer = PreparedMoE(*weights.values())
    fwd = lambda: layer.forward(x, logits, 4, deterministic=deterministic)
    outs = [fwd().clone() for _ in range(2)]        # 1332 routes: prefill path by default

    def same(a, b):
        if deterministic:
            return torch.equal(a, b)
        return torch.allclose(a.float(), b.float(), rtol=1e-2, atol=1e-2)

    assert same(outs[0], outs[1])
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        static_out = fwd()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            static_out = fwd()
    torch.cuda.current_stream().wait_stream(s)
    for _ in range(2):
        g.replay()
    torch.cuda.synchronize()
    assert same(static_out, outs[0])
    assert layer.check_device_status() == 0


def test_fused_combine_matches_the_fixed_order_pass(dev):
    """The weighted combine fused into the down projection against the separate fixed-order pass, and both against
    the oracle (Qwen3-shaped experts, 700 tokens, skewed router)."""
    from xcalibur_b200 import PreparedMoE, synth

    weights = synth.make_weights(128, 2048, 768, seed=510, device=dev)
    x, logits = synth.make_inputs(700, 2048, 128, seed=511, device=dev, bias_std=0.5)
    layer = PreparedMoE(*weights.values())
    fused, ids, wts = layer.forward(x, logits, 8, return_routing=True)
    fixed = layer.forward(x, logits, 8, deterministic=True)
    torch.cuda.synchronize()
    assert layer.check_device_status() == 0
    assert torch.allclose(fused.float(), fixed.float(), rtol=1e-2, atol=1e-2)
    rows = sample_rows(to_np(ids))
    sel = torch.as_tensor(rows, device=dev)
    want = oracle_layer(x.index_select(0, sel), weights, to_np(ids)[rows], to_np(wts)[rows])
    assert_close_bf16(fused.index_select(0, sel), want)
    assert_close_bf16(fixed.index_select(0, sel), want)


@pytest.mark.parametrize("T,k,E,ties", [(600, 4, 64, False), (3000, 8, 256, True), (1100, 3, 40, False)])
def test_chunked_router_bit_exact(dev, T, k, E, ties):
    """Above 2048 routes the router runs as three multi-CTA kernels; ids, weights and the stable permutation must
    equal the oracle's bit for bit (chunks of whole tokens, including a top-k that does not divide 1024)."""
    import ctypes

    from xcalibur_b200 import PreparedMoE

    rng = np.random.default_rng(T + k)
    H, I = 256, 256
    w = moe_ref.make_weights(rng, E, H, I)
    x, logits = moe_ref.make_inputs(rng, T, H, E)
    if ties:
        logits = rng.integers(-3, 4, (T, E)).astype(np.float32)
    layer = PreparedMoE(*_np_weights(w, dev).values())
    xd = _bf16(x, dev)
    out, ids, wts = layer.forward(xd, torch.from_numpy(logits).to(dev), k, return_routing=True)
    torch.cuda.synchronize()
    assert layer.check_device_status() == 0
    want_ids, want_w = moe_ref.route_topk(logits, k)
    assert np.array_equal(to_np(ids), want_ids)
    assert np.allclose(to_np(wts), want_w, rtol=1e-6, atol=1e-7)
    ws = layer.workspace(T, k)
    offs = (ctypes.c_size_t * 6)()
    assert layer.lib.xcb_moe_workspace_offsets(ctypes.byref(layer.shape), T, k, offs, 6) == 6
    i32 = lambda o, n: to_np(ws[o:o + 4 * n].view(torch.int32))
    order, pos, counts, offsets = moe_ref.permute(want_ids, 0, E)
    assert np.array_equal(i32(offs[2], T * k), pos)
    assert np.array_equal(i32(offs[3], T * k), order)
    assert np.array_equal(i32(offs[4], E), counts)
    assert np.array_equal(i32(offs[5], E + 1), offsets)


# ------------------------------------------------------------------------------------------------ full sizes
def sample_rows(ids: np.ndarray, n: int = 32) -> np.ndarray:
    """n token rows for an oracle check at full size: tokens on the most- and the least-loaded experts, then
    tokens chosen greedily to add as few new experts as possible (the oracle dequantises only the experts the
    sampled rows use)."""
    T, k = ids.shape
    counts = np.bincount(ids.reshape(-1), minlength=int(ids.max()) + 1)
    used = np.nonzero(counts)[0]
    picks = []
    for e in (used[np.argmax(counts[used])], used[np.argmin(counts[used])], used[np.argsort(counts[used])[1]]):
        t = int(np.nonzero((ids == e).any(axis=1))[0][0])
        if t not in picks:
            picks.append(t)
    have = np.zeros(counts.size, dtype=bool)
    for t in picks:
        have[ids[t]] = True
    while len(picks) < n:
        new = (~have[ids]).sum(axis=1)
        new[picks] = k + 1
        t = int(np.argmin(new))
        picks.append(t)
        have[ids[t]] = True
    return np.array(sorted(picks))


def _full_size_check(dev, E, H, I, T, k, seed, bias_std):
    from xcalibur_b200 import PreparedMoE, synth

    weights = synth.make_weights(E, H, I, seed=seed, device=dev)
    x, logits = synth.make_inputs(T, H, E, seed=seed + 1, device=dev, bias_std=bias_std)
    layer = PreparedMoE(*weights.values())
    out, ids, wts = layer.forward(x, logits, k, return_routing=True)      # the path the library picks
    torch.cuda.synchronize()
    assert layer.check_device_status() == 0
    want_ids, want_w = moe_ref.route_topk(to_np(logits), k)
    assert np.array_equal(to_np(ids), want_ids)                           # every row, bit for bit
    assert np.allclose(to_np(wts), want_w, rtol=1e-5, atol=1e-7)          # softmax weights: fp32 rounding only
    assert torch.isfinite(out.float()).all()
    rows = sample_rows(want_ids)
    sel = torch.as_tensor(rows, device=dev)
    want = oracle_layer(x.index_select(0, sel), weights, want_ids[rows], want_w[rows])
    assert_close_bf16(out.index_select(0, sel), want)
    return want_ids, rows


@pytest.mark.parametrize("T", [64, 96])
def test_deepseek_v3_mid_batch_on_the_decode_path(dev, T):
    """64 and 96 tokens at the DeepSeek-V3 shape (up to 3 routes per expert): the library takes the decode path with
    the separate router; ids and weights of every route exact, 32 sampled rows against the oracle."""
    import ctypes

    from xcalibur_b200 import _lib

    shape = _lib.XcbMoeShape(256, 256, 0, 7168, 2048)
    out = (ctypes.c_int32 * 8)()
    assert _lib.load().xcb_moe_plan_info(ctypes.byref(shape), T, 8, 0, 0, out, 8) == 8
    assert out[0] == 0 and out[1] == 0  # decode path, routes from the router kernel
    _full_size_check(dev, 256, 7168, 2048, T, 8, 320 + T, 0.0)


def test_prefill_deepseek_v3_t4096_sampled_rows(dev):
    """Configuration 3 at its full size (T = 4096, DeepSeek-V3 shape, router bias N(0, 0.5)): ids and weights of
    all 32768 routes bit-exact, and 32 rows (on the hottest and the coldest experts, and rows sharing experts)
    against the oracle."""
    ids, rows = _full_size_check(dev, 256, 7168, 2048, 4096, 8, 300, 0.5)
    counts = np.bincount(ids.reshape(-1), minlength=256)
    hit = np.unique(ids[rows])
    assert counts.argmax() in hit and counts[counts > 0].min() in counts[hit]


@pytest.mark.parametrize("T", [2048, 8192])
def test_qwen3_large_batches_sampled_rows(dev, T):
    """Configuration 4 at T = 2048 and 8192 (Qwen3-30B-A3B shape, H=2048, I=768, 128 experts, top-8)."""
    _full_size_check(dev, 128, 2048, 768, T, 8, 500 + T, 0.0)
