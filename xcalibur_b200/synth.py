"""Seeded synthetic NVFP4 layers on the GPU (benchmark and test inputs; no public dataset is involved).

Weights follow the recipe of the benchmark configurations: gate_up [E, 2I, H] and down [E, H, I] drawn fp32
N(0, std), quantised to NVFP4 by the library's GPU quantiser (``xcb_nvfp4_quantize``; bit-exact with the CPU
oracle's quantiser), one expert at a time so the fp32 staging stays small.  Activations are bf16 N(0, 1); router
logits fp32 N(0, 1) plus an optional per-expert bias.
"""
from __future__ import annotations

import math

import torch

from . import _lib
from ._lib import check


def quantize(w: torch.Tensor):
    """fp32 [E, R, K] CUDA tensor -> (codes uint8 [E, R, K/2], sf uint8 [E, R, K/16], gs fp32 [E])."""
    lib = _lib.load()
    E, R, K = w.shape
    w = w.contiguous()
    codes = torch.empty((E, R, K // 2), dtype=torch.uint8, device=w.device)
    sf = torch.empty((E, R, K // 16), dtype=torch.uint8, device=w.device)
    gs = torch.empty(E, dtype=torch.float32, device=w.device)
    amax = torch.empty(E, dtype=torch.float32, device=w.device)
    check(lib.xcb_nvfp4_quantize(w.data_ptr(), E, R, K, codes.data_ptr(), sf.data_ptr(), gs.data_ptr(),
                                 amax.data_ptr(), torch.cuda.current_stream(w.device).cuda_stream),
          "xcb_nvfp4_quantize")
    return codes, sf, gs


def make_weights(E: int, H: int, I: int, seed: int = 0, device="cuda", std: float = 0.02, chunk: int = 8):
    """Reference-layout NVFP4 weights dict (w13, w13_sf, w13_gs, w2, w2_sf, w2_gs) built on the GPU."""
    device = torch.device(device)
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    out = {
        "w13": torch.empty((E, 2 * I, H // 2), dtype=torch.uint8, device=device),
        "w13_sf": torch.empty((E, 2 * I, H // 16), dtype=torch.uint8, device=device),
        "w13_gs": torch.empty(E, dtype=torch.float32, device=device),
        "w2": torch.empty((E, H, I // 2), dtype=torch.uint8, device=device),
        "w2_sf": torch.empty((E, H, I // 16), dtype=torch.uint8, device=device),
        "w2_gs": torch.empty(E, dtype=torch.float32, device=device),
    }
    for e0 in range(0, E, chunk):
        n = min(chunk, E - e0)
        w = torch.randn((n, 2 * I, H), generator=g, device=device, dtype=torch.float32) * std
        c, s, gs = quantize(w)
        out["w13"][e0:e0 + n], out["w13_sf"][e0:e0 + n], out["w13_gs"][e0:e0 + n] = c, s, gs
        del w
        w = torch.randn((n, H, I), generator=g, device=device, dtype=torch.float32) * std
        c, s, gs = quantize(w)
        out["w2"][e0:e0 + n], out["w2_sf"][e0:e0 + n], out["w2_gs"][e0:e0 + n] = c, s, gs
        del w
    return out


def make_inputs(T: int, H: int, E: int, seed: int = 1, device="cuda", bias_std: float = 0.0, zipf_s: float = 0.0,
                zipf_order_seed=None):
    """bf16 N(0,1) activations [T, H] and fp32 router logits [T, E] (N(0,1) + per-expert bias).

    ``bias_std``: bias ~ N(0, bias_std) per expert (mildly uneven loads).  ``zipf_s``: bias_e = -s * ln(r_e + 1), a
    Zipf-like skew, with r_e = e (toward low expert ids: the worst case for contiguous expert sharding) or, with
    ``zipf_order_seed``, expert e's place in a seeded random order (the same on every rank and call)."""
    device = torch.device(device)
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    x = torch.randn((T, H), generator=g, device=device, dtype=torch.float32).to(torch.bfloat16)
    logits = torch.randn((T, E), generator=g, device=device, dtype=torch.float32)
    if bias_std:
        logits += torch.randn((1, E), generator=g, device=device, dtype=torch.float32) * bias_std
    if zipf_s:
        r = torch.arange(E, device=device)
        if zipf_order_seed is not None:
            gp = torch.Generator(device="cpu")
            gp.manual_seed(int(zipf_order_seed))
            r = torch.randperm(E, generator=gp).to(device)
        logits += (-zipf_s * torch.log(r.to(torch.float32) + 1.0))[None, :]
    return x, logits


def layer_bytes(U: int, H: int, I: int) -> int:
    """Algorithmic HBM bytes of the weights of U distinct experts: FP4 codes + E4M3 scales + 2 x 4 B global scales."""
    per = (2 * I * H) // 2 + (2 * I * H) // 16 + (H * I) // 2 + (H * I) // 16 + 8
    return U * per


def layer_flops(T: int, k: int, H: int, I: int) -> int:
    return 2 * T * k * (2 * I * H + H * I)


def nearest_pow2(x: int) -> int:
    return 1 << max(0, math.ceil(math.log2(max(1, x))))
