"""HBM read-bandwidth sweep on the current GPU (``python -m xcalibur_b200.probe``).

Runs ``xcb_hbm_probe`` over a few ring shapes and prints one JSON line per shape: the bulk-copy ring the decode
kernel uses (chunk x stages per CTA, with and without the L2 evict-first hint, 1 or 2 CTAs per SM) and plain
16-byte vector loads, each streaming a 4 GiB buffer (far above the 126 MB L2), best of 5 CUDA-event timings.
"""
from __future__ import annotations

import argparse
import ctypes
import json

import torch

from . import _lib


def run(mode, chunk, stages, ctas, threads, buf, status, sink, reps=5, window=0, nreg=0, seed=0):
    """Best-of-reps GB/s; with ``window`` > 0 each launch streams a different window of that many bytes."""
    lib = _lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    n = window or buf.numel()
    best = None
    g = torch.Generator().manual_seed(seed)
    for r in range(reps + 1):
        off = ((r * n) % (buf.numel() - n)) // 1024 * 1024 if window else 0
        regions = None
        if nreg:   # nreg random region starts (1 KB aligned) anywhere in the buffer, like a few random experts
            reg = n // nreg
            starts = torch.randint(0, (buf.numel() - reg) // 1024, (nreg,), generator=g) * 1024
            regions = starts.to(torch.int64).cuda()
            off = 0
        e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
        e0.record()
        _lib.check(lib.xcb_hbm_probe(buf.data_ptr() + off, n, mode, chunk, stages, ctas, threads,
                                     None if regions is None else regions.data_ptr(), nreg,
                                     status.data_ptr(), sink.data_ptr(), stream), "xcb_hbm_probe")
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1)
        best = ms if best is None else min(best, ms)
    return n / (best * 1e-3) / 1e9


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gib", type=float, default=4.0)
    ap.add_argument("--windows", default="", help="comma-separated MiB per launch (rotating offsets), e.g. 66,132,512")
    ap.add_argument("--l2-mb", type=int, default=0,
                    help="L2 read bandwidth instead: every CTA streams the same L2-resident block of this many MiB")
    a = ap.parse_args()
    if a.l2_mb:
        return l2_sweep(a.l2_mb)
    buf = torch.empty(int(a.gib * (1 << 30)), dtype=torch.uint8, device="cuda")
    buf.random_(0, 255)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    sink = torch.zeros(1, dtype=torch.float32, device="cuda")
    ap_shapes = [(2, 0, 0, 1, 256), (2, 0, 0, 2, 256), (2, 0, 0, 4, 256)]
    shapes = list(ap_shapes)
    for mode in (0, 1):
        for chunk, stages in ((4096, 16), (8192, 8), (16384, 8), (18432, 8), (32768, 6)):
            for ctas in (1, 2):
                if stages * chunk * ctas <= 220 * 1024:
                    shapes.append((mode, chunk, stages, ctas, 128))
    # the decode kernel's own shape: 18 KB stages, 16 polling consumer warps + 1 producer warp
    shapes += [(1, 18432, 8, 1, 544), (1, 16384, 8, 1, 544), (1, 18432, 8, 1, 160)]
    windows = [0] if not a.windows else [int(w) << 20 for w in a.windows.split(",")]
    if a.windows:
        shapes = [(1, 18432, 8, 1, 544), (1, 16384, 8, 1, 128), (2, 0, 0, 4, 256)]
    for window in windows:
        for nreg in ([0] + ([8] if window else [])):
            for mode, chunk, stages, ctas, threads in shapes:
                gbs = run(mode, chunk, stages, ctas, threads, buf, status, sink, reps=8 if window else 5,
                          window=window, nreg=nreg)
                print(json.dumps({"mode": ["bulk_ring", "bulk_ring_evict_first", "vector_loads"][mode],
                                  "chunk": chunk, "stages": stages, "ctas_per_sm": ctas, "threads": threads,
                                  "window_mb": window >> 20, "regions": nreg, "gbs": round(gbs, 1),
                                  "status": int(status.item())}), flush=True)


def l2_sweep(mb: int):
    """Every CTA reads the same ``mb`` MiB (regions all at offset 0), so after the first pass the stream is served
    by L2: the figure bounds how fast a kernel can refill shared memory from L2-resident operands."""
    lib = _lib.load()
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    per = mb << 20
    buf = torch.empty(per + (1 << 20), dtype=torch.uint8, device="cuda")
    buf.random_(0, 255)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    sink = torch.zeros(1, dtype=torch.float32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    for chunk, stages, ctas, threads in ((16384, 8, 1, 128), (32768, 6, 1, 128), (16384, 6, 2, 128),
                                         (4096, 16, 1, 128)):
        G = sms * ctas
        regions = torch.zeros(G, dtype=torch.int64, device="cuda")
        total = per * G
        best = None
        for r in range(4):
            e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
            e0.record()
            _lib.check(lib.xcb_hbm_probe(buf.data_ptr(), total, 0, chunk, stages, ctas, threads, regions.data_ptr(), G,
                                         status.data_ptr(), sink.data_ptr(), stream), "xcb_hbm_probe")
            e1.record()
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1)
            best = ms if best is None else min(best, ms)
        print(json.dumps({"mode": "l2_bulk_ring", "block_mb": mb, "chunk": chunk, "stages": stages, "ctas_per_sm": ctas,
                          "gbs": round(total / (best * 1e-3) / 1e9, 1), "status": int(status.item())}), flush=True)


if __name__ == "__main__":
    main()
