"""Benchmark of the B200 NVFP4 MoE layer (one JSON line on rank 0).

Default workload (N=1): the DeepSeek-V3-shaped decode layer (configuration 2: T=1, H=7168, I=2048, E=256,
top-8), HBM-bound.  ``--config prefill`` runs configuration 3 (T=4096, biased router), ``--config qwen:T`` the
Qwen3-30B-A3B shape, ``--config ep`` configuration 5 (16384 tokens per GPU, Zipf-biased router).  A step is one
full layer (router + experts + combine) over one batch.  With N > 1 GPUs (torchrun) the layer runs expert-parallel:
each GPU holds E / N experts and its own tokens, which travel to the experts' GPUs and back (weak scaling).

* ``value``: tokens/s over all ranks, inputs resident in HBM, CUDA events on the launching stream, max over ranks.
  Weights are 6.3 GB resident (>> 126 MB L2) and every step uses a different input from a pool of 64, so each
  step streams experts that the previous steps did not touch.
* ``e2e``: the same metric through the public API with pinned HOST inputs: every step copies x and the router
  logits host->device, runs the layer and copies the output device->host; on one GPU the copies run on a second
  stream against two device buffer sets (a serving loop's double buffering), on several GPUs in line with the
  captured step.
* ``roofline``: the experts kernel (``skinny_kernel``), timed with events (over the K back-to-back launches when a
  step is one launch; ``kernel_ms_bracketed`` brackets every launch):
  algorithmic bytes = distinct experts touched x (FP4 codes + E4M3 scales + global scales) + x + out.
* ``cpu_baseline``: the CPU oracle (a torch/numpy fp32 restatement of the layer; the reference has no CPU
  implementation) on the host cores, on a bounded sample (one token for decode).
* ``--impl reference``: times that same CPU restatement per step (the reference arm; rank 0 only).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

CONFIGS = {
    "decode": dict(workload="deepseek_v3_moe_decode", E=256, H=7168, I=2048, T=1, k=8, bias_std=0.0),
    "prefill": dict(workload="deepseek_v3_moe_prefill", E=256, H=7168, I=2048, T=4096, k=8, bias_std=0.5),
    # configuration 5: 16384 tokens per GPU, Zipf(s=1.1) router bias bias_e = -1.1 ln(r_e + 1) where r_e is expert
    # e's place in a seeded random order (seed 77), so the hot experts fall on different ranks of the contiguous
    # expert shards (with r_e = e, every hot expert would sit on rank 0)
    "ep": dict(workload="deepseek_v3_moe_ep", E=256, H=7168, I=2048, T=16384, k=8, bias_std=0.0, zipf=1.1,
               zipf_order_seed=77),
}
METRIC = "MoE layer tokens/s; decode HBM GB/s & prefill TFLOPS vs B200 roofline"


def config_for(name: str, experts: int = 0, tokens: int = 0) -> dict:
    if name.startswith("okc"):
        # the reference operator's own shape and contract (H = I = 4096, 32 of 256 experts local, top-8,
        # precomputed routes, post-norm), at one of its six judged loads (1, 16, 32 decode; 8, 128, 256 verify)
        T = int(name.split(":")[1]) if ":" in name else 1
        return dict(workload=f"okc_moe_w4a16_T{T}", E=256, H=4096, I=4096, T=T, k=8, bias_std=0.0, zipf=0.0,
                    local=32)
    if name.startswith("qwen"):
        T = int(name.split(":")[1]) if ":" in name else 64
        cfg = dict(workload=f"qwen3_30b_a3b_moe_T{T}", E=128, H=2048, I=768, T=T, k=8, bias_std=0.0)
    else:
        cfg = dict(CONFIGS[name])
    cfg.setdefault("zipf", 0.0)
    if experts:
        cfg["E"] = experts
        cfg["workload"] += f"_E{experts}"
    if tokens:
        cfg["T"] = tokens
        cfg["workload"] += f"_T{tokens}"
    return cfg


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="xcb", choices=["xcb", "reference"])
    ap.add_argument("--config", default=None,
                    help="decode (1 GPU default), prefill, qwen:T, ep, okc:T; with several GPUs the default prints "
                         "the ep line (configuration 5), then the expert-parallel decode line")
    ap.add_argument("--pool", type=int, default=64)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-sample-tokens", type=int, default=1)
    ap.add_argument("--experts", type=int, default=0, help="override the expert count (small profiling cases)")
    ap.add_argument("--tokens", type=int, default=0, help="override the token count (small profiling cases)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--pdl", type=int, default=1, help="1 (default): decode steps use programmatic dependent launch")
    ap.add_argument("--path", default="auto", choices=["auto", "decode", "prefill"],
                    help="okc configurations: force this library's decode or prefill path")
    return ap.parse_args()


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d["hbm_gbs"], d["bf16_tflops"], d.get("bf16_tflops_sustained", d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, 1400.0, "fallback"


def load_traffic(workload: str):
    p = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(p):
        return json.load(open(p)).get(workload)
    return None


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 100 ms during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-i", str(self.index), "-lms", "100"], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.25)
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


# ----------------------------------------------------------------------------------------------- CPU baseline
def sample_routes(logits, k, tokens: int):
    """Top-k routes of the first `tokens` tokens (CPU oracle router) and the distinct experts they use."""
    import numpy as np

    from oracle import moe_ref

    ids, wts = moe_ref.route_topk(logits[:tokens].float().cpu().numpy(), k)
    return ids, wts, np.unique(ids)


def cpu_oracle_sample(host, used, x, ids, wts, tokens: int):
    """Time the CPU oracle on the first `tokens` tokens; `host` holds the reference-layout arrays of the experts
    `used` (in that order).  Returns (seconds, tokens, cores)."""
    import numpy as np
    import torch

    from oracle import moe_ref

    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    remap = {int(e): i for i, e in enumerate(used)}
    cid = np.vectorize(remap.get)(ids).astype(np.int32)
    xb = x[:tokens].contiguous().view(torch.int16).cpu().numpy().view(np.uint16)
    t0 = time.perf_counter()
    moe_ref.moe_forward(xb, cid, wts, host["w13"], host["w13_sf"], host["w13_gs"], host["w2"], host["w2_sf"],
                        host["w2_gs"])
    return time.perf_counter() - t0, tokens, cores


def host_experts(weights_dev, used):
    """The reference-layout arrays of the experts `used`, copied to the host from the device weights."""
    import torch

    sel = torch.as_tensor(used, device=weights_dev["w13"].device)
    return {n: weights_dev[n].index_select(0, sel).cpu().numpy() for n in weights_dev}


def reference_arm_experts(cfg, used, seed: int, device, std: float = 0.02, chunk: int = 8):
    """The experts `used` of the seeded synthetic layer, built without this repository's CUDA library: the same
    fp32 draws as ``xcalibur_b200.synth.make_weights`` (one device generator, gate_up then down per chunk of
    `chunk` experts), quantised on the host by the CPU oracle's NVFP4 quantiser (bit-exact with the library's)."""
    import numpy as np
    import torch

    from oracle import nvfp4

    E, H, I = cfg["E"], cfg["H"], cfg["I"]
    want = set(int(e) for e in used)
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    got = {}
    for e0 in range(0, E, chunk):
        n = min(chunk, E - e0)
        for name, shape in (("w13", (n, 2 * I, H)), ("w2", (n, H, I))):
            w = torch.randn(shape, generator=g, device=device, dtype=torch.float32) * std
            for e in range(e0, e0 + n):
                if e in want:
                    c, sf, gs = nvfp4.quantize(w[e - e0:e - e0 + 1].cpu().numpy())
                    got[(name, e)] = (c[0], sf[0], gs[0])
            del w
    order = [int(e) for e in used]
    host = {}
    for name in ("w13", "w2"):
        host[name] = np.stack([got[(name, e)][0] for e in order])
        host[name + "_sf"] = np.stack([got[(name, e)][1] for e in order])
        host[name + "_gs"] = np.array([got[(name, e)][2] for e in order], dtype=np.float32)
    return host


# ----------------------------------------------------------------------------------------------- main arm
def run_xcb(a, cfg, rank, world, dist):
    import torch

    from xcalibur_b200 import PreparedMoE, synth

    local = int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    E, H, I, T, k = cfg["E"], cfg["H"], cfg["I"], cfg["T"], cfg["k"]
    weights = synth.make_weights(E, H, I, seed=1234, device=dev)
    layer = PreparedMoE(*weights.values())
    cpu = None
    if rank == 0 and not a.no_cpu_baseline:
        x0, l0 = synth.make_inputs(T, H, E, seed=1, device=dev, bias_std=cfg["bias_std"], zipf_s=cfg["zipf"],
                                   zipf_order_seed=cfg.get("zipf_order_seed"))
        n0 = min(T, a.cpu_sample_tokens)
        ids0, wts0, used0 = sample_routes(l0, k, n0)
        cpu = cpu_oracle_sample(host_experts(weights, used0), used0, x0, ids0, wts0, n0)
    del weights                                       # only the packed copy stays resident
    torch.cuda.empty_cache()
    P = max(1, a.pool if T <= 64 else 2)
    xs, lgs = [], []
    for i in range(P):
        x, lg = synth.make_inputs(T, H, E, seed=1000 * rank + i + 1, device=dev, bias_std=cfg["bias_std"],
                                  zipf_s=cfg["zipf"], zipf_order_seed=cfg.get("zipf_order_seed"))
        xs.append(x)
        lgs.append(lg)
    outs = [torch.empty((T, H), dtype=torch.bfloat16, device=dev) for _ in range(P)]
    calls = [layer.build_call(xs[i], lgs[i], k, out=outs[i], return_routing=True, pdl=bool(a.pdl)) for i in range(P)]
    torch.cuda.synchronize()
    # distinct experts per input (for the algorithmic byte count)
    for c in calls:
        c.launch()
    torch.cuda.synchronize()
    if layer.check_device_status():
        raise RuntimeError("device status bits set during warm-up")
    U = [int(torch.unique(c.ids_out).numel()) for c in calls]

    def step(i, ev_a=None, ev_b=None):
        c = calls[i % P]
        c.launch("route")
        if ev_a is not None:
            ev_a.record()
        c.launch("experts")
        if ev_b is not None:
            ev_b.record()

    for i in range(a.warmup):
        step(i)
    torch.cuda.synchronize()
    K = a.steps
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(K)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = ClockSampler(dev.index)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    clocks.start()
    start.record()
    for i in range(K):
        step(i)
    end.record()
    torch.cuda.synchronize()
    clk = clocks.stop()
    if dist:
        dist.barrier()
    ms = start.elapsed_time(end) / K
    # per-launch kernel time for the roofline: the same K steps again, each launch bracketed by CUDA events on its
    # stream (two event records per step cost the loop ~3 us, so the throughput above is timed without them)
    for i in range(K):
        step(i, *ev[i])
    torch.cuda.synchronize()
    kern_ms = sum(e_a.elapsed_time(e_b) for e_a, e_b in ev) / K
    u_avg = sum(U[i % P] for i in range(K)) / K
    if layer.check_device_status():
        raise RuntimeError("device status bits set in the timed region")

    # ---- end to end through the public API with pinned host buffers
    e2e_ms = None
    if not a.no_e2e:
        e2e_ms = run_e2e(a, layer, xs, lgs, k, P, dist)
    if dist:
        import torch.distributed as td

        t = torch.tensor([ms, kern_ms, e2e_ms or 0.0], dtype=torch.float64, device=dev)
        td.all_reduce(t, op=td.ReduceOp.MAX)
        ms, kern_ms, e2e_ms = t.tolist()
        e2e_ms = e2e_ms or None
    # a step of the decode path (in-kernel routing) is one launch of the kernel: its average duration is the timed
    # window over the K back-to-back launches; otherwise the kernels are timed between events around each step's
    # expert launches
    single = T * k <= 256 and T <= 32
    res = finish(a, cfg, world, ms, ms if single else kern_ms, e2e_ms, u_avg, P, clk, cpu)
    res["roofline"]["kernel_timing"] = (
        "CUDA events around the K back-to-back launches of the timed region (one launch per step)" if single else
        "CUDA events around each step's expert launches, in a second pass over the same K steps")
    res["roofline"]["kernel_ms_bracketed"] = round(kern_ms, 5)  # events around every single launch
    if res.get("e2e"):
        res["e2e"]["copies"] = ("pinned host buffers; each step's inputs uploaded and result read back on a second "
                                "stream, overlapping the neighbouring steps' compute (two device buffer sets)")
    return res


def make_ep_layer(cfg, rank, world):
    """This rank's shard of the seeded DeepSeek-V3-shaped layer, as an expert-parallel layer (collective)."""
    import torch

    from xcalibur_b200 import synth
    from xcalibur_b200.ep import ExpertParallelMoE

    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    E, H, I = cfg["E"], cfg["H"], cfg["I"]
    epr = E // world
    weights = synth.make_weights(E, H, I, seed=1234, device=dev)      # same layer on every rank; keep this shard
    shard = {n: t[rank * epr:(rank + 1) * epr].contiguous() for n, t in weights.items()}
    del weights
    torch.cuda.empty_cache()
    layer = ExpertParallelMoE(*shard.values(), total_experts=E)
    del shard
    return layer


def run_xcb_ep(a, cfg, rank, world, dist, layer):
    """N > 1: expert parallelism.  Every rank holds E / N experts and its own T tokens (weak scaling); a step is one
    layer over every rank's tokens: router, dispatch (NCCL all-to-all over NVLink), the local experts, return and
    combine.  Timed with CUDA events, max over ranks."""
    import torch
    import torch.distributed as td

    from xcalibur_b200 import synth
    from xcalibur_b200.ep import ExpertParallelMoE

    local = int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device("cuda", local)
    E, H, I, T, k = cfg["E"], cfg["H"], cfg["I"], cfg["T"], cfg["k"]
    epr = E // world
    P = max(1, a.pool if T <= 64 else 2)
    xs, lgs = [], []
    for i in range(P):
        x, lg = synth.make_inputs(T, H, E, seed=1000 * rank + i + 1, device=dev, bias_std=cfg["bias_std"],
                                  zipf_s=cfg["zipf"], zipf_order_seed=cfg.get("zipf_order_seed"))
        xs.append(x)
        lgs.append(lg)
    for i in range(max(3, a.warmup)):
        layer.forward(xs[i % P], lgs[i % P], k)
    torch.cuda.synchronize()
    if layer.ops.device_status() or layer.ops.layer.check_device_status():
        raise RuntimeError("device status bits set during warm-up")
    U, R = [], []
    for i in range(P):  # experts this rank streams and routes it computes, per input
        layer.forward(xs[i], lgs[i], k)
        rid = layer.last["recv_ids"]
        loc = rid[(rid >= rank * epr) & (rid < (rank + 1) * epr)]
        U.append(int(torch.unique(loc).numel()))
        R.append(int(loc.numel()))
    # small batches: the whole step (router, dense exchange, local experts, combine) is captured once in a CUDA graph
    # over static input buffers and replayed, so the host issues one launch per step; every rank captures the same
    # collectives in the same order
    graph = None
    if T <= ExpertParallelMoE.DENSE_MAX_TOKENS:
        xg, lg = xs[0].clone(), lgs[0].clone()
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            for _ in range(3):
                layer.forward(xg, lg, k)
        torch.cuda.current_stream(dev).wait_stream(side)
        torch.cuda.synchronize()
        td.barrier()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):
            out_g = layer.forward(xg, lg, k)
        torch.cuda.synchronize()

    def step(i):
        if graph is None:
            return layer.forward(xs[i % P], lgs[i % P], k)
        xg.copy_(xs[i % P], non_blocking=True)
        lg.copy_(lgs[i % P], non_blocking=True)
        graph.replay()
        return out_g

    for i in range(3):
        step(i)
    K = a.steps
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = ClockSampler(dev.index)
    td.barrier()
    torch.cuda.synchronize()
    clocks.start()
    start.record()
    for i in range(K):
        step(i)
    end.record()
    torch.cuda.synchronize()
    clk = clocks.stop()
    td.barrier()
    ms = start.elapsed_time(end) / K
    # end to end: pinned host inputs in, output out, every step
    e2e_ms = None
    if not a.no_e2e:
        xh = [x.cpu().pin_memory() for x in xs]
        lh = [l.cpu().pin_memory() for l in lgs]
        oh = torch.empty((T, H), dtype=torch.bfloat16).pin_memory()
        xd, ld = torch.empty_like(xs[0]), torch.empty_like(lgs[0])
        td.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(K):
            if graph is None:
                xd.copy_(xh[i % P], non_blocking=True)
                ld.copy_(lh[i % P], non_blocking=True)
                oh.copy_(layer.forward(xd, ld, k), non_blocking=True)
            else:
                xg.copy_(xh[i % P], non_blocking=True)
                lg.copy_(lh[i % P], non_blocking=True)
                graph.replay()
                oh.copy_(out_g, non_blocking=True)
        e1.record()
        torch.cuda.synchronize()
        e2e_ms = e0.elapsed_time(e1) / K
    if layer.ops.device_status() or layer.ops.layer.check_device_status():
        raise RuntimeError("device status bits set in the timed region")
    t = torch.tensor([ms, e2e_ms or 0.0], dtype=torch.float64, device=dev)
    td.all_reduce(t, op=td.ReduceOp.MAX)
    ms, e2e_ms = t[0].item(), (t[1].item() or None)
    if graph is not None:
        del graph  # a graph holding NCCL calls must be released before the process group is destroyed
        torch.cuda.synchronize()
    dense_p2p = T <= ExpertParallelMoE.DENSE_MAX_TOKENS and layer.p2p is not None
    p2p_error = layer.p2p_error
    u_avg = sum(U[i % P] for i in range(K)) / K
    r_avg = sum(R[i % P] for i in range(K)) / K
    # every rank's streamed experts and computed routes: the roofline is the per-GPU mean over the slowest rank's time
    tot = torch.tensor([u_avg, r_avg], dtype=torch.float64, device=dev)
    mx = tot.clone()
    td.all_reduce(tot, op=td.ReduceOp.SUM)
    td.all_reduce(mx, op=td.ReduceOp.MAX)
    u_mean, r_mean = tot[0].item() / world, tot[1].item() / world
    u_max, r_max = mx[0].item(), mx[1].item()
    res = finish(a, cfg, world, ms, ms, e2e_ms, u_avg, P, clk, None)
    hbm, bf16, bf16_sus, src = load_peaks()
    if T <= 64:
        achieved = (synth.layer_bytes(1, H, I) * u_mean + 2 * T * H * 2) / (ms * 1e-3) / 1e9
        busiest = (synth.layer_bytes(1, H, I) * u_max + 2 * T * H * 2) / (ms * 1e-3) / 1e9
        res["roofline"] = {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                           "frac": round(achieved / hbm, 4), "peak_source": src, "traffic": None,
                           "busiest_rank_frac": round(busiest / hbm, 4)}
    else:
        achieved = 2 * r_mean * 3 * H * I / (ms * 1e-3) / 1e12
        busiest = 2 * r_max * 3 * H * I / (ms * 1e-3) / 1e12
        res["roofline"] = {"bound": "tensor", "achieved": round(achieved, 1), "peak": bf16_sus, "unit": "TFLOP/s",
                           "frac": round(achieved / bf16_sus, 4), "peak_source": src + " (sustained)", "traffic": None,
                           "busiest_rank_frac": round(busiest / bf16_sus, 4)}
    res["roofline"]["per_rank"] = ("achieved = the mean over ranks of the routes (or experts) each computed, over the "
                                   "max-over-ranks step time; busiest_rank_frac = the rank with the most")
    res["roofline"]["kernel"] = "whole expert-parallel step per rank (router, dispatch, local experts, combine)"
    res["roofline"]["step_ms"] = round(ms, 5)
    res["config"]["parallelism"] = f"ep{world}"
    if cfg.get("zipf"):
        res["config"]["router_bias"] = (f"zipf(s={cfg['zipf']}): bias_e = -s ln(r_e + 1), r_e = place of expert e in a "
                                        f"seeded random order (seed {cfg.get('zipf_order_seed')})")
    res["config"]["step_launch"] = "one CUDA graph replay per step" if T <= 32 else "eager (planned exchange)"
    res["config"]["exchange"] = ("NVLink peer memory (dispatch/combine kernels)" if dense_p2p else
                                 "NCCL all-to-all" if T <= 32 else "NCCL all-to-all (planned, uneven splits)")
    if p2p_error:
        res["config"]["exchange"] += f" (peer exchange unavailable: {p2p_error})"
    res["config"]["experts_per_gpu"] = epr
    res["config"]["l2"] = (f"{P} rotating inputs per rank; per rank per step {u_mean:.1f} distinct local experts "
                           f"(max {u_max:.1f}) and {r_mean:.0f} local routes (max {r_max:.0f})")
    # per step: top-k, plan, gather, combine + the local layer (one decode launch, or router + gather + two grouped
    # GEMMs + combine on the prefill path)
    # this library's kernels per step: the exchange (peer dispatch with the router inside + peer combine; or router
    # top-k + NCCL + combine kernel; or router + plan + gather + combine) and the local layer (one launch up to 256
    # local routes, else 5)
    local = 1 if world * T * k <= 256 else 5
    if T <= ExpertParallelMoE.DENSE_MAX_TOKENS:
        res["gpu_launches"] = K * (2 + local)
    else:
        res["gpu_launches"] = K * (4 + local)
    return res


def run_e2e(a, layer, xs, lgs, k, P, dist):
    """End to end through the public call with pinned host buffers, as a serving loop runs it: two device buffer
    sets, the copies on a second stream, so step i + 1's inputs go up and step i's result comes down while step i
    computes.  Every step's host->device inputs and device->host result are inside the timed region (the clock
    stops after the last result has landed in host memory)."""
    import torch

    dev = layer.device
    T, H = xs[0].shape
    K = a.steps
    xh = [x.cpu().pin_memory() for x in xs]
    lh = [l.cpu().pin_memory() for l in lgs]
    oh = [torch.empty((T, H), dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    xd = [torch.empty_like(xs[0]) for _ in range(2)]
    ld = [torch.empty_like(lgs[0]) for _ in range(2)]
    od = [torch.empty((T, H), dtype=torch.bfloat16, device=dev) for _ in range(2)]
    calls = [layer.build_call(xd[b], ld[b], k, out=od[b], pdl=bool(a.pdl)) for b in range(2)]
    comp = torch.cuda.current_stream(dev)
    copy = torch.cuda.Stream(dev)
    up = [torch.cuda.Event() for _ in range(2)]    # inputs of buffer b are on the device
    done = [torch.cuda.Event() for _ in range(2)]  # the step that used buffer b has computed

    def upload(i):
        b = i % 2
        with torch.cuda.stream(copy):
            xd[b].copy_(xh[i % P], non_blocking=True)
            ld[b].copy_(lh[i % P], non_blocking=True)
            up[b].record(copy)

    def run(n, start):
        copy.wait_stream(comp)  # the first upload comes after everything already queued (the start event)
        upload(start)
        for i in range(start, start + n):
            b = i % 2
            comp.wait_event(up[b])
            calls[b].launch()
            done[b].record(comp)
            if i + 1 < start + n:
                upload(i + 1)  # buffer (i + 1) % 2: its previous step computed and was read back, in stream order
            with torch.cuda.stream(copy):
                copy.wait_event(done[b])
                oh[b].copy_(od[b], non_blocking=True)
        comp.wait_stream(copy)  # the last result is in host memory

    run(max(a.warmup, 2), 0)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(comp)
    run(K, 0)
    e1.record(comp)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / K


def finish(a, cfg, world, ms, kern_ms, e2e_ms, u_avg, P, clk, cpu):
    from xcalibur_b200 import synth

    E, H, I, T, k = cfg["E"], cfg["H"], cfg["I"], cfg["T"], cfg["k"]
    hbm, bf16, bf16_sus, src = load_peaks()
    per_expert = synth.layer_bytes(1, H, I)
    alg_bytes = u_avg * per_expert + 2 * T * H * 2
    flops = synth.layer_flops(T, k, H, I)
    if T <= 256:
        achieved = alg_bytes / (kern_ms * 1e-3) / 1e9
        roof = {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                "frac": round(achieved / hbm, 4), "peak_source": src}
    else:
        achieved = flops / (kern_ms * 1e-3) / 1e12
        peak = bf16_sus
        roof = {"bound": "tensor", "achieved": round(achieved, 1), "peak": peak, "unit": "TFLOP/s",
                "frac": round(achieved / peak, 4), "peak_source": src + " (sustained)"}
    roof["traffic"] = load_traffic(cfg["workload"])
    roof["kernel"] = "skinny_kernel" if T * k <= 256 and T <= 32 else "gather + wide_kernel x2 + combine"
    roof["kernel_ms"] = round(kern_ms, 5)
    roof["algorithmic_bytes"] = int(alg_bytes)
    roof["algorithmic_flops"] = int(flops)

    res = {
        "metric": METRIC,
        "value": round(T * world / (ms * 1e-3), 2),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": a.steps,
        "warmup": a.warmup,
        "ms_per_step": round(ms, 5),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "nvfp4 weights (e2m1 + e4m3 block scales) x bf16 activations, fp32 accumulate",
        "data": "synthetic: seeded N(0,0.02) weights quantised to NVFP4 on the GPU; bf16 N(0,1) activations; "
                "fp32 N(0,1) router logits",
        "config": {"workload": cfg["workload"], "tokens": T, "hidden": H, "inter": I, "experts": E, "top_k": k,
                   "router_bias_std": cfg["bias_std"], "parallelism": "replicas" if world > 1 else "single",
                   "pdl": bool(getattr(a, "pdl", 0)),
                   "l2": f"{P} rotating inputs; 6.3 GB of packed weights resident (>126 MB L2); "
                         f"{u_avg:.1f} distinct experts per step on average"},
        "roofline": roof,
        "e2e": None if e2e_ms is None else {
            "value": round(T * world / (e2e_ms * 1e-3), 2), "unit": "tokens/s",
            "h2d_bytes_per_step": T * H * 2 + T * E * 4, "d2h_bytes_per_step": T * H * 2},
        # decode kernel routing in-kernel (T * k <= 256, T <= 32): 1 launch per step; otherwise the prefill path:
        # router, gather, two grouped GEMMs, combine
        "gpu_launches": a.steps * (1 if T * k <= 256 and T <= 32 else 5),
        "clocks": clk,
    }
    if cpu is not None and world == 1:
        secs, n, cores = cpu
        res["cpu_baseline"] = {"value": round(n / secs, 4), "unit": "tokens/s", "cores": cores, "kind": "port",
                               "sample": f"{n} token(s) of {cfg['workload']} through the CPU oracle "
                                         f"({secs:.2f} s, dequantise + fp32 matmuls, torch threads={cores})"}
    return res


def run_reference(a, cfg):
    """Reference arm: the CPU restatement of the layer (the reference has no CPU implementation), per step.  It
    loads nothing of this repository's CUDA library: the sampled tokens' experts are drawn and quantised on the
    host (``reference_arm_experts``)."""
    import torch

    from xcalibur_b200 import synth  # noqa: F401  (torch-only input generator; the library is not loaded)

    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    E, H, I, T, k = cfg["E"], cfg["H"], cfg["I"], cfg["T"], cfg["k"]
    x, lg = synth.make_inputs(T, H, E, seed=1, device=dev, bias_std=cfg["bias_std"], zipf_s=cfg["zipf"],
                              zipf_order_seed=cfg.get("zipf_order_seed"))
    n = min(T, a.cpu_sample_tokens)
    ids, wts, used = sample_routes(lg, k, n)
    host = reference_arm_experts(cfg, used, seed=1234, device=dev)
    times = []
    for i in range(a.warmup + a.steps):
        secs, _, cores = cpu_oracle_sample(host, used, x, ids, wts, n)
        if i >= a.warmup:
            times.append(secs)
    secs = sum(times) / len(times)
    val = round(n / secs, 4)
    return {
        "impl": "reference", "metric": METRIC, "value": val, "unit": "tokens/s", "n_gpus": 1, "steps": a.steps,
        "warmup": a.warmup, "ms_per_step": round(secs * 1e3, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "fp32 (CPU restatement)", "data": "synthetic (same seeds as the main arm)",
        "config": {"workload": cfg["workload"], "tokens": T, "hidden": H, "inter": I, "experts": E, "top_k": k},
        "cpu_baseline": {"value": val, "unit": "tokens/s", "cores": cores, "kind": "port",
                         "sample": f"{n} token(s) per step of {cfg['workload']} through the CPU oracle"},
        "e2e": {"value": val, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


# ----------------------------------------------------------------------------------------------- reference shape
def okc_weights(dev, seed: int = 4096):
    """NVFP4 weights of the 32 local experts at the reference's shape (H = I = 4096), drawn with torch alone so that
    both arms time the same layer and the reference arm loads nothing of this repository's CUDA library: uniformly
    random E2M1 codes, E4M3 block scales uniform over the bytes 0x30..0x38 (0.5 .. 1, positive normals as the
    reference's PRMT-decode build requires), global scales 0.01, post-norm weights bf16 N(0, 0.1)."""
    import torch

    g = torch.Generator(device=dev).manual_seed(seed)
    E, H, I = 32, 4096, 4096
    u8 = lambda shape, lo, hi: torch.randint(lo, hi, shape, generator=g, device=dev, dtype=torch.uint8)
    return {"w13": u8((E, 2 * I, H // 2), 0, 256), "w13_sf": u8((E, 2 * I, H // 16), 0x30, 0x39),
            "w13_gs": torch.full((E,), 0.01, device=dev), "w2": u8((E, H, I // 2), 0, 256),
            "w2_sf": u8((E, H, I // 16), 0x30, 0x39), "w2_gs": torch.full((E,), 0.01, device=dev),
            "post_norm_w": (torch.randn(H, generator=g, device=dev) * 0.1).to(torch.bfloat16)}


def okc_batch(T: int, dev, seed: int):
    """bf16 N(0,1) activations and the top-8 of N(0,1) logits over 256 experts with softmax weights."""
    import torch

    g = torch.Generator(device=dev).manual_seed(seed)
    x = torch.randn((T, 4096), generator=g, device=dev).to(torch.bfloat16)
    top, ids = torch.topk(torch.randn((T, 256), generator=g, device=dev), 8, dim=1)
    cfg = {"bs": T, "d_hidden": 4096, "d_expert": 4096, "n_experts": 256, "local_start": 0, "local_count": 32,
           "top_k": 8, "sharding": "ep8"}
    return {"hidden_states": x, "topk_ids": ids.to(torch.int32), "topk_weights": torch.softmax(top, dim=1),
            "config": cfg}


HOST_LEAD_CYCLES = 400_000  # ~0.2 ms of GPU sleep before each okc step: longer than either arm's Python enqueue


def run_okc(a, cfg):
    """Configuration ``okc:T``: the reference operator's contract at its own shape, on one GPU, L2 flushed (256 MiB
    read) before every timed step as the reference's paired bench does.  ``--impl xcb`` times this library's
    ``kernel_fn``; ``--impl reference`` times the reference's own CUDA kernel (built from its sources into
    oracle/_ref/ by oracle/build_ref.py, driven by oracle/okc_ref.py).  ``e2e`` adds, every step, the host->device
    copies of x, ids and weights from pinned memory and the device->host copy of the output."""
    import torch

    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    T, H = cfg["T"], cfg["H"]
    weights = okc_weights(dev)
    if a.impl == "reference":
        from oracle import okc_ref

        try:
            state = okc_ref.prepare(weights)
            okc_ref.module(okc_ref.build_for(T))
        except okc_ref.Unavailable as e:
            return {"impl": "reference", "unavailable": str(e), "config": {"workload": cfg["workload"]}}
        fn = lambda d: okc_ref.kernel_fn(d, state)
        launches = (T + okc_ref.CHUNK_TOKENS - 1) // okc_ref.CHUNK_TOKENS
        what = f"the reference's own CUDA kernel ({okc_ref.build_for(T)} build, oracle/_ref)"
    else:
        from xcalibur_b200 import kernel_fn, prepare

        state = prepare(weights, local_start=0, local_count=32, n_experts=256)
        if a.path == "auto":
            fn = lambda d: kernel_fn(d, state)
        else:
            lay = state["layer"]
            fn = lambda d: lay.forward(d["hidden_states"], None, topk_ids=d["topk_ids"],
                                       topk_weights=d["topk_weights"], post_norm=True, path=a.path)
        # decode kernel alone (in-kernel routing), router + decode kernel (up to ~192 expected held routes), or
        # router + gather + two grouped GEMMs + final pass
        launches = 1 if T * 8 <= 256 and T <= 32 else (2 if T * 8 * 32 // 256 <= 192 else 5)
        what = "xcalibur_b200 kernel_fn"
    del weights
    torch.cuda.empty_cache()
    P = 16
    batches = [okc_batch(T, dev, seed=100 + i) for i in range(P)]
    U = [int(torch.unique(b["topk_ids"][b["topk_ids"] < 32]).numel()) for b in batches]
    flush = torch.empty(64 << 20, dtype=torch.float32, device=dev)   # 256 MiB, twice the L2
    flush.fill_(1.0)
    for i in range(max(3, a.warmup)):
        fn(batches[i % P])
    torch.cuda.synchronize()
    K = a.steps
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(K)]
    clocks = ClockSampler(dev.index)
    clocks.start()
    for i in range(K):
        flush.sum()
        torch.cuda._sleep(HOST_LEAD_CYCLES)  # the host enqueues the step meanwhile: no idle GPU inside the window
        ev[i][0].record()
        fn(batches[i % P])
        ev[i][1].record()
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = sum(e0.elapsed_time(e1) for e0, e1 in ev) / K
    # end to end: pinned host inputs in, output out, every step (after the same flush)
    host = [{k: (v.cpu().pin_memory() if torch.is_tensor(v) else v) for k, v in b.items()} for b in batches]
    oh = torch.empty((T, H), dtype=torch.bfloat16).pin_memory()
    ev2 = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(K)]
    for i in range(K):
        hb = host[i % P]
        flush.sum()
        torch.cuda._sleep(HOST_LEAD_CYCLES)
        ev2[i][0].record()
        d = {k: (v.to(dev, non_blocking=True) if torch.is_tensor(v) else v) for k, v in hb.items()}
        oh.copy_(fn(d), non_blocking=True)
        ev2[i][1].record()
    torch.cuda.synchronize()
    e2e_ms = sum(e0.elapsed_time(e1) for e0, e1 in ev2) / K
    u_avg = sum(U[i % P] for i in range(K)) / K
    from xcalibur_b200 import synth

    hbm, _, _, src = load_peaks()
    alg = u_avg * synth.layer_bytes(1, H, H) + 2 * T * H * 2 + T * 8 * 8
    achieved = alg / (ms * 1e-3) / 1e9
    res = {
        "metric": METRIC, "value": round(T / (ms * 1e-3), 2), "unit": "tokens/s", "n_gpus": 1, "steps": K,
        "warmup": max(3, a.warmup), "ms_per_step": round(ms, 5), "us_per_step": round(ms * 1e3, 2),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "nvfp4 weights (e2m1 + e4m3 block scales) x bf16 activations, fp32 accumulate",
        "data": "synthetic: random NVFP4 codes and scales, bf16 N(0,1) activations, top-8 of N(0,1) logits",
        "config": {"workload": cfg["workload"], "tokens": T, "hidden": H, "inter": H, "experts": 256,
                   "local_experts": 32, "top_k": 8, "contract": "reference kernel_fn: precomputed routes, post-norm",
                   "implementation": what,
                   "l2": f"256 MiB read flush before every timed step; {u_avg:.1f} distinct local experts per step"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                     "frac": round(achieved / hbm, 4), "peak_source": src, "traffic": None,
                     "kernel_timing": "CUDA events around each step's launches, a GPU sleep before each step so the host enqueue is hidden", "algorithmic_bytes": int(alg)},
        "e2e": {"value": round(T / (e2e_ms * 1e-3), 2), "unit": "tokens/s",
                "h2d_bytes_per_step": T * H * 2 + T * 8 * 8, "d2h_bytes_per_step": T * H * 2},
        "gpu_launches": K * launches, "clocks": clk,
    }
    if a.impl == "reference":
        res["impl"] = "reference"
        res["cpu_baseline"] = {"value": res["value"], "unit": "tokens/s", "cores": 0, "kind": "reference",
                               "device": "GPU", "sample": f"{K} steps of {cfg['workload']} through {what}"}
    return res


def main():
    a = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    names = [a.config] if a.config else (["decode"] if world == 1 else ["ep", "decode"])
    cfg = config_for(names[0], a.experts, a.tokens)
    if "local" in cfg:                 # the reference's own shape: one GPU, both arms on the GPU
        if rank == 0:
            print(json.dumps(run_okc(a, cfg)), flush=True)
        return
    if a.impl == "reference":
        if rank == 0:
            # reduce the per-step sample so the whole run stays within a few minutes
            a.steps = min(a.steps, 3)
            a.warmup = min(a.warmup, 1)
            print(json.dumps(run_reference(a, cfg)), flush=True)
        return
    dist = None
    if world > 1:
        import datetime

        import torch
        import torch.distributed as td

        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
        td.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
        dist = td
    layer = None
    try:
        if world == 1:
            res = run_xcb(a, cfg, rank, world, dist)
            if rank == 0:
                print(json.dumps(res), flush=True)
        else:
            layer = make_ep_layer(cfg, rank, world)
            for name in names:            # one JSON line per configuration, configuration 5 first
                res = run_xcb_ep(a, config_for(name, a.experts, a.tokens), rank, world, dist, layer)
                if rank == 0:
                    print(json.dumps(res), flush=True)
    finally:
        if layer is not None:
            layer.close()  # the peer exchange's buffers (collective)
        if dist:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
