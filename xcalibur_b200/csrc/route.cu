// Router and token permutation (one CTA of 1024 threads).
//
// Replaces the reference's per-CTA route() (kernels/moe_w4a16_h200/moe_w4a16.py:491-611), which rebuilds the same
// per-expert lists redundantly in every CTA from precomputed topk ids, and adds the router the north_star
// signature needs (absent from the reference, which receives topk_ids/topk_weights, moe_w4a16.py:93-97):
//
//   1. top-k per token, one warp per token: rank by raw logit descending, ties to the lower expert id; the route
//      weights are the softmax over the k selected logits (== softmax -> top-k -> renormalise);
//   2. per-expert histogram of local routes (shared-memory atomics), exclusive scan -> offsets;
//   3. stable permutation: position of flat route f = t*k + s is offsets[e] + #{f' < f : id[f'] = e}, computed
//      1024 routes at a time with __match_any_sync ranks and a per-warp prefix (bit-exact with a stable sort);
//   4. the decode-path job list: each expert's routes cut into jobs of at most kJobTokens tokens.
#include "common.cuh"
#include "kernels.cuh"
#include "workspace.cuh"

namespace xcb {

constexpr int kRouteThreads = 1024;

__global__ void __launch_bounds__(kRouteThreads, 1) route_kernel(RouteParams p) {
  extern __shared__ int route_smem[];
  __shared__ int tot_routes, tot_jobs;
  const int EL = p.E_loc;
  int* cnt = route_smem;            // [EL]
  int* base = cnt + EL;             // [EL + 1]
  int* jcnt = base + EL + 1;        // [EL]
  int* wc = jcnt + EL;              // [32][EL]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int R = p.T * p.k;
  for (int e = tid; e < p.E_loc; e += kRouteThreads) cnt[e] = 0;
  __syncthreads();

  // ---- 1. routes and histogram
  if (p.logits) {
    for (int t = warp; t < p.T; t += kRouteThreads / 32) {
      int my_i;
      float w;
      warp_topk(p.logits + (size_t)t * p.E_tot, p.E_tot, p.k, my_i, w);
      if (lane < p.k) {
        const int f = t * p.k + lane;
        p.ids[f] = my_i;
        p.wts[f] = w;
        if (p.ids_out) p.ids_out[f] = my_i;
        if (p.wts_out) p.wts_out[f] = w;
        const int el = my_i - p.lo;
        if (el >= 0 && el < p.E_loc) atomicAdd(&cnt[el], 1);
      }
    }
  } else {
    for (int f = tid; f < R; f += kRouteThreads) {
      int id = p.ids_in[f];
      const float w = p.wts_in[f];
      if (id < 0 || id >= p.E_tot) {
        set_status(p.ctl + kCtlStatus, XCB_STATUS_BAD_EXPERT);
        id = -1;
      }
      p.ids[f] = id;
      p.wts[f] = w;
      if (p.ids_out) p.ids_out[f] = id;
      if (p.wts_out) p.wts_out[f] = w;
      const int el = id - p.lo;
      if (id >= 0 && el >= 0 && el < p.E_loc) atomicAdd(&cnt[el], 1);
    }
  }
  __syncthreads();

  // ---- 2. offsets and jobs
  for (int e = tid; e < p.E_loc; e += kRouteThreads) {
    base[e] = cnt[e];
    jcnt[e] = (cnt[e] + kJobTokens - 1) / kJobTokens;
  }
  __syncthreads();
  if (warp == 0) {
    const int tot = warp_exclusive_scan(base, p.E_loc);
    if (lane == 0) tot_routes = tot;
  }
  if (warp == 1) {
    const int tot = warp_exclusive_scan(jcnt, p.E_loc);
    if (lane == 0) tot_jobs = tot;
  }
  __syncthreads();
  for (int e = tid; e < p.E_loc; e += kRouteThreads) {
    p.counts[e] = cnt[e];
    p.offsets[e] = base[e];
    const int c = cnt[e];
    int j = jcnt[e];
    for (int s0 = 0; s0 < c; s0 += kJobTokens, ++j) {
      p.jobs[j] = make_int4(e, base[e] + s0, min(kJobTokens, c - s0), 0);
      p.doneA[j] = 0;
    }
  }
  if (tid == 0) {
    p.offsets[p.E_loc] = tot_routes;
    p.ctl[kCtlJobs] = tot_jobs;
    p.ctl[kCtlRoutes] = tot_routes;
  }
  for (int i = tid; i < tot_routes; i += kRouteThreads) p.ss[i] = 0.f;
  __syncthreads();

  // ---- 3. stable ranks, 1024 routes per pass
  const uint32_t lt = (1u << lane) - 1u;
  for (int c0 = 0; c0 < R; c0 += kRouteThreads) {
    for (int i = tid; i < 32 * p.E_loc; i += kRouteThreads) wc[i] = 0;
    __syncthreads();
    const int f = c0 + tid;
    int el = -1;
    if (f < R) {
      const int id = p.ids[f];
      el = id - p.lo;
      if (id < 0 || el < 0 || el >= p.E_loc) el = -1;
    }
    const uint32_t peers = __match_any_sync(0xffffffffu, el);
    const int rank = __popc(peers & lt);
    if (el >= 0 && rank == 0) wc[warp * EL + el] = __popc(peers);
    __syncthreads();
    for (int e = tid; e < p.E_loc; e += kRouteThreads) {
      int run = base[e];
#pragma unroll 8
      for (int w = 0; w < 32; ++w) {
        const int v = wc[w * EL + e];
        wc[w * EL + e] = run;
        run += v;
      }
      base[e] = run;
    }
    __syncthreads();
    if (f < R) {
      if (el >= 0) {
        const int q = wc[warp * EL + el] + rank;
        p.pos[f] = q;
        p.order[q] = f;
      } else {
        p.pos[f] = -1;
      }
    }
    __syncthreads();
  }
}

size_t route_smem_bytes(int E_loc) { return (size_t)(3 * E_loc + 1 + 32 * E_loc) * sizeof(int); }

int launch_route(const RouteParams& p, cudaStream_t stream) {
  const size_t smem = route_smem_bytes(p.E_loc);
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute(route_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return XCB_ERR_CUDA;
  route_kernel<<<1, kRouteThreads, smem, stream>>>(p);
  return cudaGetLastError() == cudaSuccess ? XCB_OK : XCB_ERR_CUDA;
}

}  // namespace xcb
