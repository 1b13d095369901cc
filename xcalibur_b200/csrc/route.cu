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
//   4. the decode-path job list: each expert's routes cut into jobs of at most p.job_tokens tokens.
// Above kChunkedRouteMin routes the same steps run as three multi-CTA kernels (below).
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
    jcnt[e] = (cnt[e] + p.job_tokens - 1) / p.job_tokens;
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
    for (int s0 = 0; s0 < c; s0 += p.job_tokens, ++j) {
      p.jobs[j] = make_int4(e, base[e] + s0, min(p.job_tokens, c - s0), 0);
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

// ------------------------------------------------------------------------------------------------ many tokens
// The same routing split over chunks of whole tokens (at most 1024 routes each), so that it scales with T:
//   route_chunk_kernel   one CTA per chunk: top-k (one warp per token) and the chunk's expert histogram;
//   route_scan_kernel    one CTA: expert counts and offsets, each chunk's first position per expert, the
//                        decode-path job list;
//   route_place_kernel   one CTA per chunk: stable ranks inside the chunk (as in route_kernel) + chunk base.
// The permutation equals route_kernel's (a stable sort of the flat route index by expert).
__global__ void __launch_bounds__(kRouteThreads) route_chunk_kernel(RouteParams p) {
  extern __shared__ int rc_hist[];  // [E_loc]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int CT = route_chunk_tokens(p.k);
  const int t0 = blockIdx.x * CT, t1 = min(p.T, t0 + CT);
  for (int e = tid; e < p.E_loc; e += kRouteThreads) rc_hist[e] = 0;
  __syncthreads();
  if (p.logits) {
    for (int t = t0 + warp; t < t1; t += kRouteThreads / 32) {
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
        if (el >= 0 && el < p.E_loc) atomicAdd(&rc_hist[el], 1);
      }
    }
  } else {
    for (int f = t0 * p.k + tid; f < t1 * p.k; f += kRouteThreads) {
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
      if (id >= 0 && el >= 0 && el < p.E_loc) atomicAdd(&rc_hist[el], 1);
    }
  }
  __syncthreads();
  for (int e = tid; e < p.E_loc; e += kRouteThreads) p.hist[(size_t)blockIdx.x * p.E_loc + e] = rc_hist[e];
}

__global__ void __launch_bounds__(kRouteThreads, 1) route_scan_kernel(RouteParams p) {
  extern __shared__ int rs_smem[];
  __shared__ int tot_routes, tot_jobs;
  int* base = rs_smem;              // [E_loc + 1]
  int* jcnt = base + p.E_loc + 1;   // [E_loc]
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nch = (int)route_chunks(p.T, p.k);
  for (int e = tid; e < p.E_loc; e += kRouteThreads) {  // per-expert prefix over chunks (exclusive), counts
    int run = 0;
    for (int c = 0; c < nch; ++c) {
      int* h = p.hist + (size_t)c * p.E_loc + e;
      const int v = *h;
      *h = run;
      run += v;
    }
    base[e] = run;
    jcnt[e] = (run + p.job_tokens - 1) / p.job_tokens;
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
    const int b0 = base[e];
    for (int ch = 0; ch < nch; ++ch) p.hist[(size_t)ch * p.E_loc + e] += b0;
    const int c = (e + 1 < p.E_loc ? base[e + 1] : tot_routes) - b0;
    p.counts[e] = c;
    p.offsets[e] = b0;
    int j = jcnt[e];
    for (int s0 = 0; s0 < c; s0 += p.job_tokens, ++j) {
      p.jobs[j] = make_int4(e, b0 + s0, min(p.job_tokens, c - s0), 0);
      p.doneA[j] = 0;
    }
  }
  if (tid == 0) {
    p.offsets[p.E_loc] = tot_routes;
    p.ctl[kCtlJobs] = tot_jobs;
    p.ctl[kCtlRoutes] = tot_routes;
  }
}

__global__ void __launch_bounds__(kRouteThreads) route_place_kernel(RouteParams p) {
  extern __shared__ int rp_wc[];  // [32][E_loc]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int EL = p.E_loc;
  const int CR = route_chunk_tokens(p.k) * p.k;
  const int R = p.T * p.k;
  for (int i = tid; i < 32 * EL; i += kRouteThreads) rp_wc[i] = 0;
  __syncthreads();
  const int f = blockIdx.x * CR + tid;
  int el = -1;
  if (tid < CR && f < R) {
    const int id = p.ids[f];
    el = id - p.lo;
    if (id < 0 || el < 0 || el >= EL) el = -1;
  }
  const uint32_t peers = __match_any_sync(0xffffffffu, el);
  const int rank = __popc(peers & ((1u << lane) - 1u));
  if (el >= 0 && rank == 0) rp_wc[warp * EL + el] = __popc(peers);
  __syncthreads();
  for (int e = tid; e < EL; e += kRouteThreads) {
    int run = p.hist[(size_t)blockIdx.x * EL + e];
#pragma unroll 8
    for (int w = 0; w < 32; ++w) {
      const int v = rp_wc[w * EL + e];
      rp_wc[w * EL + e] = run;
      run += v;
    }
  }
  __syncthreads();
  if (tid < CR && f < R) {
    if (el >= 0) {
      const int q = rp_wc[warp * EL + el] + rank;
      p.pos[f] = q;
      p.order[q] = f;
      p.ss[q] = 0.f;
    } else {
      p.pos[f] = -1;
    }
  }
}

size_t route_smem_bytes(int E_loc) { return (size_t)(3 * E_loc + 1 + 32 * E_loc) * sizeof(int); }

// Routes above which the chunked (multi-CTA) router replaces the single-CTA one.
constexpr long long kChunkedRouteMin = 2048;

int launch_route(const RouteParams& p, cudaStream_t stream) {
  const long long R = (long long)p.T * p.k;
  if (R > kChunkedRouteMin) {
    const int nch = (int)route_chunks(p.T, p.k);
    const size_t s1 = (size_t)p.E_loc * 4, s2 = (size_t)(2 * p.E_loc + 1) * 4, s3 = (size_t)32 * p.E_loc * 4;
    if (s3 > 48 * 1024 &&
        cudaFuncSetAttribute(route_place_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)s3) != cudaSuccess)
      return XCB_ERR_CUDA;
    route_chunk_kernel<<<nch, kRouteThreads, s1, stream>>>(p);
    route_scan_kernel<<<1, kRouteThreads, s2, stream>>>(p);
    route_place_kernel<<<nch, kRouteThreads, s3, stream>>>(p);
    return cudaGetLastError() == cudaSuccess ? XCB_OK : XCB_ERR_CUDA;
  }
  const size_t smem = route_smem_bytes(p.E_loc);
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute(route_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return XCB_ERR_CUDA;
  route_kernel<<<1, kRouteThreads, smem, stream>>>(p);
  return cudaGetLastError() == cudaSuccess ? XCB_OK : XCB_ERR_CUDA;
}

}  // namespace xcb
