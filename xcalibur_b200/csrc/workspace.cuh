// Workspace layout shared by the host launcher and the kernels.  The caller allocates xcb_moe_workspace_bytes()
// and zeroes it once (xcb_moe_workspace_init).  The control words sit at offset 0 whatever the call's size; the
// kernel that uses them returns them to zero before it exits.  Every other region is rewritten by each call
// before it is read (the router zeroes the per-job counters), so consecutive calls of any size on one stream
// need no host-side reset and stay graph-capturable.
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace xcb {

constexpr int kJobTokens = 8;  // tokens per decode-path job (one m16n8k16 n-tile)

// Fixed header at the start of the workspace (same offsets whatever the call's size).
enum CtlWord : int {
  kCtlStatus = 0,      // XCB_STATUS_* bits
  kCtlGridArrive = 1,  // grid barrier of the decode-path kernel
  kCtlExit = 2,        // CTAs that finished the decode-path kernel (the last one resets the counters)
  kCtlJobs = 3,        // number of jobs written by the router
  kCtlRoutes = 4,      // number of local routes
  kCtlWideTile = 5,    // [2] prefill GEMM tile claims and finished CTAs (the last CTA resets both)
  kCtlDoneA = 64,      // [256] per-job phase-A counters when the decode kernel routes in-kernel
  kCtlSS = 320,        // [256] fp32 per-route sums of squares (post-norm) when routing in-kernel
  kCtlRowBlock = 576,  // [512] per-16-row-block phase-B arrival counters (H <= 8192)
  kCtlWords = 1280
};
constexpr int kSmallRoutes = 256;  // T*k up to which the decode kernel routes in-kernel (one launch per call)
constexpr int kSmallTokens = 32;

// The many-token router works on chunks of whole tokens, at most 1024 routes each.
__host__ __device__ inline int route_chunk_tokens(int top_k) { return top_k > 0 && top_k <= 1024 ? 1024 / top_k : 1; }
__host__ __device__ inline size_t route_chunks(int tokens, int top_k) {
  const int ct = route_chunk_tokens(top_k);
  return ((size_t)tokens + ct - 1) / ct;
}

struct WsLayout {
  size_t ctl, ids, wts, pos, order, counts, offsets, jobs, doneA, ss, hist, inter, y, total;
  int max_routes, max_jobs;
};

inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

inline WsLayout ws_layout(int E_loc, int H, int I, int max_tokens, int top_k) {
  WsLayout L;
  const size_t R = (size_t)max_tokens * (size_t)top_k;
  L.max_routes = (int)R;
  // every job holds at least one route, and the in-kernel router may cut jobs as narrow as one route
  L.max_jobs = (int)(R + 1);
  size_t o = 0;
  auto take = [&](size_t bytes) {
    size_t at = o;
    o = align_up(o + bytes, 256);
    return at;
  };
  L.ctl = take(kCtlWords * 4);
  L.ids = take(R * 4);
  L.wts = take(R * 4);
  L.pos = take(R * 4);
  L.order = take(R * 4);
  L.counts = take((size_t)E_loc * 4);
  L.offsets = take(((size_t)E_loc + 1) * 4);
  L.jobs = take((size_t)L.max_jobs * 16);
  L.doneA = take((size_t)L.max_jobs * 4);
  L.ss = take(R * 4);
  L.hist = take(route_chunks(max_tokens, top_k) * (size_t)E_loc * 4);
  L.inter = take(R * (size_t)I * 2);
  L.y = take(R * (size_t)H * 4);
  L.total = o;
  return L;
}

}  // namespace xcb
