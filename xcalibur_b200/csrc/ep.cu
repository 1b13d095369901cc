// Expert-parallel helpers: router top-k on its own, the dispatch plan, the gather of the send buffer and the combine
// of returned partial sums.  The reference has no exchange step (an EP rank only masks non-local routes,
// kernels/moe_w4a16_h200/moe_w4a16.py:513-520, and the cross-rank sum was its harness's job); these kernels give
// the expert-parallel layer its dispatch and combine around the local experts, with the transport (NCCL all-to-all
// or peer stores) chosen by the host.
//
//   plan     a token goes once to every rank that holds one of its experts (rank of expert e = e / experts per
//            rank), in token order: counts[d], send_tok[d][i] = token, send_pos[t][d] = i (or -1);
//   gather   destination-major send rows: x[send_tok[d][i]] with the token's full top-k ids and weights (the
//            receiving rank masks the experts it does not hold);
//   combine  out[t] = bf16(sum over ranks d, in rank order, of the partial returned for (t, d)).
#include "common.cuh"
#include "kernels.cuh"

namespace xcb {

constexpr int kEpThreads = 1024;
constexpr int kEpMaxRanks = 32;

__global__ void topk_kernel(const float* logits, int T, int E, int k, int* ids, float* wts) {
  const int lane = threadIdx.x & 31;
  const int nw = (gridDim.x * blockDim.x) >> 5;
  for (int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; t < T; t += nw) {
    int id;
    float w;
    warp_topk(logits + (size_t)t * E, E, k, id, w);
    if (lane < k) {
      ids[t * k + lane] = id;
      wts[t * k + lane] = w;
    }
  }
}

// One CTA: tokens in chunks of 1024 (one per thread); per destination rank a warp ballot, a per-warp prefix and a
// scan over the 32 warps give each token its position in that rank's list (token order, deterministic).
__global__ void __launch_bounds__(kEpThreads, 1) ep_plan_kernel(const int* ids, int T, int k, int epr, int G,
                                                                int* counts, int* send_tok, int* send_pos,
                                                                int* status) {
  __shared__ int wsum[32][kEpMaxRanks];
  __shared__ int run[kEpMaxRanks];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid < G) run[tid] = 0;
  __syncthreads();
  for (int c0 = 0; c0 < T; c0 += kEpThreads) {
    const int t = c0 + tid;
    uint32_t mask = 0;
    if (t < T) {
      for (int s = 0; s < k; ++s) {
        const int id = ids[t * k + s];
        if (id < 0 || id >= epr * G) {
          set_status(status, XCB_STATUS_BAD_EXPERT);
          continue;
        }
        mask |= 1u << (id / epr);
      }
    }
    for (int d = 0; d < G; ++d) {
      const uint32_t b = __ballot_sync(0xffffffffu, (mask >> d) & 1u);
      if (lane == 0) wsum[warp][d] = __popc(b);
    }
    __syncthreads();
    if (tid < G) {  // scan over warps for rank tid
      int r = run[tid];
      for (int w = 0; w < 32; ++w) {
        const int v = wsum[w][tid];
        wsum[w][tid] = r;
        r += v;
      }
      run[tid] = r;
    }
    __syncthreads();
    for (int d = 0; d < G; ++d) {
      const uint32_t b = __ballot_sync(0xffffffffu, (mask >> d) & 1u);
      if (t < T) {
        int pos = -1;
        if ((mask >> d) & 1u) {
          pos = wsum[warp][d] + __popc(b & ((1u << lane) - 1u));
          send_tok[(size_t)d * T + pos] = t;
        }
        send_pos[(size_t)t * G + d] = pos;
      }
    }
    __syncthreads();
  }
  if (tid < G) counts[tid] = run[tid];
}

// Row r of the send buffer: rank d = the last with base[d] <= r (base = exclusive scan of counts).
__device__ __forceinline__ int ep_rank_of(int r, const int* counts, int G, int& base) {
  int b = 0, d = 0;
  for (; d < G - 1; ++d) {
    if (r < b + counts[d]) break;
    b += counts[d];
  }
  base = b;
  return d;
}

__global__ void ep_gather_kernel(const uint16_t* __restrict__ x, const int* __restrict__ ids,
                                 const float* __restrict__ wts, int T, int H, int k, int G,
                                 const int* __restrict__ counts, const int* __restrict__ send_tok,
                                 uint16_t* __restrict__ x_out, int* __restrict__ ids_out, float* __restrict__ w_out) {
  int total = 0;
  for (int d = 0; d < G; ++d) total += counts[d];
  const int lane = threadIdx.x & 31;
  const int nw = (gridDim.x * blockDim.x) >> 5;
  const int nv = H / 8;
  for (int r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < total; r += nw) {
    int base;
    const int d = ep_rank_of(r, counts, G, base);
    const int t = send_tok[(size_t)d * T + (r - base)];
    const uint4* src = reinterpret_cast<const uint4*>(x + (size_t)t * H);
    uint4* dst = reinterpret_cast<uint4*>(x_out + (size_t)r * H);
    for (int v = lane; v < nv; v += 32) dst[v] = __ldg(src + v);
    if (lane < k) {
      ids_out[(size_t)r * k + lane] = ids[(size_t)t * k + lane];
      w_out[(size_t)r * k + lane] = wts[(size_t)t * k + lane];
    }
  }
}

__global__ void ep_combine_kernel(const uint16_t* __restrict__ parts, const int* __restrict__ counts,
                                  const int* __restrict__ send_pos, int T, int H, int G, uint16_t* __restrict__ out) {
  __shared__ int base[kEpMaxRanks];
  if (threadIdx.x == 0) {
    int b = 0;
    for (int d = 0; d < G; ++d) {
      base[d] = b;
      b += counts[d];
    }
  }
  __syncthreads();
  const int per_row = H / 4;
  const size_t n = (size_t)T * per_row;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const int t = (int)(i / per_row), col = (int)(i % per_row) * 4;
    float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
    for (int d = 0; d < G; ++d) {  // rank order: deterministic
      const int pos = send_pos[(size_t)t * G + d];
      if (pos >= 0) {
        const uint2 v = *reinterpret_cast<const uint2*>(parts + (size_t)(base[d] + pos) * H + col);
        a0 += bf2f((uint16_t)(v.x & 0xFFFFu));
        a1 += bf2f((uint16_t)(v.x >> 16));
        a2 += bf2f((uint16_t)(v.y & 0xFFFFu));
        a3 += bf2f((uint16_t)(v.y >> 16));
      }
    }
    uint2 o;
    o.x = (uint32_t)f2bf(a0) | ((uint32_t)f2bf(a1) << 16);
    o.y = (uint32_t)f2bf(a2) | ((uint32_t)f2bf(a3) << 16);
    *reinterpret_cast<uint2*>(out + (size_t)t * H + col) = o;
  }
}

int ep_sm_count() {
  static int cached_dev = -1, cached = 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  if (dev != cached_dev) {
    if (cudaDeviceGetAttribute(&cached, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
    cached_dev = dev;
  }
  return cached;
}

}  // namespace xcb

using namespace xcb;

extern "C" {

int xcb_moe_topk(const float* logits, int32_t T, int32_t E, int32_t k, int32_t* ids, float* wts,
                 cudaStream_t stream) {
  if (T < 0 || E <= 0 || E > 512 || k <= 0 || k > 16 || k > E) return XCB_ERR_INVALID_ARG;
  if (T == 0) return XCB_OK;
  if (!logits || !ids || !wts) return XCB_ERR_INVALID_ARG;
  const int sms = ep_sm_count();
  if (!sms) return XCB_ERR_CUDA;
  const int want = (T + 7) / 8;  // 8 warps (tokens) per CTA
  const int blocks = want < sms * 8 ? want : sms * 8;
  topk_kernel<<<blocks, 256, 0, stream>>>(logits, T, E, k, ids, wts);
  return cudaGetLastError() == cudaSuccess ? XCB_OK : XCB_ERR_CUDA;
}

int xcb_ep_plan(const int32_t* ids, int32_t T, int32_t k, int32_t experts_per_rank, int32_t G, int32_t* counts,
                int32_t* send_tok, int32_t* send_pos, int32_t* status, cudaStream_t stream) {
  if (T < 0 || k <= 0 || k > 16 || experts_per_rank <= 0 || G <= 0 || G > kEpMaxRanks) return XCB_ERR_INVALID_ARG;
  if (!counts || !status || (T > 0 && (!ids || !send_tok || !send_pos))) return XCB_ERR_INVALID_ARG;
  ep_plan_kernel<<<1, kEpThreads, 0, stream>>>(ids, T, k, experts_per_rank, G, counts, send_tok, send_pos, status);
  return cudaGetLastError() == cudaSuccess ? XCB_OK : XCB_ERR_CUDA;
}

int xcb_ep_gather(const uint16_t* x, const int32_t* ids, const float* wts, int32_t T, int32_t H, int32_t k, int32_t G,
                  const int32_t* counts, const int32_t* send_tok, uint16_t* x_out, int32_t* ids_out, float* w_out,
                  cudaStream_t stream) {
  if (T < 0 || H <= 0 || H % 8 || k <= 0 || k > 16 || G <= 0 || G > kEpMaxRanks) return XCB_ERR_INVALID_ARG;
  if (T == 0) return XCB_OK;
  if (!x || !ids || !wts || !counts || !send_tok || !x_out || !ids_out || !w_out) return XCB_ERR_INVALID_ARG;
  if (((uintptr_t)x & 15u) || ((uintptr_t)x_out & 15u)) return XCB_ERR_INVALID_ARG;
  const int sms = ep_sm_count();
  if (!sms) return XCB_ERR_CUDA;
  ep_gather_kernel<<<sms * 4, 256, 0, stream>>>(x, ids, wts, T, H, k, G, counts, send_tok, x_out, ids_out, w_out);
  return cudaGetLastError() == cudaSuccess ? XCB_OK : XCB_ERR_CUDA;
}

int xcb_ep_combine(const uint16_t* parts, const int32_t* counts, const int32_t* send_pos, int32_t T, int32_t H,
                   int32_t G, uint16_t* out, cudaStream_t stream) {
  if (T < 0 || H <= 0 || H % 4 || G <= 0 || G > kEpMaxRanks) return XCB_ERR_INVALID_ARG;
  if (T == 0) return XCB_OK;
  if (!counts || !send_pos || !out) return XCB_ERR_INVALID_ARG;
  if (((uintptr_t)parts & 7u) || ((uintptr_t)out & 7u)) return XCB_ERR_INVALID_ARG;
  const int sms = ep_sm_count();
  if (!sms) return XCB_ERR_CUDA;
  ep_combine_kernel<<<sms * 4, 256, 0, stream>>>(parts, counts, send_pos, T, H, G, out);
  return cudaGetLastError() == cudaSuccess ? XCB_OK : XCB_ERR_CUDA;
}

}  // extern "C"
