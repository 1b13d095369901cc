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
#include <cstring>

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

// ------------------------------------------------------------------------------------------------ peer exchange
// Dense exchange for small batches over NVLink peer memory, without NCCL: every rank holds one buffer (same layout
// on every rank, mapped into every peer through CUDA IPC) with, per source rank d, a slot for d's token rows and
// their top-k row (written by d) and a slot for the partial sums this rank's tokens got on d (written by d).
// dispatch: push this rank's rows into slot [rank] of every peer, fence, raise the peer's x flag; wait until every
// peer has raised this rank's.  combine: push each peer's partial rows into slot [rank] of that peer, fence, raise
// its part flag; wait for all; out = bf16(sum over d in rank order).  Flags count block arrivals and only grow: the
// number of pushing blocks per peer (nb) depends on the buffer's T_max alone, never on a step's T (a block whose
// share of a small step is empty still raises its flag), so after e steps every flag of a rank stands at e * nb and
// no reset is needed between steps of any size.  Every wait is bounded; on timeout the status word gets
// XCB_STATUS_DEVICE_TIMEOUT and the combine writes NaN rows, so a failed step cannot pass for a valid result.
namespace xcb {

struct P2pLayout {
  size_t x, ids, wts, part, flag, total;
};
__host__ __device__ inline P2pLayout p2p_layout(int G, int Tm, int H, int k) {
  P2pLayout L;
  size_t o = 0;
  auto take = [&](size_t b) { size_t at = o; o = (o + b + 255) / 256 * 256; return at; };
  L.x = take((size_t)G * Tm * H * 2);
  L.ids = take((size_t)G * Tm * k * 4);
  L.wts = take((size_t)G * Tm * k * 4);
  L.part = take((size_t)G * Tm * H * 2);
  L.flag = take((size_t)(2 * G + 4) * 4);  // x flags [G], part flags [G], epoch, block counter
  L.total = o;
  return L;
}

constexpr int kP2pRowBytesPerBlock = 65536;  // rows per pushing block: about 64 KB

__device__ __forceinline__ unsigned p2p_load_acquire(const unsigned* a) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(a) : "memory");
  return v;
}
__device__ __forceinline__ void p2p_red_release(unsigned* a, unsigned v) {
  asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(a), "r"(v) : "memory");
}

// Wait (bounded) until every flag [0, G) of `flags` reaches `target`; false on timeout (status bit set).
__device__ bool p2p_wait_all(const unsigned* flags, int G, unsigned target, uint64_t timeout_ns, int* status) {
  const uint64_t t0 = gtimer();
  for (int d = 0; d < G; ++d) {
    while ((int)(p2p_load_acquire(flags + d) - target) < 0) {
      __nanosleep(64);
      if (gtimer() - t0 > timeout_ns) {
        set_status(status, XCB_STATUS_DEVICE_TIMEOUT);
        return false;
      }
    }
  }
  return true;
}

__global__ void ep_p2p_dispatch_kernel(const uint16_t* __restrict__ x, const float* __restrict__ logits, int T, int Tm,
                                       int H, int E, int k, int G, int rank, const uint64_t* __restrict__ peers,
                                       int nb, P2pLayout L, uint64_t timeout_ns, int* status) {
  (void)Tm;
  const int d = blockIdx.x / nb, sub = blockIdx.x % nb;
  uint8_t* mine = reinterpret_cast<uint8_t*>(peers[rank]);
  const unsigned e = *reinterpret_cast<volatile unsigned*>(mine + L.flag + 2 * G * 4) + 1;  // this step's epoch
  uint8_t* dst = reinterpret_cast<uint8_t*>(peers[d]);
  const int r0 = T * sub / nb, r1 = T * (sub + 1) / nb;
  const int nv = H / 8;
  const uint4* src = reinterpret_cast<const uint4*>(x);
  // slots are T rows apart (every rank sends T rows this step), so the received rows form one [G T, H] matrix
  uint4* dx = reinterpret_cast<uint4*>(dst + L.x + (size_t)rank * T * H * 2);
  for (int i = r0 * nv + threadIdx.x; i < r1 * nv; i += blockDim.x) dx[i] = __ldg(src + i);
  // the router: top-k of each of this block's tokens (one warp per token; every block sending these rows computes
  // the same selection), written straight into the peer's ids / weights slots
  int* di = reinterpret_cast<int*>(dst + L.ids + (size_t)rank * T * k * 4);
  float* dw = reinterpret_cast<float*>(dst + L.wts + (size_t)rank * T * k * 4);
  const int lane = threadIdx.x & 31;
  for (int t = r0 + (threadIdx.x >> 5); t < r1; t += blockDim.x >> 5) {
    int id;
    float w;
    warp_topk(logits + (size_t)t * E, E, k, id, w);
    if (lane < k) {
      di[t * k + lane] = id;
      dw[t * k + lane] = w;
    }
  }
  // the block's stores, then one system-scope fence and the release by thread 0 (the barrier orders every thread's
  // stores before it; a fence in every thread would wait for NVLink acknowledgements 256 times over)
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    p2p_red_release(reinterpret_cast<unsigned*>(dst + L.flag) + rank, 1u);
  }
  // one block waits for every peer's rows in this rank's buffer; the kernels after this one read them
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    p2p_wait_all(reinterpret_cast<const unsigned*>(mine + L.flag), G, e * (unsigned)nb, timeout_ns, status);
    __threadfence_system();
  }
}

__global__ void ep_p2p_combine_kernel(const uint16_t* __restrict__ parts, int T, int Tm, int H, int G, int rank,
                                      const uint64_t* __restrict__ peers, int nb, P2pLayout L, uint16_t* __restrict__ out,
                                      uint64_t timeout_ns, int* status) {
  (void)Tm;
  const int d = blockIdx.x / nb, sub = blockIdx.x % nb;
  uint8_t* mine = reinterpret_cast<uint8_t*>(peers[rank]);
  unsigned* epoch = reinterpret_cast<unsigned*>(mine + L.flag + 2 * G * 4);
  const unsigned e = *reinterpret_cast<volatile unsigned*>(epoch) + 1;
  uint8_t* dst = reinterpret_cast<uint8_t*>(peers[d]);
  const int r0 = T * sub / nb, r1 = T * (sub + 1) / nb;
  const int nv = H / 8;
  // rank d's tokens are rows [d T, (d + 1) T) of this rank's partial sums
  const uint4* src = reinterpret_cast<const uint4*>(parts + (size_t)d * T * H);
  uint4* dp = reinterpret_cast<uint4*>(dst + L.part + (size_t)rank * T * H * 2);
  for (int i = r0 * nv + threadIdx.x; i < r1 * nv; i += blockDim.x) dp[i] = __ldg(src + i);
  __syncthreads();  // as in the dispatch: the block's stores, then one fence and the release by thread 0
  __shared__ int ok;
  if (threadIdx.x == 0) {
    __threadfence_system();
    p2p_red_release(reinterpret_cast<unsigned*>(dst + L.flag) + G + rank, 1u);
    ok = p2p_wait_all(reinterpret_cast<const unsigned*>(mine + L.flag) + G, G, e * (unsigned)nb, timeout_ns, status);
    // a dispatch of this step that timed out left the local layer with incomplete rows: the sums are invalid too
    if (*reinterpret_cast<volatile int*>(status) & XCB_STATUS_DEVICE_TIMEOUT) ok = 0;
  }
  __syncthreads();
  if (!ok) {
    // NaN rows instead of stale or partial sums (bf16 quiet NaN 0x7FC0)
    const int nq = T * (H / 4);
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < nq; i += gridDim.x * blockDim.x) {
      const int t = i / (H / 4), c = (i % (H / 4)) * 4;
      *reinterpret_cast<uint2*>(out + (size_t)t * H + c) = make_uint2(0x7FC07FC0u, 0x7FC07FC0u);
    }
  } else {
    // out = bf16(sum over source ranks in rank order), this block's slice of the T x H outputs
    const uint16_t* pin = reinterpret_cast<const uint16_t*>(mine + L.part);
    const int nq = T * (H / 4);
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < nq; i += gridDim.x * blockDim.x) {
      const int t = i / (H / 4), c = (i % (H / 4)) * 4;
      float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
      for (int s = 0; s < G; ++s) {
        const uint2 v = __ldcv(reinterpret_cast<const uint2*>(pin + ((size_t)s * T + t) * H + c));
        a0 += bf2f((uint16_t)(v.x & 0xFFFFu));
        a1 += bf2f((uint16_t)(v.x >> 16));
        a2 += bf2f((uint16_t)(v.y & 0xFFFFu));
        a3 += bf2f((uint16_t)(v.y >> 16));
      }
      uint2 o;
      o.x = (uint32_t)f2bf(a0) | ((uint32_t)f2bf(a1) << 16);
      o.y = (uint32_t)f2bf(a2) | ((uint32_t)f2bf(a3) << 16);
      *reinterpret_cast<uint2*>(out + (size_t)t * H + c) = o;
    }
  }
  // the last block to finish advances this rank's epoch (every block has read it by then)
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned* cnt = epoch + 1;
    __threadfence();
    if (atomicAdd(cnt, 1u) == gridDim.x - 1) {
      *cnt = 0;
      *epoch = e;
      __threadfence();
    }
  }
}

}  // namespace xcb

extern "C" {

size_t xcb_ep_p2p_bytes(int32_t G, int32_t T_max, int32_t H, int32_t k) {
  if (G <= 0 || G > kEpMaxRanks || T_max <= 0 || H <= 0 || k <= 0) return 0;
  return p2p_layout(G, T_max, H, k).total;
}

int xcb_p2p_alloc(size_t bytes, void** ptr, void* handle) {
  if (!ptr || !handle || bytes == 0) return XCB_ERR_INVALID_ARG;
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) return XCB_ERR_CUDA;
  if (cudaMemset(p, 0, bytes) != cudaSuccess ||
      cudaIpcGetMemHandle(reinterpret_cast<cudaIpcMemHandle_t*>(handle), p) != cudaSuccess) {
    cudaFree(p);
    return XCB_ERR_CUDA;
  }
  *ptr = p;
  return XCB_OK;
}

int xcb_p2p_open(const void* handle, void** ptr) {
  if (!handle || !ptr) return XCB_ERR_INVALID_ARG;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  return cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess ? XCB_OK : XCB_ERR_CUDA;
}

int xcb_p2p_close(void* ptr) {
  if (!ptr) return XCB_ERR_INVALID_ARG;
  return cudaIpcCloseMemHandle(ptr) == cudaSuccess ? XCB_OK : XCB_ERR_CUDA;
}

int xcb_p2p_free(void* ptr) {
  if (!ptr) return XCB_ERR_INVALID_ARG;
  return cudaFree(ptr) == cudaSuccess ? XCB_OK : XCB_ERR_CUDA;
}

// Pushing blocks per peer for a buffer of T_max rows per rank (about 64 KB of rows each).  It must not depend on
// a step's T: the flags' targets are (steps so far) x nb.
static int p2p_blocks(int T_max, int H) {
  const long long bytes = (long long)T_max * H * 2;
  long long nb = (bytes + kP2pRowBytesPerBlock - 1) / kP2pRowBytesPerBlock;
  nb = nb < 1 ? 1 : nb;
  return (int)(nb > T_max ? T_max : nb);
}

static uint64_t p2p_timeout(uint64_t timeout_ns) { return timeout_ns ? timeout_ns : 2000000000ull; }

int xcb_ep_p2p_dispatch(const uint16_t* x, const float* logits, int32_t T, int32_t T_max, int32_t H, int32_t E,
                        int32_t k, int32_t G, int32_t rank, const uint64_t* peers, int32_t* status,
                        uint64_t timeout_ns, cudaStream_t stream) {
  if (T <= 0 || T > T_max || H <= 0 || H % 8 || E <= 0 || E > 512 || k <= 0 || k > 16 || k > E || G <= 0 ||
      G > kEpMaxRanks || rank < 0 || rank >= G)
    return XCB_ERR_INVALID_ARG;
  if (!x || !logits || !peers || !status || ((uintptr_t)x & 15u)) return XCB_ERR_INVALID_ARG;
  const int nb = p2p_blocks(T_max, H);
  ep_p2p_dispatch_kernel<<<G * nb, 256, 0, stream>>>(x, logits, T, T_max, H, E, k, G, rank, peers, nb,
                                                     p2p_layout(G, T_max, H, k), p2p_timeout(timeout_ns), status);
  return cudaGetLastError() == cudaSuccess ? XCB_OK : XCB_ERR_CUDA;
}

int xcb_ep_p2p_combine(const uint16_t* parts, int32_t T, int32_t T_max, int32_t H, int32_t k, int32_t G,
                       int32_t rank, const uint64_t* peers, uint16_t* out, int32_t* status, uint64_t timeout_ns,
                       cudaStream_t stream) {
  if (T <= 0 || T > T_max || H <= 0 || H % 8 || k <= 0 || k > 16 || G <= 0 || G > kEpMaxRanks || rank < 0 ||
      rank >= G)
    return XCB_ERR_INVALID_ARG;
  if (!parts || !peers || !out || !status || ((uintptr_t)parts & 15u) || ((uintptr_t)out & 7u))
    return XCB_ERR_INVALID_ARG;
  const int nb = p2p_blocks(T_max, H);
  ep_p2p_combine_kernel<<<G * nb, 256, 0, stream>>>(parts, T, T_max, H, G, rank, peers, nb,
                                                    p2p_layout(G, T_max, H, k), out, p2p_timeout(timeout_ns), status);
  return cudaGetLastError() == cudaSuccess ? XCB_OK : XCB_ERR_CUDA;
}

}  // extern "C"
