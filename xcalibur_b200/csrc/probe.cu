// HBM read-bandwidth probes for sm_100a: the two ways the decode kernel can stream weights.
//
//   mode 0: 1-D bulk-copy ring on the TMA engine (one issuing thread, `stages` x `chunk` bytes in flight per CTA),
//           consumers release each stage after touching one word of it;
//   mode 1: mode 0 with an L2 evict-first cache hint on every copy;
//   mode 2: vector loads (16 B per thread, `stages` independent loads in flight per thread), summed so the loads
//           cannot be removed.
//
// Every CTA streams a contiguous share of `bytes`.  Reference counterpart: the BW_SRC bulk-copy probes of
// kernels/moe_w4a16_h200/moe_w4a16.py:2890-3061 (dead code there); here they measure the roofline denominators
// and the ring shapes the decode kernel is sized from.
#include "common.cuh"

namespace xcb {

struct ProbeParams {
  const uint8_t* src;
  size_t bytes;
  const long long* regions;  // optional: byte offsets of `nreg` regions of bytes/nreg each (expert-like layout)
  int nreg;
  int mode, chunk, stages;
  unsigned long long timeout_ns;
  int* status;
  float* sink;
};

__global__ void __launch_bounds__(1024) probe_kernel(ProbeParams p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const size_t per = (p.bytes / gridDim.x) / p.chunk * p.chunk;
  const uint8_t* base = p.src + per * blockIdx.x;
  if (p.regions) {  // CTA c streams its slice of region c * nreg / G, like the decode kernel's expert ranges
    const int r = (int)((long long)blockIdx.x * p.nreg / gridDim.x);
    const int c0 = (int)(((long long)r * gridDim.x + p.nreg - 1) / p.nreg);
    base = p.src + p.regions[r] + per * (blockIdx.x - c0);
  }
  const int tid = threadIdx.x;
  uint32_t* sum = reinterpret_cast<uint32_t*>(p.sink);
  if (p.mode == 2) {
    uint32_t acc = 0;
    const uint4* v = reinterpret_cast<const uint4*>(base);
    const size_t n = per / 16;
    const int U = 8;
    for (size_t i = tid; i < n; i += (size_t)blockDim.x * U) {
      uint4 r[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const size_t j = i + (size_t)u * blockDim.x;
        r[u] = j < n ? __ldcs(v + j) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int u = 0; u < U; ++u) acc ^= r[u].x ^ r[u].y ^ r[u].z ^ r[u].w;
    }
    acc = __reduce_xor_sync(0xffffffffu, acc);
    if ((tid & 31) == 0) atomicXor(sum, acc);
    return;
  }
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)p.stages * p.chunk);
  uint64_t* empty = full + p.stages;
  const int nconsumer_warps = blockDim.x / 32 - 1;
  if (tid == 0) {
    for (int i = 0; i < p.stages; ++i) {
      mbar_init(full + i, 1);
      mbar_init(empty + i, nconsumer_warps);
    }
    fence_mbar_init();
  }
  __syncthreads();
  const int nch = (int)(per / p.chunk);
  const int warp = tid >> 5, lane = tid & 31;
  if (warp == nconsumer_warps) {
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      for (int it = 0; it < nch; ++it) {
        const int st = it % p.stages;
        if (it >= p.stages && !mbar_wait(empty + st, ((it / p.stages) + 1) & 1, p.timeout_ns, p.status)) break;
        mbar_arrive_expect_tx(full + st, p.chunk);
        if (p.mode == 1)
          bulk_g2s_stream(smem + (size_t)st * p.chunk, base + (size_t)it * p.chunk, p.chunk, full + st, pol);
        else
          bulk_g2s(smem + (size_t)st * p.chunk, base + (size_t)it * p.chunk, p.chunk, full + st);
      }
      for (int i = max(0, nch - p.stages); i < nch; ++i)
        mbar_wait(full + (i % p.stages), (i / p.stages) & 1, p.timeout_ns, p.status);
    }
  } else {
    // the consumer warps read every word of every stage (a streaming reduction, as a GEMV reads its weights)
    uint32_t acc = 0;
    const int words = p.chunk / 16;
    for (int it = 0; it < nch; ++it) {
      const int st = it % p.stages;
      mbar_wait(full + st, (it / p.stages) & 1, p.timeout_ns, p.status);
      const uint4* w = reinterpret_cast<const uint4*>(smem + (size_t)st * p.chunk);
      for (int i = lane + 32 * warp; i < words; i += 32 * nconsumer_warps) {
        const uint4 v = w[i];
        acc ^= v.x ^ v.y ^ v.z ^ v.w;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(empty + st);
    }
    acc = __reduce_xor_sync(0xffffffffu, acc);
    if (lane == 0) atomicXor(sum, acc);
  }
}

}  // namespace xcb

using namespace xcb;

extern "C" int xcb_hbm_probe(const void* src, size_t bytes, int mode, int chunk, int stages, int ctas_per_sm,
                             int threads, const long long* regions, int nreg, int32_t* status, float* sink,
                             cudaStream_t stream) {
  if (!src || !status || !sink || bytes == 0 || mode < 0 || mode > 2 || ctas_per_sm < 1 || ctas_per_sm > 8)
    return XCB_ERR_INVALID_ARG;
  if (mode != 2 && (chunk < 1024 || chunk % 1024 || stages < 1 || stages > 64)) return XCB_ERR_INVALID_ARG;
  if (threads < 64 || threads > 1024 || threads % 32) return XCB_ERR_INVALID_ARG;
  if (((uintptr_t)src & 1023u) != 0) return XCB_ERR_INVALID_ARG;
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return XCB_ERR_CUDA;
  const size_t smem = mode == 2 ? 0 : (size_t)stages * chunk + 2 * 64 * 8;
  if (smem > 227 * 1024) return XCB_ERR_UNSUPPORTED;
  if (cudaFuncSetAttribute(probe_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return XCB_ERR_CUDA;
  if (regions && (nreg < 1 || nreg > sms * ctas_per_sm)) return XCB_ERR_INVALID_ARG;
  ProbeParams p{(const uint8_t*)src, bytes, regions, nreg, mode, chunk < 16 ? 16 : chunk, stages, 2000000000ull, status, sink};
  probe_kernel<<<sms * ctas_per_sm, threads, smem, stream>>>(p);
  return cudaGetLastError() == cudaSuccess ? XCB_OK : XCB_ERR_CUDA;
}
