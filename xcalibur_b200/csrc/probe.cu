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
//
// The tensor-pipe probe (xcb_mma_probe) times back-to-back tcgen05.mma kind::f16 (M = 128, K = 16) the way the
// prefill kernel issues them: 64-k chunks of four MMAs cycling four A and four B slots, A from tensor memory or
// shared memory, with a tcgen05.commit after every `commit_every` chunks (a power of two; 0: none); one CTA per SM,
// cycles per CTA.
#include "common.cuh"
#include "tcgen05.cuh"

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
  if (p.mode == 2) {
    float acc = 0.f;
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
      for (int u = 0; u < U; ++u) acc += __uint_as_float(r[u].x ^ r[u].y ^ r[u].z ^ r[u].w);
    }
    if (acc == 1.2345f) p.sink[0] = acc;
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
    float acc = 0.f;
    for (int it = 0; it < nch; ++it) {
      const int st = it % p.stages;
      mbar_wait(full + st, (it / p.stages) & 1, p.timeout_ns, p.status);
      acc += __uint_as_float(reinterpret_cast<const uint32_t*>(smem + (size_t)st * p.chunk)[(lane + 32 * warp) % (p.chunk / 4)]);
      __syncwarp();
      if (lane == 0) mbar_arrive(empty + st);
    }
    if (acc == 1.2345f) p.sink[0] = acc;
  }
}

constexpr int kMpA = 4 * 16384, kMpB = 4 * 32768;  // four A slots (128 x 64 bf16), four B slots (256 x 64 bf16)

__device__ __forceinline__ void mma_ss(uint32_t d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc)
      : "memory");
}

__global__ void __launch_bounds__(128, 1) mma_probe_kernel(int a_smem, int n, int chunks, int commit_every,
                                                           unsigned long long* cycles, int* status) {
  extern __shared__ uint8_t mp_raw[];
  uint8_t* sm = mp_raw + ((1024u - (smem_u32(mp_raw) & 1023u)) & 1023u);
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + kMpA + kMpB);  // [0]: per-window commits, [1]: the final one
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bar + 2);
  const int warp = threadIdx.x >> 5;
  for (int i = threadIdx.x; i < (kMpA + kMpB) / 16; i += blockDim.x)  // operand values do not matter
    reinterpret_cast<uint4*>(sm)[i] = make_uint4(0x3f803f80u, 0x3f803f80u, 0x3f803f80u, 0x3f803f80u);
  if (threadIdx.x == 0) {
    mbar_init(bar, 1);
    mbar_init(bar + 1, 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(tslot, 512);
    tmem_relinquish();
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  if (warp == 0) {
    const uint32_t idesc = idesc_bf16_m128(n);
    const uint64_t ad0 = sdesc_sw128(smem_u32(sm)), bd0 = sdesc_sw128(smem_u32(sm + kMpA));
    const unsigned long long t0 = clock64();
    for (int c = 0; c < chunks; ++c) {
      const uint32_t s = c & 3;
      if (elect_one()) {
        const uint64_t bd = bd0 + (uint64_t)(s * (32768 >> 4));
        if (!a_smem) {
          const uint32_t ta = tmem + s * 32;  // A ring in columns [0, 128), D from column 128
          tc_mma_ts(tmem + 128, ta, bd, idesc, c > 0);
          tc_mma_ts(tmem + 128, ta + 8, bd + 2, idesc, 1u);
          tc_mma_ts(tmem + 128, ta + 16, bd + 4, idesc, 1u);
          tc_mma_ts(tmem + 128, ta + 24, bd + 6, idesc, 1u);
        } else {
          const uint64_t ad = ad0 + (uint64_t)(s * (16384 >> 4));
          mma_ss(tmem + 128, ad, bd, idesc, c > 0);
          mma_ss(tmem + 128, ad + 2, bd + 2, idesc, 1u);
          mma_ss(tmem + 128, ad + 4, bd + 4, idesc, 1u);
          mma_ss(tmem + 128, ad + 6, bd + 6, idesc, 1u);
        }
        if (commit_every && (c & (commit_every - 1)) == commit_every - 1) tc_commit(bar);
      }
      __syncwarp();
    }
    if (elect_one()) tc_commit(bar + 1);  // completes once every MMA above has
    __syncwarp();
    mbar_wait(bar + 1, 0, 2000000000ull, status);
    if (threadIdx.x == 0) cycles[blockIdx.x] = clock64() - t0;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace xcb

using namespace xcb;

extern "C" int xcb_mma_probe(int a_smem, int n, int chunks, int commit_every, unsigned long long* cycles,
                             int32_t* status, cudaStream_t stream) {
  if (!cycles || !status || n < 16 || n > 256 || n % 16 || chunks < 1 || commit_every < 0 ||
      (commit_every & (commit_every - 1)))
    return XCB_ERR_INVALID_ARG;
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return XCB_ERR_CUDA;
  const int smem = kMpA + kMpB + 64 + 1024;
  if (cudaFuncSetAttribute(mma_probe_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return XCB_ERR_CUDA;
  mma_probe_kernel<<<sms, 128, smem, stream>>>(a_smem, n, chunks, commit_every, cycles, status);
  return cudaGetLastError() == cudaSuccess ? XCB_OK : XCB_ERR_CUDA;
}

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
