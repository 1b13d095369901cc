// Shared device helpers for the sm_100a MoE kernels: PTX wrappers for mbarriers, 1-D bulk copies (TMA engine),
// bounded spin-waits, the legacy m16n8k16 tensor-core step used by the decode path, and the FP4 decoder.
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "../../include/xcb_moe.h"

namespace xcb {

// ------------------------------------------------------------------------------------------------ time / status
__device__ __forceinline__ uint64_t gtimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Record an error bit in the workspace status word (read back by xcb_moe_read_status).
__device__ __forceinline__ void set_status(int* status, int bit) { atomicOr(status, bit); }

// Programmatic dependent launch: a kernel launched with the programmatic-serialisation attribute may start while
// the previous kernel of its stream is still running; it must wait for that kernel (and its memory) before it
// reads anything another kernel wrote.  launch_dependents lets the next kernel be scheduled early.  Both are no-ops
// for a kernel launched without the attribute.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ int ld_acquire(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Spin until *p >= target or the deadline passes.  Returns false (and sets the status bit) on timeout.
__device__ __forceinline__ bool wait_geq(const int* p, int target, uint64_t timeout_ns, int* status) {
  if (ld_acquire(p) >= target) return true;
  const uint64_t t0 = gtimer();
  while (ld_acquire(p) < target) {
    __nanosleep(64);
    if (gtimer() - t0 > timeout_ns) {
      set_status(status, XCB_STATUS_DEVICE_TIMEOUT);
      return false;
    }
  }
  return true;
}

// ------------------------------------------------------------------------------------------------ mbarrier
__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("{\n .reg .b64 st;\n mbarrier.arrive.shared::cta.b64 st, [%0];\n}" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("{\n .reg .b64 st;\n mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n}" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait for the phase with the given parity to complete.  Returns false on timeout (status bit set).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint64_t timeout_ns, int* status) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = gtimer();
  while (!mbar_try_wait(bar, parity)) {
    if (gtimer() - t0 > timeout_ns) {
      set_status(status, XCB_STATUS_DEVICE_TIMEOUT);
      return false;
    }
  }
  return true;
}

// 1-D bulk copy global -> shared through the TMA engine, completing on an mbarrier (16-byte aligned, size % 16 == 0).
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
// Same with an L2 evict-first policy (weights are streamed once per call).
__device__ __forceinline__ void bulk_g2s_stream(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                                uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}
// Fire-and-forget bulk prefetch of [src, src + bytes) into L2 (16-byte aligned, size % 16 == 0).
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}
__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// Named barrier over a subset of warps (id 0 is __syncthreads).
__device__ __forceinline__ void named_bar(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// ------------------------------------------------------------------------------------------------ math
// D = A(16x16 bf16, row) * B(16x8 bf16, col) + D, fp32 accumulate.
__device__ __forceinline__ void mma_16816(float* d, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                          uint32_t b1) {
  asm(  // not volatile: no side effects, so the compiler may interleave it with the decode of other words
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t bf16x2_mul_lo(uint32_t a, uint32_t s) {  // a * (s.lo, s.lo)
  __nv_bfloat162 r = __hmul2(*reinterpret_cast<__nv_bfloat162*>(&a), __low2bfloat162(*reinterpret_cast<__nv_bfloat162*>(&s)));
  return *reinterpret_cast<uint32_t*>(&r);
}
__device__ __forceinline__ uint32_t bf16x2_mul_hi(uint32_t a, uint32_t s) {  // a * (s.hi, s.hi)
  __nv_bfloat162 r = __hmul2(*reinterpret_cast<__nv_bfloat162*>(&a), __high2bfloat162(*reinterpret_cast<__nv_bfloat162*>(&s)));
  return *reinterpret_cast<uint32_t*>(&r);
}

// FP4 decoder D (its GF(2) rows and the packing transform T = D^-1 P live in xcalibur_b200/packer.py): one packed
// word -> four bf16x2 registers, each field e2m1 * 2^-126.  8 integer ops: two shifts (IMAD-able), two
// rotations, four LOP3 with the field mask.
__device__ __forceinline__ void decode_fp4x8(uint32_t q, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  constexpr uint32_t M = 0x81C081C0u;
  const uint32_t u6 = q << 6;
  r0 = q & M;
  r1 = (q << 4) & M;
  r2 = (u6 ^ __funnelshift_l(q, q, 10)) & M;
  r3 = (u6 ^ __funnelshift_l(q, q, 12)) & M;
}

// Two canonical scale codes (row g in byte 0, row g + 8 in byte 1) -> bf16x2 (scale * 2^74 each).
__device__ __forceinline__ uint32_t scale_pair(uint32_t two_codes) {
  return __byte_perm(two_codes, 0u, 0x4140u) * 16u + 0x60006000u;
}

// 2^52 as fp32: the decoded weights carry 2^-52, the epilogue multiplies it back with the global scale.
constexpr float kTwo52 = 4503599627370496.0f;

__device__ __forceinline__ uint16_t f2bf(float v) {
  __nv_bfloat16 b = __float2bfloat16_rn(v);
  return *reinterpret_cast<uint16_t*>(&b);
}
__device__ __forceinline__ float bf2f(uint16_t v) { return __uint_as_float((uint32_t)v << 16); }

// Exclusive scan of n <= 1024 ints in shared memory by one warp (each lane owns a contiguous run); every lane
// returns the total.
__device__ __forceinline__ int warp_exclusive_scan(int* a, int n) {
  const int lane = threadIdx.x & 31;
  const int per = (n + 31) / 32;
  const int b = min(n, lane * per), e = min(n, b + per);
  int s = 0;
  for (int i = b; i < e; ++i) s += a[i];
  int incl = s;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  int run = incl - s;
  for (int i = b; i < e; ++i) {
    const int v = a[i];
    a[i] = run;
    run += v;
  }
  return __shfl_sync(0xffffffffu, incl, 31);
}

// Order-preserving map float -> uint32 (larger float, larger key; -0 and +0 share a key, so they tie).
__device__ __forceinline__ uint32_t float_key(float f) {
  const uint32_t b = __float_as_uint(f == 0.f ? 0.f : f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float key_float(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
}

// Top-k of one token's logits by one warp: rank by value descending, ties to the lower index; weights = softmax
// over the selected logits (summed in route order).  Lane s < k returns route s in (id, w).  E <= 512.
// Each round is two warp reductions: the largest key, then the lowest index holding it.  The first half loads the
// row into registers (split out so a caller can issue the loads early).
__device__ __forceinline__ void warp_topk_load(const float* row, int E, uint32_t (&key)[16]) {
  const int lane = threadIdx.x & 31;
  const int per = (E + 31) / 32;
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const int e = lane + 32 * j;
    key[j] = (j < per && e < E) ? float_key(row[e]) : 0u;  // 0 is below every real key
  }
}
__device__ __forceinline__ void warp_topk_select(const uint32_t (&key)[16], int k, int& id, float& w) {
  const int lane = threadIdx.x & 31;
  uint32_t used = 0, my_key = 0;
  int my_i = -1;
  for (int s = 0; s < k; ++s) {
    uint32_t bk = 0;
    int bj = -1;
#pragma unroll
    for (int j = 0; j < 16; ++j)
      if (!((used >> j) & 1u) && key[j] > bk) {  // strict: the lower j (lower index) wins a tie
        bk = key[j];
        bj = j;
      }
    const uint32_t mk = __reduce_max_sync(0xffffffffu, bk);
    const uint32_t mi = __reduce_min_sync(0xffffffffu, (bj >= 0 && bk == mk) ? (uint32_t)(lane + 32 * bj) : 0xffffffffu);
    if ((int)(mi & 31) == lane) used |= 1u << (mi >> 5);
    if (lane == s) {
      my_key = mk;
      my_i = (int)mi;
    }
  }
  const float top = key_float(__shfl_sync(0xffffffffu, my_key, 0));
  const float ex = (lane < k) ? expf(key_float(my_key) - top) : 0.f;
  float den = 0.f;
  for (int s = 0; s < k; ++s) den += __shfl_sync(0xffffffffu, ex, s);
  id = my_i;
  w = ex / den;
}
__device__ __forceinline__ void warp_topk(const float* row, int E, int k, int& id, float& w) {
  uint32_t key[16];
  warp_topk_load(row, E, key);
  warp_topk_select(key, k, id, w);
}

}  // namespace xcb
