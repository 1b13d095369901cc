// GPU weight packer and NVFP4 quantiser.
//
// The packer replaces the reference's host-side torch repack (kernels/moe_w4a16_h200/moe_w4a16.py:3168-3190
// _pack_codes/_pack_scales, GF(2) word transform :3903-3933), which takes ~0.8 s per 8192x4096 tensor on a CPU;
// here one thread writes one packed word and the 6.3 GB of DeepSeek-V3-shaped weights pack in well under a
// second.  Two layouts per tensor: the decode-path layout (raw codes in m16n8k16 fragment order for the hardware
// FP4 converter) and, after it, the prefill-path layout (GF(2)-transformed words for the tensor-memory kernel).
// Layouts and bit map: xcalibur_b200/packer.py (module docstring).
#include <cuda_fp8.h>

#include "common.cuh"
#include "kernels.cuh"

namespace xcb {

// Canonical scale code of an E4M3 byte (see packer.scale_code); fold: 0 none, 1 zero block, 2 negative, 3 NaN.
__device__ __forceinline__ uint32_t scale_code(uint32_t b, int& fold) {
  const uint32_t e = (b >> 3) & 15u, m = b & 7u;
  if ((b & 0x7Fu) == 0x7Fu) { fold = 3; return 0; }
  if (e == 0 && m == 0) { fold = 1; return (7u + 2u) << 3; }
  fold = (b & 0x80u) ? 2 : 0;
  if (e >= 1) return ((e + 2u) << 3) | m;
  // subnormal m * 2^-9 -> normalised: 1:0 2:8 3:12 4:16 5:18 6:20 7:22
  const uint32_t sub = 0x16141210u;  // codes for m = 4..7 packed as bytes
  if (m >= 4) return (sub >> (8 * (m - 4))) & 0xFFu;
  return m == 1 ? 0u : (m == 2 ? 8u : 12u);
}

__device__ __forceinline__ int orig_row(int pr, int R, int gate_up) {
  if (!gate_up) return pr;
  const int blk = pr >> 4, r = pr & 15;
  return r < 8 ? blk * 8 + r : (R >> 1) + blk * 8 + (r - 8);
}

// Decode-path layout: per 16-row unit, K/64 slice records of 576 bytes, [32 lanes][4 words] of codes then
// [32 lanes][2] scale bytes.  Word j of lane L = 4g + t in slice S holds the raw code bytes
// (row g, row g + 8, row g, row g + 8) at code byte 32S + 8t + 2j, +0, +1, +1 (low nibble = even k): exactly the
// f16x2 registers cvt.rn.f16x2.e2m1x2 produces for the four m16n8k16 A fragments.  The scale bytes of lane L are
// the raw E4M3 scales of rows g and g + 8 for block 4S + t (cvt.rn.f16x2.e4m3x2 takes them as they are).
__global__ void pack_codes_kernel(PackParams p) {
  const int nS = p.K / 64, nb = p.R / 16;
  const size_t words_per_unit = (size_t)nS * 128;
  const size_t total = (size_t)p.E * nb * words_per_unit;
  const size_t K2 = p.K / 2;
  for (size_t w = (size_t)blockIdx.x * blockDim.x + threadIdx.x; w < total; w += (size_t)gridDim.x * blockDim.x) {
    const int j = (int)(w & 3), lane = (int)((w >> 2) & 31);
    const size_t rest = w >> 7;
    const int S = (int)(rest % nS);
    const size_t ub = rest / nS;          // e * nb + rb
    const int rb = (int)(ub % nb), e = (int)(ub / nb);
    const int g = lane >> 2, t = lane & 3;
    const int ro0 = orig_row(rb * 16 + g, p.R, p.gate_up), ro1 = orig_row(rb * 16 + g + 8, p.R, p.gate_up);
    const size_t bidx = (size_t)32 * S + 8 * t + 2 * j;
    const uint8_t* c0 = p.codes + ((size_t)e * p.R + ro0) * K2;
    const uint8_t* c1 = p.codes + ((size_t)e * p.R + ro1) * K2;
    const uint32_t word = (uint32_t)c0[bidx] | ((uint32_t)c1[bidx] << 8) | ((uint32_t)c0[bidx + 1] << 16) |
                          ((uint32_t)c1[bidx + 1] << 24);
    reinterpret_cast<uint32_t*>(p.out + ub * (size_t)9 * p.K + (size_t)S * 576)[lane * 4 + j] = word;
  }
}

__global__ void pack_scales_kernel(PackParams p) {
  const int nS = p.K / 64, nb = p.R / 16;
  const size_t total = (size_t)p.E * nb * nS * 32;  // one thread per (unit, slice, lane): two bytes
  const size_t K16 = p.K / 16;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int lane = (int)(i & 31);
    const size_t rest = i >> 5;
    const int S = (int)(rest % nS);
    const size_t ub = rest / nS;
    const int rb = (int)(ub % nb), e = (int)(ub / nb);
    const int g = lane >> 2, t = lane & 3;
    const int ro0 = orig_row(rb * 16 + g, p.R, p.gate_up), ro1 = orig_row(rb * 16 + g + 8, p.R, p.gate_up);
    const int blk = 4 * S + t;
    const uint8_t s0 = p.sf[((size_t)e * p.R + ro0) * K16 + blk], s1 = p.sf[((size_t)e * p.R + ro1) * K16 + blk];
    if ((s0 & 0x7Fu) == 0x7Fu || (s1 & 0x7Fu) == 0x7Fu) set_status(p.status, XCB_STATUS_NAN_SCALE);
    uint8_t* dst = p.out + ub * (size_t)9 * p.K + (size_t)S * 576 + 512 + lane * 2;
    dst[0] = s0;
    dst[1] = s1;
  }
}

// ------------------------------------------------------------------------------------------------ prefill layout
// Original row of wide-layout packed row pr: per 128-row block, lanes 0-31 gate / 32-63 up / 64-95 gate / 96-127 up
// of the block's 64 features (gate_up); identity for down.
__device__ __forceinline__ int wide_orig_row(int pr, int R, int gate_up) {
  if (!gate_up) return pr;
  const int b = pr >> 7, q = (pr >> 5) & 3, i = pr & 31;
  return 64 * b + 32 * (q >> 1) + i + ((q & 1) ? (R >> 1) : 0);
}

// One thread per packed word: the row's 4 code bytes at k/2 (k = 8 consecutive weights of one row), folded by the
// block's scale and sent through T.
__global__ void pack_wide_codes_kernel(PackParams p) {
  __shared__ uint32_t tab[4][256];
  for (int i = threadIdx.x; i < 1024; i += blockDim.x) tab[i >> 8][i & 255] = p.tabs[i];
  __syncthreads();
  const int ns = p.K / 256, nb = p.R / 128;
  const size_t total = (size_t)p.E * p.R * (p.K / 8);
  const size_t K2 = p.K / 2, K16 = p.K / 16;
  for (size_t w = (size_t)blockIdx.x * blockDim.x + threadIdx.x; w < total; w += (size_t)gridDim.x * blockDim.x) {
    const int wq = (int)(w & 3), row = (int)((w >> 2) & 127), j = (int)((w >> 9) & 1), c = (int)((w >> 10) & 3);
    const size_t rest = w >> 12;
    const int s = (int)(rest % ns);
    const size_t ub = rest / ns;  // e * nb + b
    const int b = (int)(ub % nb), e = (int)(ub / nb);
    const int ro = wide_orig_row(128 * b + row, p.R, p.gate_up);
    const int k = 256 * s + 64 * c + 32 * j + 8 * wq;
    const size_t rbase = (size_t)e * p.R + ro;
    int f;
    scale_code(p.sf[rbase * K16 + k / 16], f);
    if (f == 3) set_status(p.status, XCB_STATUS_NAN_SCALE);
    uint32_t word = *reinterpret_cast<const uint32_t*>(p.codes + rbase * K2 + k / 2);
    word = f == 1 ? 0u : (f == 2 ? word ^ 0x88888888u : word);
    const uint32_t packed = tab[0][word & 255] ^ tab[1][(word >> 8) & 255] ^ tab[2][(word >> 16) & 255] ^ tab[3][word >> 24];
    reinterpret_cast<uint32_t*>(p.out + ((ub * ns + s) * 4 + c) * 4608)[(j * 128 + row) * 4 + wq] = packed;
  }
}

__global__ void pack_wide_scales_kernel(PackParams p) {
  const int ns = p.K / 256, nb = p.R / 128;
  const size_t total = (size_t)p.E * p.R * (p.K / 16);
  const size_t K16 = p.K / 16;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int blk = (int)(i & 3), row = (int)((i >> 2) & 127), c = (int)((i >> 9) & 3);
    const size_t rest = i >> 11;
    const int s = (int)(rest % ns);
    const size_t ub = rest / ns;
    const int b = (int)(ub % nb), e = (int)(ub / nb);
    const int ro = wide_orig_row(128 * b + row, p.R, p.gate_up);
    int f;
    const uint32_t code = scale_code(p.sf[((size_t)e * p.R + ro) * K16 + 16 * s + 4 * c + blk], f);
    p.out[((ub * ns + s) * 4 + c) * 4608 + 4096 + row * 4 + blk] = (uint8_t)code;
  }
}

int launch_pack(const PackParams& p, cudaStream_t stream) {
  pack_codes_kernel<<<148 * 8, 256, 0, stream>>>(p);
  if (cudaGetLastError() != cudaSuccess) return XCB_ERR_CUDA;
  pack_scales_kernel<<<148 * 4, 256, 0, stream>>>(p);
  if (cudaGetLastError() != cudaSuccess) return XCB_ERR_CUDA;
  PackParams q = p;
  q.out = p.out + (size_t)p.E * (p.R / 16) * 9 * (size_t)p.K;  // the prefill layout follows the decode layout
  pack_wide_codes_kernel<<<148 * 8, 256, 0, stream>>>(q);
  if (cudaGetLastError() != cudaSuccess) return XCB_ERR_CUDA;
  pack_wide_scales_kernel<<<148 * 4, 256, 0, stream>>>(q);
  return cudaGetLastError() == cudaSuccess ? XCB_OK : XCB_ERR_CUDA;
}

// ------------------------------------------------------------------------------------------------ quantiser
__global__ void amax_kernel(QuantParams p) {
  const size_t per = (size_t)p.R * p.K;
  const int e = blockIdx.y;
  float m = 0.f;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < per; i += (size_t)gridDim.x * blockDim.x)
    m = fmaxf(m, fabsf(p.w[(size_t)e * per + i]));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) atomicMax(reinterpret_cast<int*>(p.amax + e), __float_as_int(m));
}

// E2M1 round-to-nearest-even with saturation; a value that rounds to zero is +0.
__device__ __forceinline__ uint32_t e2m1_rne(float q) {
  const float a = fabsf(q);
  uint32_t c = (a > 0.25f) + (a > 0.75f) + (a > 1.25f) + (a > 1.75f) + (a > 2.5f) + (a > 3.5f) + (a > 5.0f);
  c += (a == 0.75f) | (a == 1.75f) | (a == 3.5f);
  return (c != 0 && signbit(q)) ? (c | 8u) : c;
}

__global__ void quant_kernel(QuantParams p) {
  const size_t nblk = (size_t)p.E * p.R * (p.K / 16);
  const size_t blk_per_e = (size_t)p.R * (p.K / 16);
  for (size_t b = (size_t)blockIdx.x * blockDim.x + threadIdx.x; b < nblk; b += (size_t)gridDim.x * blockDim.x) {
    const int e = (int)(b / blk_per_e);
    float gsv = p.amax[e] / 2688.0f;
    if (gsv == 0.f) gsv = 1.f;
    const float4* src = reinterpret_cast<const float4*>(p.w + b * 16);
    float v[16];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float4 f = src[i];
      v[4 * i] = f.x; v[4 * i + 1] = f.y; v[4 * i + 2] = f.z; v[4 * i + 3] = f.w;
    }
    float bm = 0.f;
#pragma unroll
    for (int i = 0; i < 16; ++i) bm = fmaxf(bm, fabsf(v[i]));
    const float sval = (bm / 6.0f) / gsv;
    const __nv_fp8_storage_t s8 = __nv_cvt_float_to_fp8(sval, __NV_SATFINITE, __NV_E4M3);
    const __half_raw hr = __nv_cvt_fp8_to_halfraw(s8, __NV_E4M3);
    const float sdec = __half2float(*reinterpret_cast<const __half*>(&hr));
    const float scale = sdec * gsv;
    uint8_t* cd = p.codes + b * 8;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float q0 = scale == 0.f ? 0.f : v[2 * i] / scale;
      const float q1 = scale == 0.f ? 0.f : v[2 * i + 1] / scale;
      cd[i] = (uint8_t)(e2m1_rne(q0) | (e2m1_rne(q1) << 4));
    }
    p.sf[b] = (uint8_t)s8;
    if ((b % blk_per_e) == 0) p.gs[e] = gsv;
  }
}

int launch_quantize(const QuantParams& p, cudaStream_t stream) {
  if (cudaMemsetAsync(p.amax, 0, sizeof(float) * p.E, stream) != cudaSuccess) return XCB_ERR_CUDA;
  amax_kernel<<<dim3(64, p.E), 256, 0, stream>>>(p);
  if (cudaGetLastError() != cudaSuccess) return XCB_ERR_CUDA;
  quant_kernel<<<148 * 8, 256, 0, stream>>>(p);
  return cudaGetLastError() == cudaSuccess ? XCB_OK : XCB_ERR_CUDA;
}

}  // namespace xcb
