// Decode-path MoE kernel: one persistent launch runs gate_up + SwiGLU (phase A), down (phase B) and the
// weighted combine for jobs of at most 8 tokens.  This is the HBM-bound path (T = 1 decode streams ~200 MB of
// FP4 weights for 8 experts), so it is built around the weight stream:
//
// * One CTA per SM (1 x 288 threads): warp 8 is a producer that streams packed units through an 8-stage
//   shared-memory ring with 1-D bulk copies (TMA engine, L2 evict-first), 9 KB per stage (16 slices of 64 k).
// * Warps 0..7 split each unit's k slices; per 4 packed words a lane runs the GF(2) decoder (8 integer ops per
//   8 weights), one bf16x2 multiply per register by the block scale pair, and one m16n8k16 tensor-core step
//   whose A operand comes straight from registers.  A register-fed MMA reads no shared memory for the weights,
//   which is why this path does not use tcgen05: at T <= 8 the weights are used once, and staging decoded bf16
//   tiles through shared memory for tcgen05 would double the shared-memory traffic per weight.
// * Work: CTA c owns a contiguous range of phase-A units (job, 16-row block) and of phase-B units.  A phase-B
//   unit waits (bounded spin) until all phase-A units of its job are done; meanwhile the producer keeps
//   streaming phase-B weights, so HBM stays busy across the phase boundary.
// * After a grid barrier (bounded) every CTA combines (token, 1024-column) items:
//   out = bf16(sum_s w_s * y_s) or the post-norm form.  The last CTA to exit zeroes the grid counters; the
//   per-job counters are zeroed by the router launch that precedes every call.
//
// Reference counterpart: moe_fused's skinny path (kernels/moe_w4a16_h200/moe_w4a16.py:754-1133 skinny ring,
// :1602-1785 warp-specialised epilogues, :2617-2641 grid barrier, :2654-2796 final combine).
#include "common.cuh"
#include "kernels.cuh"
#include "workspace.cuh"

namespace xcb {

constexpr int SK_NW = 8;
constexpr int SK_THREADS = (SK_NW + 1) * 32;
constexpr int SK_CS = 16;                               // slices (64 k) per stage
constexpr int SK_CODE_BYTES = SK_CS * 512;              // 8 KB codes
constexpr int SK_STAGE_BYTES = SK_CODE_BYTES + SK_CS * 64;  // + 1 KB scale codes
constexpr int SK_NSTAGE = 8;

struct SkSmemOffsets {
  int ring, xs, red, bars, total, pitch_max;
};

__host__ __device__ inline SkSmemOffsets sk_smem(int H, int I) {
  SkSmemOffsets o;
  const int kmax = H > I ? H : I;
  o.pitch_max = kmax * 2 + 16;
  o.ring = 0;
  o.xs = SK_NSTAGE * SK_STAGE_BYTES;
  o.red = o.xs + 8 * o.pitch_max;
  o.bars = o.red + 2 * SK_NW * 32 * 4 * 4;
  o.total = o.bars + 2 * SK_NSTAGE * 8 + 16;
  return o;
}

// One 64-k slice for one warp: 4 packed words -> 4 tensor-core steps.
__device__ __forceinline__ void sk_slice(const uint8_t* stage, int s, const uint8_t* xrow, int S, int lane, int t,
                                         float* acc) {
  const uint4 cw = *reinterpret_cast<const uint4*>(stage + s * 512 + lane * 16);
  const uint32_t sc = *reinterpret_cast<const uint16_t*>(stage + SK_CODE_BYTES + (s >> 2) * 256 + lane * 8 + (s & 3) * 2);
  const uint4 xa = *reinterpret_cast<const uint4*>(xrow + S * 128 + t * 32);
  const uint4 xb = *reinterpret_cast<const uint4*>(xrow + S * 128 + t * 32 + 16);
  const uint32_t s2 = scale_pair(sc);
  const uint32_t qw[4] = {cw.x, cw.y, cw.z, cw.w};
  const uint32_t xv[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint32_t r0, r1, r2, r3;
    decode_fp4x8(qw[j], r0, r1, r2, r3);
    mma_16816(acc, bf16x2_mul_lo(r0, s2), bf16x2_mul_hi(r1, s2), bf16x2_mul_lo(r2, s2), bf16x2_mul_hi(r3, s2),
              xv[2 * j], xv[2 * j + 1]);
  }
}

__global__ void __launch_bounds__(SK_THREADS, 1) skinny_kernel(SkinnyParams p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const SkSmemOffsets so = sk_smem(p.H, p.I);
  uint8_t* ring = smem + so.ring;
  uint8_t* xs = smem + so.xs;
  float* red = reinterpret_cast<float*>(smem + so.red);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + so.bars);
  uint64_t* empty = full + SK_NSTAGE;
  int* status = p.ctl + kCtlStatus;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = gridDim.x, bid = blockIdx.x;
  const int njobs = p.ctl[kCtlJobs];
  const int nrbA = (2 * p.I) / 16, nrbB = p.H / 16;
  const int nSA = p.H / 64, nSB = p.I / 64;           // slices per unit
  const int nchA = (nSA + SK_CS - 1) / SK_CS, nchB = (nSB + SK_CS - 1) / SK_CS;
  const long long nA = (long long)njobs * nrbA, nB = (long long)njobs * nrbB;
  const long long a0 = nA * bid / G, a1 = nA * (bid + 1) / G;
  const long long b0 = nB * bid / G, b1 = nB * (bid + 1) / G;
  const size_t unitA = (size_t)9 * p.H, unitB = (size_t)9 * p.I;

  if (tid == 0) {
    for (int i = 0; i < SK_NSTAGE; ++i) {
      mbar_init(full + i, 1);
      mbar_init(empty + i, SK_NW);
    }
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == SK_NW) {
    // ------------------------------------------------------------------ producer
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      int it = 0;
      bool ok = true;
      for (int ph = 0; ph < 2 && ok; ++ph) {
        const long long u0 = ph ? b0 : a0, u1 = ph ? b1 : a1;
        const int nrb = ph ? nrbB : nrbA, nS = ph ? nSB : nSA, nch = ph ? nchB : nchA;
        const uint8_t* wbase = ph ? p.wB : p.wA;
        const size_t ub = ph ? unitB : unitA;
        const size_t code_bytes = (size_t)nS * 512;
        for (long long u = u0; u < u1 && ok; ++u) {
          const int jidx = (int)(u / nrb), rb = (int)(u % nrb);
          const int e = p.jobs[jidx].x;
          const uint8_t* unit = wbase + ((size_t)e * nrb + rb) * ub;
          for (int c = 0; c < nch; ++c, ++it) {
            const int ns = min(SK_CS, nS - c * SK_CS);
            const int st = it % SK_NSTAGE;
            if (it >= SK_NSTAGE && !mbar_wait(empty + st, ((it / SK_NSTAGE) + 1) & 1, p.timeout_ns, status)) {
              ok = false;
              break;
            }
            uint8_t* dst = ring + st * SK_STAGE_BYTES;
            mbar_arrive_expect_tx(full + st, ns * 576);
            bulk_g2s_stream(dst, unit + (size_t)c * SK_CODE_BYTES, ns * 512, full + st, pol);
            bulk_g2s_stream(dst + SK_CODE_BYTES, unit + code_bytes + (size_t)c * SK_CS * 64, ns * 64, full + st, pol);
          }
        }
      }
      // drain: every copy issued must have landed before this CTA may exit
      for (int i = max(0, it - SK_NSTAGE); i < it; ++i)
        mbar_wait(full + (i % SK_NSTAGE), (i / SK_NSTAGE) & 1, p.timeout_ns, status);
    }
    return;
  }

  // -------------------------------------------------------------------- consumers (warps 0..7)
  const int g = lane >> 2, t = lane & 3;
  int it = 0, rbuf = 0;
  for (int ph = 0; ph < 2; ++ph) {
    const long long u0 = ph ? b0 : a0, u1 = ph ? b1 : a1;
    const int nrb = ph ? nrbB : nrbA, nS = ph ? nSB : nSA, nch = ph ? nchB : nchA;
    const int K = ph ? p.I : p.H;
    const int pitch = K * 2 + 16;
    int cur = -1;
    for (long long u = u0; u < u1; ++u) {
      const int jidx = (int)(u / nrb), rb = (int)(u % nrb);
      const int4 job = p.jobs[jidx];
      if (jidx != cur) {
        // stage this job's activation rows (x for phase A, inter for phase B) into shared memory
        named_bar(1, SK_NW * 32);
        if (ph == 1 && tid == 0) wait_geq(p.doneA + jidx, nrbA, p.timeout_ns, status);
        named_bar(1, SK_NW * 32);
        const int vec_per_row = K / 8;  // 16-byte vectors
        for (int i = tid; i < 8 * vec_per_row; i += SK_NW * 32) {
          const int n = i / vec_per_row, v = i % vec_per_row;
          uint4 val = make_uint4(0, 0, 0, 0);
          if (n < job.z) {
            if (ph == 0) {
              const int tok = p.order[job.y + n] / p.k;
              val = __ldg(reinterpret_cast<const uint4*>(p.x + (size_t)tok * p.H) + v);
            } else {
              val = __ldcg(reinterpret_cast<const uint4*>(p.inter + (size_t)(job.y + n) * p.I) + v);
            }
          }
          *reinterpret_cast<uint4*>(xs + n * pitch + v * 16) = val;
        }
        named_bar(1, SK_NW * 32);
        cur = jidx;
      }
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
      const uint8_t* xrow = xs + g * pitch;
      for (int c = 0; c < nch; ++c, ++it) {
        const int ns = min(SK_CS, nS - c * SK_CS);
        const int st = it % SK_NSTAGE;
        mbar_wait(full + st, (it / SK_NSTAGE) & 1, p.timeout_ns, status);
        const uint8_t* stage = ring + st * SK_STAGE_BYTES;
        for (int s = warp; s < ns; s += SK_NW) sk_slice(stage, s, xrow, c * SK_CS + s, lane, t, acc);
        __syncwarp();
        if (lane == 0) mbar_arrive(empty + st);
      }
      // cross-warp reduction and epilogue (warp 0)
      float* rb_buf = red + rbuf * (SK_NW * 32 * 4);
      *reinterpret_cast<float4*>(rb_buf + (warp * 32 + lane) * 4) = make_float4(acc[0], acc[1], acc[2], acc[3]);
      named_bar(1, SK_NW * 32);
      if (warp == 0) {
        float v[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int w = 0; w < SK_NW; ++w) {
          const float4 r = *reinterpret_cast<const float4*>(rb_buf + (w * 32 + lane) * 4);
          v[0] += r.x; v[1] += r.y; v[2] += r.z; v[3] += r.w;
        }
        const int e = job.x;
        if (ph == 0) {
          const float gsc = p.gsA[e] * kTwo52;
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int n = 2 * t + h;
            if (n < job.z) {
              const float gt = v[h] * gsc, up = v[2 + h] * gsc;
              const float hv = gt / (1.f + expf(-gt)) * up;
              p.inter[(size_t)(job.y + n) * p.I + rb * 8 + g] = f2bf(hv);
            }
          }
          __threadfence();
          __syncwarp();
          if (lane == 0) atomicAdd(p.doneA + jidx, 1);
        } else {
          const float gsc = p.gsB[e] * kTwo52;
          const int r0 = rb * 16 + g, r1 = r0 + 8;
          float n0 = 1.f, n1 = 1.f;
          if (p.post_norm) {
            n0 += bf2f(p.normw[r0]);
            n1 += bf2f(p.normw[r1]);
          }
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int n = 2 * t + h;
            const float y0 = v[h] * gsc * n0, y1 = v[2 + h] * gsc * n1;
            float sq = y0 * y0 + y1 * y1;
            if (n < job.z) {
              p.y[(size_t)(job.y + n) * p.H + r0] = y0;
              p.y[(size_t)(job.y + n) * p.H + r1] = y1;
            }
            if (p.post_norm) {
              sq += __shfl_xor_sync(0xffffffffu, sq, 4);
              sq += __shfl_xor_sync(0xffffffffu, sq, 8);
              sq += __shfl_xor_sync(0xffffffffu, sq, 16);
              if (g == 0 && n < job.z) atomicAdd(p.ss + job.y + n, sq);
            }
          }
        }
      }
      rbuf ^= 1;
    }
  }

  // -------------------------------------------------------------------- grid barrier, combine, exit
  named_bar(1, SK_NW * 32);
  if (tid == 0) {
    __threadfence();
    atomicAdd(p.ctl + kCtlGridArrive, 1);
    wait_geq(p.ctl + kCtlGridArrive, G, p.timeout_ns, status);
  }
  named_bar(1, SK_NW * 32);
  const int nseg = (p.H + 1023) / 1024;
  for (int item = bid; item < p.T * nseg; item += G) {
    const int tk = item / nseg, col = (item % nseg) * 1024 + tid * 4;
    if (col < p.H) {
      float a[4] = {0.f, 0.f, 0.f, 0.f};
      for (int s = 0; s < p.k; ++s) {
        const int q = p.pos[tk * p.k + s];
        if (q >= 0) {
          float r = p.wts[tk * p.k + s];
          if (p.post_norm) r *= rsqrtf(__ldcg(p.ss + q) / (float)p.H + 1e-8f);
          const float4 yv = __ldcg(reinterpret_cast<const float4*>(p.y + (size_t)q * p.H + col));
          a[0] += r * yv.x; a[1] += r * yv.y; a[2] += r * yv.z; a[3] += r * yv.w;
        }
      }
      uint2 o;
      o.x = (uint32_t)f2bf(a[0]) | ((uint32_t)f2bf(a[1]) << 16);
      o.y = (uint32_t)f2bf(a[2]) | ((uint32_t)f2bf(a[3]) << 16);
      *reinterpret_cast<uint2*>(p.out + (size_t)tk * p.H + col) = o;
    }
  }
  named_bar(1, SK_NW * 32);
  if (tid == 0) {
    __threadfence();
    const int done = atomicAdd(p.ctl + kCtlExit, 1);
    if (done == G - 1) {
      p.ctl[kCtlGridArrive] = 0;
      p.ctl[kCtlExit] = 0;
      __threadfence();
    }
  }
}

int skinny_grid(int* grid_out, int* smem_out, int H, int I) {
  static int cached_dev = -1, cached_sms = 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return XCB_ERR_CUDA;
  const SkSmemOffsets so = sk_smem(H, I);
  if (cudaFuncSetAttribute(skinny_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, so.total) != cudaSuccess)
    return XCB_ERR_CUDA;
  if (dev != cached_dev) {
    if (cudaDeviceGetAttribute(&cached_sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return XCB_ERR_CUDA;
    cached_dev = dev;
  }
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, skinny_kernel, SK_THREADS, so.total) != cudaSuccess ||
      per_sm < 1)
    return XCB_ERR_CUDA;
  *grid_out = cached_sms * per_sm;
  *smem_out = so.total;
  return XCB_OK;
}

size_t skinny_smem_bytes(int H, int I) { return (size_t)sk_smem(H, I).total; }

int launch_skinny(const SkinnyParams& p, cudaStream_t stream) {
  int grid = 0, smem = 0;
  int rc = skinny_grid(&grid, &smem, p.H, p.I);
  if (rc != XCB_OK) return rc;
  skinny_kernel<<<grid, SK_THREADS, smem, stream>>>(p);
  return cudaGetLastError() == cudaSuccess ? XCB_OK : XCB_ERR_CUDA;
}

}  // namespace xcb
