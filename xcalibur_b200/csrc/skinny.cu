// Decode-path MoE kernel: one persistent launch runs (for small batches) the router, gate_up + SwiGLU (phase A),
// down (phase B) and the weighted combine, for jobs of at most 8 tokens.  This is the HBM-bound path (T = 1
// decode streams ~200 MB of FP4 weights for 8 experts), so the kernel is one continuous weight stream per SM
// whose arithmetic must keep up with HBM:
//
// * Arithmetic per 64-k slice of 16 rows (one warp): the hardware FP4 converter (cvt.rn.f16x2.e2m1x2, one
//   instruction per two weights), one f16x2 multiply per register by the block-scale pair (itself converted from
//   E4M3 by cvt.rn.f16x2.e4m3x2), and four m16n8k16 f16 tensor-core steps fed from registers.  Every product
//   e2m1 * e4m3 has at most 6 significant bits and lies in [2^-10, 2688], so the f16 weight is exact.  The
//   activations are converted to f16 once per segment in shared memory, each token scaled by a power of two
//   2^-e that puts its largest magnitude in [2^14, 2^15), so it neither overflows f16 nor sinks into f16's
//   subnormal range; the epilogue multiplies the fp32 sums back by 2^e.  At T <= 8 tokens per expert the weights are used once, and a
//   register-fed MMA reads no shared memory for them.
// * Weight stream: warp 16 copies packed weights into a ring of 3-8 stages with 1-D bulk copies (TMA engine,
//   L2 evict-first).  A stage holds PER consecutive slices for each of the 16 compute warps, PER chosen per
//   phase so that a unit (16 rows x the full reduction) either spans whole stages or a stage holds whole units
//   and no warp's slices straddle two units (DeepSeek-V3: 7 slices = 64.5 KB stages for gate_up, 4 for down).
//   Both phases stream from HBM: prefetching the down-projection weights into L2 during gate_up was measured
//   slower (it delays the latency-critical gate_up stream more than phase B gains).
// * Partial sums leave the compute warps only at stage ends: at every flush point a warp sums its accumulator's
//   two chains into four pending partials and clears it, and writes the partials one stage later (or at the end
//   of its segment) into a reduction slot; one accumulator set keeps a single copy of the unrolled hot loop per
//   stage size.  Two epilogue warps consume the slots in order: they add the partials of each unit in warp order
//   (deterministic) and apply the epilogue (SwiGLU -> inter, or y and the post-norm sums).
// * Warp 17 stages each segment's activation rows (x for phase A, the job's SwiGLU output for phase B, after an
//   acquire on that job's phase-A counter) with bulk copies and converts them to f16 in place; the epilogue warp
//   that finishes a segment's last unit publishes it GPU-wide (one fence and one counter update per segment).
// * Combine: the CTA whose phase-B units complete a 16-row block forms out = bf16(sum_s w_s * y_s) for it; with the
//   post-norm, or for large batches, a bounded grid barrier precedes a combine spread over all CTAs.
// * Small batches (T*k <= 256) route inside the kernel (every CTA computes the same tables; up to 32 routes with
//   one warp), so a decode step is a single launch.  Every wait is bounded by %globaltimer; on timeout a status
//   bit is set and the kernel drains.
//
// Reference counterpart: moe_fused's skinny path (kernels/moe_w4a16_h200/moe_w4a16.py:491-611 route,
// :754-1133 skinny ring, :1602-1785 warp-specialised epilogues, :2617-2641 grid barrier, :2654-2796 final sum).
#include <cuda_fp16.h>

#include "common.cuh"
#include "kernels.cuh"
#include "workspace.cuh"

namespace xcb {

// Optional timeline trace, read back with xcb_trace_read (off in the shipped library): -DXCB_TRACE=1 records
// %globaltimer stamps, clock64 spans and counters per CTA; -DXCB_TRACE=2 only each CTA's start and exit times and
// its SM (light enough not to change the timing); -DXCB_TRACE=3 the stamps of mode 1 with the clock64 spans and
// counters summed in per-thread registers and written once at kernel end.
#ifndef XCB_TRACE
#define XCB_TRACE 0
#endif
#if XCB_TRACE
constexpr int kTraceSlots = 48;
__device__ unsigned long long g_trace[1024 * kTraceSlots];
#define TRACE_EDGE(slot) (g_trace[blockIdx.x * kTraceSlots + (slot)] = gtimer())
#endif
#if XCB_TRACE == 1 || XCB_TRACE == 3
#define TRACE_AT(slot) (g_trace[blockIdx.x * kTraceSlots + (slot)] = gtimer())
#if XCB_TRACE == 1
#define TRACE_ADD(slot, v) atomicAdd(&g_trace[blockIdx.x * kTraceSlots + (slot)], (unsigned long long)(v))
#else
#define TRACE_ADD(slot, v) (tr_acc[(slot)] += (unsigned long long)(v))
#endif
#define TRACE_GET(slot) (*(volatile unsigned long long*)&g_trace[blockIdx.x * kTraceSlots + (slot)])
#define TRACE_T0(name) const unsigned long long name = clock64()
#define TRACE_SPAN(slot, name) TRACE_ADD(slot, clock64() - (name))
#define TRACE_ONCE(slot) ((trace_once & (1u << (slot))) ? (void)0 : (void)(trace_once |= 1u << (slot), TRACE_AT(slot)))
#else
#ifndef TRACE_EDGE
#define TRACE_EDGE(slot) ((void)0)
#endif
#define TRACE_AT(slot) ((void)0)
#define TRACE_ADD(slot, v) ((void)0)
#define TRACE_T0(name) ((void)0)
#define TRACE_SPAN(slot, name) ((void)0)
#define TRACE_ONCE(slot) ((void)0)
#endif

#ifndef XCB_SK_WAVES
#define XCB_SK_WAVES 2  // job waves of the static schedule
#endif
#ifndef XCB_SK_NOCOMPUTE
#define XCB_SK_NOCOMPUTE 0  // experiments only: skip the slice arithmetic
#endif
#ifndef XCB_SK_MUL
#define XCB_SK_MUL 41  // share permutation multiplier (prime)
#endif
constexpr int SK_NW = 16;                               // compute warps
constexpr int SK_W_PROD = SK_NW;                        // weight producer warp
constexpr int SK_W_ACT = SK_NW + 1;                     // activation staging warp
constexpr int SK_W_EPI = SK_NW + 2;                     // reduction + epilogue warps (SK_NEPI of them)
constexpr int SK_NEPI = 2;                              // epilogue warp e takes the flush events f with f % 2 == e
constexpr int SK_THREADS = (SK_NW + 2 + SK_NEPI) * 32;  // 20 warps: at most 5 per SM sub-partition
constexpr int SK_SLICE = 576;                           // 512 B of codes + 64 B of scale bytes per 64-k slice
#ifndef XCB_SK_PER_MAX
#define XCB_SK_PER_MAX 7
#endif
#ifndef XCB_SK_MAX_STAGES
#define XCB_SK_MAX_STAGES 8
#endif
constexpr int SK_PER_MAX = XCB_SK_PER_MAX;              // slices per compute warp per stage
constexpr int SK_MAX_STAGES = XCB_SK_MAX_STAGES;
constexpr int SK_NSLOT = 2;                             // reduction slots
constexpr int SK_NBUF_MAX = 2;                          // activation buffers
constexpr int SK_SEG_RING = 64;                         // per-segment completion counters
constexpr int SK_WARP_ROUTES = 32;                      // up to this many routes one warp builds the tables
constexpr int SK_COPY_SPLIT = 36864;                    // stages above this many bytes go as two bulk copies
constexpr int SK_SMEM_LIMIT = 227 * 1024;

// Slices per warp per stage for a unit of U slices: U % PER == 0 (a warp's slices never straddle a unit) and
// either U % (16 PER) == 0 (a unit spans whole stages) or (16 PER) % U == 0 (a stage holds whole units).
__host__ __device__ inline int sk_per(int U, int per_max) {
  for (int per = per_max; per >= 1; --per) {
    if (per == 5 || per == 3) continue;  // not instantiated (sk_run_per): fewer copies of the hot loop
    if (U % per == 0 && ((16 * per) % U == 0 || U % (16 * per) == 0)) return per;
  }
  return 0;
}

// The units of one CTA, cut into segments of one job and one phase, in processing order.  The jobs are split into
// two waves (first and second half of the job list) and the work runs as four sequences: gate_up of wave 0,
// gate_up of wave 1, down of wave 0, down of wave 1; every CTA takes a contiguous share of each sequence.  The
// down projection of a wave thus depends on gate_up work that finished one sequence earlier on every CTA, so the
// phase A -> B handoff costs no wait.  A unit is numbered job * nrb + rb within its phase.
struct SkSegments {
  // per sequence q (as scalars, so no array is indexed at run time): unit range, first job, jobs touched
  long long u0_0, u0_1, u0_2, u0_3, u1_0, u1_1, u1_2, u1_3;
  int jf_0, jf_1, jf_2, jf_3, nj_0, nj_1, nj_2, nj_3;
  int nrbA, nrbB;

  template <typename T>
  __device__ static T pick(int q, T a, T b, T c, T d) { return q == 0 ? a : (q == 1 ? b : (q == 2 ? c : d)); }

  __device__ void init(int njobs, int nA_rb, int nB_rb, int G, int bid) {
    nrbA = nA_rb;
    nrbB = nB_rb;
    const int W = njobs >= 2 ? XCB_SK_WAVES : 1;
    long long a[4], b[4];
    int f[4], n[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int ph = q >> 1, w = q & 1;
      const int nrb = ph ? nrbB : nrbA;
      const int j0 = w < W ? njobs * w / W : njobs, j1 = w < W ? njobs * (w + 1) / W : njobs;
      const long long cnt = (long long)(j1 - j0) * nrb;
      // the share a CTA takes differs per sequence (a bijection of the CTA index: 41 is prime, so coprime with G
      // unless G is a multiple of it): a CTA whose share of one sequence streams slowly (the slow part of the
      // address space) gets other parts of the others, which evens the CTAs' finish times (measured 1.5 %)
      const int mul = G % XCB_SK_MUL ? XCB_SK_MUL : 1;
      const int sb = (int)(((long long)bid * mul + q * 17) % G);
      a[q] = (long long)j0 * nrb + cnt * sb / G;
      b[q] = (long long)j0 * nrb + cnt * (sb + 1) / G;
      f[q] = (int)(a[q] / nrb);
      n[q] = b[q] > a[q] ? (int)((b[q] - 1) / nrb) - f[q] + 1 : 0;
    }
    u0_0 = a[0]; u0_1 = a[1]; u0_2 = a[2]; u0_3 = a[3];
    u1_0 = b[0]; u1_1 = b[1]; u1_2 = b[2]; u1_3 = b[3];
    jf_0 = f[0]; jf_1 = f[1]; jf_2 = f[2]; jf_3 = f[3];
    nj_0 = n[0]; nj_1 = n[1]; nj_2 = n[2]; nj_3 = n[3];
  }
  __device__ int count() const { return nj_0 + nj_1 + nj_2 + nj_3; }
  // Segment i: phase, job, unit range [v0, v1).
  __device__ void at(int i, int& ph, int& job, long long& v0, long long& v1) const {
    int q = 0;
    if (i >= nj_0) {
      i -= nj_0;
      q = 1;
      if (i >= nj_1) {
        i -= nj_1;
        q = 2;
        if (i >= nj_2) {
          i -= nj_2;
          q = 3;
        }
      }
    }
    ph = q >> 1;
    job = pick(q, jf_0, jf_1, jf_2, jf_3) + i;
    const long long nrb = ph ? nrbB : nrbA;
    const long long a = pick(q, u0_0, u0_1, u0_2, u0_3), b = pick(q, u1_0, u1_1, u1_2, u1_3);
    v0 = a > job * nrb ? a : job * nrb;
    v1 = b < (job + 1) * nrb ? b : (job + 1) * nrb;
  }
};

// Control block: mbarriers and bookkeeping.
struct SkCtl {
  uint64_t full[SK_MAX_STAGES], empty[SK_MAX_STAGES];
  uint64_t act_land[SK_NBUF_MAX], act_full[SK_NBUF_MAX], act_empty[SK_NBUF_MAX];
  uint64_t slot_full[SK_NSLOT], slot_free[SK_NSLOT];
  uint64_t x_land;                    // one-token calls: the token's row, copied at kernel start
  int xpart[SK_NW];                   // per-warp partial maxima of that row's conversion
  int seg_cnt[SK_SEG_RING];           // units of segment k finished (slot k % SK_SEG_RING)
  int xexp[SK_NBUF_MAX][kJobTokens];  // per activation buffer and row: x was multiplied by 2^-xexp
  int list[512];                      // 16-row blocks this CTA completed (H <= 8192)
  int nlist;
  int njobs, nroutes;
  SkSegments segs;                    // written once by thread 0, read by every role (keeps it out of registers)
};

struct SkLayout {
  int ring, buf, red, route, ctl, total;
  int nstage, nbuf, rows, pitch, slot_bytes, perA, perB, rl, red_slot, route_cap;
};

// Shared-memory plan: the weight ring (at offset 0; the many-route router's scratch aliases it before the first
// copy), activation buffers, reduction slots, routing tables, control block.
__host__ __device__ inline SkLayout sk_layout(int H, int I, int job_tokens, int route_R) {
  SkLayout o{};
  o.rows = job_tokens < 1 ? 1 : (job_tokens > kJobTokens ? kJobTokens : job_tokens);
  o.pitch = (H > I ? H : I) * 2 + (o.rows > 1 ? 16 : 0);
  o.rl = o.rows <= 2 ? 8 : (o.rows <= 4 ? 16 : 32);  // lanes holding useful accumulator columns (t < rl / 8)
  o.red_slot = SK_NW * o.rl * 16;
  o.route_cap = (route_R + 3) & ~3;
  const int route = route_R ? o.route_cap * 32 : 0;  // ids, wts, pos, order (4 B each) + jobs (16 B)
  for (int per_max = SK_PER_MAX; per_max >= 1; --per_max) {
    o.perA = sk_per(H / 64, per_max);
    o.perB = sk_per(I / 64, per_max);
    if (!o.perA || !o.perB) break;
    o.slot_bytes = 16 * (o.perA > o.perB ? o.perA : o.perB) * SK_SLICE;
    for (int nbuf = SK_NBUF_MAX; nbuf >= 1; --nbuf) {
      o.nbuf = nbuf;
      const int rest = nbuf * o.rows * o.pitch + SK_NSLOT * o.red_slot + route + (int)sizeof(SkCtl) + 64;
      int ns = (SK_SMEM_LIMIT - rest) / o.slot_bytes;
      ns = ns > SK_MAX_STAGES ? SK_MAX_STAGES : ns;
      if (ns >= 3) {
        o.nstage = ns;
        o.ring = 0;
        o.buf = ns * o.slot_bytes;
        o.red = (o.buf + nbuf * o.rows * o.pitch + 15) & ~15;
        o.route = o.red + SK_NSLOT * o.red_slot;
        o.ctl = (o.route + route + 15) & ~15;
        o.total = o.ctl + (int)sizeof(SkCtl);
        return o;
      }
    }
  }
  o.nstage = 0;
  return o;
}

// Shared routing tables of the in-kernel router (route_cap entries each).
struct SkTables {
  int4* jobs;
  int* ids;
  float* wts;
  int* pos;
  int* order;
  __device__ SkTables(uint8_t* base, int cap)
      : jobs(reinterpret_cast<int4*>(base)),
        ids(reinterpret_cast<int*>(base + cap * 16)),
        wts(reinterpret_cast<float*>(base + cap * 20)),
        pos(reinterpret_cast<int*>(base + cap * 24)),
        order(reinterpret_cast<int*>(base + cap * 28)) {}
};

// ------------------------------------------------------------------------------------------------ arithmetic
__device__ __forceinline__ void cvt_e2m1x8(uint32_t q, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm("{\n .reg .b8 b0, b1, b2, b3;\n mov.b32 {b0, b1, b2, b3}, %4;\n"
      " cvt.rn.f16x2.e2m1x2 %0, b0;\n cvt.rn.f16x2.e2m1x2 %1, b1;\n cvt.rn.f16x2.e2m1x2 %2, b2;\n"
      " cvt.rn.f16x2.e2m1x2 %3, b3;\n}"
      : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
      : "r"(q));
}
// Two E4M3 scale bytes (row g in the low byte, row g + 8 in the high byte) -> f16x2.
__device__ __forceinline__ uint32_t cvt_e4m3x2(uint32_t two) {
  uint32_t s;
  asm("{\n .reg .b16 h;\n cvt.u16.u32 h, %1;\n cvt.rn.f16x2.e4m3x2 %0, h;\n}" : "=r"(s) : "r"(two));
  return s;
}
__device__ __forceinline__ void mma_16816_f16(float* d, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                              uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t h2mul_lo(uint32_t a, uint32_t s) {  // a * (s.lo, s.lo)
  __half2 r = __hmul2(*reinterpret_cast<__half2*>(&a), __low2half2(*reinterpret_cast<__half2*>(&s)));
  return *reinterpret_cast<uint32_t*>(&r);
}
__device__ __forceinline__ uint32_t h2mul_hi(uint32_t a, uint32_t s) {  // a * (s.hi, s.hi)
  __half2 r = __hmul2(*reinterpret_cast<__half2*>(&a), __high2half2(*reinterpret_cast<__half2*>(&s)));
  return *reinterpret_cast<uint32_t*>(&r);
}

// One 64-k slice of one unit for one warp: lane (g, t) holds the codes of rows g and g + 8 at k = 16t + 4i + 0..3
// of the slice for step i, and the scale pair of block t; xs = the f16 activation row at the slice's first k.
// Steps alternate between the set's two chains.  (Four chains would need more than the 80 registers a thread
// may hold when six warps of this CTA share one SM sub-partition.)
__device__ __forceinline__ void sk_slice(const uint8_t* sl, const uint8_t* xs, int lane, int t, float (&c)[2][4]) {
  const uint4 cw = *reinterpret_cast<const uint4*>(sl + lane * 16);
  const uint32_t sc = *reinterpret_cast<const uint16_t*>(sl + 512 + lane * 2);
  const uint4 xa = *reinterpret_cast<const uint4*>(xs + t * 32);
  const uint4 xb = *reinterpret_cast<const uint4*>(xs + t * 32 + 16);
  const uint32_t s2 = cvt_e4m3x2(sc);
  uint32_t r0, r1, r2, r3;
  cvt_e2m1x8(cw.x, r0, r1, r2, r3);
  mma_16816_f16(c[0], h2mul_lo(r0, s2), h2mul_hi(r1, s2), h2mul_lo(r2, s2), h2mul_hi(r3, s2), xa.x, xa.y);
  cvt_e2m1x8(cw.y, r0, r1, r2, r3);
  mma_16816_f16(c[1], h2mul_lo(r0, s2), h2mul_hi(r1, s2), h2mul_lo(r2, s2), h2mul_hi(r3, s2), xa.z, xa.w);
  cvt_e2m1x8(cw.z, r0, r1, r2, r3);
  mma_16816_f16(c[0], h2mul_lo(r0, s2), h2mul_hi(r1, s2), h2mul_lo(r2, s2), h2mul_hi(r3, s2), xb.x, xb.y);
  cvt_e2m1x8(cw.w, r0, r1, r2, r3);
  mma_16816_f16(c[1], h2mul_lo(r0, s2), h2mul_hi(r1, s2), h2mul_lo(r2, s2), h2mul_hi(r3, s2), xb.z, xb.w);
}

// PER consecutive slices of one warp into one accumulator set (compile-time PER so the slices interleave).
template <int PER>
__device__ __forceinline__ void sk_run(const uint8_t* sl, const uint8_t* xs, int lane, int t, float (&c)[2][4]) {
#pragma unroll
  for (int j = 0; j < PER; ++j) sk_slice(sl + j * SK_SLICE, xs + j * 128, lane, t, c);
}
__device__ __forceinline__ void sk_run_per(int per, const uint8_t* sl, const uint8_t* xs, int lane, int t,
                                           float (&c)[2][4]) {
  switch (per) {  // the slice counts sk_per can return
    case 7: sk_run<7>(sl, xs, lane, t, c); break;
    case 6: sk_run<6>(sl, xs, lane, t, c); break;
    case 4: sk_run<4>(sl, xs, lane, t, c); break;
    case 2: sk_run<2>(sl, xs, lane, t, c); break;
    default: sk_run<1>(sl, xs, lane, t, c); break;
  }
}

// ------------------------------------------------------------------------------------------------ router
// In-kernel router for T*k <= kSmallRoutes (every CTA computes the same tables).  `scratch` (the ring, unused
// yet) holds the per-expert counts of the many-route variant.
__device__ void sk_route_small(const SkinnyParams& p, SkTables& rt, SkCtl& cb, int* scratch) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nthr = blockDim.x;
  const int R = p.T * p.k;
  const int JC = p.job_tokens;  // tokens per job
  for (int t = warp; t < p.T; t += nthr / 32) {
    int id = -1;
    float w = 0.f;
    if (p.logits) {
      warp_topk(p.logits + (size_t)t * p.E_tot, p.E_tot, p.k, id, w);
    } else if (lane < p.k) {
      id = p.ids_in[t * p.k + lane];
      w = p.wts_in[t * p.k + lane];
      if (id < 0 || id >= p.E_tot) {
        if (blockIdx.x == 0) set_status(p.ctl + kCtlStatus, XCB_STATUS_BAD_EXPERT);
        id = -1;
      }
    }
    if (lane < p.k) {
      rt.ids[t * p.k + lane] = id;
      rt.wts[t * p.k + lane] = w;
    }
  }
  __syncthreads();
  if (tid == 0) TRACE_AT(15);
  if (R <= SK_WARP_ROUTES) {
    // one warp: lane f owns route f; ranks by __match_any_sync, offsets and job bases by a 32-step scan
    if (warp == 0) {
      int el = -1;
      if (lane < R) {
        const int id = rt.ids[lane];
        el = id - p.lo;
        if (id < 0 || el < 0 || el >= p.E_loc) el = -1;
      }
      const uint32_t peers = __match_any_sync(0xffffffffu, el);
      const int rank = __popc(peers & ((1u << lane) - 1u));
      const int cnt = __popc(peers);
      int less = 0, jbase = 0;
      for (int g2 = 0; g2 < 32; ++g2) {
        const int eg = __shfl_sync(0xffffffffu, el, g2);
        const int cg = __shfl_sync(0xffffffffu, cnt, g2);
        const int rg = __shfl_sync(0xffffffffu, rank, g2);
        if (eg >= 0 && el >= 0 && eg < el) {
          ++less;
          if (rg == 0) jbase += (cg + JC - 1) / JC;
        }
      }
      const bool lead = el >= 0 && rank == 0;
      const int nj = lead ? (cnt + JC - 1) / JC : 0;
      if (lane < R) {
        rt.pos[lane] = el >= 0 ? less + rank : -1;
        if (el >= 0) rt.order[less + rank] = lane;
      }
      for (int i = 0; i < nj; ++i) rt.jobs[jbase + i] = make_int4(el, less + JC * i, min(JC, cnt - JC * i), 0);
      const int njobs = __reduce_add_sync(0xffffffffu, nj);
      const int nroutes = __popc(__ballot_sync(0xffffffffu, el >= 0));
      if (lane == 0) {
        cb.njobs = njobs;
        cb.nroutes = nroutes;
        TRACE_AT(4);
      }
    }
  } else {
    int* counts = scratch;              // [E_loc]
    int* offs = counts + p.E_loc;       // [E_loc + 1]
    int* jcnt = offs + p.E_loc + 1;     // [E_loc]
    for (int e = tid; e < p.E_loc; e += nthr) {
      int c = 0;
      for (int f = 0; f < R; ++f) c += (rt.ids[f] == p.lo + e);
      counts[e] = c;
      offs[e] = c;
      jcnt[e] = (c + JC - 1) / JC;
    }
    for (int f = tid; f < R; f += nthr) {
      const int id = rt.ids[f];
      int rank = 0;
      for (int g2 = 0; g2 < f; ++g2) rank += (rt.ids[g2] == id);
      rt.pos[f] = rank;
    }
    __syncthreads();
    if (warp == 0) {
      const int tot = warp_exclusive_scan(offs, p.E_loc);
      if (lane == 0) {
        cb.nroutes = tot;
        offs[p.E_loc] = tot;
      }
    } else if (warp == 1) {
      const int tot = warp_exclusive_scan(jcnt, p.E_loc);
      if (lane == 0) cb.njobs = tot;
    }
    __syncthreads();
    for (int f = tid; f < R; f += nthr) {
      const int el = rt.ids[f] - p.lo;
      if (rt.ids[f] >= 0 && el >= 0 && el < p.E_loc) {
        const int q = offs[el] + rt.pos[f];
        rt.pos[f] = q;
        rt.order[q] = f;
      } else {
        rt.pos[f] = -1;
      }
    }
    for (int e = tid; e < p.E_loc; e += nthr) {
      const int c = counts[e];
      int j = jcnt[e];
      for (int s0 = 0; s0 < c; s0 += JC, ++j) rt.jobs[j] = make_int4(e, offs[e] + s0, min(JC, c - s0), 0);
    }
  }
}

// CTA 0 publishes the routing tables to the workspace (tests and callers read them there); all its threads.
__device__ void sk_publish(const SkinnyParams& p, const SkTables& rt, const SkCtl& cb) {
  const int tid = threadIdx.x, nthr = blockDim.x;
  const int R = p.T * p.k;
  {
    for (int f = tid; f < R; f += nthr) {
      p.g_ids[f] = rt.ids[f];
      p.g_wts[f] = rt.wts[f];
      p.g_pos[f] = rt.pos[f];
      if (p.ids_out) p.ids_out[f] = rt.ids[f];
      if (p.wts_out) p.wts_out[f] = rt.wts[f];
    }
    for (int q = tid; q < cb.nroutes; q += nthr) p.g_order[q] = rt.order[q];
    for (int e = tid; e <= p.E_loc; e += nthr) {
      int c = 0, below = 0;
      for (int f = 0; f < R; ++f) {
        const int id = rt.ids[f], el = id - p.lo;
        if (id >= 0 && el >= 0 && el < p.E_loc) {
          c += (el == e);
          below += (el < e);
        }
      }
      if (e < p.E_loc) p.g_counts[e] = c;
      p.g_offsets[e] = below;
    }
  }
}

// One token with router logits (warp 0; the keys were loaded before the barrier set-up): the top-k routes name
// distinct experts, so each local route is one job of one token, and a route's position in the expert order is the
// number of local routes with a lower expert id.
__device__ void sk_route_one(const SkinnyParams& p, const uint32_t (&key)[16], SkTables& rt, SkCtl& cb) {
  const int lane = threadIdx.x & 31;
  int id;
  float w;
  warp_topk_select(key, p.k, id, w);
  const int el = id - p.lo;
  const bool loc = lane < p.k && el >= 0 && el < p.E_loc;
  int below = 0;
  for (int j = 0; j < p.k; ++j) {
    const int e2 = __shfl_sync(0xffffffffu, loc ? el : 0x7fffffff, j);
    below += (e2 < el);
  }
  if (lane < p.k) {
    rt.ids[lane] = id;
    rt.wts[lane] = w;
    rt.pos[lane] = loc ? below : -1;
    if (loc) {
      rt.order[below] = lane;
      rt.jobs[below] = make_int4(el, below, 1, 0);
    }
  }
  const int n = __popc(__ballot_sync(0xffffffffu, loc));
  if (lane == 0) {
    cb.njobs = n;
    cb.nroutes = n;
  }
}

__device__ __forceinline__ void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }

// Convert `ntok` staged bf16 rows of K values to f16 in place (one warp), each row scaled by 2^-e with e chosen
// from its largest magnitude so that the result neither overflows f16 nor loses bits in its subnormal range; e is
// returned per row in xexp.
__device__ void sk_rows_to_f16(uint8_t* buf, int pitch, int ntok, int K, int* xexp) {
  const int lane = threadIdx.x & 31, nv = K / 8;
  for (int n = 0; n < ntok; ++n) {
    uint4* row = reinterpret_cast<uint4*>(buf + (size_t)n * pitch);
    uint32_t m = 0;
    for (int v = lane; v < nv; v += 32) {
      const uint4 q = row[v];
      const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) m = max(m, max(w[i] & 0x7FFFu, (w[i] >> 16) & 0x7FFFu));
    }
    m = __reduce_max_sync(0xffffffffu, m);
    const int E = (int)(m >> 7);           // bf16 exponent field of the largest magnitude: |x| < 2^(E - 126)
    // the row's largest magnitude lands in [2^14, 2^15): a large row cannot overflow f16 and a small one does not
    // sink into its subnormal range (e = -126 at most, so 2^e and 2^-e stay normal fp32 numbers)
    const int e = max(E - 141, -126);
    const float sc = __uint_as_float((uint32_t)(127 - e) << 23);
    for (int v = lane; v < nv; v += 32) {
      const uint4 q = row[v];
      const uint32_t w[4] = {q.x, q.y, q.z, q.w};
      uint32_t o[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        __half2 h = __floats2half2_rn(__uint_as_float(w[i] << 16) * sc, __uint_as_float(w[i] & 0xFFFF0000u) * sc);
        o[i] = *reinterpret_cast<uint32_t*>(&h);
      }
      row[v] = make_uint4(o[0], o[1], o[2], o[3]);
    }
    if (lane == 0) xexp[n] = e;
  }
}

// Convert one staged bf16 row of K values to f16 in place with `nw` warps (this one is number `wid`), the same
// power-of-two scaling as sk_rows_to_f16, writing a second copy to `copy` when it is not null; named barrier `bar`
// joins the warps between the max pass and the conversion.  Returns the exponent e.
__device__ int sk_row_to_f16_warps(uint8_t* row, uint8_t* copy, int K, int* part, int wid, int nw, int bar) {
  const int lane = threadIdx.x & 31, nv = K / 8;
  const int v0 = nv * wid / nw, v1 = nv * (wid + 1) / nw;
  uint4* r = reinterpret_cast<uint4*>(row);
  uint4* c = reinterpret_cast<uint4*>(copy);
  uint32_t m = 0;
  for (int v = v0 + lane; v < v1; v += 32) {
    const uint4 q = r[v];
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) m = max(m, max(w[i] & 0x7FFFu, (w[i] >> 16) & 0x7FFFu));
  }
  m = __reduce_max_sync(0xffffffffu, m);
  if (lane == 0) part[wid] = (int)m;
  named_bar(bar, nw * 32);
  int mm = 0;
  for (int i = 0; i < nw; ++i) mm = max(mm, part[i]);
  const int E = mm >> 7;
  const int e = max(E - 141, -126);  // as in sk_rows_to_f16
  const float sc = __uint_as_float((uint32_t)(127 - e) << 23);
  for (int v = v0 + lane; v < v1; v += 32) {
    const uint4 q = r[v];
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
    uint32_t o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __half2 h = __floats2half2_rn(__uint_as_float(w[i] << 16) * sc, __uint_as_float(w[i] & 0xFFFF0000u) * sc);
      o[i] = *reinterpret_cast<uint32_t*>(&h);
    }
    r[v] = make_uint4(o[0], o[1], o[2], o[3]);
    if (copy) c[v] = make_uint4(o[0], o[1], o[2], o[3]);
  }
  return e;
}

// TWO: a call of two tokens whose jobs hold one token each, with two activation buffers (the host checks): both
// token rows are staged at kernel start, token n in buffer n, so the phase-A segments need no staging.  The other
// instantiation is the general kernel.
template <bool TWO>
__global__ void __launch_bounds__(SK_THREADS, 1) skinny_kernel(const SkinnyParams p, const SkLayout L) {
  extern __shared__ __align__(1024) uint8_t smem[];
  uint8_t* ring = smem + L.ring;
  uint8_t* bufs = smem + L.buf;
  float* red = reinterpret_cast<float*>(smem + L.red);
  SkCtl& cb = *reinterpret_cast<SkCtl*>(smem + L.ctl);
  SkTables rt(smem + L.route, L.route_cap);
  int* status = p.ctl + kCtlStatus;
  const int NST = L.nstage, NBUF = L.nbuf;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = gridDim.x, bid = blockIdx.x;
  // one token and one row per job (so not an expert named twice by precomputed routing): every phase-A segment
  // uses that token's row, staged before routing into row 0 of buffers 0 and 1
  const bool xpre = p.T == 1;
#if XCB_TRACE == 3
  unsigned long long tr_acc[kTraceSlots] = {};  // spans and counters of this thread
#endif
#if XCB_TRACE == 1 || XCB_TRACE == 3
  unsigned trace_once = 0;  // TRACE_ONCE slots this thread has stamped
#endif

  // with programmatic dependent launch this CTA may be resident before the previous kernel of the stream is done:
  // every global read below (inputs, workspace) comes after the wait; the next kernel may be scheduled from now on
  // (it waits for this whole grid before it reads anything)
  if (p.pdl) {
    pdl_wait();
    if (threadIdx.x == 0) pdl_launch_dependents();
  }
  // one token with logits: warp 0 loads the row now, so the load overlaps the set-up below
  const bool route_one = p.small_route && p.T == 1 && p.logits != nullptr;
  uint32_t key[16];
  if (route_one && warp == 0) warp_topk_load(p.logits, p.E_tot, key);
  if (tid == 0) {
    TRACE_EDGE(0);
#if XCB_TRACE
    {
      uint32_t smid;
      asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
      g_trace[blockIdx.x * kTraceSlots + 2] = smid;
    }
#endif
    for (int i = 0; i < NST; ++i) {
      mbar_init(cb.full + i, 1);
      mbar_init(cb.empty + i, SK_NW);
    }
    for (int i = 0; i < NBUF; ++i) {
      mbar_init(cb.act_land + i, 1);
      mbar_init(cb.act_full + i, 1);
      mbar_init(cb.act_empty + i, SK_NW);
    }
    for (int i = 0; i < SK_NSLOT; ++i) {
      mbar_init(cb.slot_full + i, SK_NW);
      mbar_init(cb.slot_free + i, 1);
    }
    mbar_init(&cb.x_land, 1);
    fence_mbar_init();
    cb.nlist = 0;
    if (xpre) {  // one token: every phase-A segment uses its row, so copy it now and convert it while routing
      mbar_arrive_expect_tx(&cb.x_land, p.H * 2);
      bulk_g2s(bufs, p.x, p.H * 2, &cb.x_land);
    }
    if constexpr (TWO) {  // two tokens: row n into buffer n
      mbar_arrive_expect_tx(&cb.x_land, 2 * p.H * 2);
      bulk_g2s(bufs, p.x, p.H * 2, &cb.x_land);
      bulk_g2s(bufs + (size_t)L.rows * L.pitch, p.x + p.H, p.H * 2, &cb.x_land);
    }
  }
  for (int i = tid; i < SK_SEG_RING; i += SK_THREADS) cb.seg_cnt[i] = 0;
  __syncthreads();  // barrier initialisation visible to every warp
  if (xpre && warp >= SK_NW - 12 && warp < SK_NW) {
    // 12 compute warps convert the token's row while warp 0 (and the router) pick its experts
    mbar_wait(&cb.x_land, 0, p.timeout_ns, status);
    const int e = sk_row_to_f16_warps(bufs, NBUF > 1 ? bufs + (size_t)L.rows * L.pitch : nullptr, p.H, cb.xpart,
                                      warp - (SK_NW - 12), 12, 1);
    if (warp == SK_NW - 12 && lane == 0) {
      cb.xexp[0][0] = e;
      cb.xexp[1][0] = e;
    }
  }
  if constexpr (TWO) {
    if (warp >= SK_NW - 12 && warp < SK_NW) {  // six warps per token row (named barriers 1 and 2)
      const int w = warp - (SK_NW - 12), n = w / 6;
      mbar_wait(&cb.x_land, 0, p.timeout_ns, status);
      const int e = sk_row_to_f16_warps(bufs + (size_t)n * L.rows * L.pitch, nullptr, p.H, cb.xpart + 8 * n, w % 6,
                                        6, 1 + n);
      if (w % 6 == 0 && lane == 0) cb.xexp[n][0] = e;
    }
  }
  if (route_one) {
    if (warp == 0) sk_route_one(p, key, rt, cb);
  } else if (p.small_route) {
    sk_route_small(p, rt, cb, reinterpret_cast<int*>(ring));
  }
  if (tid == 0) TRACE_AT(21);
  __syncthreads();
  if (tid == 0) TRACE_AT(27);
  if (p.small_route && bid == 0) sk_publish(p, rt, cb);
  if (tid == 0) TRACE_AT(1);

  const int njobs = p.small_route ? cb.njobs : p.ctl[kCtlJobs];
  const int4* jobs = p.small_route ? rt.jobs : p.jobs;
  const int* order = p.small_route ? rt.order : p.order;
  const int* pos = p.small_route ? rt.pos : p.pos;
  const float* wts = p.small_route ? rt.wts : p.wts;
  const int nrbA = (2 * p.I) / 16, nrbB = p.H / 16;
  const int UA = p.H / 64, UB = p.I / 64;  // slices per unit
  const size_t unitA = (size_t)9 * p.H, unitB = (size_t)9 * p.I;
  if (tid == 0) cb.segs.init(njobs, nrbA, nrbB, G, bid);
  __syncthreads();
  const SkSegments& segs = cb.segs;
  const int nseg = segs.count();

  if (warp == SK_W_PROD) {
    // ------------------------------------------------------------------ weight producer
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      int it = 0;
      bool ok = true;
      for (int s = 0; s < nseg && ok; ++s) {
        int ph, job;
        long long u0, u1;
        segs.at(s, ph, job, u0, u1);
        if (u1 <= u0) continue;
        const int nrb = ph ? nrbB : nrbA, U = ph ? UB : UA, SS = 16 * (ph ? L.perB : L.perA);
        const int nsl = (int)(u1 - u0) * U;
        const uint8_t* seg = (ph ? p.wB : p.wA) +
                             ((size_t)jobs[job].x * nrb + (size_t)(u0 - (long long)job * nrb)) * (ph ? unitB : unitA);
        for (int base = 0; base < nsl; base += SS, ++it) {
          const uint32_t bytes = (uint32_t)min(SS, nsl - base) * SK_SLICE;
          const int st = it % NST;
          TRACE_T0(t_e);
          if (it >= NST && !mbar_wait(cb.empty + st, ((it / NST) + 1) & 1, p.timeout_ns, status)) {
            ok = false;
            break;
          }
          TRACE_SPAN(13, t_e);
          uint8_t* dst = ring + (size_t)st * L.slot_bytes;
          const uint8_t* src = seg + (size_t)base * SK_SLICE;
          mbar_arrive_expect_tx(cb.full + st, bytes);
          if (bytes > (uint32_t)SK_COPY_SPLIT) {
            const uint32_t h = (bytes / 2 + 15u) & ~15u;
            bulk_g2s_stream(dst, src, h, cb.full + st, pol);
            bulk_g2s_stream(dst + h, src + h, bytes - h, cb.full + st, pol);
          } else {
            bulk_g2s_stream(dst, src, bytes, cb.full + st, pol);
          }
        }
      }
      TRACE_AT(3);
      for (int i = max(0, it - NST); i < it; ++i) mbar_wait(cb.full + (i % NST), (i / NST) & 1, p.timeout_ns, status);
    }
  } else if (warp == SK_W_ACT) {
    // ------------------------------------------------------------------ activation staging + f16 conversion
    int k = 0;                 // non-empty segments so far
    uint32_t land0 = 0, land1 = 0;  // landings per buffer (phase parity of act_land)
    TRACE_T0(t_act);
    for (int s = 0; s < nseg; ++s) {
      int ph, job;
      long long u0, u1;
      segs.at(s, ph, job, u0, u1);
      if (u1 <= u0) continue;
      const int b = k % NBUF;
      const int4 jb = jobs[job];
      const int K = ph ? p.I : p.H;
      const int ntok = min(jb.z, L.rows);
      uint8_t* dst = bufs + (size_t)b * L.rows * L.pitch;
      if ((xpre || TWO) && ph == 0) {  // phase-A segments precede every phase-B one: the staged rows stay put
        if (lane == 0) {
          if (k >= NBUF) mbar_wait(cb.act_empty + b, ((k / NBUF) + 1) & 1, p.timeout_ns, status);
          mbar_arrive(cb.act_full + b);
        }
        __syncwarp();
        ++k;
        continue;
      }
      if (lane == 0) {
        if (k >= NBUF) mbar_wait(cb.act_empty + b, ((k / NBUF) + 1) & 1, p.timeout_ns, status);
        // two tokens: the previous segment read the buffer of its job's token, whichever that was; both buffers
        // must be released before the first phase-B staging overwrites one
        if (TWO && k >= 1) mbar_wait(cb.act_empty + (k - 1) % NBUF, ((k - 1) / NBUF) & 1, p.timeout_ns, status);
        if (ph == 1) {
          TRACE_ONCE(5);
          wait_geq(p.doneA + job, nrbA, p.timeout_ns, status);  // every phase-A unit of this job is published
          TRACE_ONCE(6);
          fence_proxy_async_global();
        }
        mbar_arrive_expect_tx(cb.act_land + b, ntok * K * 2);
        for (int n = 0; n < ntok; ++n) {
          const uint16_t* src = ph ? p.inter + (size_t)(jb.y + n) * p.I : p.x + (size_t)(order[jb.y + n] / p.k) * p.H;
          bulk_g2s(dst + (size_t)n * L.pitch, src, K * 2, cb.act_land + b);
        }
      }
      __syncwarp();
      const uint32_t lpar = (b ? land1++ : land0++) & 1;
      TRACE_T0(t_al);
      mbar_wait(cb.act_land + b, lpar, p.timeout_ns, status);
      if (lane == 0) {
        TRACE_ONCE(17);
        TRACE_SPAN(35, t_al);
      }
      TRACE_T0(t_cv);
      sk_rows_to_f16(dst, L.pitch, ntok, K, cb.xexp[b]);
      if (lane == 0) TRACE_SPAN(36, t_cv);
      __syncwarp();
      if (lane == 0) {
        TRACE_ONCE(16);
        mbar_arrive(cb.act_full + b);
      }
      ++k;
    }
    if (lane == 0) {
      TRACE_AT(20);
      TRACE_SPAN(37, t_act);
    }
  } else if (warp >= SK_W_EPI) {
    // ------------------------------------------------------------------ reduction + epilogue
    // slot lane l holds the partial of accumulator lane (g, t) = (l % 8, l / 8): rows g, g + 8; tokens 2t, 2t + 1
    const int epi = warp - SK_W_EPI;
    const int g = lane & 7, t = lane >> 3;
    const bool act = lane < L.rl;
    int f = 0, k = 0;
    TRACE_T0(t_epi);
    for (int s = 0; s < nseg; ++s) {
      int ph, job;
      long long u0, u1;
      segs.at(s, ph, job, u0, u1);
      if (u1 <= u0) continue;
      const int nrb = ph ? nrbB : nrbA, U = ph ? UB : UA, PER = ph ? L.perB : L.perA, SS = 16 * PER;
      const int nunits = (int)(u1 - u0);
      const int4 jb = jobs[job];
      const float gsc = (ph ? p.gsB : p.gsA)[jb.x];
      const int upe = U >= SS ? 1 : SS / U;            // units per flush event
      const int wpu = U >= SS ? SK_NW : U / PER;       // contributing warps per unit
      const int nev = (nunits + upe - 1) / upe;
      for (int ev = 0; ev < nev; ++ev, ++f) {
        if (f % SK_NEPI != epi) continue;
        const int slot = f % SK_NSLOT;
        TRACE_T0(t_sl);
        mbar_wait(cb.slot_full + slot, (f / SK_NSLOT) & 1, p.timeout_ns, status);
        if (lane == 0) {
          TRACE_SPAN(24, t_sl);
          TRACE_ADD(26, 1);
        }
        TRACE_T0(t_ew);
        const float* sb = red + slot * (L.red_slot / 4);
        const int i0 = ev * upe, i1 = min(nunits, i0 + upe);
        for (int i = i0; i < i1; ++i) {
          const int w0 = (i - i0) * wpu;
          float v[4] = {0.f, 0.f, 0.f, 0.f};
          if (act) {
            for (int w = w0; w < w0 + wpu; ++w) {  // fixed warp order: deterministic sums
              const float4 r = *reinterpret_cast<const float4*>(sb + (w * L.rl + lane) * 4);
              v[0] += r.x; v[1] += r.y; v[2] += r.z; v[3] += r.w;
            }
          }
          if (i + 1 == i1) {
            __syncwarp();
            if (lane == 0) mbar_arrive(cb.slot_free + slot);
          }
          const int rb = (int)(u0 + i - (long long)job * nrb);
          if (ph == 0) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const int n = 2 * t + h;
              if (act && n < jb.z) {
                const float gt = v[h] * gsc, up = v[2 + h] * gsc;
                const float hv = __fdividef(gt, 1.f + __expf(-gt)) * up;  // SiLU(g) * u (fast exp / divide)
                p.inter[(size_t)(jb.y + n) * p.I + rb * 8 + g] = f2bf(hv);
              }
            }
          } else {
            const int r0 = rb * 16 + g, r1 = r0 + 8;
            float n0 = 1.f, n1 = 1.f;
            if (p.post_norm) {
              n0 += bf2f(p.normw[r0]);
              n1 += bf2f(p.normw[r1]);
            }
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const int n = 2 * t + h;
              const bool ok = act && n < jb.z;
              const float y0 = v[h] * gsc * n0, y1 = v[2 + h] * gsc * n1;
              if (ok) {
                p.y[(size_t)(jb.y + n) * p.H + r0] = y0;
                p.y[(size_t)(jb.y + n) * p.H + r1] = y1;
              }
              if (p.post_norm) {
                float sq = ok ? y0 * y0 + y1 * y1 : 0.f;
                sq += __shfl_xor_sync(0xffffffffu, sq, 1);
                sq += __shfl_xor_sync(0xffffffffu, sq, 2);
                sq += __shfl_xor_sync(0xffffffffu, sq, 4);
                if (g == 0 && ok) atomicAdd(p.ss + jb.y + n, sq);
              }
            }
          }
          // count the finished unit; the warp that completes the segment publishes it GPU-wide (the CTA-scope
          // fence orders this warp's writes before its count; the other warp's GPU-scope fence, issued after it
          // observed every count of the segment, is cumulative)
          __syncwarp();
          int done = 0;
          if (lane == 0) {
            __threadfence_block();
            done = atomicAdd(&cb.seg_cnt[k % SK_SEG_RING], 1) + 1;
          }
          done = __shfl_sync(0xffffffffu, done, 0);
          if (done == nunits) {
            TRACE_T0(t_sc);
            __threadfence();
            if (lane == 0) cb.seg_cnt[k % SK_SEG_RING] = 0;
            if (ph == 0) {
              if (lane == 0) atomicAdd(p.doneA + job, nunits);
            } else if (!p.grid_combine) {
              // one count per 16-row block; the CTA that completes a block combines it (all threads, at the end)
              for (long long u = u0 + lane; u < u1; u += 32) {
                const int rb2 = (int)(u - (long long)job * nrbB);
                if (atomicAdd(p.rbcnt + rb2, 1) == njobs - 1) cb.list[atomicAdd(&cb.nlist, 1)] = rb2;
              }
            }
            __syncwarp();
            if (lane == 0) TRACE_SPAN(34, t_sc);
          }
        }
        if (lane == 0) TRACE_SPAN(ph ? 33 : 32, t_ew);
      }
      ++k;
    }
    if (lane == 0) {
      TRACE_AT(22);
      TRACE_SPAN(41, t_epi);
    }
  } else {
    // ------------------------------------------------------------------ compute warps
    // Stage i of a segment holds slices [i SS, i SS + ns); warp w takes [i SS + w PER, + PER), all in one unit.
    // At a flush point the set's two chains are summed into four pending partials and the set is cleared; the
    // partials are written one stage later (one hot-loop instantiation per stage size).
    const int g = lane >> 2, t = lane & 3;
    const bool wr = t < L.rl / 8;  // this lane's columns are read by the epilogue
    int st = 0, f = 0, k = 0;
    uint32_t sphase = 0;
    bool pend = false;
    int fpend = 0;
    float psc0 = 1.f, psc1 = 1.f;
    float sa[2][4] = {};                 // the accumulator set, two chains
    float pv[4] = {0.f, 0.f, 0.f, 0.f};  // partials of the last flush, not yet written
    auto deposit = [&]() {               // write the pending partials into their slot
      const int slot = fpend % SK_NSLOT;
      TRACE_T0(t_sf);
      if (fpend >= SK_NSLOT) mbar_wait(cb.slot_free + slot, ((fpend / SK_NSLOT) + 1) & 1, p.timeout_ns, status);
      if (warp == 0 && lane == 0) {
        TRACE_SPAN(14, t_sf);
        TRACE_ADD(18, 1);
      }
      if (wr)
        *reinterpret_cast<float4*>(red + slot * (L.red_slot / 4) + (warp * L.rl + t * 8 + g) * 4) =
            make_float4(pv[0] * psc0, pv[1] * psc1, pv[2] * psc0, pv[3] * psc1);
      __syncwarp();
      if (lane == 0) mbar_arrive(cb.slot_full + slot);
      pend = false;
    };
    TRACE_T0(t_cw);
    for (int s = 0; s < nseg; ++s) {
      int ph, job;
      long long u0, u1;
      segs.at(s, ph, job, u0, u1);
      if (u1 <= u0) continue;
      const int b = k % NBUF;
      const int U = ph ? UB : UA, PER = ph ? L.perB : L.perA, SS = 16 * PER;
      const int nsl = (int)(u1 - u0) * U;
      const int nst = (nsl + SS - 1) / SS;
      const int spe = U >= SS ? U / SS : 1;  // stages per flush event
      const int4 jb = jobs[job];
      const int ntok = min(jb.z, L.rows);
      TRACE_T0(t_x);
      mbar_wait(cb.act_full + b, (k / NBUF) & 1, p.timeout_ns, status);
      if (warp == 0 && lane == 0) {
        TRACE_SPAN(12, t_x);
        if (ph == 1) TRACE_ONCE(10);
      }
      // one token: every route of a job (an expert named twice by precomputed routing gives a job two routes) is
      // that token, whose row is row 0 (staged once at kernel start for phase A)
      const bool one = p.T == 1;
      const uint8_t* xrow = bufs + (size_t)b * L.rows * L.pitch + (size_t)(g < ntok && !one ? g : 0) * L.pitch;
      // column scales 2^e of this lane's tokens 2t, 2t + 1 (rows past the job's tokens are discarded)
      float sc0 = __uint_as_float((uint32_t)(127 + cb.xexp[b][one ? 0 : min(2 * t, ntok - 1)]) << 23);
      float sc1 = __uint_as_float((uint32_t)(127 + cb.xexp[b][one ? 0 : min(2 * t + 1, ntok - 1)]) << 23);
      if constexpr (TWO) {
        if (ph == 0) {  // the job's one token n = its route's token, staged in buffer n
          const int n = order[jb.y] / p.k;
          xrow = bufs + (size_t)n * L.rows * L.pitch;
          sc0 = sc1 = __uint_as_float((uint32_t)(127 + cb.xexp[n][0]) << 23);
        }
      }
      for (int i = 0; i < nst; ++i) {
        TRACE_T0(t_f);
        mbar_wait(cb.full + st, sphase, p.timeout_ns, status);
        TRACE_T0(t_it);
        if (warp == 0 && lane == 0) {
          TRACE_SPAN(ph ? 30 : 11, t_f);
          TRACE_ONCE(9);
        }
        const int my0 = i * SS + warp * PER;
        if (my0 < nsl) {
          const uint8_t* sl = ring + (size_t)st * L.slot_bytes + (size_t)warp * PER * SK_SLICE;
          const uint8_t* xs = xrow + (size_t)(my0 % U) * 128;
          TRACE_T0(t_c);
          if (!XCB_SK_NOCOMPUTE) sk_run_per(PER, sl, xs, lane, t, sa);
          if (warp == 0) {
            __syncwarp();
            if (lane == 0) TRACE_SPAN(ph ? 31 : 23, t_c);
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(cb.empty + st);
        if (warp == 0 && lane == 0) TRACE_ADD(19, 1);
        if (++st == NST) {
          st = 0;
          sphase ^= 1;
        }
        if (pend) {
          TRACE_T0(t_d);
          deposit();
          if (warp == 0 && lane == 0) TRACE_SPAN(25, t_d);
        }
        if ((i + 1) % spe == 0) {
          pend = true;
          fpend = f++;
          psc0 = sc0;
          psc1 = sc1;
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            pv[i] = sa[0][i] + sa[1][i];
            sa[0][i] = 0.f;
            sa[1][i] = 0.f;
          }
        }
        if (warp == 0 && lane == 0) TRACE_SPAN(ph ? 29 : 28, t_it);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(cb.act_empty + b);
      // the segment's last set is written now, not after the next segment's first stage: the next segment's
      // activations may wait (phase B) on phase-A counters that this very set completes
      if (pend) {
        deposit();
      }
      ++k;
    }
    if (warp == 0 && lane == 0) TRACE_SPAN(40, t_cw);
  }

  if (tid == 0) TRACE_AT(7);
  // 16-row blocks this CTA completed: combine them for every token with all threads (one L2 round trip)
  __syncthreads();
  if (!p.grid_combine && cb.nlist > 0) {
    __threadfence();
    const int nl = cb.nlist, items = nl * 16 * p.T;
    for (int i = tid; i < items; i += SK_THREADS) {
      const int rb = cb.list[i / (16 * p.T)], rem = i % (16 * p.T);
      const int tk = rem / 16, row = rb * 16 + rem % 16;
      float yv[16], wv[16];
#pragma unroll
      for (int s = 0; s < 16; ++s) {
        yv[s] = 0.f;
        wv[s] = 0.f;
        if (s < p.k) {
          const int q = pos[tk * p.k + s];
          if (q >= 0) {
            yv[s] = __ldcg(p.y + (size_t)q * p.H + row);
            wv[s] = wts[tk * p.k + s];
          }
        }
      }
      float a = 0.f;
#pragma unroll
      for (int s = 0; s < 16; ++s) a += wv[s] * yv[s];
      p.out[(size_t)tk * p.H + row] = f2bf(a);
    }
    __syncthreads();
    for (int i = tid; i < nl; i += SK_THREADS) p.rbcnt[cb.list[i]] = 0;
  }
  // no local route at all: no unit will combine, so the output is zero
  if (!p.grid_combine && njobs == 0) {
    const size_t n2 = (size_t)p.T * p.H / 2;
    for (size_t i = (size_t)bid * SK_THREADS + tid; i < n2; i += (size_t)G * SK_THREADS)
      reinterpret_cast<uint32_t*>(p.out)[i] = 0u;
  }

  // -------------------------------------------------------------------- grid combine (post-norm / large batch)
  if (p.grid_combine) {
    __threadfence();
    __syncthreads();
    if (tid == 0) {
      atomicAdd(p.ctl + kCtlGridArrive, 1);
      wait_geq(p.ctl + kCtlGridArrive, G, p.timeout_ns, status);
    }
    __syncthreads();
    const int nsegc = (p.H + 1023) / 1024;
    for (int item = bid; item < p.T * nsegc; item += G) {
      const int tk = item / nsegc, col = (item % nsegc) * 1024 + tid * 4;
      if (tid < 256 && col < p.H) {
        float a[4] = {0.f, 0.f, 0.f, 0.f};
        for (int s = 0; s < p.k; ++s) {
          const int q = pos[tk * p.k + s];
          if (q >= 0) {
            float r = wts[tk * p.k + s];
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
  }

#if XCB_TRACE == 3
  for (int s = 0; s < kTraceSlots; ++s)
    if (tr_acc[s]) atomicAdd(&g_trace[blockIdx.x * kTraceSlots + s], tr_acc[s]);
#endif
  // -------------------------------------------------------------------- exit: the last CTA resets the counters
  __syncthreads();
  if (tid == 0) {
    TRACE_EDGE(8);
    __threadfence();
    const int done = atomicAdd(p.ctl + kCtlExit, 1);
    if (done == G - 1) {
      if (p.small_route) {
        for (int j = 0; j < njobs; ++j) p.doneA[j] = 0;
        if (p.post_norm)
          for (int q = 0; q < cb.nroutes; ++q) p.ss[q] = 0.f;
      }
      p.ctl[kCtlGridArrive] = 0;
      p.ctl[kCtlExit] = 0;
      __threadfence();
    }
  }
}

#if XCB_TRACE
extern "C" int xcb_trace_read(void* host, size_t bytes) {
  return cudaMemcpyFromSymbol(host, g_trace, bytes) == cudaSuccess ? 0 : 4;
}
extern "C" int xcb_trace_clear() {
  static unsigned long long zero[1024 * kTraceSlots];
  return cudaMemcpyToSymbol(g_trace, zero, sizeof(zero)) == cudaSuccess ? 0 : 4;
}
#endif

int skinny_config(int* grid_out, SkLayout* plan, int H, int I, int job_tokens, int route_R) {
  static int cached_dev = -1, cached_sms = 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return XCB_ERR_CUDA;
  const SkLayout L = sk_layout(H, I, job_tokens, route_R);
  if (L.nstage < 3) return XCB_ERR_UNSUPPORTED;
  if (cudaFuncSetAttribute(skinny_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, L.total) !=
          cudaSuccess ||
      cudaFuncSetAttribute(skinny_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, L.total) != cudaSuccess)
    return XCB_ERR_CUDA;
  if (dev != cached_dev) {
    if (cudaDeviceGetAttribute(&cached_sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return XCB_ERR_CUDA;
    cached_dev = dev;
  }
  *grid_out = cached_sms;  // one CTA per SM (the kernel takes nearly all shared memory)
  *plan = L;
  return XCB_OK;
}

// Tokens per job for the decode path: the most (up to `want`) whose shared-memory plan keeps the stage sizes of the
// one-token plan, so that batches of a few tokens do not fall back to small copies, and also its two activation
// buffers (with one, a segment's rows are staged while no other segment computes) as long as that width still
// holds `min_rows` routes, the expected routes per expert (narrower jobs would stream an expert's weights once per
// job).  At the reference's shape (H = I = 4096) this gives 6-token jobs with two buffers rather than 8-token jobs
// with one: 91 -> 83 us at 8 tokens, 126 -> 117 us at 16.
int skinny_job_cap(int H, int I, int want, int route_R, int min_rows) {
  const SkLayout one = sk_layout(H, I, 1, route_R);
  int same_stages = 1;
  bool found = false;
  for (int r = want < kJobTokens ? want : kJobTokens; r > 1; --r) {
    const SkLayout L = sk_layout(H, I, r, route_R);
    if (L.nstage < 3 || L.perA != one.perA || L.perB != one.perB) continue;
    if (!found) {
      same_stages = r;
      found = true;
    }
    if (L.nbuf >= one.nbuf) return r >= min_rows ? r : same_stages;
  }
  return 1 >= min_rows ? 1 : same_stages;  // one-token jobs keep the one-token plan itself
}

// Two tokens: one-token jobs are worth an expert the tokens share being streamed twice when they keep two activation
// buffers and two-token jobs would not.  The kernel then stages both rows at start (the two-token instantiation).
bool skinny_two_one_token_jobs(int H, int I, int route_R) {
  const SkLayout one = sk_layout(H, I, 1, route_R), two = sk_layout(H, I, 2, route_R);
  return one.nstage >= 3 && one.nbuf == 2 && (two.nstage < 3 || two.nbuf < 2);
}

void skinny_plan_fields(int H, int I, int job_tokens, int route_R, int T, int* out) {
  const SkLayout L = sk_layout(H, I, job_tokens, route_R);
  out[0] = L.rows;
  out[1] = L.nbuf;
  out[2] = L.nstage;
  out[3] = L.slot_bytes;
  out[4] = T == 2 && L.rows == 1 && L.nbuf == 2 ? 1 : 0;  // launch_skinny's choice of instantiation
}

bool skinny_supported(int H, int I) {
  return sk_layout(H, I, kJobTokens, kSmallRoutes).nstage >= 3 && sk_layout(H, I, 1, kSmallRoutes).nstage >= 3;
}

int launch_skinny(const SkinnyParams& p, cudaStream_t stream) {
  int grid = 0;
  SkLayout plan;
  int rc = skinny_config(&grid, &plan, p.H, p.I, p.job_tokens, p.small_route ? p.T * p.k : 0);
  if (rc != XCB_OK) return rc;
  // two tokens with one token per job and two activation buffers: the instantiation that stages both rows at start
  const bool two = p.T == 2 && plan.rows == 1 && plan.nbuf == 2;
  if (!p.pdl) {
    if (two)
      skinny_kernel<true><<<grid, SK_THREADS, plan.total, stream>>>(p, plan);
    else
      skinny_kernel<false><<<grid, SK_THREADS, plan.total, stream>>>(p, plan);
    return cudaGetLastError() == cudaSuccess ? XCB_OK : XCB_ERR_CUDA;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(SK_THREADS);
  cfg.dynamicSmemBytes = (size_t)plan.total;
  cfg.stream = stream;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, two ? skinny_kernel<true> : skinny_kernel<false>, p, plan) == cudaSuccess
             ? XCB_OK
             : XCB_ERR_CUDA;
}

}  // namespace xcb
