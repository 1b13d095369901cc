// Decode-path MoE kernel: one persistent launch runs (for small batches) the router, gate_up + SwiGLU (phase A),
// down (phase B) and the weighted combine, for jobs of at most 8 tokens.  This is the HBM-bound path (T = 1
// decode streams ~200 MB of FP4 weights for 8 experts), so the kernel is one continuous weight stream per SM:
//
// * 19 warps per CTA, one CTA per SM, each warp one role:
//   - warp 16 streams packed weights through a shared-memory ring (18 KB stages, one 1-D bulk copy on the TMA
//     engine each, L2 evict-first); 18 KB copies are what a single issuing thread needs to reach HBM rate;
//   - warp 17 stages each segment's activation rows (x for phase A, the job's SwiGLU output for phase B, after an
//     acquire on that job's phase-A counter) into double-buffered shared memory, also with bulk copies;
//   - warp 18 publishes finished work: one GPU-scope fence and one counter update per segment (phase A: the
//     job's unit credits; phase B: the 16-row blocks' counts, combining a block when it completes);
//   - warps 0..15 only compute: slice w of every 16-slice group, the GF(2) decoder (8 integer ops per 8
//     weights), one bf16x2 multiply per register by the block-scale pair and an m16n8k16 tensor-core step fed
//     from registers.  At T <= 8 tokens per expert the weights are used once, and staging decoded bf16 tiles
//     through shared memory for tcgen05 would add 4 B of shared-memory traffic per weight.
// * Units (16 output rows x full K) are reduced without a barrier: each warp drops its partial sums into a slot,
//   the last to arrive sums the 16 partials in warp order (deterministic) and writes the epilogue.
// * Wave schedule for few jobs: every CTA takes an equal share of every job, in the order A0 A1 B0 A2 B1 ...,
//   so phase B of a job starts about one job after its phase A and the weight stream never waits for it.  With
//   many jobs each CTA takes contiguous unit ranges instead.
// * Combine: the CTA whose phase-B units complete a 16-row block forms out = bf16(sum_s w_s * y_s) for it; with the
//   post-norm, or for large batches, a bounded grid barrier precedes a combine spread over all CTAs.
// * Small batches (T*k <= 256) route inside the kernel (every CTA computes the same tables), so a decode step is
//   a single launch.  Every wait is bounded by %globaltimer; on timeout a status bit is set and the kernel drains.
//
// Reference counterpart: moe_fused's skinny path (kernels/moe_w4a16_h200/moe_w4a16.py:491-611 route,
// :754-1133 skinny ring, :1602-1785 warp-specialised epilogues, :2617-2641 grid barrier, :2654-2796 final sum).
#include "common.cuh"
#include "kernels.cuh"
#include "workspace.cuh"

namespace xcb {

// Optional timeline trace (builds with -DXCB_TRACE=1 only): %globaltimer stamps and wait counters per CTA, read back
// with xcb_trace_read.  Off in the shipped library.
#ifndef XCB_TRACE
#define XCB_TRACE 0
#endif
#if XCB_TRACE
constexpr int kTraceSlots = 32;
__device__ unsigned long long g_trace[1024 * kTraceSlots];
#define TRACE_AT(slot) (g_trace[blockIdx.x * kTraceSlots + (slot)] = gtimer())
#define TRACE_ADD(slot, v) atomicAdd(&g_trace[blockIdx.x * kTraceSlots + (slot)], (unsigned long long)(v))
#define TRACE_GET(slot) (*(volatile unsigned long long*)&g_trace[blockIdx.x * kTraceSlots + (slot)])
#else
#define TRACE_AT(slot) ((void)0)
#define TRACE_ADD(slot, v) ((void)0)
#endif

#ifndef XCB_SK_NW
#define XCB_SK_NW 16
#endif
constexpr int SK_NW = XCB_SK_NW;                        // compute warps (each takes slices w, w + SK_NW, ... of a group)
constexpr int SK_W_PROD = SK_NW;                        // weight producer warp
constexpr int SK_W_ACT = SK_NW + 1;                     // activation staging warp
constexpr int SK_W_SIG = SK_NW + 2;                     // signalling warp
constexpr int SK_W_EPI = SK_NW + 3;                     // reduction + epilogue warps (SK_NEPI of them)
constexpr int SK_NEPI = 2;                              // epilogue warp e takes the units with useq % SK_NEPI == e
constexpr int SK_THREADS = (SK_NW + 3 + SK_NEPI) * 32;
constexpr int SK_SLICE_BYTES = 576;                     // 512 B of codes + 64 B of scale codes per 64-k slice
#ifndef XCB_SK_PER
#define XCB_SK_PER 2
#endif
constexpr int SK_PER = XCB_SK_PER;                      // slices per compute warp per stage
constexpr int SK_STAGE_SLICES = SK_PER * SK_NW;         // slices per full stage (18 KB at 2 x 16)
constexpr int SK_MAX_STAGES = 16;
constexpr int SK_MAX_SLOTS = 4;                         // reduction slots
constexpr int SK_SLOT_FLOATS = SK_NW * 32 * 4;
constexpr int SK_MAX_BUFS = 2;                          // activation buffers
constexpr int SK_SEG_RING = 64;                         // per-segment completion counters
constexpr int SK_WAVE_JOBS = 0;                         // at most this many jobs: wave schedule (measured slower:
                                                        // per-job staging and dependency stalls; kept switchable)
constexpr long long SK_L2_PREFETCH_BYTES = 96ll << 20;  // phase-B weights up to this size are prefetched into L2
constexpr int SK_SMEM_LIMIT = 227 * 1024;

// Shared-memory routing tables of the in-kernel router.
struct SkRoute {
  int ids[kSmallRoutes];
  float wts[kSmallRoutes];
  int pos[kSmallRoutes];
  int order[kSmallRoutes];
  int4 jobs[kSmallRoutes];
  int counts[512];
  int offsets[513];
  int jcnt[512];
  int njobs, nroutes;
};

// Control block: mbarriers, reduction-slot and segment bookkeeping.
struct SkCtl {
  uint64_t full[SK_MAX_STAGES], empty[SK_MAX_STAGES];
  uint64_t act_full[SK_MAX_BUFS], act_empty[SK_MAX_BUFS];
  uint64_t slot_full[SK_MAX_SLOTS];  // 16 compute warps deposited their partial sums of a unit
  uint64_t slot_free[SK_MAX_SLOTS];  // the epilogue warp has consumed the slot
  int seg_cnt[SK_SEG_RING];
  int seg_gen[SK_SEG_RING];
  float gs[2][kSmallRoutes];  // phase A / B global scale (x 2^52) of each job (jobs < kSmallRoutes; else global)
  int list[1024];             // scratch: row blocks a segment completed
  int nlist;
};

struct SkLayout {
  int buf, red, route, ctl, ring, total, nstage, nbuf, nslot, rows, pitch, stage_slices;
};

__host__ __device__ inline SkLayout sk_layout(int H, int I, int job_tokens, int small_route) {
  SkLayout o;
  o.pitch = (H > I ? H : I) * 2 + 16;
  o.rows = job_tokens < kJobTokens ? job_tokens : kJobTokens;
  if (o.rows < 1) o.rows = 1;
  const int route = small_route ? (int)sizeof(SkRoute) : 0;
  o.nstage = 0;
  // full-size stages when at least 4 fit, else half-size stages
  for (int ss = SK_STAGE_SLICES; ss >= SK_STAGE_SLICES / 2; ss /= 2) {
    for (int nbuf = SK_MAX_BUFS; nbuf >= 1; --nbuf) {
      for (int nslot = SK_MAX_SLOTS; nslot >= 2; nslot /= 2) {
        o.stage_slices = ss;
        o.nbuf = nbuf;
        o.nslot = nslot;
        o.buf = 0;
        o.red = o.buf + nbuf * o.rows * o.pitch;
        o.route = o.red + nslot * SK_SLOT_FLOATS * 4;
        o.ctl = (o.route + route + 15) & ~15;
        o.ring = (o.ctl + (int)sizeof(SkCtl) + 1023) & ~1023;
        const int ns = (SK_SMEM_LIMIT - o.ring) / (ss * SK_SLICE_BYTES);
        o.nstage = ns > SK_MAX_STAGES ? SK_MAX_STAGES : ns;
        o.total = o.ring + o.nstage * ss * SK_SLICE_BYTES;
        if (o.nstage >= 4) return o;
      }
    }
  }
  return o;
}

// The units of one CTA, cut into segments of one job and one phase, in processing order.
struct SkSegments {
  int wave, njobs, nrbA, nrbB, G, bid;
  long long a0, a1, b0, b1;  // contiguous mode: this CTA's unit ranges
  int jA0, nAj, jB0, nBj;    // contiguous mode: jobs the ranges touch

  __device__ void init(int nj, int nA_rb, int nB_rb, int grid, int b, int wave_mode) {
    njobs = nj;
    nrbA = nA_rb;
    nrbB = nB_rb;
    G = grid;
    bid = b;
    wave = wave_mode;
    const long long nA = (long long)njobs * nrbA, nB = (long long)njobs * nrbB;
    a0 = nA * bid / G;
    a1 = nA * (bid + 1) / G;
    b0 = nB * bid / G;
    b1 = nB * (bid + 1) / G;
    jA0 = (int)(a0 / nrbA);
    nAj = a1 > a0 ? (int)((a1 - 1) / nrbA) - jA0 + 1 : 0;
    jB0 = (int)(b0 / nrbB);
    nBj = b1 > b0 ? (int)((b1 - 1) / nrbB) - jB0 + 1 : 0;
  }
  __device__ int count() const { return wave ? 2 * njobs : nAj + nBj; }
  // Segment i (possibly empty): phase, job, unit range [u0, u1) in the phase's unit numbering (job * nrb + rb).
  __device__ void at(int i, int& ph, int& job, long long& u0, long long& u1) const {
    if (wave) {
      if (i == 0) { ph = 0; job = 0; }
      else if (i == 2 * njobs - 1) { ph = 1; job = njobs - 1; }
      else if (i & 1) { ph = 0; job = (i + 1) / 2; }
      else { ph = 1; job = (i + 1) / 2 - 1; }
      const int nrb = ph ? nrbB : nrbA;
      u0 = (long long)job * nrb + (long long)nrb * bid / G;
      u1 = (long long)job * nrb + (long long)nrb * (bid + 1) / G;
    } else if (i < nAj) {
      ph = 0;
      job = jA0 + i;
      u0 = a0 > (long long)job * nrbA ? a0 : (long long)job * nrbA;
      u1 = a1 < (long long)(job + 1) * nrbA ? a1 : (long long)(job + 1) * nrbA;
    } else {
      ph = 1;
      job = jB0 + i - nAj;
      u0 = b0 > (long long)job * nrbB ? b0 : (long long)job * nrbB;
      u1 = b1 < (long long)(job + 1) * nrbB ? b1 : (long long)(job + 1) * nrbB;
    }
  }
};

// One 64-k slice for one warp: 4 packed words -> 4 tensor-core steps on two accumulator chains.  `grp` is the
// group (ns slices: codes, then scale codes) in shared memory, s the slice within it, S its index in the unit.
__device__ __forceinline__ void sk_slice(const uint8_t* grp, int ns, int s, const uint8_t* xrow, int S, int lane, int t,
                                         float* acc0, float* acc1) {
  const uint4 cw = *reinterpret_cast<const uint4*>(grp + s * 512 + lane * 16);
  const uint32_t sc = *reinterpret_cast<const uint16_t*>(grp + ns * 512 + (s >> 2) * 256 + lane * 8 + (s & 3) * 2);
  const uint4 xa = *reinterpret_cast<const uint4*>(xrow + S * 128 + t * 32);
  const uint4 xb = *reinterpret_cast<const uint4*>(xrow + S * 128 + t * 32 + 16);
  const uint32_t s2 = scale_pair(sc);
  uint32_t r0, r1, r2, r3;
  decode_fp4x8(cw.x, r0, r1, r2, r3);
  mma_16816(acc0, bf16x2_mul_lo(r0, s2), bf16x2_mul_hi(r1, s2), bf16x2_mul_lo(r2, s2), bf16x2_mul_hi(r3, s2), xa.x, xa.y);
  decode_fp4x8(cw.y, r0, r1, r2, r3);
  mma_16816(acc1, bf16x2_mul_lo(r0, s2), bf16x2_mul_hi(r1, s2), bf16x2_mul_lo(r2, s2), bf16x2_mul_hi(r3, s2), xa.z, xa.w);
  decode_fp4x8(cw.z, r0, r1, r2, r3);
  mma_16816(acc0, bf16x2_mul_lo(r0, s2), bf16x2_mul_hi(r1, s2), bf16x2_mul_lo(r2, s2), bf16x2_mul_hi(r3, s2), xb.x, xb.y);
  decode_fp4x8(cw.w, r0, r1, r2, r3);
  mma_16816(acc1, bf16x2_mul_lo(r0, s2), bf16x2_mul_hi(r1, s2), bf16x2_mul_lo(r2, s2), bf16x2_mul_hi(r3, s2), xb.z, xb.w);
}

// In-kernel router for T*k <= kSmallRoutes (all warps; every CTA computes the same tables).
__device__ void sk_route_small(const SkinnyParams& p, SkRoute& r) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nthr = blockDim.x;
  const int R = p.T * p.k;
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
      r.ids[t * p.k + lane] = id;
      r.wts[t * p.k + lane] = w;
    }
  }
  __syncthreads();
  if (tid == 0) TRACE_AT(15);
  // per-expert counts and each route's rank among the earlier routes of its expert (stable order)
  for (int e = tid; e < p.E_loc; e += nthr) {
    int c = 0;
    for (int f = 0; f < R; ++f) c += (r.ids[f] == p.lo + e);
    r.counts[e] = c;
    r.offsets[e] = c;
    r.jcnt[e] = (c + kJobTokens - 1) / kJobTokens;
  }
  for (int f = tid; f < R; f += nthr) {
    const int id = r.ids[f];
    int rank = 0;
    for (int g = 0; g < f; ++g) rank += (r.ids[g] == id);
    r.pos[f] = rank;
  }
  __syncthreads();
  if (warp == 0) {
    const int tot = warp_exclusive_scan(r.offsets, p.E_loc);
    if (lane == 0) {
      r.nroutes = tot;
      r.offsets[p.E_loc] = tot;
    }
  } else if (warp == 1) {
    const int tot = warp_exclusive_scan(r.jcnt, p.E_loc);
    if (lane == 0) r.njobs = tot;
  }
  __syncthreads();
  if (tid == 0) TRACE_AT(16);
  for (int f = tid; f < R; f += nthr) {
    const int el = r.ids[f] - p.lo;
    if (r.ids[f] >= 0 && el >= 0 && el < p.E_loc) {
      const int q = r.offsets[el] + r.pos[f];
      r.pos[f] = q;
      r.order[q] = f;
    } else {
      r.pos[f] = -1;
    }
  }
  for (int e = tid; e < p.E_loc; e += nthr) {
    const int c = r.counts[e];
    int j = r.jcnt[e];
    for (int s0 = 0; s0 < c; s0 += kJobTokens, ++j) r.jobs[j] = make_int4(e, r.offsets[e] + s0, min(kJobTokens, c - s0), 0);
  }
  __syncthreads();
  if (blockIdx.x == 0) {  // publish the routing (tests and callers read it from the workspace)
    for (int f = tid; f < R; f += nthr) {
      p.g_ids[f] = r.ids[f];
      p.g_wts[f] = r.wts[f];
      p.g_pos[f] = r.pos[f];
      if (p.ids_out) p.ids_out[f] = r.ids[f];
      if (p.wts_out) p.wts_out[f] = r.wts[f];
    }
    for (int q = tid; q < r.nroutes; q += nthr) p.g_order[q] = r.order[q];
    for (int e = tid; e <= p.E_loc; e += nthr) {
      if (e < p.E_loc) p.g_counts[e] = r.counts[e];
      p.g_offsets[e] = r.offsets[e];
    }
  }
}



__device__ __forceinline__ void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }

__global__ void __launch_bounds__(SK_THREADS, 1) skinny_kernel(SkinnyParams p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const SkLayout L = sk_layout(p.H, p.I, p.job_tokens, p.small_route);
  uint8_t* bufs = smem + L.buf;
  float* red = reinterpret_cast<float*>(smem + L.red);
  SkRoute& rt = *reinterpret_cast<SkRoute*>(smem + L.route);
  SkCtl& cb = *reinterpret_cast<SkCtl*>(smem + L.ctl);
  uint8_t* ring = smem + L.ring;
  int* status = p.ctl + kCtlStatus;
  const int NST = L.nstage, NBUF = L.nbuf, NSLOT = L.nslot;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = gridDim.x, bid = blockIdx.x;

  if (tid == 0) {
    TRACE_AT(0);
    for (int i = 0; i < NST; ++i) {
      mbar_init(cb.full + i, 1);
      mbar_init(cb.empty + i, SK_NW);
    }
    for (int i = 0; i < NBUF; ++i) {
      mbar_init(cb.act_full + i, 1);
      mbar_init(cb.act_empty + i, SK_NW);
    }
    fence_mbar_init();
  }
  if (tid == 0) {
    for (int i = 0; i < NSLOT; ++i) {
      mbar_init(cb.slot_full + i, SK_NW);
      mbar_init(cb.slot_free + i, 1);
    }
    fence_mbar_init();
  }
  for (int i = tid; i < SK_SEG_RING; i += SK_THREADS) {
    cb.seg_cnt[i] = 0;
    cb.seg_gen[i] = 0;
  }
  if (tid == 0) cb.nlist = 0;
  if (p.small_route) sk_route_small(p, rt);
  __syncthreads();
  if (tid == 0) TRACE_AT(1);

  const int njobs = p.small_route ? rt.njobs : p.ctl[kCtlJobs];
  const int4* jobs = p.small_route ? rt.jobs : p.jobs;
  const int* order = p.small_route ? rt.order : p.order;
  const int* pos = p.small_route ? rt.pos : p.pos;
  const float* wts = p.small_route ? rt.wts : p.wts;
  const int nrbA = (2 * p.I) / 16, nrbB = p.H / 16;
  const int nSA = p.H / 64, nSB = p.I / 64;  // slices per unit
  const int gsA = group_slices(p.H), gsB = group_slices(p.I);
  const int ssA = L.stage_slices / gsA * gsA, ssB = L.stage_slices / gsB * gsB;  // slices per full stage (whole groups)
  const size_t unitA = (size_t)9 * p.H, unitB = (size_t)9 * p.I;
  SkSegments segs;
  segs.init(njobs, nrbA, nrbB, G, bid, njobs <= SK_WAVE_JOBS);
  const int nseg = segs.count();
  const bool gs_cached = njobs <= kSmallRoutes;
  if (gs_cached) {
    for (int j = tid; j < njobs; j += SK_THREADS) {
      const int e = jobs[j].x;
      cb.gs[0][j] = p.gsA[e] * kTwo52;
      cb.gs[1][j] = p.gsB[e] * kTwo52;
    }
  }
  __syncthreads();

  if (warp == SK_W_PROD) {
    // ------------------------------------------------------------------ weight producer
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      int it = 0;
      bool ok = true;
      // phase-B weights do not depend on phase A: when they fit in L2, stream them into L2 right behind this CTA's
      // phase-A weights, so HBM sees one continuous stream and phase B reads L2 after the A -> B handoff
      const bool prefetch_b = (long long)njobs * nrbB * (long long)unitB <= SK_L2_PREFETCH_BYTES;
      bool prefetched = false;
      for (int s = 0; s < nseg && ok; ++s) {
        int ph, job;
        long long u0, u1;
        segs.at(s, ph, job, u0, u1);
        if (ph == 1 && prefetch_b && !prefetched) {
          prefetched = true;
          for (int s2 = s; s2 < nseg; ++s2) {
            int ph2, job2;
            long long v0, v1;
            segs.at(s2, ph2, job2, v0, v1);
            if (ph2 != 1 || v1 <= v0) continue;
            const uint8_t* first = p.wB + ((size_t)jobs[job2].x * nrbB + (size_t)(v0 - (long long)job2 * nrbB)) * unitB;
            const size_t total = (size_t)(v1 - v0) * unitB;  // consecutive units of one job are contiguous
            for (size_t off = 0; off < total; off += (size_t)1 << 20)
              bulk_prefetch_l2(first + off, (uint32_t)min(total - off, (size_t)1 << 20));
          }
        }
        // the segment's units are one contiguous byte range; stream it in stages of whole groups
        const int nrb = ph ? nrbB : nrbA, ss = ph ? ssB : ssA;
        const long long nsl = (u1 - u0) * (ph ? nSB : nSA);
        const uint8_t* seg = (ph ? p.wB : p.wA) +
                             ((size_t)jobs[job].x * nrb + (size_t)(u0 - (long long)job * nrb)) * (ph ? unitB : unitA);
        for (long long base = 0; base < nsl && ok; base += ss, ++it) {
          const int ns = (int)min((long long)ss, nsl - base);
          const int st = it % NST;
          if (it >= NST && !mbar_wait(cb.empty + st, ((it / NST) + 1) & 1, p.timeout_ns, status)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(cb.full + st, ns * SK_SLICE_BYTES);
          bulk_g2s_stream(ring + (size_t)st * L.stage_slices * SK_SLICE_BYTES, seg + (size_t)base * SK_SLICE_BYTES,
                          ns * SK_SLICE_BYTES, cb.full + st, pol);
        }
      }
      TRACE_AT(3);
      for (int i = max(0, it - NST); i < it; ++i) mbar_wait(cb.full + (i % NST), (i / NST) & 1, p.timeout_ns, status);
    }
  } else if (warp == SK_W_ACT) {
    // ------------------------------------------------------------------ activation staging
    if (lane == 0) {
      int k = 0;  // non-empty segments so far
      for (int s = 0; s < nseg; ++s) {
        int ph, job;
        long long u0, u1;
        segs.at(s, ph, job, u0, u1);
        if (u1 <= u0) continue;
        const int b = k % NBUF;
        if (k >= NBUF) mbar_wait(cb.act_empty + b, ((k / NBUF) + 1) & 1, p.timeout_ns, status);
        const int4 jb = jobs[job];
        const int K = ph ? p.I : p.H;
        if (ph == 1) {
          wait_geq(p.doneA + job, nrbA, p.timeout_ns, status);  // every phase-A unit of this job is published
          fence_proxy_async_global();
        }
        uint8_t* dst = bufs + (size_t)b * L.rows * L.pitch;
        const int ntok = min(jb.z, L.rows);
        mbar_arrive_expect_tx(cb.act_full + b, ntok * K * 2);
        for (int n = 0; n < ntok; ++n) {
          const uint16_t* src = ph ? p.inter + (size_t)(jb.y + n) * p.I : p.x + (size_t)(order[jb.y + n] / p.k) * p.H;
          bulk_g2s(dst + n * (size_t)(K * 2 + 16), src, K * 2, cb.act_full + b);
        }
        ++k;
      }
      for (int i = max(0, k - NBUF); i < k; ++i) mbar_wait(cb.act_full + (i % NBUF), (i / NBUF) & 1, p.timeout_ns, status);
      TRACE_AT(20);
    }
  } else if (warp == SK_W_SIG) {
    // ------------------------------------------------------------------ signalling
    int k = 0;
    for (int s = 0; s < nseg; ++s) {
      int ph, job;
      long long u0, u1;
      segs.at(s, ph, job, u0, u1);
      if (u1 <= u0) continue;
      const int slot = k % SK_SEG_RING;
      const int want = (int)(u1 - u0);
      // all units of the segment reduced and written by the compute warps (CTA-scope release, acquire here)
      if (lane == 0) {
        const uint64_t t0 = gtimer();
        while (*reinterpret_cast<volatile int*>(&cb.seg_cnt[slot]) < want) {
          __nanosleep(200);
          if (gtimer() - t0 > p.timeout_ns) {
            set_status(status, XCB_STATUS_DEVICE_TIMEOUT);
            break;
          }
        }
      }
      __syncwarp();
      __threadfence();  // cumulative: publishes the compute warps' epilogue writes GPU-wide before the counters move
      if (lane == 0) {
        cb.seg_cnt[slot] = 0;
        *reinterpret_cast<volatile int*>(&cb.seg_gen[slot]) = k / SK_SEG_RING + 1;
      }
      if (ph == 0) {
        if (lane == 0) atomicAdd(p.doneA + job, want);
      } else if (!p.grid_combine) {
        // one count per 16-row block; the CTA that completes a block combines it (all its threads, at the end)
        for (long long u = u0 + lane; u < u1; u += 32) {
          const int rb = (int)(u - (long long)job * nrbB);
          if (atomicAdd(p.rbcnt + rb, 1) == njobs - 1) cb.list[atomicAdd(&cb.nlist, 1)] = rb;
        }
        __syncwarp();
      }
      ++k;
    }
    if (lane == 0) TRACE_AT(21);
  } else if (warp >= SK_W_EPI) {
    // ------------------------------------------------------------------ reduction + epilogue
    const int g = lane >> 2, t = lane & 3;
    const int epi = warp - SK_W_EPI;
    int useq = 0, k = 0;
    for (int s = 0; s < nseg; ++s) {
      int ph, job;
      long long u0, u1;
      segs.at(s, ph, job, u0, u1);
      if (u1 <= u0) continue;
      const int nrb = ph ? nrbB : nrbA;
      const int4 jb = jobs[job];
      const float gsc = gs_cached ? cb.gs[ph][job] : (ph ? p.gsB : p.gsA)[jb.x] * kTwo52;
      for (long long u = u0; u < u1; ++u, ++useq) {
        if (useq % SK_NEPI != epi) continue;
        const int rb = (int)(u - (long long)job * nrb);
        const int slot = useq % NSLOT;
        mbar_wait(cb.slot_full + slot, (useq / NSLOT) & 1, p.timeout_ns, status);
        const float* sb = red + slot * SK_SLOT_FLOATS;
        float v[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 8
        for (int w = 0; w < SK_NW; ++w) {  // fixed warp order: deterministic sums
          const float4 r = *reinterpret_cast<const float4*>(sb + (w * 32 + lane) * 4);
          v[0] += r.x; v[1] += r.y; v[2] += r.z; v[3] += r.w;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(cb.slot_free + slot);
        if (ph == 0) {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int n = 2 * t + h;
            if (n < jb.z) {
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
            const float y0 = v[h] * gsc * n0, y1 = v[2 + h] * gsc * n1;
            float sq = y0 * y0 + y1 * y1;
            if (n < jb.z) {
              p.y[(size_t)(jb.y + n) * p.H + r0] = y0;
              p.y[(size_t)(jb.y + n) * p.H + r1] = y1;
            }
            if (p.post_norm) {
              sq += __shfl_xor_sync(0xffffffffu, sq, 4);
              sq += __shfl_xor_sync(0xffffffffu, sq, 8);
              sq += __shfl_xor_sync(0xffffffffu, sq, 16);
              if (g == 0 && n < jb.z) atomicAdd(p.ss + jb.y + n, sq);
            }
          }
        }
        // hand the finished unit to the signalling warp (CTA-scope release of the epilogue writes)
        __syncwarp();
        if (lane == 0) {
          const int sl = k % SK_SEG_RING;
          const int want = k / SK_SEG_RING;
          if (*reinterpret_cast<volatile int*>(&cb.seg_gen[sl]) < want) {
            const uint64_t t0 = gtimer();
            while (*reinterpret_cast<volatile int*>(&cb.seg_gen[sl]) < want) {
              __nanosleep(100);
              if (gtimer() - t0 > p.timeout_ns) {
                set_status(status, XCB_STATUS_DEVICE_TIMEOUT);
                break;
              }
            }
          }
          __threadfence_block();
          atomicAdd(&cb.seg_cnt[sl], 1);
        }
      }
      ++k;
    }
    if (lane == 0) TRACE_AT(22);
  } else {
    // ------------------------------------------------------------------ compute warps
    // A segment's slices are streamed in stages of whole groups; warp w takes stage slices w, w + SK_NW, ...
    // Each slice belongs to one unit (its 16 rows); a warp hands its partial sums of a unit to the epilogue warps
    // when its slices move past the unit (a unit none of whose slices this warp saw gets a zero partial).
    const int g = lane >> 2, t = lane & 3;
    const int grow = g < L.rows ? g : L.rows - 1;  // MMA columns past the job's tokens are computed and discarded
    int st = 0, useq = 0, k = 0;
    uint32_t sphase = 0;
    float a0[4] = {0.f, 0.f, 0.f, 0.f}, a1[4] = {0.f, 0.f, 0.f, 0.f};
    float a2[4] = {0.f, 0.f, 0.f, 0.f}, a3[4] = {0.f, 0.f, 0.f, 0.f};
    auto flush = [&]() {  // deposit this warp's partial of unit `useq` and start the next unit
      const int slot = useq % NSLOT;
      if (useq >= NSLOT) mbar_wait(cb.slot_free + slot, ((useq / NSLOT) + 1) & 1, p.timeout_ns, status);
      *reinterpret_cast<float4*>(red + slot * SK_SLOT_FLOATS + (warp * 32 + lane) * 4) =
          make_float4(a0[0] + a2[0] + (a1[0] + a3[0]), a0[1] + a2[1] + (a1[1] + a3[1]),
                      a0[2] + a2[2] + (a1[2] + a3[2]), a0[3] + a2[3] + (a1[3] + a3[3]));
      __syncwarp();
      if (lane == 0) mbar_arrive(cb.slot_full + slot);
#pragma unroll
      for (int i = 0; i < 4; ++i) a0[i] = a1[i] = a2[i] = a3[i] = 0.f;
      ++useq;
    };
    for (int s = 0; s < nseg; ++s) {
      int ph, job;
      long long u0, u1;
      segs.at(s, ph, job, u0, u1);
      if (u1 <= u0) continue;
      const int b = k % NBUF;
      const int spu = ph ? nSB : nSA, gs = ph ? gsB : gsA, ss = ph ? ssB : ssA;
      const int pitch = (ph ? p.I : p.H) * 2 + 16;
      const long long nsl = (u1 - u0) * spu;
      mbar_wait(cb.act_full + b, (k / NBUF) & 1, p.timeout_ns, status);
      const uint8_t* xrow = bufs + (size_t)b * L.rows * L.pitch + grow * pitch;
      // per-warp constants of the segment: where each of its stage slices sits (group offset, slice in group)
      int goff[SK_PER], gsl[SK_PER];
#pragma unroll
      for (int j = 0; j < SK_PER; ++j) {
        const int i = warp + j * SK_NW, q = i / gs;
        goff[j] = q * gs * SK_SLICE_BYTES;
        gsl[j] = i - q * gs;
      }
      const int nsl32 = (int)nsl;
      int ucur = 0, uend = spu;  // unit this warp is accumulating, and the segment slice where it ends
      for (int base = 0; base < nsl32; base += ss) {
        mbar_wait(cb.full + st, sphase, p.timeout_ns, status);
        const uint8_t* stage = ring + (size_t)st * L.stage_slices * SK_SLICE_BYTES;
        const int ns = min(ss, nsl32 - base);
#pragma unroll
        for (int j = 0; j < SK_PER; ++j) {
          const int i = warp + j * SK_NW;
          if (i < ns) {
            const int gi = base + i;
            while (gi >= uend) {
              flush();
              ++ucur;
              uend += spu;
            }
            if (j & 1)
              sk_slice(stage + goff[j], gs, gsl[j], xrow, gi - (uend - spu), lane, t, a2, a3);
            else
              sk_slice(stage + goff[j], gs, gsl[j], xrow, gi - (uend - spu), lane, t, a0, a1);
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(cb.empty + st);
        if (++st == NST) {
          st = 0;
          sphase ^= 1;
        }
      }
      while (ucur < (int)(u1 - u0)) {
        flush();
        ++ucur;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(cb.act_empty + b);
      ++k;
    }
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

  // -------------------------------------------------------------------- exit: the last CTA resets the counters
  __syncthreads();
  if (tid == 0) {
    TRACE_AT(8);
    __threadfence();
    const int done = atomicAdd(p.ctl + kCtlExit, 1);
    if (done == G - 1) {
      if (p.small_route) {
        for (int j = 0; j < njobs; ++j) p.doneA[j] = 0;
        if (p.post_norm)
          for (int q = 0; q < rt.nroutes; ++q) p.ss[q] = 0.f;
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

int skinny_config(int* grid_out, int* smem_out, int H, int I, int job_tokens, int small_route) {
  static int cached_dev = -1, cached_sms = 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return XCB_ERR_CUDA;
  const SkLayout L = sk_layout(H, I, job_tokens, small_route);
  if (L.nstage < 4) return XCB_ERR_UNSUPPORTED;
  if (cudaFuncSetAttribute(skinny_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, L.total) != cudaSuccess)
    return XCB_ERR_CUDA;
  if (dev != cached_dev) {
    if (cudaDeviceGetAttribute(&cached_sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return XCB_ERR_CUDA;
    cached_dev = dev;
  }
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, skinny_kernel, SK_THREADS, L.total) != cudaSuccess ||
      per_sm < 1)
    return XCB_ERR_CUDA;
  *grid_out = cached_sms * per_sm;
  *smem_out = L.total;
  return XCB_OK;
}

size_t skinny_smem_bytes(int H, int I) {
  const SkLayout L = sk_layout(H, I, kJobTokens, 1);
  return L.nstage >= 4 ? (size_t)L.total : (size_t)1 << 30;
}

int launch_skinny(const SkinnyParams& p, cudaStream_t stream) {
  int grid = 0, smem = 0;
  int rc = skinny_config(&grid, &smem, p.H, p.I, p.job_tokens, p.small_route);
  if (rc != XCB_OK) return rc;
  skinny_kernel<<<grid, SK_THREADS, smem, stream>>>(p);
  return cudaGetLastError() == cudaSuccess ? XCB_OK : XCB_ERR_CUDA;
}

}  // namespace xcb
