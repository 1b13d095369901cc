// Prefill path (many tokens per expert): per-expert grouped GEMMs on the fifth-generation tensor core.
//
// Replaces the reference's large-M variants — the "fat" and warp-specialised grouped GEMMs
// (kernels/moe_w4a16_h200/moe_w4a16.py:1136-1566, :1824-2358) with their epilogues epi_A (SwiGLU, :616-627) and
// epi_B (down projection, post-norm partial sums, :628-657), and the final weighted combine (:2654-2796) — with
// four launches on top of the router:
//
//   gather   xperm[q] = x[token of route q]                (routes in expert order, so each expert's rows are one
//                                                           contiguous block a 2-D TMA box can fetch)
//   wide(0)  inter[q] = SiLU(gate_e x) * up_e x             (bf16, rounded as the reference rounds inter)
//   wide(1)  y[q] = down_e inter[q] * gs (* (1 + post_norm_w)), ss[q] += sum y^2 in post-norm mode   (fp32)
//   combine  out[t] = bf16(sum_s w_s (* rsqrt(ss/H + 1e-8)) y[pos[t, s]])          (slot order, as the reference)
//
// wide_kernel is persistent (one CTA per SM, 640 threads; the weight-stream warp claims tiles in order from one
// counter shared by all CTAs and hands them to the other roles through a shared-memory ring).  A tile is 128 packed
// weight rows of one expert x up to 192 of its tokens, the full reduction length:
//
//   warp 0       streams the tile's packed weights (18 KB bulk copies, the prefill layout) into a 4-stage ring;
//   warp 2       loads the tokens' activation rows into a 4-stage ring: one 2-D TMA box (64 k x 64, 128 or 256
//                rows, 128-byte swizzle) per 64-k chunk;
//   warps 4-11   two dequantising warpgroups, alternating 64-k chunks: each thread owns one weight row (= one
//                tensor-memory lane), decodes 8 FP4 codes per word with the GF(2) decoder, applies the exact
//                bf16 scale, and writes 64 bf16 weights into tensor memory with one tcgen05.st — the MMA's A
//                operand never touches shared memory;
//   warp 1       allocates tensor memory and issues tcgen05.mma (M = 128, N = tokens rounded up to 16, K = 16)
//                from tensor-memory A and shared-memory B; its loop is kept lean because one thread must issue
//                an MMA every 64-128 clocks to keep the tensor core busy;
//   warps 12-19  drain the fp32 accumulator (tcgen05.ld; two warps per lane quarter, one per 128-token half)
//                through the epilogue and release it.
//
// Tensor memory (512 columns): an A ring of 4 chunks x 32 columns, then two 192-column accumulators, so the MMAs
// of the next tile run while the epilogue drains the last one (with one accumulator the MMA warp waited for every
// drain, ~16 % of the GEMM time at the DeepSeek-V3 prefill size).  The MMA issue rate sets the shape: a
// 128 x N x 16 bf16 MMA takes N/2 clocks for N >= 64 (44 clocks below), so wide tiles amortise the per-instruction
// cost.  Every wait is bounded; a wait that runs out sets
// XCB_STATUS_DEVICE_TIMEOUT and an abort flag that ends every role, and the kernel drains its copies and MMAs
// before it frees tensor memory.
#include <cudaTypedefs.h>

#include <mutex>

#include "kernels.cuh"
#include "tcgen05.cuh"
#include "workspace.cuh"

namespace xcb {

// Tile shape knobs (compile time): tokens per tile, tensor-memory A slots, activation stages.  Tensor memory holds
// the A ring (32 columns a slot) and two accumulators of kWdTok columns: 4 x 32 + 2 x 192 = 512.
#ifndef XCB_WD_TOK
#define XCB_WD_TOK 192
#endif
#ifndef XCB_WD_ASLOTS
#define XCB_WD_ASLOTS 4
#endif
#ifndef XCB_WD_BST
#define XCB_WD_BST 4
#endif
constexpr int kWdTok = XCB_WD_TOK;  // tokens per tile (MMA N upper bound; two accumulators of this width)
constexpr int kWdStage = 18432;   // packed bytes of 256 k x 128 rows
constexpr int kWdChunk = 4608;    // packed bytes of 64 k x 128 rows
constexpr int kWdWSt = 4;         // weight ring stages (power of two)
constexpr int kWdBSt = XCB_WD_BST;  // activation ring stages, 64 k x (the widest box) bf16 each
constexpr int kWdBBytes = (kWdTok > 128 ? 256 : (kWdTok > 64 ? 128 : 64)) * 128;
constexpr int kWdASlots = XCB_WD_ASLOTS;  // tensor-memory A ring, 32 columns each (power of two)
constexpr int kWdEpiHalf = kWdTok > 128 ? 128 : kWdTok / 2;  // columns of one epilogue column half
#ifndef XCB_WD_NDQ
#define XCB_WD_NDQ 2
#endif
constexpr int kWdDq = XCB_WD_NDQ;  // dequantising warpgroups
constexpr int kWdEpiWarp0 = 4 + 4 * kWdDq;
constexpr int kWdEpiWarps = 8;     // two per tensor-memory lane quarter, one per 128-column half
constexpr int kWdThreads = 32 * (kWdEpiWarp0 + kWdEpiWarps);
constexpr int kWdXbuf = 4 * 2 * 32 * 17;  // SwiGLU exchange: [pair][gate|up][32 lanes][16 tokens + 1]
constexpr int kWdTQ = 8;  // tile ring: tiles claimed by the weight-stream warp, read in order by every other role
constexpr int kWdTQReaders = 2 + 4 * kWdDq + kWdEpiWarps;  // activation producer, MMA, dequantising, epilogue warps
constexpr int kWdNBar = 2 * kWdWSt + 2 * kWdASlots + 4 + 1 + 2 * kWdTQ;
constexpr size_t kWdOffB = (size_t)kWdWSt * kWdStage;  // 1024-aligned (swizzle atoms)
constexpr size_t kWdOffX = kWdOffB + (size_t)kWdBSt * kWdBBytes;
constexpr size_t kWdOffBar = kWdOffX + (size_t)kWdXbuf * 4;
constexpr size_t kWdOffTab = kWdOffBar + (size_t)kWdNBar * 8;
constexpr size_t kWdOffMisc = kWdOffTab + 2 * 516 * 4;
constexpr size_t kWdOffCol = kWdOffMisc + 64;       // fused combine: [2 tiles][kWdTok] token ids, then route weights
constexpr size_t kWdSmem = kWdOffCol + 2 * kWdTok * 8 + 1024;  // + slack to align the base to 1024
// Tensor memory (512 columns): the A ring [0, 128), accumulator 0 [128, 320), accumulator 1 [320, 512): the MMAs
// of tile i + 1 fill one accumulator while the epilogue drains tile i from the other.
constexpr uint32_t kWdDCol = 32 * kWdASlots;
static_assert(kWdDCol + 2 * kWdTok <= 512, "tensor memory columns");
static_assert(kWdOffB % 1024 == 0, "activation ring must be 1024-aligned");
static_assert(kWdSmem <= 227 * 1024, "prefill kernel shared memory");

// Activation boxes: 64 k x {64, 128, 256} rows; a tile loads the smallest box that covers its tokens.
struct WdMaps {
  CUtensorMap m64, m128, m256;
};

struct WdTile {
  int e, rb, q0, n;
};

// Compile-time role profile (-DXCB_WD_PROFILE=1): per CTA, clock64 cycles each role spends waiting and working,
// read back with xcb_wide_profile_read.  Off in the shipped build.
#ifndef XCB_WD_PROFILE
#define XCB_WD_PROFILE 0
#endif
#if XCB_WD_PROFILE
constexpr int kWdProfSlots = 16;
__device__ unsigned long long g_wd_prof[1024 * kWdProfSlots];
#define WD_PROF_T0(name) const unsigned long long name = clock64()
#define WD_PROF_ADD(slot, since) atomicAdd(&g_wd_prof[blockIdx.x * kWdProfSlots + (slot)], clock64() - (since))
#define WD_PROF_INC(slot) atomicAdd(&g_wd_prof[blockIdx.x * kWdProfSlots + (slot)], 1ull)
#else
#define WD_PROF_T0(name)
#define WD_PROF_ADD(slot, since)
#define WD_PROF_INC(slot)
#endif

// Tile i -> (expert, row block, first permuted route, tokens).  Tiles run expert by expert, token tile by token
// tile, row block fastest: the row blocks sharing one token tile run side by side and read its activation box from
// L2 (a 192-token box is 5.3x the bytes of a 128-row weight block per k), and the expert's weights (16.5 MB for
// gate_up at the DeepSeek-V3 shape) stay in L2 across the few token tiles in flight.  With the token tile fastest,
// the ~148 tiles in flight on a wide expert would each read a different box, and every row block would re-read
// the activations from HBM.
__device__ __forceinline__ WdTile wd_tile(int i, const int* tpre, const int* offs, int E, int RB) {
  int lo = 0, hi = E - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (tpre[mid] <= i) lo = mid; else hi = mid - 1;
  }
  const int cnt = offs[lo + 1] - offs[lo];
  const int local = i - tpre[lo];
  WdTile t;
  t.e = lo;
  const int tt = local / RB;
  t.rb = local - tt * RB;
  t.q0 = offs[lo] + tt * kWdTok;
  t.n = min(kWdTok, cnt - tt * kWdTok);
  return t;
}

// Bounded wait that also gives up as soon as another role has aborted.
__device__ __forceinline__ bool wd_wait(uint64_t* bar, uint32_t par, volatile int* abrt, const WideParams& p) {
  if (mbar_try_wait(bar, par)) return true;
  const uint64_t t0 = gtimer();
  while (!mbar_try_wait(bar, par)) {
    if (*abrt) return false;
    if (gtimer() - t0 > p.timeout_ns) {
      set_status(p.status, XCB_STATUS_DEVICE_TIMEOUT);
      *abrt = 1;
      return false;
    }
  }
  return true;
}

// Tile n of this CTA's sequence, as published by the weight-stream warp (-1: no more tiles, or an abort).  The
// whole warp calls wd_next_tile_warp (every lane gets lane 0's read, taken before lane 0 releases the slot); a
// single thread calls wd_next_tile_one.
__device__ __forceinline__ int wd_next_tile_warp(uint64_t* full, uint64_t* empty, volatile int* tq, uint32_t n,
                                                 volatile int* abrt, const WideParams& p) {
  const uint32_t s = n % kWdTQ;
  const bool ok = __all_sync(0xffffffffu, wd_wait(full + s, (n / kWdTQ) & 1, abrt, p));
  int i = ok ? tq[s] : -1;
  i = __shfl_sync(0xffffffffu, i, 0);
  if ((threadIdx.x & 31) == 0 && ok) mbar_arrive(empty + s);
  return i;
}
__device__ __forceinline__ int wd_next_tile_one(uint64_t* full, uint64_t* empty, volatile int* tq, uint32_t n,
                                                volatile int* abrt, const WideParams& p) {
  const uint32_t s = n % kWdTQ;
  if (!wd_wait(full + s, (n / kWdTQ) & 1, abrt, p)) return -1;
  const int i = tq[s];
  mbar_arrive(empty + s);
  return i;
}

__device__ __forceinline__ uint32_t bf16x2_mul(uint32_t a, uint32_t b) {
  __nv_bfloat162 r = __hmul2(*reinterpret_cast<__nv_bfloat162*>(&a), *reinterpret_cast<__nv_bfloat162*>(&b));
  return *reinterpret_cast<uint32_t*>(&r);
}

// One row's 64 weights of a chunk: 8 packed words (k = 8i .. 8i+7) and 4 scale codes (16 k each) -> 32 bf16x2
// tensor-memory columns, each weight exactly e2m1 * sf * 2^-52.
__device__ __forceinline__ void dequant_row64(const uint4& h0, const uint4& h1, uint32_t sc, uint32_t (&r)[32]) {
  const uint32_t w[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
  uint32_t s[4];
#pragma unroll
  for (int b = 0; b < 4; ++b) s[b] = __byte_perm(sc, 0u, 0x4040u + 0x101u * b) * 16u + 0x60006000u;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    uint32_t a0, a1, a2, a3;
    decode_fp4x8(w[i], a0, a1, a2, a3);
    const uint32_t f = s[i >> 1];
    r[4 * i + 0] = bf16x2_mul(a0, f);
    r[4 * i + 1] = bf16x2_mul(a1, f);
    r[4 * i + 2] = bf16x2_mul(a2, f);
    r[4 * i + 3] = bf16x2_mul(a3, f);
  }
}

__global__ void __launch_bounds__(kWdThreads, 1) wide_kernel(const WideParams p, const __grid_constant__ WdMaps maps) {
  extern __shared__ uint8_t wd_raw[];
  uint8_t* sm = wd_raw + ((1024u - (smem_u32(wd_raw) & 1023u)) & 1023u);
  uint8_t* wring = sm;
  uint8_t* bring = sm + kWdOffB;
  float* xbuf = reinterpret_cast<float*>(sm + kWdOffX);
  uint64_t* w_full = reinterpret_cast<uint64_t*>(sm + kWdOffBar);
  uint64_t* w_empty = w_full + kWdWSt;
  // chunk gc: ab_full[gc % 8] completes when its A slot (4 dequantising warps) and its activation box (TMA
  // bytes) are in place; ab_empty[gc % 8] when the MMAs that read them have completed (one commit), which frees
  // both the A slot (reused by chunk gc + 8) and the activation slot (reused by chunk gc + 4)
  uint64_t* ab_full = w_empty + kWdWSt;
  uint64_t* ab_empty = ab_full + kWdASlots;
  uint64_t* d_full = ab_empty + kWdASlots;  // [2]: accumulator b holds a finished tile
  uint64_t* d_empty = d_full + 2;           // [2]: the epilogue drained accumulator b
  uint64_t* drain = d_empty + 2;
  uint64_t* tq_full = drain + 1;           // [kWdTQ]: tile slot published
  uint64_t* tq_empty = tq_full + kWdTQ;    // [kWdTQ]: every reader has taken it
  volatile int* tq = reinterpret_cast<volatile int*>(sm + kWdOffMisc + 32);
  int* offs = reinterpret_cast<int*>(sm + kWdOffTab);
  int* tpre = offs + 516;
  volatile int* abrt = reinterpret_cast<volatile int*>(sm + kWdOffMisc);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + kWdOffMisc + 16);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int E = p.E_loc, RB = p.R / 128, nK = p.K / 64, nS = p.K / 256;

  if (tid == 0) {
    for (int i = 0; i < kWdWSt; ++i) {
      mbar_init(w_full + i, 1);
      mbar_init(w_empty + i, 16);  // 4 chunks x 4 warps read each stage
    }
    for (int i = 0; i < kWdASlots; ++i) {
      mbar_init(ab_full + i, 5);  // 4 dequantising warps + the activation producer (with the box's bytes)
      mbar_init(ab_empty + i, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(d_full + b, 1);
      mbar_init(d_empty + b, kWdEpiWarps);
    }
    mbar_init(drain, 1);
    for (int i = 0; i < kWdTQ; ++i) {
      mbar_init(tq_full + i, 1);
      mbar_init(tq_empty + i, kWdTQReaders);
    }
    *abrt = 0;
    fence_mbar_init();
  }
  if (warp == 3) {  // tile table: tiles of expert e start at tpre[e]
    for (int e = lane; e <= E; e += 32) offs[e] = p.offsets[e];
    __syncwarp();
    for (int e = lane; e < E; e += 32) tpre[e] = (offs[e + 1] - offs[e] + kWdTok - 1) / kWdTok * RB;
    __syncwarp();
    const int tot = warp_exclusive_scan(tpre, E);
    if (lane == 0) tpre[E] = tot;
  }
  if (warp == 1) {
    tmem_alloc(tslot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  const int ntiles = tpre[E];

  if (warp == 0) {
    // ---------------------------------------------------------------- weight stream
    if (lane == 0) {
      uint32_t ws = 0, nq = 0;
      bool ok = true;
      // tiles are claimed in order from one counter shared by all CTAs (a CTA on a slower SM, or with narrower
      // tiles, simply claims fewer), and published to this CTA's other roles through the tile ring
      auto publish = [&](int i) -> bool {
        const uint32_t s = nq % kWdTQ;
        if (nq >= (uint32_t)kWdTQ && !wd_wait(tq_empty + s, ((nq / kWdTQ) + 1) & 1, abrt, p)) return false;
        tq[s] = i;
        mbar_arrive(tq_full + s);
        ++nq;
        return true;
      };
      for (;;) {
        const int i = atomicAdd(p.tilectl, 1);
        if (i >= ntiles) {
          publish(-1);
          break;
        }
        if (!publish(i)) {
          ok = false;
          break;
        }
        const WdTile t = wd_tile(i, tpre, offs, E, RB);
        const uint8_t* src = p.w + ((size_t)t.e * RB + t.rb) * (size_t)nS * kWdStage;
        for (int s = 0; s < nS; ++s) {
          const uint32_t slot = ws & (kWdWSt - 1);
          WD_PROF_T0(t_w);
          if (ws >= (uint32_t)kWdWSt && !wd_wait(w_empty + slot, ((ws / kWdWSt) + 1) & 1, abrt, p)) {
            ok = false;
            break;
          }
          WD_PROF_ADD(10, t_w);
          mbar_arrive_expect_tx(w_full + slot, kWdStage);
          bulk_g2s(wring + (size_t)slot * kWdStage, src + (size_t)s * kWdStage, kWdStage, w_full + slot);
          ++ws;
        }
        if (!ok) break;
      }
      for (uint32_t u = ws > (uint32_t)kWdWSt ? ws - kWdWSt : 0; u < ws; ++u)  // copies still landing
        mbar_wait(w_full + (u & (kWdWSt - 1)), (u / kWdWSt) & 1, p.timeout_ns, p.status);
    }
  } else if (warp == 2) {
    // ---------------------------------------------------------------- activation rows
    if (lane == 0) {
      uint32_t bs = 0;
      bool ok = true;
      for (uint32_t n = 0; ok; ++n) {
        const int i = wd_next_tile_one(tq_full, tq_empty, tq, n, abrt, p);
        if (i < 0) break;
        const WdTile t = wd_tile(i, tpre, offs, E, RB);
        const CUtensorMap* tm = t.n <= 64 ? &maps.m64 : (t.n <= 128 ? &maps.m128 : &maps.m256);
        const uint32_t bytes = (t.n <= 64 ? 64u : (t.n <= 128 ? 128u : 256u)) * 128u;
        for (int c = 0; c < nK; ++c) {
          const uint32_t slot = bs % kWdBSt, bar = bs & (kWdASlots - 1);
          WD_PROF_T0(t_b);
          // the activation slot was last read by chunk bs - kWdBSt, whose MMAs complete ab_empty[that % 8]
          if (bs >= (uint32_t)kWdBSt &&
              !wd_wait(ab_empty + ((bs - kWdBSt) & (kWdASlots - 1)), ((bs - kWdBSt) / kWdASlots) & 1, abrt, p)) {
            ok = false;
            break;
          }
          WD_PROF_ADD(13, t_b);
          mbar_arrive_expect_tx(ab_full + bar, bytes);
          tma_load_2d(bring + (size_t)slot * kWdBBytes, tm, c * 64, t.q0, ab_full + bar);
          ++bs;
        }
      }
      // copies still landing: the last chunks' barriers complete once both halves arrived, so wait for the TMA
      // bytes alone through the last phase of each (bounded)
      for (uint32_t u = bs > (uint32_t)kWdASlots ? bs - kWdASlots : 0; u < bs; ++u)
        mbar_wait(ab_full + (u & (kWdASlots - 1)), (u / kWdASlots) & 1, p.timeout_ns, p.status);
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issue
    // The whole warp runs the loop, so its warp-uniform slot indices and descriptors live in uniform registers;
    // one elected lane issues each tcgen05 instruction (and the commits, which track that lane's MMAs).
    uint32_t aslot = 0, aph = 0, bslot = 0, tc = 0;
    const uint64_t bdesc0 = sdesc_sw128(smem_u32(bring));
    bool ok = true;
    WD_PROF_T0(t_all);
    for (uint32_t n = 0; ok; ++n, ++tc) {
      const int i = wd_next_tile_warp(tq_full, tq_empty, tq, n, abrt, p);
      if (i < 0) break;
      const WdTile t = wd_tile(i, tpre, offs, E, RB);
      const uint32_t idesc = idesc_bf16_m128(max(16, (t.n + 15) & ~15));
      WD_PROF_T0(t_d);
      const uint32_t db = tc & 1, dcol = tmem + kWdDCol + db * kWdTok;
      // accumulator db was last used by tile tc - 2: its epilogue must have drained it
      const bool d_ok = tc < 2 || wd_wait(d_empty + db, ((tc >> 1) + 1) & 1, abrt, p);
      if (!__all_sync(0xffffffffu, d_ok)) break;
      if (lane == 0) WD_PROF_ADD(2, t_d);
      if (lane == 0) WD_PROF_INC(12);
      tc_fence_after();
      uint32_t acc = 0;
      for (int c = 0; c < nK; ++c) {
        WD_PROF_T0(t_a);
        const bool a_ok = __all_sync(0xffffffffu, wd_wait(ab_full + aslot, aph, abrt, p));
        if (lane == 0) WD_PROF_ADD(0, t_a);
        if (lane == 0) WD_PROF_INC(11);
        if (!a_ok) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t ta = tmem + aslot * 32;
        const uint64_t bd = bdesc0 + (uint64_t)(bslot * (kWdBBytes >> 4));
        if (elect_one()) {
          tc_mma_ts(dcol, ta, bd, idesc, acc);
          tc_mma_ts(dcol, ta + 8, bd + 2, idesc, 1u);
          tc_mma_ts(dcol, ta + 16, bd + 4, idesc, 1u);
          tc_mma_ts(dcol, ta + 24, bd + 6, idesc, 1u);
          tc_commit(ab_empty + aslot);
        }
        __syncwarp();
        acc = 1u;
        aslot = (aslot + 1) & (kWdASlots - 1);
        aph ^= (aslot == 0);
        bslot = bslot + 1 == (uint32_t)kWdBSt ? 0u : bslot + 1;
      }
      if (ok && elect_one()) tc_commit(d_full + db);
      __syncwarp();
    }
    if (lane == 0) WD_PROF_ADD(3, t_all);
    if (elect_one()) tc_commit(drain);  // every MMA issued has completed once this arrives
    __syncwarp();
    mbar_wait(drain, 0, p.timeout_ns, p.status);
  } else if (warp >= 4 && warp < kWdEpiWarp0) {
    // ---------------------------------------------------------------- dequantise into tensor memory
    const int grp = (warp - 4) >> 2, wq = warp & 3, row = 32 * wq + lane;
    const uint32_t tlane = (uint32_t)(32 * wq) << 16;
    uint32_t gc = 0;
    bool ok = true;
    WD_PROF_T0(t_all);
    for (uint32_t n = 0; ok; ++n) {
      if (wd_next_tile_warp(tq_full, tq_empty, tq, n, abrt, p) < 0) break;
      for (int c = 0; c < nK; ++c, ++gc) {
        if ((int)(gc % kWdDq) != grp) continue;
        const uint32_t st = gc >> 2, wslot = st & (kWdWSt - 1), aslot = gc & (kWdASlots - 1);
        WD_PROF_T0(t_w);
        bool good = wd_wait(w_full + wslot, (st / kWdWSt) & 1, abrt, p);
        if (warp == 4 && lane == 0) WD_PROF_ADD(4, t_w);
        WD_PROF_T0(t_a);
        if (good && gc >= (uint32_t)kWdASlots) good = wd_wait(ab_empty + aslot, ((gc / kWdASlots) + 1) & 1, abrt, p);
        if (warp == 4 && lane == 0) WD_PROF_ADD(5, t_a);
        if (!__all_sync(0xffffffffu, good)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint8_t* ch = wring + (size_t)wslot * kWdStage + (gc & 3) * kWdChunk;
        const uint4 h0 = *reinterpret_cast<const uint4*>(ch + row * 16);
        const uint4 h1 = *reinterpret_cast<const uint4*>(ch + 2048 + row * 16);
        const uint32_t sc = *reinterpret_cast<const uint32_t*>(ch + 4096 + row * 4);
        __syncwarp();
        if (lane == 0) mbar_arrive(w_empty + wslot);
        uint32_t r[32];
        dequant_row64(h0, h1, sc, r);
        WD_PROF_T0(t_s);
        tc_st_x32(tmem + tlane + aslot * 32, r);
        tc_wait_st();
        if (warp == 4 && lane == 0) WD_PROF_ADD(7, t_s);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(ab_full + aslot);
      }
    }
    if (warp == 4 && lane == 0) WD_PROF_ADD(6, t_all);
  } else if (warp >= kWdEpiWarp0) {
    // ---------------------------------------------------------------- epilogue: 8 warps, lane quarter x column half
    const int ew = warp - kWdEpiWarp0, wq = warp & 3, chalf = ew >> 2;
    const uint32_t tlane = (uint32_t)(32 * wq) << 16;
    int* ctok = reinterpret_cast<int*>(sm + kWdOffCol);        // [2][kWdTok]
    float* cwt = reinterpret_cast<float*>(ctok + 2 * kWdTok);   // [2][kWdTok]
    uint32_t tc = 0;
    WD_PROF_T0(t_all);
    for (uint32_t n = 0;; ++n, ++tc) {
      const int i = wd_next_tile_warp(tq_full, tq_empty, tq, n, abrt, p);
      if (i < 0) break;
      const WdTile t = wd_tile(i, tpre, offs, E, RB);
      const float gsc = p.gs[t.e] * kTwo52;  // loaded while the MMAs run
      if (p.fuse) {
        // the tile's tokens and route weights (buffer tc & 1: a warp one tile ahead fills the other buffer; the
        // barrier below keeps any warp from running two tiles ahead)
        for (int c = 32 * ew + lane; c < t.n; c += 32 * kWdEpiWarps) {
          const int f = p.order[t.q0 + c];
          ctok[(tc & 1) * kWdTok + c] = f / p.k;
          cwt[(tc & 1) * kWdTok + c] = p.wts[f] * gsc;
        }
      }
      WD_PROF_T0(t_d);
      const uint32_t db = tc & 1;
      const bool good = wd_wait(d_full + db, (tc >> 1) & 1, abrt, p);
      if (ew == 0 && lane == 0) WD_PROF_ADD(8, t_d);
      __syncwarp();
      (void)good;
      named_bar(1, 32 * kWdEpiWarps);  // the epilogue warps leave together when any of them gave up
      if (*abrt) break;
      tc_fence_after();
      const int cend = min(t.n, kWdEpiHalf * (chalf + 1));
      for (int c0 = kWdEpiHalf * chalf; c0 < cend; c0 += 32) {
        uint32_t v[32];
        WD_PROF_T0(t_l);
        tc_ld_x32(tmem + tlane + kWdDCol + db * kWdTok + c0, v);
        tc_wait_ld();
        if (ew == 0 && lane == 0) WD_PROF_ADD(14, t_l);
        WD_PROF_T0(t_m);
        if (p.mode == 0) {
          // rows: lanes 0-31 gate / 32-63 up (features 64rb..+31), 64-95 gate / 96-127 up (features +32..+63)
          const int pair = wq >> 1, isup = wq & 1;
          float* xg = xbuf + (2 * chalf + pair) * (2 * 32 * 17);  // gate values of tokens c0+16..c0+31
          float* xu = xg + 32 * 17;                               // up values of tokens c0..c0+15
          if (!isup) {
#pragma unroll
            for (int j = 0; j < 16; ++j) xg[lane * 17 + j] = __uint_as_float(v[16 + j]);
          } else {
#pragma unroll
            for (int j = 0; j < 16; ++j) xu[lane * 17 + j] = __uint_as_float(v[j]);
          }
          named_bar(2 + 2 * chalf + pair, 64);
          const int f = 64 * t.rb + 32 * pair + lane;
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int n = c0 + (isup ? 16 : 0) + j;
            if (n < t.n) {
              const float g = (isup ? xg[lane * 17 + j] : __uint_as_float(v[j])) * gsc;
              const float u = (isup ? __uint_as_float(v[16 + j]) : xu[lane * 17 + j]) * gsc;
              const float h = __fdividef(g, 1.f + __expf(-g)) * u;  // SiLU(g) * u
              p.inter[(size_t)(t.q0 + n) * p.I + f] = f2bf(h);
            }
          }
          named_bar(2 + 2 * chalf + pair, 64);
        } else if (p.fuse) {
          // weighted combine fused into the down projection: each column's token gets w * y for this warp's 32
          // rows (one coalesced 128-byte reduction per column; the order of the k additions is not fixed)
          const int h = 128 * t.rb + 32 * wq + lane;
          const int* tk = ctok + (tc & 1) * kWdTok;
          const float* wk = cwt + (tc & 1) * kWdTok;
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int n = c0 + j;
            if (n < t.n) atomicAdd(p.out32 + (size_t)tk[n] * p.H + h, __uint_as_float(v[j]) * wk[n]);
          }
        } else {
          const int h = 128 * t.rb + 32 * wq + lane;
          const float sc = gsc * (p.post_norm ? 1.f + bf2f(p.normw[h]) : 1.f);
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int n = c0 + j;
            if (n < t.n) {
              const float yv = __uint_as_float(v[j]) * sc;
              p.y[(size_t)(t.q0 + n) * p.H + h] = yv;
              if (p.post_norm) {
                float sq = yv * yv;
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
                if (lane == 0) atomicAdd(p.ss + t.q0 + n, sq);
              }
            }
          }
        }
        if (ew == 0 && lane == 0) WD_PROF_ADD(15, t_m);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(d_empty + db);
    }
    if (ew == 0 && lane == 0) WD_PROF_ADD(9, t_all);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
  // the last CTA to finish returns the tile counter and its own count to zero for the next launch
  if (tid == 0) {
    __threadfence();
    if (atomicAdd(p.tilectl + 1, 1) == (int)gridDim.x - 1) {
      p.tilectl[0] = 0;
      p.tilectl[1] = 0;
      __threadfence();
    }
  }
}

// ------------------------------------------------------------------------------------------------ gather / combine
__global__ void gather_kernel(const uint16_t* __restrict__ x, const int* __restrict__ order, const int* ctl, int k,
                              int H, uint16_t* __restrict__ xp, float* __restrict__ zero, size_t nzero4) {
  const int nroutes = ctl[kCtlRoutes];
  const int nwarps = (gridDim.x * blockDim.x) >> 5;
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  const int nv = H / 8;
  for (int q = gw; q < nroutes; q += nwarps) {
    const uint4* src = reinterpret_cast<const uint4*>(x + (size_t)(order[q] / k) * H);
    uint4* dst = reinterpret_cast<uint4*>(xp + (size_t)q * H);
    for (int v = lane; v < nv; v += 32) dst[v] = __ldg(src + v);
  }
  // the fused combine's fp32 accumulator starts at zero
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < nzero4; i += (size_t)gridDim.x * blockDim.x)
    reinterpret_cast<float4*>(zero)[i] = make_float4(0.f, 0.f, 0.f, 0.f);
}

// out = bf16(out32), 4 values per thread (the end of the fused combine)
__global__ void to_bf16_kernel(const float* __restrict__ out32, size_t n4, uint16_t* __restrict__ out) {
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (size_t)gridDim.x * blockDim.x) {
    const float4 a = __ldcs(reinterpret_cast<const float4*>(out32) + i);
    uint2 o;
    o.x = (uint32_t)f2bf(a.x) | ((uint32_t)f2bf(a.y) << 16);
    o.y = (uint32_t)f2bf(a.z) | ((uint32_t)f2bf(a.w) << 16);
    reinterpret_cast<uint2*>(out)[i] = o;
  }
}

__global__ void combine_kernel(const float* __restrict__ y, const float* __restrict__ wts, const int* __restrict__ pos,
                               const float* __restrict__ ss, int T, int k, int H, int post_norm,
                               uint16_t* __restrict__ out) {
  const int per_row = H / 4;
  const size_t total = (size_t)T * per_row;
  for (size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += (size_t)gridDim.x * blockDim.x) {
    const int t = (int)(idx / per_row), col = (int)(idx % per_row) * 4;
    float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
    for (int s = 0; s < k; ++s) {
      const int q = pos[t * k + s];
      if (q >= 0) {
        float r = wts[t * k + s];
        if (post_norm) r *= rsqrtf(ss[q] / (float)H + 1e-8f);
        const float4 yv = __ldcs(reinterpret_cast<const float4*>(y + (size_t)q * H + col));
        a0 += r * yv.x;
        a1 += r * yv.y;
        a2 += r * yv.z;
        a3 += r * yv.w;
      }
    }
    uint2 o;
    o.x = (uint32_t)f2bf(a0) | ((uint32_t)f2bf(a1) << 16);
    o.y = (uint32_t)f2bf(a2) | ((uint32_t)f2bf(a3) << 16);
    *reinterpret_cast<uint2*>(out + (size_t)t * H + col) = o;
  }
}

// ------------------------------------------------------------------------------------------------ host side
namespace {
std::mutex g_encode_mu;
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

bool encode_2d(CUtensorMap* tm, const void* base, int rows, int cols, int box_cols, int box_rows, bool f32,
               bool swizzle) {
  {
    std::lock_guard<std::mutex> lock(g_encode_mu);
    if (!g_encode) {
      void* fn = nullptr;
      cudaDriverEntryPointQueryResult q;
      if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault, &q) != cudaSuccess ||
          q != cudaDriverEntryPointSuccess || !fn)
        return false;
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
  }
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)cols * (f32 ? 4 : 2)};
  const cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return g_encode(tm, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                  const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int launch_wide_gemm(const WideParams& p, const void* b_rows, int rows, int cols, int sms, cudaStream_t stream) {
  WdMaps maps;
  if (!encode_2d(&maps.m64, b_rows, rows, cols, 64, 64, false, true) ||
      !encode_2d(&maps.m128, b_rows, rows, cols, 64, 128, false, true) ||
      !encode_2d(&maps.m256, b_rows, rows, cols, 64, 256, false, true))
    return XCB_ERR_CUDA;
  wide_kernel<<<sms, kWdThreads, kWdSmem, stream>>>(p, maps);
  return cudaGetLastError() == cudaSuccess ? XCB_OK : XCB_ERR_CUDA;
}
}  // namespace

size_t wide_smem_bytes() { return kWdSmem; }

#if XCB_WD_PROFILE
extern "C" int xcb_wide_profile_read(void* host, size_t bytes) {
  return cudaMemcpyFromSymbol(host, g_wd_prof, bytes) == cudaSuccess ? 0 : 4;
}
extern "C" int xcb_wide_profile_clear() {
  static unsigned long long zero[1024 * kWdProfSlots];
  return cudaMemcpyToSymbol(g_wd_prof, zero, sizeof(zero)) == cudaSuccess ? 0 : 4;
}
#endif

int launch_wide_path(const WidePathParams& a, cudaStream_t stream) {
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return XCB_ERR_CUDA;
  if (cudaFuncSetAttribute(wide_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kWdSmem) != cudaSuccess)
    return XCB_ERR_CUDA;
  const int R = a.T * a.k;
  const size_t n4 = (size_t)a.T * a.H / 4;
  gather_kernel<<<sms * 4, 256, 0, stream>>>(a.x, a.order, a.ctl, a.k, a.H, a.xperm, a.fuse ? a.out32 : nullptr,
                                              a.fuse ? n4 : 0);
  if (cudaGetLastError() != cudaSuccess) return XCB_ERR_CUDA;

  WideParams g{};
  g.offsets = a.offsets;
  g.E_loc = a.E_loc;
  g.I = a.I;
  g.H = a.H;
  g.status = a.ctl + kCtlStatus;
  g.tilectl = a.ctl + kCtlWideTile;
  g.timeout_ns = a.timeout_ns;
  g.normw = a.normw;
  g.post_norm = a.post_norm;
  g.inter = a.inter;
  g.y = a.y;
  g.ss = a.ss;
  g.order = a.order;
  g.wts = a.wts;
  g.out32 = a.out32;
  g.k = a.k;

  g.w = a.wA;
  g.gs = a.gsA;
  g.R = 2 * a.I;
  g.K = a.H;
  g.mode = 0;
  int rc = launch_wide_gemm(g, a.xperm, R, a.H, sms, stream);
  if (rc != XCB_OK) return rc;

  g.w = a.wB;
  g.gs = a.gsB;
  g.R = a.H;
  g.K = a.I;
  g.mode = 1;
  g.fuse = a.fuse;
  rc = launch_wide_gemm(g, a.inter, R, a.I, sms, stream);
  if (rc != XCB_OK) return rc;

  if (a.fuse)
    to_bf16_kernel<<<sms * 8, 256, 0, stream>>>(a.out32, n4, a.out);
  else
    combine_kernel<<<sms * 8, 256, 0, stream>>>(a.y, a.wts, a.pos, a.ss, a.T, a.k, a.H, a.post_norm, a.out);
  return cudaGetLastError() == cudaSuccess ? XCB_OK : XCB_ERR_CUDA;
}

}  // namespace xcb
