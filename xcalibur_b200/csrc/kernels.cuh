// Parameter blocks and launchers of the kernels behind the C-ABI (one definition, shared by all translation units).
#pragma once
#include <stddef.h>
#include <stdint.h>
#include <cuda_runtime.h>

namespace xcb {

struct RouteParams {
  const float* logits;     // [T, E_tot] or null
  const int* ids_in;       // [T, k] or null
  const float* wts_in;     // [T, k] or null
  int T, k, E_tot, lo, E_loc;
  int job_tokens;           // decode-path jobs hold at most this many routes (1..kJobTokens)
  int* ctl;
  int* ids;
  float* wts;
  int* pos;
  int* order;
  int* counts;
  int* offsets;
  int4* jobs;
  int* doneA;              // per-job phase-A counters, zeroed here for the kernel that follows
  float* ss;
  int* hist;               // [chunks][E_loc] per-chunk expert histograms, then chunk bases (many-token router)
  int* ids_out;
  float* wts_out;
};

struct SkinnyParams {
  const uint8_t* wA;      // packed gate_up units
  const uint8_t* wB;      // packed down units
  const float* gsA;
  const float* gsB;
  const uint16_t* normw;  // bf16 [H] or null
  const uint16_t* x;      // bf16 [T, H]
  // routing produced by route_kernel (small_route == 0)
  const int* order;       // permuted position -> flat route
  const float* wts;       // flat route weights
  const int* pos;         // flat route -> permuted position (-1: not local)
  const int4* jobs;       // (expert, p0, ntok, 0)
  // in-kernel routing (small_route == 1): inputs, and where CTA 0 publishes the tables
  int small_route;
  const float* logits;
  const int* ids_in;
  const float* wts_in;
  int E_tot, lo, E_loc;
  int* g_ids;
  float* g_wts;
  int* g_pos;
  int* g_order;
  int* g_counts;
  int* g_offsets;
  int* ids_out;
  float* wts_out;
  int* ctl;
  int* doneA;             // per-job phase-A counters
  int* rbcnt;             // per-16-row-block phase-B counters
  uint16_t* inter;        // bf16 [routes, I]
  float* y;               // fp32 [routes, H]
  float* ss;              // fp32 [routes]
  uint16_t* out;          // bf16 [T, H]
  int T, k, H, I;
  int job_tokens;         // most tokens one job holds (sizes the activation staging; the in-kernel router's job split)
  int post_norm;
  int grid_combine;       // 1: grid barrier + distributed combine; 0: per-row-block combine by the CTA completing it
  int pdl;                // launched with programmatic dependent launch (griddepcontrol.wait before any read)
  unsigned long long timeout_ns;
};

struct PackParams {
  const uint8_t* codes;  // [E, R, K/2]
  const uint8_t* sf;     // [E, R, K/16]
  uint8_t* out;          // [E, R/16, 9K]
  const uint32_t* tabs;  // [4][256]
  int* status;
  int E, R, K;
  int gate_up;           // rows interleaved gate/up in 8-row groups
};

struct QuantParams {
  const float* w;
  int E, R, K;
  uint8_t* codes;
  uint8_t* sf;
  float* gs;
  float* amax;
};

// One prefill-path GEMM (wide_kernel): mode 0 = gate_up + SwiGLU -> inter, mode 1 = down -> y.
struct WideParams {
  const uint8_t* w;        // prefill-layout packed weights of this GEMM
  const float* gs;         // per-expert global scale
  const int* offsets;      // [E_loc + 1] first permuted route of each expert
  const uint16_t* normw;   // bf16 [H] (post-norm) or null
  uint16_t* inter;         // mode 0 output, bf16 [routes, I]
  float* y;                // mode 1 output, fp32 [routes, H]
  float* ss;               // mode 1 post-norm sums of squares [routes]
  // mode 1 fused with the weighted combine (fuse != 0): out32[token][h] += w_route * y instead of writing y
  const int* order;        // permuted position -> flat route (token = route / k)
  const float* wts;        // flat route weights
  float* out32;            // fp32 [T, H], zeroed before the launch
  int k, fuse;
  int* status;
  int* tilectl;            // [2] tiles claimed so far, CTAs finished (zero between launches)
  int E_loc, R, K, I, H;
  int mode, post_norm;
  unsigned long long timeout_ns;
};

// The whole prefill path after the router: gather, gate_up GEMM, down GEMM, combine.
struct WidePathParams {
  const uint16_t* x;
  const int* order;
  const int* pos;
  const float* wts;
  const int* offsets;
  int* ctl;
  const uint8_t* wA;       // prefill-layout regions of the packed buffers
  const uint8_t* wB;
  const float* gsA;
  const float* gsB;
  const uint16_t* normw;
  uint16_t* xperm;
  uint16_t* inter;
  float* y;
  float* ss;
  float* out32;            // fp32 [T, H] accumulator of the fused combine (fuse != 0)
  uint16_t* out;
  int T, k, H, I, E_loc, post_norm, fuse;
  unsigned long long timeout_ns;
};

int launch_route(const RouteParams& p, cudaStream_t stream);
int launch_wide_path(const WidePathParams& p, cudaStream_t stream);
size_t wide_smem_bytes();
size_t route_smem_bytes(int E_loc);
int launch_skinny(const SkinnyParams& p, cudaStream_t stream);
bool skinny_supported(int H, int I);  // the decode kernel has a stage plan for this shape
int skinny_job_cap(int H, int I, int want, int route_R, int min_rows);
bool skinny_two_one_token_jobs(int H, int I, int route_R);
// rows, buffers, stages, stage bytes and the two-token instantiation flag of the decode kernel's plan
void skinny_plan_fields(int H, int I, int job_tokens, int route_R, int T, int* out);
int launch_pack(const PackParams& p, cudaStream_t stream);
int launch_quantize(const QuantParams& p, cudaStream_t stream);

}  // namespace xcb
