// extern "C" boundary (include/xcb_moe.h): argument validation, workspace carving, launch sequencing.
#include <string.h>

#include <mutex>

#include "common.cuh"
#include "workspace.cuh"

#include "kernels.cuh"

using namespace xcb;

namespace {
constexpr unsigned long long kTimeoutNs = 2000000000ull;  // 2 s per bounded wait unless the call sets its own

bool aligned16(const void* p) { return ((uintptr_t)p & 15u) == 0; }

int shape_ok(const XcbMoeShape* s) {
  if (!s) return XCB_ERR_INVALID_ARG;
  if (s->num_experts <= 0 || s->total_experts <= 0 || s->hidden <= 0 || s->inter <= 0 || s->expert_offset < 0)
    return XCB_ERR_INVALID_ARG;
  if (s->expert_offset + s->num_experts > s->total_experts) return XCB_ERR_INVALID_ARG;
  if (s->hidden % 256 || s->inter % 256) return XCB_ERR_UNSUPPORTED;
  if (s->total_experts > 512 || s->num_experts > 512) return XCB_ERR_UNSUPPORTED;
  if (wide_smem_bytes() > 227 * 1024) return XCB_ERR_UNSUPPORTED;
  return XCB_OK;
}
}  // namespace

extern "C" {

const char* xcb_status_str(int code) {
  switch (code) {
    case XCB_OK: return "ok";
    case XCB_ERR_INVALID_ARG: return "invalid argument";
    case XCB_ERR_UNSUPPORTED: return "unsupported shape";
    case XCB_ERR_WORKSPACE: return "workspace too small";
    case XCB_ERR_CUDA: return "CUDA error";
    case XCB_ERR_DEVICE: return "device status bits set";
    default: return "unknown status";
  }
}

int xcb_moe_check_shape(const XcbMoeShape* shape) { return shape_ok(shape); }

size_t xcb_moe_packed_bytes(const XcbMoeShape* s, int which) {
  if (shape_ok(s) != XCB_OK) return 0;
  const size_t E = (size_t)s->num_experts, H = (size_t)s->hidden, I = (size_t)s->inter;
  // decode-path layout followed by the prefill-path layout, equal sizes
  return 2 * (which == 0 ? E * (2 * I / 16) * 9 * H : E * (H / 16) * 9 * I);
}

int xcb_moe_pack_weights(const XcbMoeShape* s, const uint8_t* w13, const uint8_t* w13_sf, const uint8_t* w2,
                         const uint8_t* w2_sf, const uint32_t* xor_tables, void* gate_up_out, void* down_out,
                         int32_t* status, cudaStream_t stream) {
  int rc = shape_ok(s);
  if (rc != XCB_OK) return rc;
  if (!w13 || !w13_sf || !w2 || !w2_sf || !xor_tables || !gate_up_out || !down_out || !status)
    return XCB_ERR_INVALID_ARG;
  if (!aligned16(gate_up_out) || !aligned16(down_out)) return XCB_ERR_INVALID_ARG;
  PackParams a{w13, w13_sf, (uint8_t*)gate_up_out, xor_tables, status, s->num_experts, 2 * s->inter, s->hidden, 1};
  rc = launch_pack(a, stream);
  if (rc != XCB_OK) return rc;
  PackParams b{w2, w2_sf, (uint8_t*)down_out, xor_tables, status, s->num_experts, s->hidden, s->inter, 0};
  return launch_pack(b, stream);
}

size_t xcb_moe_workspace_bytes(const XcbMoeShape* s, int32_t max_tokens, int32_t top_k) {
  if (shape_ok(s) != XCB_OK || max_tokens < 0 || top_k <= 0) return 0;
  return ws_layout(s->num_experts, s->hidden, s->inter, max_tokens, top_k).total;
}

int xcb_moe_workspace_offsets(const XcbMoeShape* s, int32_t max_tokens, int32_t top_k, size_t* out, int n) {
  if (shape_ok(s) != XCB_OK || max_tokens < 0 || top_k <= 0 || !out || n < 6) return -1;
  const WsLayout L = ws_layout(s->num_experts, s->hidden, s->inter, max_tokens, top_k);
  out[0] = L.ids;
  out[1] = L.wts;
  out[2] = L.pos;
  out[3] = L.order;
  out[4] = L.counts;
  out[5] = L.offsets;
  return 6;
}

int xcb_moe_workspace_init(void* ws, size_t bytes, int32_t max_tokens, int32_t top_k, cudaStream_t stream) {
  (void)max_tokens;
  (void)top_k;
  if (!ws) return XCB_ERR_INVALID_ARG;
  return cudaMemsetAsync(ws, 0, bytes, stream) == cudaSuccess ? XCB_OK : XCB_ERR_CUDA;
}

namespace {
// Routes per call from which xcb_moe_forward takes the prefill path (tensor-core grouped GEMMs) instead of the
// decode kernel, unless a XCB_FLAG_*_PATH flag forces one.
constexpr long long kPrefillMinRoutes = kSmallRoutes + 1;
constexpr long long kShardDecodeMaxRoutes = 192;  // expected held routes up to which a shard stays on the decode path
// A layer holding every expert stays on the decode path up to this many routes per expert on average: its weight
// stream then beats the tensor-core path's dequantisation (DeepSeek-V3 shape: 48 tokens 1.22 against 1.75 ms,
// 64 tokens 1.57 against 2.01 ms, 96 tokens 2.12 against 2.16 ms, 128 tokens 2.74 against 2.26 ms).
constexpr long long kDecodeMaxRoutesPerExpert = 3;

struct CallPlan {
  RouteParams rp;
  SkinnyParams sp;
  WidePathParams wp;
  bool wide;
};

// Validate a forward call, pick its path and carve its workspace; shared by route / experts / forward.
int prepare_call(const XcbMoeWeights* w, const XcbMoeArgs* a, void* ws, size_t ws_bytes, CallPlan* plan) {
  if (!w || !a || !ws) return XCB_ERR_INVALID_ARG;
  RouteParams* rp = &plan->rp;
  SkinnyParams* sp = &plan->sp;
  const XcbMoeShape* s = &w->shape;
  int rc = shape_ok(s);
  if (rc != XCB_OK) return rc;
  if (a->tokens < 0 || a->top_k <= 0 || a->top_k > 16 || a->top_k > s->total_experts) return XCB_ERR_INVALID_ARG;
  if (a->wait_limit_us < 0) return XCB_ERR_INVALID_ARG;
  if (a->tokens == 0) return XCB_OK;
  const unsigned long long timeout_ns = a->wait_limit_us ? (unsigned long long)a->wait_limit_us * 1000ull : kTimeoutNs;
  if (!a->hidden_states || !a->out || !w->gate_up || !w->down || !w->gate_up_gs || !w->down_gs)
    return XCB_ERR_INVALID_ARG;
  const bool have_logits = a->router_logits != nullptr;
  const bool have_ids = a->topk_ids != nullptr && a->topk_weights != nullptr;
  if (have_logits == have_ids) return XCB_ERR_INVALID_ARG;
  const bool post_norm = (a->flags & XCB_FLAG_POST_NORM) != 0;
  if (post_norm && !w->post_norm_w) return XCB_ERR_INVALID_ARG;
  if (a->flags &
      ~(XCB_FLAG_POST_NORM | XCB_FLAG_DECODE_PATH | XCB_FLAG_PREFILL_PATH | XCB_FLAG_PDL | XCB_FLAG_DETERMINISTIC))
    return XCB_ERR_INVALID_ARG;
  if ((a->flags & XCB_FLAG_DECODE_PATH) && (a->flags & XCB_FLAG_PREFILL_PATH)) return XCB_ERR_INVALID_ARG;
  if (!aligned16(a->hidden_states) || !aligned16(a->out) || !aligned16(w->gate_up) || !aligned16(w->down) ||
      !aligned16(ws))
    return XCB_ERR_INVALID_ARG;
  const WsLayout L = ws_layout(s->num_experts, s->hidden, s->inter, a->tokens, a->top_k);
  if (ws_bytes < L.total) return XCB_ERR_WORKSPACE;
  uint8_t* b = (uint8_t*)ws;
  const long long routes = (long long)a->tokens * a->top_k;
  // A layer that holds only some of the router's experts (an expert-parallel shard, the reference's local range)
  // sees about routes * held / total of them: the decode kernel streams each held expert once per job of up to 8
  // tokens, and stays ahead of the tensor-core path up to ~192 such routes (measured at the reference's shape:
  // 128 tokens x top-8 over 32 of 256 experts 280 us against 359 us; 256 tokens 384 against 369 us).
  const bool shard = s->num_experts < s->total_experts;
  const long long est_local = routes * s->num_experts / s->total_experts;
  plan->wide = (a->flags & XCB_FLAG_PREFILL_PATH) ||
               (!(a->flags & XCB_FLAG_DECODE_PATH) &&
                (shard ? est_local > kShardDecodeMaxRoutes
                       : ((routes >= kPrefillMinRoutes || a->tokens > kSmallTokens) &&
                          routes > kDecodeMaxRoutesPerExpert * s->total_experts)));
  if (!plan->wide && !skinny_supported(s->hidden, s->inter)) {
    // no stage plan of the decode kernel fits this shape: the tensor-core path serves every batch size
    if (a->flags & XCB_FLAG_DECODE_PATH) return XCB_ERR_UNSUPPORTED;
    plan->wide = true;
  }

  rp->logits = a->router_logits;
  rp->ids_in = a->topk_ids;
  rp->wts_in = a->topk_weights;
  rp->T = a->tokens;
  rp->k = a->top_k;
  rp->E_tot = s->total_experts;
  rp->lo = s->expert_offset;
  rp->E_loc = s->num_experts;
  rp->job_tokens = kJobTokens;  // the decode path sets its own width below
  rp->ctl = (int*)(b + L.ctl);
  rp->ids = (int*)(b + L.ids);
  rp->wts = (float*)(b + L.wts);
  rp->pos = (int*)(b + L.pos);
  rp->order = (int*)(b + L.order);
  rp->counts = (int*)(b + L.counts);
  rp->offsets = (int*)(b + L.offsets);
  rp->jobs = (int4*)(b + L.jobs);
  rp->doneA = (int*)(b + L.doneA);
  rp->ss = (float*)(b + L.ss);
  rp->hist = (int*)(b + L.hist);
  rp->ids_out = a->topk_ids_out;
  rp->wts_out = a->topk_weights_out;

  const bool small = !plan->wide && routes <= (long long)kSmallRoutes && a->tokens <= kSmallTokens;
  int* ctl = rp->ctl;
  *sp = SkinnyParams{};
  sp->wA = (const uint8_t*)w->gate_up;
  sp->wB = (const uint8_t*)w->down;
  sp->gsA = w->gate_up_gs;
  sp->gsB = w->down_gs;
  sp->normw = w->post_norm_w;
  sp->x = a->hidden_states;
  sp->order = rp->order;
  sp->wts = rp->wts;
  sp->pos = rp->pos;
  sp->jobs = rp->jobs;
  sp->small_route = small ? 1 : 0;
  sp->logits = a->router_logits;
  sp->ids_in = a->topk_ids;
  sp->wts_in = a->topk_weights;
  sp->E_tot = s->total_experts;
  sp->lo = s->expert_offset;
  sp->E_loc = s->num_experts;
  sp->g_ids = rp->ids;
  sp->g_wts = rp->wts;
  sp->g_pos = rp->pos;
  sp->g_order = rp->order;
  sp->g_counts = rp->counts;
  sp->g_offsets = rp->offsets;
  sp->ids_out = a->topk_ids_out;
  sp->wts_out = a->topk_weights_out;
  sp->ctl = ctl;
  sp->doneA = small ? ctl + kCtlDoneA : rp->doneA;
  sp->rbcnt = ctl + kCtlRowBlock;
  sp->inter = (uint16_t*)(b + L.inter);
  sp->y = (float*)(b + L.y);
  sp->ss = small ? (float*)(ctl + kCtlSS) : rp->ss;
  sp->out = a->out;
  sp->T = a->tokens;
  sp->k = a->top_k;
  sp->H = s->hidden;
  sp->I = s->inter;
  {
    // with precomputed ids one expert may repeat within a token, so a job can hold up to T*k tokens
    const long long per_job = have_logits ? a->tokens : (long long)a->tokens * a->top_k;
    sp->job_tokens = (int)(per_job < kJobTokens ? per_job : kJobTokens);
    // jobs may be cut finer, so that the shared-memory plan keeps its large stages and two activation buffers
    const int per_expert = (int)((routes + s->total_experts - 1) / s->total_experts);  // expected routes per expert
    sp->job_tokens = skinny_job_cap(s->hidden, s->inter, sp->job_tokens, small ? (int)routes : 0, per_expert);
    if (small && a->tokens == 2 && skinny_two_one_token_jobs(s->hidden, s->inter, (int)routes)) sp->job_tokens = 1;
    if (!plan->wide) rp->job_tokens = sp->job_tokens;  // the separate router cuts the jobs at the same width
  }
  sp->post_norm = post_norm ? 1 : 0;
  sp->grid_combine = (post_norm || !small) ? 1 : 0;
  // programmatic dependent launch for the single-launch decode step (a step that runs the router first keeps
  // plain stream order: its router kernel is what the experts kernel waits for)
  sp->pdl = (a->flags & XCB_FLAG_PDL) && small ? 1 : 0;
  sp->timeout_ns = timeout_ns;

  WidePathParams* wp = &plan->wp;
  *wp = WidePathParams{};
  const size_t E = (size_t)s->num_experts, H = (size_t)s->hidden, I = (size_t)s->inter;
  wp->x = a->hidden_states;
  wp->order = rp->order;
  wp->pos = rp->pos;
  wp->wts = rp->wts;
  wp->offsets = rp->offsets;
  wp->ctl = ctl;
  wp->wA = (const uint8_t*)w->gate_up + E * (2 * I / 16) * 9 * H;  // prefill layout after the decode layout
  wp->wB = (const uint8_t*)w->down + E * (H / 16) * 9 * I;
  wp->gsA = w->gate_up_gs;
  wp->gsB = w->down_gs;
  wp->normw = w->post_norm_w;
  wp->xperm = (uint16_t*)(b + L.y);  // gathered rows live in the y region: read by the gate_up GEMM before y is written
  wp->inter = sp->inter;
  wp->y = sp->y;
  // the down projection adds w * y straight into a fp32 [T, H] accumulator (after the gathered rows in the y region,
  // which holds R*H*4 bytes: room for T*H*4 more when k >= 2); the post-norm needs every y row whole first, and
  // XCB_FLAG_DETERMINISTIC asks for the fixed-order combine pass
  wp->fuse = (!post_norm && a->top_k >= 2 && !(a->flags & XCB_FLAG_DETERMINISTIC)) ? 1 : 0;
  wp->out32 = (float*)(b + L.y + (size_t)a->tokens * a->top_k * s->hidden * 2);
  wp->ss = rp->ss;
  wp->out = a->out;
  wp->T = a->tokens;
  wp->k = a->top_k;
  wp->H = s->hidden;
  wp->I = s->inter;
  wp->E_loc = s->num_experts;
  wp->post_norm = post_norm ? 1 : 0;
  wp->timeout_ns = timeout_ns;
  return XCB_OK;
}

int run_experts(const CallPlan& plan, cudaStream_t stream) {
  return plan.wide ? launch_wide_path(plan.wp, stream) : launch_skinny(plan.sp, stream);
}
}  // namespace

// The planner of a forward call (prepare_call, unchanged), run on placeholder pointers: it only checks them for
// null and alignment, and nothing here reads or launches anything.
int xcb_moe_plan_info(const XcbMoeShape* shape, int32_t tokens, int32_t top_k, int32_t flags, int32_t given_routes,
                      int32_t* out, int32_t n) {
  if (!shape || !out || n <= 0 || tokens <= 0) return XCB_ERR_INVALID_ARG;
  int rc = shape_ok(shape);
  if (rc != XCB_OK) return rc;
  const uintptr_t fake = 256;  // 16-byte aligned, never dereferenced
  XcbMoeWeights w{};
  w.shape = *shape;
  w.gate_up = w.down = (const void*)fake;
  w.gate_up_gs = w.down_gs = (const float*)fake;
  w.post_norm_w = (flags & XCB_FLAG_POST_NORM) ? (const uint16_t*)fake : nullptr;
  XcbMoeArgs a{};
  a.tokens = tokens;
  a.top_k = top_k;
  a.flags = flags & ~XCB_FLAG_PDL;
  a.hidden_states = (const uint16_t*)fake;
  a.out = (uint16_t*)fake;
  if (given_routes) {
    a.topk_ids = (const int32_t*)fake;
    a.topk_weights = (const float*)fake;
  } else {
    a.router_logits = (const float*)fake;
  }
  if (top_k <= 0 || top_k > 16) return XCB_ERR_INVALID_ARG;
  CallPlan plan;
  rc = prepare_call(&w, &a, (void*)fake, xcb_moe_workspace_bytes(shape, tokens, top_k), &plan);
  if (rc != XCB_OK) return rc;
  int v[8] = {plan.wide ? 1 : 0, 0, 0, 0, 0, 0, 0, 0};
  if (!plan.wide) {
    v[1] = plan.sp.small_route;
    v[2] = plan.sp.job_tokens;
    skinny_plan_fields(shape->hidden, shape->inter, plan.sp.job_tokens, plan.sp.small_route ? tokens * top_k : 0,
                       tokens, v + 3);
  }
  const int m = n < 8 ? n : 8;
  for (int i = 0; i < m; ++i) out[i] = v[i];
  return m;
}

int xcb_moe_route(const XcbMoeWeights* w, const XcbMoeArgs* a, void* ws, size_t ws_bytes, cudaStream_t stream) {
  CallPlan plan;
  int rc = prepare_call(w, a, ws, ws_bytes, &plan);
  if (rc != XCB_OK || a->tokens == 0) return rc;
  if (plan.sp.small_route) return XCB_OK;  // small batches are routed inside the experts kernel
  return launch_route(plan.rp, stream);
}

int xcb_moe_experts(const XcbMoeWeights* w, const XcbMoeArgs* a, void* ws, size_t ws_bytes, cudaStream_t stream) {
  CallPlan plan;
  int rc = prepare_call(w, a, ws, ws_bytes, &plan);
  if (rc != XCB_OK || a->tokens == 0) return rc;
  return run_experts(plan, stream);
}

int xcb_moe_forward(const XcbMoeWeights* w, const XcbMoeArgs* a, void* ws, size_t ws_bytes, cudaStream_t stream) {
  CallPlan plan;
  int rc = prepare_call(w, a, ws, ws_bytes, &plan);
  if (rc != XCB_OK || a->tokens == 0) return rc;
  if (!plan.sp.small_route) {
    rc = launch_route(plan.rp, stream);
    if (rc != XCB_OK) return rc;
  }
  return run_experts(plan, stream);
}

// ------------------------------------------------------------------------------------------------ allocation-free
// Scratch for xcb_moe_forward_static: a file-scope device array, so callers that may not allocate device memory
// still get a workspace.  Every GPU that loads this library reserves it until the process exits.
static __device__ __align__(256) unsigned char g_static_scratch[XCB_STATIC_SCRATCH_BYTES];

namespace {
std::mutex g_static_mu;
constexpr int kMaxDevices = 128;
void* g_static_ptr[kMaxDevices] = {};

// Device address of g_static_scratch on the current device.  In host code the array's name is only a host-side
// stand-in, so the address is looked up once per device (with that device current) and cached.
int static_scratch_address(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return XCB_ERR_CUDA;
  std::lock_guard<std::mutex> lock(g_static_mu);
  if (!g_static_ptr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_static_scratch) != cudaSuccess || !p) return XCB_ERR_CUDA;
    g_static_ptr[dev] = p;
  }
  *out = g_static_ptr[dev];
  return XCB_OK;
}
}  // namespace

int xcb_moe_forward_static(const XcbMoeWeights* w, const XcbMoeArgs* a, cudaStream_t stream) {
  if (!w || !a) return XCB_ERR_INVALID_ARG;
  int rc = shape_ok(&w->shape);
  if (rc != XCB_OK) return rc;
  if (a->tokens < 0 || a->top_k <= 0) return XCB_ERR_INVALID_ARG;
  if (a->tokens == 0) return XCB_OK;
  const WsLayout L = ws_layout(w->shape.num_experts, w->shape.hidden, w->shape.inter, a->tokens, a->top_k);
  if (L.total > (size_t)XCB_STATIC_SCRATCH_BYTES) return XCB_ERR_WORKSPACE;  // call too large for the fixed scratch
  void* ws = nullptr;
  rc = static_scratch_address(&ws);
  if (rc != XCB_OK) return rc;
  // The array keeps the previous call's contents: clear the control words (counters) that the kernels expect to
  // start at zero; every other region is rewritten by the call before it is read.  Word 0, the status bits, is
  // kept, so device errors of earlier calls accumulate until xcb_moe_static_read_status reads and clears them.
  if (cudaMemsetAsync((int*)ws + 1, 0, (kCtlWords - 1) * sizeof(int), stream) != cudaSuccess) return XCB_ERR_CUDA;
  return xcb_moe_forward(w, a, ws, (size_t)XCB_STATIC_SCRATCH_BYTES, stream);
}

int xcb_moe_static_read_status(int32_t* device_status, cudaStream_t stream) {
  if (!device_status) return XCB_ERR_INVALID_ARG;
  void* ws = nullptr;
  const int rc = static_scratch_address(&ws);
  if (rc != XCB_OK) return rc;
  return xcb_moe_read_status(ws, device_status, stream);
}

int xcb_moe_read_status(void* ws, int32_t* device_status, cudaStream_t stream) {
  if (!ws || !device_status) return XCB_ERR_INVALID_ARG;
  int v = 0;
  if (cudaMemcpyAsync(&v, ws, sizeof(int), cudaMemcpyDeviceToHost, stream) != cudaSuccess) return XCB_ERR_CUDA;
  if (cudaStreamSynchronize(stream) != cudaSuccess) return XCB_ERR_CUDA;
  *device_status = v;
  if (v) {
    if (cudaMemsetAsync(ws, 0, sizeof(int), stream) != cudaSuccess) return XCB_ERR_CUDA;
    if (cudaStreamSynchronize(stream) != cudaSuccess) return XCB_ERR_CUDA;
    return XCB_ERR_DEVICE;
  }
  return XCB_OK;
}

int xcb_nvfp4_quantize(const float* w, int32_t E, int32_t R, int32_t K, uint8_t* codes, uint8_t* sf, float* gs,
                       float* amax_scratch, cudaStream_t stream) {
  if (!w || !codes || !sf || !gs || !amax_scratch || E <= 0 || R <= 0 || K <= 0 || K % 16) return XCB_ERR_INVALID_ARG;
  if (!aligned16(w)) return XCB_ERR_INVALID_ARG;
  QuantParams q{w, E, R, K, codes, sf, gs, amax_scratch};
  return launch_quantize(q, stream);
}

}  // extern "C"
