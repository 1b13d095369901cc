/* C-ABI of the B200 (sm_100a) NVFP4-weight / BF16-activation mixture-of-experts layer.
 *
 * Drop-in for the native boundary of xCalibur's kernels/moe_w4a16_h200 operator.  The reference binds one pybind
 * entry point, okc_run(w, scratch, x, topk_ids, topk_weights, out, lo, nloc, grid) (moe_w4a16.py:2812, declared
 * at :3063-3068), builds its packed weights in Python in prepare() (moe_w4a16.py:3292-3351) and allocates its
 * scratch in _make_scratch() (moe_w4a16.py:3353-3367).  Here every argument is a plain device pointer plus sizes,
 * every call takes an explicit cudaStream_t, and the compute calls never allocate: the caller provides the packed
 * weight buffers and the workspace, sized by the *_bytes queries (the expert-parallel set-up call xcb_p2p_alloc
 * is the one call that allocates, once, the peer-exchange buffer).
 *
 * All calls return XCB_OK or an XCB_ERR_* code; argument and shape errors are detected on the host before any
 * launch.  Errors that only the device can see (a NaN block scale, an expert id out of range, a spin-wait that
 * ran out of time) set bits in a status word inside the workspace; xcb_moe_read_status() reads and clears it.
 */
#ifndef XCB_MOE_H_
#define XCB_MOE_H_

#include <stddef.h>
#include <stdint.h>
#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- return codes ---- */
#define XCB_OK 0
#define XCB_ERR_INVALID_ARG 1       /* null pointer, negative size, misaligned pointer, bad flag     */
#define XCB_ERR_UNSUPPORTED 2       /* shape outside what the kernels support (see xcb_moe_check_shape) */
#define XCB_ERR_WORKSPACE 3         /* workspace smaller than xcb_moe_workspace_bytes()               */
#define XCB_ERR_CUDA 4              /* a CUDA runtime call or launch failed                            */
#define XCB_ERR_DEVICE 5            /* xcb_moe_read_status found device-side status bits               */

/* ---- device status bits (xcb_moe_read_status) ---- */
#define XCB_STATUS_DEVICE_TIMEOUT 1 /* a bounded spin-wait gave up (the output of that call is invalid) */
#define XCB_STATUS_BAD_EXPERT 2     /* a topk id outside [0, total_experts): that route was dropped   */
#define XCB_STATUS_NAN_SCALE 4      /* the packer met a NaN E4M3 block scale                          */
#define XCB_STATUS_CAPACITY 8       /* more routes than the workspace was sized for                   */

/* ---- forward flags ---- */
#define XCB_FLAG_POST_NORM 1        /* reference contract: y *= (1 + post_norm_w); out = sum w * y / rms(y) */
#define XCB_FLAG_DECODE_PATH 2      /* force the decode kernel (default below 257 routes and 33 tokens; for a
                                       layer holding some of the router's experts, up to ~192 expected held
                                       routes)                                                                  */
#define XCB_FLAG_PREFILL_PATH 4     /* force the prefill path: tcgen05 grouped GEMMs (default above)         */
#define XCB_FLAG_DETERMINISTIC 16   /* prefill path: combine the routes in a separate pass, in slot order, so the
                                       output is bit-reproducible; by default (without the post-norm) the down
                                       projection adds w * y into a fp32 accumulator itself, whose order of
                                       additions varies from run to run                                       */
#define XCB_FLAG_PDL 8              /* single-launch decode calls use programmatic dependent launch: the kernel
                                       may start before the previous kernel of the stream ends and waits
                                       (griddepcontrol.wait) before its first global read; the reference's
                                       PDL switch, moe_w4a16.py:169, :2864-2878                                */

/* Shape of one prepared layer.  total_experts is the router width (logits columns, valid topk ids);
 * experts [expert_offset, expert_offset + num_experts) are held in the packed buffers (the reference's
 * local_start / local_count, moe_w4a16.py:105-110). */
typedef struct XcbMoeShape {
  int32_t num_experts;    /* experts held in the packed buffers                                           */
  int32_t total_experts;  /* router width                                                                  */
  int32_t expert_offset;  /* global id of held expert 0                                                    */
  int32_t hidden;         /* H: x and out row length; K of gate_up; rows of down                           */
  int32_t inter;          /* I: rows of gate (and of up); K of down                                        */
} XcbMoeShape;

/* Packed weights (device memory owned by the caller) + per-expert fp32 global scales + optional bf16 post-norm. */
typedef struct XcbMoeWeights {
  XcbMoeShape shape;
  const void* gate_up;        /* xcb_moe_packed_bytes(shape, 0) bytes, written by xcb_moe_pack_weights */
  const void* down;           /* xcb_moe_packed_bytes(shape, 1) bytes                                   */
  const float* gate_up_gs;    /* [num_experts]  (reference w13_gs, moe_w4a16.py:72-79)                 */
  const float* down_gs;       /* [num_experts]  (reference w2_gs)                                       */
  const uint16_t* post_norm_w;/* bf16 [hidden] or NULL (reference post_norm_w)                          */
} XcbMoeWeights;

/* One forward call.  Either router_logits (north_star form: softmax -> top-k -> renormalise, ties to the lower
 * expert id) or topk_ids + topk_weights (reference form, moe_w4a16.py:93-97) must be given. */
typedef struct XcbMoeArgs {
  int32_t tokens;                 /* T (0 is allowed: nothing is launched)                      */
  int32_t top_k;                  /* routes per token, 1..16                                    */
  int32_t flags;                  /* XCB_FLAG_*                                                 */
  int32_t wait_limit_us;          /* bound of every device-side wait, microseconds (0: 2 s)     */
  const uint16_t* hidden_states;  /* bf16 [T, hidden], rows 16-byte aligned                     */
  const float* router_logits;     /* fp32 [T, total_experts] or NULL                            */
  const int32_t* topk_ids;        /* int32 [T, top_k] global ids, or NULL                       */
  const float* topk_weights;      /* fp32 [T, top_k], or NULL                                   */
  uint16_t* out;                  /* bf16 [T, hidden]                                           */
  int32_t* topk_ids_out;          /* optional int32 [T, top_k]: the routing used                */
  float* topk_weights_out;        /* optional fp32 [T, top_k]                                   */
} XcbMoeArgs;

/* Human-readable name of a return code. */
const char* xcb_status_str(int code);

/* XCB_OK if the kernels support this shape (hidden and inter multiples of 256, hidden <= 8192, ...). */
int xcb_moe_check_shape(const XcbMoeShape* shape);

/* Bytes of one packed tensor: which = 0 gate_up [E, 2I, H], 1 down [E, H, I].  The buffer holds two layouts of
 * the same weights: the decode-path layout (first half) and the prefill-path layout (second half).
 * Replaces the reference's packed copies built in prepare() (moe_w4a16.py:3292-3351). */
size_t xcb_moe_packed_bytes(const XcbMoeShape* shape, int which);

/* Repack reference-layout NVFP4 weights into the kernels' layout on the GPU (lossless; never requantises).
 * w13: uint8 [E, 2I, H/2] (gate rows then up rows, low nibble = even k), w13_sf: E4M3 bytes [E, 2I, H/16],
 * w2: uint8 [E, H, I/2], w2_sf: [E, H, I/16] (moe_w4a16.py:72-79, nibble order :3151-3158); E = shape.num_experts
 * experts starting at the pointers given.  xor_tables: device uint32 [4*256], the GF(2) packing transform of the
 * decoder (xcalibur_b200/packer.py).  status: device int32, gets XCB_STATUS_NAN_SCALE on a NaN scale.
 * Replaces _pack_codes/_pack_scales and the GF(2) word transform (moe_w4a16.py:3168-3190, :3903-3933). */
int xcb_moe_pack_weights(const XcbMoeShape* shape, const uint8_t* w13, const uint8_t* w13_sf, const uint8_t* w2,
                         const uint8_t* w2_sf, const uint32_t* xor_tables, void* gate_up_out, void* down_out,
                         int32_t* status, cudaStream_t stream);

/* Workspace bytes for calls of up to max_tokens tokens with top_k routes each (reference scratch:
 * _make_scratch, moe_w4a16.py:3353-3367). */
size_t xcb_moe_workspace_bytes(const XcbMoeShape* shape, int32_t max_tokens, int32_t top_k);

/* Byte offsets of the routing arrays inside a workspace sized for (max_tokens, top_k), for inspection by tests and
 * callers that want the permutation: out[0] ids int32 [T*k], out[1] weights fp32 [T*k], out[2] pos int32 [T*k]
 * (permuted position of each flat route, -1 if not local), out[3] order int32 [routes] (flat route at each
 * permuted position), out[4] counts int32 [num_experts], out[5] offsets int32 [num_experts + 1].
 * Returns the number of entries written (6) or -1 on bad arguments. */
int xcb_moe_workspace_offsets(const XcbMoeShape* shape, int32_t max_tokens, int32_t top_k, size_t* out, int n);

/* How a forward call of this shape and size would run, without touching the GPU (a diagnostic, for tests and for
 * callers sizing their batches; no counterpart in the reference, whose kernel_fn picks a build by token count,
 * moe_w4a16.py:3384-3393).  given_routes: 1 for topk_ids/topk_weights, 0 for router logits.  out[0] path (0 decode,
 * 1 prefill), out[1] routes computed inside the decode kernel (1) or by the router kernel (0), out[2] routes per
 * decode job, out[3] activation rows per buffer, out[4] activation buffers, out[5] weight-ring stages, out[6] bytes
 * per stage, out[7] the decode kernel stages both rows of a two-token call at start (1).  Decode fields are 0 on
 * the prefill path.  Returns the number of entries written (8, or n if smaller) or an XCB_ERR_* code. */
int xcb_moe_plan_info(const XcbMoeShape* shape, int32_t tokens, int32_t top_k, int32_t flags, int32_t given_routes,
                      int32_t* out, int32_t n);

/* Zero a fresh workspace (once, before its first forward call).  Calls keep it consistent afterwards. */
int xcb_moe_workspace_init(void* workspace, size_t bytes, int32_t max_tokens, int32_t top_k, cudaStream_t stream);

/* One MoE layer: out = sum_k w_k * down_e(SiLU(gate_e x) * up_e x) (or the post-norm form with
 * XCB_FLAG_POST_NORM).  Asynchronous on `stream`; no host synchronisation; graph-capturable.
 * Replaces okc_run (moe_w4a16.py:2812-2886) and kernel_fn's variant dispatch (moe_w4a16.py:3370-3399).
 * Calls that share a workspace must be ordered on one stream. */
int xcb_moe_forward(const XcbMoeWeights* weights, const XcbMoeArgs* args, void* workspace, size_t workspace_bytes,
                    cudaStream_t stream);

/* The two halves of xcb_moe_forward, for callers that time or schedule them separately: xcb_moe_route runs the
 * router, the expert histogram and the stable permutation into the workspace; xcb_moe_experts then runs the
 * expert MLPs and the weighted combine.  They must be called with the same arguments, in this order, on one
 * stream. */
int xcb_moe_route(const XcbMoeWeights* weights, const XcbMoeArgs* args, void* workspace, size_t workspace_bytes,
                  cudaStream_t stream);
int xcb_moe_experts(const XcbMoeWeights* weights, const XcbMoeArgs* args, void* workspace, size_t workspace_bytes,
                    cudaStream_t stream);

/* Size of the fixed scratch behind xcb_moe_forward_static (8 MiB, reserved on every GPU that loads the library). */
#define XCB_STATIC_SCRATCH_BYTES (8u << 20)

/* xcb_moe_forward without a caller-provided workspace, for callers that cannot allocate device memory: a host
 * framework that owns every device byte through its own allocator and forbids plugins to call cudaMalloc, or a
 * latency-critical decode loop where cudaMalloc/cudaFree would stall or synchronise the device.  No counterpart in
 * the reference (its scratch is always allocated by prepare(), moe_w4a16.py:3353-3367).
 * The scratch is one file-scope device array of XCB_STATIC_SCRATCH_BYTES per GPU, held until the process exits;
 * a call whose workspace would exceed it (xcb_moe_workspace_bytes(shape, tokens, top_k) > XCB_STATIC_SCRATCH_BYTES,
 * e.g. more than 31 tokens x top-8 at the DeepSeek-V3 shape) returns XCB_ERR_WORKSPACE before any launch.  The
 * function allocates nothing.  Its first call on a device looks up the array's device address (with that device
 * current) and caches it; make that first call before any stream capture.  All calls on a device share the one
 * array: calls that overlap on the GPU (other streams, other threads) race and must be serialised by the caller.
 * Device-side status bits (XCB_STATUS_*) of these calls stay in the array until xcb_moe_static_read_status reads
 * them. */
int xcb_moe_forward_static(const XcbMoeWeights* weights, const XcbMoeArgs* args, cudaStream_t stream);

/* Status bits that xcb_moe_forward_static calls on the current device have set since the last read (a bounded wait
 * that expired, an expert id out of range): synchronises `stream`, writes them to *device_status and clears them.
 * Returns XCB_OK if none were set, XCB_ERR_DEVICE otherwise.  Like xcb_moe_forward_static it allocates nothing and
 * has no counterpart in the reference. */
int xcb_moe_static_read_status(int32_t* device_status, cudaStream_t stream);

/* Synchronise `stream`, read the workspace status bits into *device_status, clear them.
 * Returns XCB_OK if none were set, XCB_ERR_DEVICE otherwise. */
int xcb_moe_read_status(void* workspace, int32_t* device_status, cudaStream_t stream);

/* HBM read-bandwidth probe (diagnostic; replaces the reference's bulk-copy probes, moe_w4a16.py:2890-3061):
 * streams `bytes` from `src` (1 KB aligned) with mode 0 = 1-D bulk-copy ring (stages x chunk bytes per CTA, chunk a
 * multiple of 1 KB),
 * 1 = the same with an L2 evict-first hint, 2 = 16-byte vector loads; ctas_per_sm CTAs of `threads` threads per SM.
 * With `regions` (device int64 byte offsets, `nreg` of them) the CTAs split into nreg groups that each stream one
 * region of bytes/nreg bytes, as the decode kernel streams a few experts.  Time it with events on `stream`;
 * status gets XCB_STATUS_DEVICE_TIMEOUT if a ring wait expired.  Every byte streamed is read: `sink` (4 bytes, zeroed
 * by the caller) receives the XOR of every 32-bit word read, so a caller can check that the probe streamed what it
 * claims (each CTA streams (bytes / CTAs) rounded down to a multiple of chunk, 16 for mode 2). */
int xcb_hbm_probe(const void* src, size_t bytes, int mode, int chunk, int stages, int ctas_per_sm, int threads,
                  const long long* regions, int nreg, int32_t* status, float* sink, cudaStream_t stream);

/* ---- expert parallelism ----
 * The reference models an expert-parallel rank only as a local expert range whose non-local routes are masked
 * (moe_w4a16.py:105-110, :513-520); the exchange between ranks was its harness's job.  These helpers give the
 * expert-parallel layer its dispatch and combine: experts are held contiguously, experts_per_rank per rank, and a
 * token is sent once to every rank holding one of its experts, with its full top-k row (the receiving rank's
 * xcb_moe_forward masks the experts it does not hold). */

/* Router alone: softmax -> top-k -> renormalise per token (ties to the lower expert id), ids int32 [T, k] and
 * weights fp32 [T, k] for all E experts.  Same selection and weights as xcb_moe_forward's router. */
int xcb_moe_topk(const float* logits, int32_t T, int32_t E, int32_t k, int32_t* ids, float* wts, cudaStream_t stream);

/* Dispatch plan of one rank's T tokens over G ranks (G <= 32): counts int32 [G] (tokens for each rank),
 * send_tok int32 [G, T] (row d: the tokens for rank d in token order, first counts[d] valid), send_pos int32 [T, G]
 * (position of token t in rank d's list, or -1).  status gets XCB_STATUS_BAD_EXPERT for an id outside
 * [0, G * experts_per_rank). */
int xcb_ep_plan(const int32_t* ids, int32_t T, int32_t k, int32_t experts_per_rank, int32_t G, int32_t* counts,
                int32_t* send_tok, int32_t* send_pos, int32_t* status, cudaStream_t stream);

/* Send buffer in destination order (rank 0's rows first): x_out bf16 [sum(counts), H], ids_out int32 [.., k],
 * w_out fp32 [.., k]. */
int xcb_ep_gather(const uint16_t* x, const int32_t* ids, const float* wts, int32_t T, int32_t H, int32_t k, int32_t G,
                  const int32_t* counts, const int32_t* send_tok, uint16_t* x_out, int32_t* ids_out, float* w_out,
                  cudaStream_t stream);

/* out[t] = bf16(sum over ranks d in rank order of parts[row of (t, d)]), parts bf16 [sum(counts), H] in the send
 * buffer's order (each rank returns the partial sums of the rows it received, in the order received). */
int xcb_ep_combine(const uint16_t* parts, const int32_t* counts, const int32_t* send_pos, int32_t T, int32_t H,
                   int32_t G, uint16_t* out, cudaStream_t stream);

/* Peer exchange for small batches (every rank sends the same T <= T_max tokens to every rank), over NVLink peer
 * memory instead of a collective library.  Each rank allocates one buffer of xcb_ep_p2p_bytes() with
 * xcb_p2p_alloc (zeroed; handle = 64-byte CUDA IPC handle to share with the other ranks), opens the others'
 * with xcb_p2p_open, and passes peers = device uint64 [G] (peers[d] = rank d's buffer in this process, peers[rank]
 * its own).  Layout of a buffer for a step of T tokens: x bf16 [G * T, H] (row d*T + t = token t of rank d),
 * top-k ids int32 [G * T, k], top-k weights fp32 [G * T, k], partial sums bf16 [G * T, H], flags.
 * xcb_ep_p2p_dispatch routes this rank's tokens (router logits fp32 [T, E], E <= 512: the same softmax -> top-k
 * -> renormalise as xcb_moe_topk), writes their rows and top-k rows into every buffer and returns once (in stream
 * order) every rank's rows are in this rank's buffer; the local layer then runs on them in place;
 * xcb_ep_p2p_combine sends partial rows
 * [d*T, (d+1)*T) to rank d and writes out bf16 [T, H] = sum over source ranks in rank order.  Every rank must make
 * the same calls in the same order; T may change from step to step (up to T_max).  Waits are bounded by timeout_ns
 * (0: 2 s): on timeout status gets XCB_STATUS_DEVICE_TIMEOUT and xcb_ep_p2p_combine writes NaN rows (also when the
 * step's dispatch timed out), so a failed step cannot pass for a valid result. */
size_t xcb_ep_p2p_bytes(int32_t G, int32_t T_max, int32_t H, int32_t k);
int xcb_p2p_alloc(size_t bytes, void** ptr, void* handle);
int xcb_p2p_open(const void* handle, void** ptr);
int xcb_p2p_close(void* ptr);
int xcb_p2p_free(void* ptr);
int xcb_ep_p2p_dispatch(const uint16_t* x, const float* logits, int32_t T, int32_t T_max, int32_t H, int32_t E,
                        int32_t k, int32_t G, int32_t rank, const uint64_t* peers, int32_t* status,
                        uint64_t timeout_ns, cudaStream_t stream);
int xcb_ep_p2p_combine(const uint16_t* parts, int32_t T, int32_t T_max, int32_t H, int32_t k, int32_t G,
                       int32_t rank, const uint64_t* peers, uint16_t* out, int32_t* status, uint64_t timeout_ns,
                       cudaStream_t stream);

/* Quantise fp32 weights [E, R, K] to NVFP4 (gs = amax/(6*448) per expert, sf = e4m3(block_amax/6/gs),
 * codes RNE to E2M1): codes [E, R, K/2], sf [E, R, K/16], gs [E].  A utility for synthetic weights; the
 * reference receives already-quantised weights.  amax_scratch: device float [E] (zeroed by this call). */
int xcb_nvfp4_quantize(const float* w, int32_t E, int32_t R, int32_t K, uint8_t* codes, uint8_t* sf, float* gs,
                       float* amax_scratch, cudaStream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* XCB_MOE_H_ */
