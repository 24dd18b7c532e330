/*
 * pw_cuda.h -- C ABI of the B200 (sm_100a) block-FP8 routed-MoE path.
 *
 * This is the drop-in boundary for Prismwing's routed-MoE / projection
 * runtime.  Each entry point names the reference interface it replaces
 * (path:line inside the x3haloed/mimo-prismwing tree).  A Rust caller binds
 * these with an `extern "C"` block, exactly as the reference already binds
 * its C++ top-k bridge (src/text_endpoint.rs:2466-2472 declaring
 * src/pytorch_topk.cpp:7).
 *
 * Conventions
 *  - Every function returns an int status: PW_OK (0) or a negative PW_ERR_*.
 *    No C++ exception crosses the boundary.  pw_last_error() gives the text.
 *  - Weight and scale pointers inside pw_fp8_tensor / pw_router are DEVICE
 *    pointers owned by the caller (uploaded once; never freed by the library).
 *  - Activation inputs and outputs are host or device pointers, chosen per
 *    call by `mem` (PW_MEM_HOST or PW_MEM_DEVICE).  With PW_MEM_HOST the call
 *    copies inputs in, runs, copies outputs out and returns after the stream
 *    has finished (the reference's commit + wait_until_completed).  With
 *    PW_MEM_DEVICE the call is asynchronous on the runtime's stream unless
 *    stats are requested (stats imply a stream synchronisation).
 *  - One runtime per (thread, device).  Calls on one runtime are not
 *    re-entrant.  The runtime owns its stream, its scratch arena and the
 *    device error-flag word.
 */
#ifndef PW_CUDA_H
#define PW_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PW_ABI_VERSION 2

/* ---- status codes (reference: Result<_, String>, src/wide_metal_moe.rs) ---- */
#define PW_OK 0
#define PW_ERR_ARGUMENT (-1)     /* null pointer, bad enum, bad runtime        */
#define PW_ERR_SHAPE (-2)        /* shape / layout / scale-grid mismatch       */
#define PW_ERR_NONFINITE (-3)    /* non-finite input, scale, weight or output  */
#define PW_ERR_DEVICE_FLAGS (-4) /* a kernel set a bit in the error-flag word  */
#define PW_ERR_CUDA (-5)         /* CUDA runtime error                         */
#define PW_ERR_NCCL (-6)         /* NCCL error (expert-parallel calls)         */
#define PW_ERR_TIMEOUT (-7)      /* a bounded device wait gave up              */
#define PW_ERR_SCHEDULE (-8)     /* invalid expert schedule / route table      */
#define PW_ERR_UNSUPPORTED (-9)  /* valid request outside this build's limits  */
#define PW_ERR_FORMAT (-10)      /* malformed or inconsistent checkpoint file  */
#define PW_ERR_IO (-11)          /* file open / read / write failure           */

/* ---- device error-flag bits (reference kernels/block_fp8_gemv.metal:40-229;
 *      bits 1..128 keep the reference meanings, 256+ are new) ---- */
#define PW_FLAG_BAD_LAUNCH 1u          /* launch geometry mismatch            */
#define PW_FLAG_NONFINITE_INPUT 2u     /* non-finite activation               */
#define PW_FLAG_NONFINITE_SWIGLU 4u    /* non-finite staged SwiGLU value      */
#define PW_FLAG_BAD_EXPERT_COUNT 8u    /* schedule row count mismatch         */
#define PW_FLAG_NONFINITE_COMBINE 16u  /* non-finite weighted combine         */
#define PW_FLAG_NONFINITE_ROUND 32u    /* non-finite bf16-rounded output      */
#define PW_FLAG_NONFINITE_FUSED 128u   /* non-finite fused gate/up result     */
#define PW_FLAG_ROUTE_WEIGHTS 256u     /* route weights not finite / sum != 1 */
#define PW_FLAG_WAIT_TIMEOUT 512u      /* bounded pipeline wait ran out       */
#define PW_FLAG_BAD_WEIGHT 1024u       /* weight byte 0x7f/0xff or bad scale  */

/* ---- runtime flags (reference: compile vs compile_with_fused_gate_up,
 *      src/wide_metal_moe.rs:165-171) ---- */
#define PW_RUNTIME_FUSED_GATE_UP 1u

/* ---- projection layouts (reference: execute_fp8_linear's full_qkv_layout
 *      flag and its 14848-row SWA dispatch, src/wide_metal_moe.rs:300-306) ---- */
#define PW_LAYOUT_PLAIN 0u
#define PW_LAYOUT_FULL_QKV 1u /* [13568,4096], 4 shards [Q3072|K192|V128], grid [108,32] */
#define PW_LAYOUT_SWA_QKV 2u  /* [14848,4096], 4 shards [Q3072|K384|V256], grid [116,32] */
/* OR-able with a layout in pw_fp8_linear: return the f32 pre-round projection
 * instead of the reference's bf16-rounded one. */
#define PW_OUTPUT_F32 0x100u

/* ---- where caller activation buffers live (the `mem` argument) ---- */
#define PW_MEM_DEVICE 0u
#define PW_MEM_HOST 1u
/* OR-able with PW_MEM_DEVICE: enqueue on the runtime's stream and return
 * without waiting (CUDA-graph capturable).  Errors surface through
 * pw_read_error_flags(); stats must be NULL. */
#define PW_MEM_ASYNC 2u

typedef struct pw_runtime pw_runtime;
typedef struct pw_expert_bank pw_expert_bank;

/* One e4m3 weight matrix with its 128x128 f32 scale grid (reference:
 * WideProjectionBinding src/wide_metal_moe.rs:80 + GemvShape :131).  Device
 * pointers.  scale_rows x scale_cols must be ceil(rows/128) x cols/128 for
 * PLAIN, [108,32] for FULL_QKV and [116,32] for SWA_QKV. */
typedef struct pw_fp8_tensor {
  const uint8_t *weight;
  const float *scale;
  uint32_t rows, cols;
  uint32_t scale_rows, scale_cols;
} pw_fp8_tensor;

/* gate [I,H], up [I,H], down [H,I] (reference: WideExpertBinding's three
 * projections, src/wide_metal_moe.rs:88). */
typedef struct pw_expert_weights {
  pw_fp8_tensor gate, up, down;
} pw_expert_weights;

/* Host-built schedule entry (reference: WideExpertBinding
 * src/wide_metal_moe.rs:88-95: expert id, positions, route weights). */
typedef struct pw_expert_binding {
  uint32_t expert;
  uint32_t count;
  const uint32_t *positions;    /* host memory, [count], < rows */
  const float *route_weights;   /* host memory, [count] */
  pw_expert_weights weights;    /* device pointers */
} pw_expert_binding;

/* Router weight storage (pw_router.weight_dtype).  The reference reads the
 * checkpoint's model.layers.N.mlp.gate.weight as F32 and runs an f32 linear
 * (src/text_endpoint.rs:4350-4358, f32_linear :3458-3476): pass that tensor as
 * PW_ROUTER_F32.  PW_ROUTER_BF16 takes bf16 bits, widened to f32 exactly
 * (a bf16 copy of the checkpoint's weight is a different router). */
#define PW_ROUTER_F32 0u
#define PW_ROUTER_BF16 1u

/* Router (reference: route_mlp src/text_endpoint.rs:4342 with gate.weight
 * [256,4096] and e_score_correction_bias [256]).  Device pointers. */
typedef struct pw_router {
  const void *weight;    /* [experts, hidden], f32 or bf16 bits per weight_dtype */
  const float *bias;     /* [experts] f32 */
  uint32_t experts, hidden, top_k;
  uint32_t weight_dtype; /* PW_ROUTER_F32 or PW_ROUTER_BF16 */
} pw_router;

/* RMSNorm weight storage (pw_norm.weight_dtype).  The checkpoint stores
 * model.layers.N.post_attention_layernorm.weight as BF16 (read by bf16_vector,
 * src/text_endpoint.rs:5507-5512). */
#define PW_NORM_F32 0u
#define PW_NORM_BF16 1u

/* An RMSNorm (reference: rms_norm src/text_endpoint.rs:2939 with
 * stable_rms_inverse src/lib.rs:1890).  Device pointer. */
typedef struct pw_norm {
  const void *weight;    /* [hidden], f32 or bf16 bits per weight_dtype */
  uint32_t hidden;       /* a multiple of 256, at most 16384 */
  uint32_t weight_dtype; /* PW_NORM_F32 or PW_NORM_BF16 */
  float epsilon;         /* layernorm_epsilon (1e-5 for MiMo-V2.5), finite and > 0 */
} pw_norm;

/* Per-call accounting (reference: WideMoeExecution / WideLinearExecution,
 * src/wide_metal_moe.rs:97-111). */
typedef struct pw_stats {
  double wall_ms;             /* host wall time of the call                */
  float device_ms;            /* CUDA-event time of the call's device work */
  uint32_t error_flags;       /* PW_FLAG_* bits seen                       */
  uint32_t unique_experts;    /* experts with >= 1 placement               */
  uint32_t expert_rows;       /* placements (rows * top_k)                 */
  uint32_t boundary_tie_rows; /* rows whose k-th/(k+1)-th scores tie       */
  uint64_t weight_bytes;      /* FP8 weight + scale bytes the call reads   */
} pw_stats;

/* Device time per kernel class of the last profiled call (CUDA events on the
 * runtime's stream around each launch; 0 for classes the call did not run).
 * The reference's equivalent is its per-projection tomography
 * (ProjectionTomography / ExpertTomography, src/staged_metal_expert.rs:198-236). */
typedef struct pw_profile {
  float quantize_ms;   /* activation quantization (input + hidden)      */
  float router_ms;     /* router logits + sigmoid top-k                 */
  float schedule_ms;   /* device-side expert schedule                   */
  float gate_up_ms;    /* gate/up projection (+ SwiGLU)                 */
  float down_ms;       /* down projection                               */
  float combine_ms;    /* weighted combine                              */
  float projection_ms; /* single projections (pw_fp8_linear / gemv)     */
  uint32_t launches;   /* kernels this library launched in the call     */
} pw_profile;

/* ---------------------------------------------------------------- runtime */

/* Reference: WideMetalMoeRuntime::compile / compile_with_fused_gate_up
 * (src/wide_metal_moe.rs:165-171).  Selects `device`, creates a stream,
 * the error-flag word and an empty scratch arena. */
int pw_runtime_create(int device, uint32_t flags, pw_runtime **out);
void pw_runtime_destroy(pw_runtime *rt);
/* Text of the last error on this runtime ("" if none); valid until the next call. */
const char *pw_last_error(const pw_runtime *rt);
/* Run subsequent calls on a caller stream (a cudaStream_t passed as void*); NULL restores the runtime's own. */
int pw_set_stream(pw_runtime *rt, void *cuda_stream);
int pw_synchronize(pw_runtime *rt);
/* Device error-flag word accumulated since the last call that reset it (0 = clean). */
int pw_read_error_flags(pw_runtime *rt, uint32_t *flags);
int pw_abi_version(void);
/* Turn per-kernel event timing on (1) or off (0) for subsequent synchronous calls. */
int pw_set_profiling(pw_runtime *rt, int enable);
int pw_last_profile(pw_runtime *rt, pw_profile *out);

/* ------------------------------------------------------------- primitives */

/* Reference: dynamic_fp8_activations src/text_endpoint.rs:3008 and the
 * kernel dynamic_fp8_quantized_group128 kernels/block_fp8_gemv.metal:84.
 * x f32 [rows, cols] -> codes e4m3 [rows, cols], scales f32 [rows, cols/128].
 * cols % 128 == 0.  Bit-exact with the reference. */
int pw_quantize_fp8(pw_runtime *rt, const float *x, uint32_t rows, uint32_t cols, uint8_t *codes,
                    float *scales, uint32_t mem);

/* Reference: validate_fp8_views_internal src/lib.rs:1217 (scan of every
 * weight byte for 0x7f/0xff and of every scale for finiteness).
 * *bad_offset receives the first bad weight byte offset, or UINT64_MAX. */
int pw_validate_fp8(pw_runtime *rt, const pw_fp8_tensor *w, uint64_t *bad_offset);

/* Reference: mapped_fp8_gemv src/lib.rs:1272 / block_fp8_gemv src/lib.rs:7469
 * (the readable projection: activation NOT quantized, f32 output, no bf16
 * rounding).  x f32 [width, cols], y f32 [width, rows], width 1..=8. */
int pw_fp8_gemv(pw_runtime *rt, const pw_fp8_tensor *w, const float *x, uint32_t width, float *y,
                uint32_t mem, pw_stats *stats);

/* Reference: WideMetalMoeRuntime::execute_fp8_linear src/wide_metal_moe.rs:241
 * (dynamic FP8 activation quantization, block-scaled projection, bf16 round).
 * x f32 [width, cols], y f32 [width, rows] (bf16-valued).  `layout` selects the
 * plain, full-QKV or SWA-QKV row/scale map.  Widths 1..=8 take the width-
 * specialised GEMV; wider inputs run in chunks of 8 (reference limit: 8). */
int pw_fp8_linear(pw_runtime *rt, const pw_fp8_tensor *w, uint32_t layout, const float *x,
                  uint32_t width, float *y, uint32_t mem, pw_stats *stats);

/* One routed expert at weight 1: quantize -> gate/up -> staged bf16 SwiGLU ->
 * quantize -> down -> bf16 (reference: the per-expert body of
 * routed_mlp_traced src/text_endpoint.rs:5311-5346 and of execute_configured
 * src/wide_metal_moe.rs:1081-1240).  x [width, H] -> y [width, H]. */
int pw_expert_forward(pw_runtime *rt, const pw_expert_weights *w, const float *x, uint32_t width,
                      float *y, uint32_t mem, pw_stats *stats);

/* Reference: dense_mlp src/text_endpoint.rs:4266, the dense MLP of layer 0:
 * gate and up [I, H], staged bf16 SwiGLU, down [H, I], each projection an
 * fp8_linear (dynamic FP8 input, block-scaled, bf16-rounded output); for
 * MiMo-V2.5 I = 16384, H = 4096.  x [rows, H] -> y [rows, H].  The same
 * arithmetic as pw_expert_forward; intermediate sizes above 4096 (up to
 * 65536) run the down projection over 4096-column slices of its input axis,
 * whose sums are added in slice order before the bf16 round. */
int pw_dense_mlp(pw_runtime *rt, const pw_expert_weights *w, const float *x, uint32_t rows, float *y, uint32_t mem,
                 pw_stats *stats);

/* Reference: route_mlp src/text_endpoint.rs:4342 + pytorch_noaux_routes :4394
 * (f32 logits, SLEEF-u10 sigmoid, top-k of score+bias, weights = score /
 * (pairwise sum of the k chosen + 1e-20)).  top_k must be 8.  Logits are f32
 * in one fixed order: the hidden axis is cut into 256-column slices, each
 * slice sum is a chain of fused multiply-adds from +0 over its columns in
 * ascending order, and the logit adds the slice sums in slice order (the
 * reference's SGEMM order is unspecified; this one is reproducible on CPU and
 * GPU).  Selected experts are emitted in canonical order (corrected score
 * descending, index ascending).  selected u32 [tokens, 8], weights f32
 * [tokens, 8]. */
int pw_route(pw_runtime *rt, const pw_router *router, const float *x, uint32_t tokens,
             uint32_t *selected, float *weights, uint32_t mem, pw_stats *stats);

/* Reference: rms_norm src/text_endpoint.rs:2939.  Per row of x f32 [rows,
 * hidden]: inv = 1 / sqrt(sum(x^2) / hidden + epsilon), the sum in PyTorch's
 * vectorised cascade order (pytorch_contiguous_inner_square_sum_f32,
 * src/lib.rs:1905), then y = bf16(bf16(x * inv) * weight).  `inverse`
 * (optional, same `mem` as x) receives each row's inv.  Non-finite input is
 * PW_ERR_NONFINITE (stable_rms_inverse's Err). */
int pw_rms_norm(pw_runtime *rt, const pw_norm *norm, const float *x, uint32_t rows, float *y, float *inverse,
                uint32_t mem, pw_stats *stats);

/* ------------------------------------------------------------ MoE layers */

/* Reference: WideMetalMoeRuntime::execute / execute_fused_gate_up
 * src/wide_metal_moe.rs:836-1316 (host-built schedule, whole routed layer
 * in one device transaction).  x f32 [rows, H], y f32 [rows, H] bf16-valued.
 * sum(count) must equal rows * 8; positions < rows; counts >= 1. */
int pw_moe_execute(pw_runtime *rt, const float *x, uint32_t rows, const pw_expert_binding *experts,
                   uint32_t n_experts, float *y, uint32_t mem, pw_stats *stats);

/* Register an expert bank (256 experts for MiMo-V2.5) once; the library keeps
 * a device table of the caller's weight pointers and validates every weight
 * byte and scale (the reference's fail-closed checkpoint validation,
 * src/lib.rs:1217).  The weights stay caller-owned. */
int pw_bank_create(pw_runtime *rt, const pw_expert_weights *experts, uint32_t n_experts,
                   pw_expert_bank **out);
void pw_bank_destroy(pw_expert_bank *bank);

/* Whole routed layer on the device, router included (reference:
 * routed_mlp_metal_wide_configured src/text_endpoint.rs:4750, with route_mlp,
 * the BTreeMap schedule :4768-4776 and execute_configured folded into one
 * stream of kernels with no host round trip).  x [tokens, H] -> y [tokens, H].
 * Optional selected/weights (same `mem` as x) receive the routing. */
int pw_moe_layer(pw_runtime *rt, const pw_router *router, const pw_expert_bank *bank, const float *x,
                 uint32_t tokens, float *y, uint32_t *selected, float *weights, uint32_t mem,
                 pw_stats *stats);

/* The MoE half of a decoder layer (reference: src/text_endpoint.rs:5507-5580):
 *   moe_input = rms_norm(post_attention, post_attention_layernorm)
 *   mlp       = routed layer of moe_input (as pw_moe_layer)
 *   out       = bf16(post_attention + mlp)
 * The RMSNorm runs fused with the experts' input quantization (one kernel
 * writes the normalized rows for the router and their FP8 codes), and the
 * residual add runs in the combine's epilogue.  residual = post_attention f32
 * [tokens, H] (bf16-valued); out [tokens, H] may not alias it. */
int pw_moe_block(pw_runtime *rt, const pw_norm *post_norm, const pw_router *router, const pw_expert_bank *bank,
                 const float *residual, uint32_t tokens, float *out, uint32_t *selected, float *weights,
                 uint32_t mem, pw_stats *stats);

/* ------------------------------------------------- expert parallelism */

/* The reference runs all experts of a layer on one device
 * (routed_mlp_metal_wide_configured, src/text_endpoint.rs:4750); these calls
 * split a layer's experts over the GPUs of one node, one process (and one
 * runtime) per GPU, over NCCL.  NCCL is loaded on first use (libnccl.so.2);
 * without it these calls return PW_ERR_UNSUPPORTED.
 *
 * pw_ep_unique_id: one rank creates the communicator id (128 bytes) and sends
 * it to the others by any out-of-band channel.
 * pw_ep_init: collective; rank `rank` of `world` joins.  `timeout_ms` (0 = 60 s)
 * bounds every wait of this and later expert-parallel calls; a call that runs
 * out of time, or sees an NCCL error, aborts the communicator and returns
 * PW_ERR_TIMEOUT / PW_ERR_NCCL, after which the runtime refuses further
 * expert-parallel calls. */
/* max_tokens (0 = 2048, at most 2048) bounds the tokens any rank passes per
 * layer; every rank must pass the same value.  The expert rows travel by
 * peer-memory stores: each rank's receive window, sized for max_tokens,
 * `hidden` and `local_experts` (experts per rank), is mapped into the other
 * ranks through CUDA IPC here (hidden = 0 defers that to the first layer
 * call, which is then collective too).  With PW_EP_NCCL_TRANSPORT in `flags`
 * the rows travel by NCCL send/recv instead, planned on the host. */
#define PW_EP_NCCL_TRANSPORT 1u
int pw_ep_unique_id(void *id, uint32_t bytes);
int pw_ep_init(pw_runtime *rt, int rank, int world, const void *id, uint32_t bytes, uint32_t timeout_ms,
               uint32_t max_tokens, uint32_t hidden, uint32_t local_experts, uint32_t flags);
int pw_ep_rank(const pw_runtime *rt, int *rank, int *world);

/* Collective routed layer.  Every rank passes its own tokens (x [tokens, H],
 * tokens may be 0) and a bank holding its experts: rank g owns experts
 * [g * n, (g + 1) * n) of the router's E = n * world.  Routing is local; token
 * codes and scales go to the expert owners and bf16 expert outputs come back;
 * the combine runs on the token's rank in ascending expert order, so y is
 * bit-identical to pw_moe_layer on one GPU.  With PW_MEM_DEVICE | PW_MEM_ASYNC
 * it returns once its work is enqueued (the peer-memory transport needs no
 * host round trip; the NCCL transport waits for the all-gathered per-expert
 * counts first), otherwise when the layer is done.
 * stats->unique_experts / expert_rows count this rank's local work. */
int pw_ep_moe_layer(pw_runtime *rt, const pw_router *router, const pw_expert_bank *bank, const float *x,
                    uint32_t tokens, float *y, uint32_t *selected, float *weights, uint32_t mem,
                    pw_stats *stats);

/* Collective form of pw_moe_block: the RMSNorm and the residual add run on
 * each token's own rank, the routed layer as in pw_ep_moe_layer. */
int pw_ep_moe_block(pw_runtime *rt, const pw_norm *post_norm, const pw_router *router, const pw_expert_bank *bank,
                    const float *residual, uint32_t tokens, float *out, uint32_t *selected, float *weights,
                    uint32_t mem, pw_stats *stats);

/* Host-only helper (no GPU): the transfer plan pw_ep_moe_layer derives for
 * rank `rank` from every rank's expert offsets.  all_offsets[g * (E + 1) + e]
 * is the first of rank g's placements (expert-major) routed to expert e, with
 * all_offsets[g * (E + 1) + E] its placement count.  Outputs: n_send[world],
 * n_recv[world], recv_base[world + 1] (where each source's rows land),
 * perm[rows received] (received row of each row in expert order: local expert,
 * then source rank, then the source's order) and expert_begin[E / world + 1]. */
int pw_ep_plan(const uint32_t *all_offsets, uint32_t world, uint32_t rank, uint32_t experts, uint32_t *n_send,
               uint32_t *n_recv, uint32_t *recv_base, uint32_t *perm, uint32_t *expert_begin);

/* ------------------------------------------------- checkpoint ingestion */

/* A read-only mapped tensor file: a safetensors checkpoint shard or a PWEXPRT1
 * expert container.  Tensor bytes stay in the mapping (host memory) until
 * uploaded. */
typedef struct pw_tensor_file pw_tensor_file;

typedef struct pw_tensor_view {
  const char *name;   /* valid while the file is open */
  const char *dtype;  /* safetensors dtype string: "F8_E4M3", "F32", "BF16", ... */
  uint32_t rank;
  uint64_t shape[8];
  const void *data;   /* host pointer into the mapping */
  uint64_t bytes;
} pw_tensor_view;

/* Reference: MappedSafetensors::open (src/lib.rs:784-905), fail-closed: the
 * 8-byte header length (non-zero, <= 256 MiB, a multiple of 8, inside the
 * file), a strict JSON header with unique keys, known dtypes, non-empty
 * shapes without zero dimensions, byte counts matching shape x dtype,
 * in-range non-overlapping payloads, at least one tensor.  `err` (optional)
 * receives the reason on failure.  Returns PW_ERR_FORMAT / PW_ERR_IO. */
int pw_safetensors_open(const char *path, pw_tensor_file **out, char *err, size_t err_len);
/* Reference: verify_expert_container (src/lib.rs:7282-7345) and
 * docs/EXPERT_CONTAINER.md: PWEXPRT1 magic, schema 1, 64-byte aligned
 * increasing payloads, every tensor's SHA-256, no trailing bytes. */
int pw_container_open(const char *path, pw_tensor_file **out, char *err, size_t err_len);
/* Reference: repack_expert_container (src/lib.rs:7190-7280): copy the named
 * tensors of a safetensors file, byte for byte, into a new PWEXPRT1 file;
 * refuses to overwrite; writes a same-directory temporary file, verifies it
 * and publishes it with a hard link. */
int pw_container_repack(const char *source, const char *output, const char *const *names, uint32_t n_names,
                        char *err, size_t err_len);
void pw_tensor_file_close(pw_tensor_file *f);
int pw_tensor_file_count(const pw_tensor_file *f, uint32_t *n);
/* i-th tensor in name order. */
int pw_tensor_file_at(const pw_tensor_file *f, uint32_t i, pw_tensor_view *out);
/* Reference: MappedSafetensors::tensor (src/lib.rs:907).  PW_ERR_FORMAT if absent. */
int pw_tensor_file_find(const pw_tensor_file *f, const char *name, pw_tensor_view *out);

/* Copy one tensor, found in exactly one of `files`, into a new device buffer
 * on the runtime's device (free it with pw_device_free).  dtype / shape
 * (optional) must match.  The router's model.layers.N.mlp.gate.weight (F32)
 * and e_score_correction_bias (F32), and post_attention_layernorm.weight
 * (BF16) load this way. */
int pw_tensor_upload(pw_runtime *rt, const pw_tensor_file *const *files, uint32_t n_files, const char *name,
                     const char *dtype, const uint64_t *shape, uint32_t rank, void **device_ptr, char *err,
                     size_t err_len);
int pw_device_free(pw_runtime *rt, void *device_ptr);

/* Load routed experts [first_expert, first_expert + n_experts) of `layer`
 * from the checkpoint's tensors model.layers.{layer}.mlp.experts.{e}.
 * {gate,up,down}_proj.weight (F8_E4M3) and their "_scale_inv" grids (F32)
 * (src/text_endpoint.rs:3067), found across `files`, into one device
 * allocation, and register them as a bank (pw_bank_create, which validates
 * every weight byte and scale).  The bank owns that memory; pw_bank_destroy
 * frees it.  Shapes must agree across experts: gate/up [I, H], down [H, I]. */
int pw_bank_load(pw_runtime *rt, const pw_tensor_file *const *files, uint32_t n_files, uint32_t layer,
                 uint32_t first_expert, uint32_t n_experts, pw_expert_bank **out, char *err, size_t err_len);

/* ------------------------------------------------- allocation-free variant */

/* No counterpart in the reference: an addition of this library.
 *
 * pw_expert_forward_static is pw_expert_forward for callers that must not
 * allocate device memory when they call in: code running inside a memory
 * budget that was reserved up front, plug-in hosts that own the allocator,
 * and serving loops that must stay free of cudaMalloc/cudaFree because those
 * calls synchronise the device.  It allocates nothing (no cudaMalloc, no
 * cudaFree, no allocating library call) and needs no pw_runtime: its scratch
 * (activation and hidden FP8 codes and scales, TMA descriptors, group records,
 * the error-flag word; about 70 KB) is one fixed __device__ array in the
 * library, which every GPU that loads the library holds until the process
 * exits.
 *
 * Limits: width 1..=8 tokens; hidden and intermediate sizes multiples of 128
 * and at most 4096; larger requests return PW_ERR_UNSUPPORTED.  x and y are
 * DEVICE pointers ([width, H] f32); weights as in pw_expert_forward.  The call
 * runs on `cuda_stream` (a cudaStream_t, NULL = legacy default stream) and
 * waits for it before returning the status.
 *
 * The first call on a device looks up the array's device address
 * (cudaGetSymbolAddress) with that device current; make that first call before
 * any stream capture.  The address is kept until the process exits: do not
 * call this after cudaDeviceReset.  `cuda_stream` must belong to the current
 * device (else PW_ERR_ARGUMENT).  All calls share the one array and it keeps
 * the last call's contents, so calls that overlap on the GPU (different
 * streams or threads at once) race with each other: serialise them. */
int pw_expert_forward_static(const pw_expert_weights *w, const float *x, uint32_t width, float *y,
                             void *cuda_stream);

#ifdef __cplusplus
}
#endif

#endif /* PW_CUDA_H */
