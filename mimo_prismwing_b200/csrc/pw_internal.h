// pw_internal.h -- host-side declarations shared by the kernels and the C ABI.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>
#include <nccl.h>

#include <string>

#include "pw_cuda.h"

namespace pw {

// The CUDA device of a runtime (PW_ERR_ARGUMENT for a null runtime).
int runtime_device(const pw_runtime *rt, int *device);
// A bank loaded from checkpoint files owns its weights' device memory
// (one allocation, freed by pw_bank_destroy).
void bank_adopt_memory(pw_expert_bank *bank, void *device_block);

// Launch a kernel, marked for programmatic dependent launch when the calling
// thread has enabled it (routed-layer chains); otherwise a plain launch.
bool pdl_enabled();
void set_pdl(bool on);
struct PdlScope {
  bool prev;
  explicit PdlScope(bool on) : prev(pdl_enabled()) { set_pdl(on); }
  ~PdlScope() { set_pdl(prev); }
};

template <typename... KArgs, typename... Args>
cudaError_t launch_kernel(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                          Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
  return e != cudaSuccess ? e : cudaGetLastError();
}

// One group of tokens sharing one weight matrix (a projection call, or one
// expert's placements in a routed layer).  count <= 8 per group: wider token
// sets are split into several groups over the same weights.
struct GemvGroup {
  const uint8_t *w0;        // weight (gate for the fused kernel)
  const float *s0;          // its scale grid
  const uint8_t *w1;        // up weight (fused kernel only)
  const float *s1;          // its scale grid
  const CUtensorMap *tm0;   // 2-D TMA maps of w0 / w1 in device memory
  const CUtensorMap *tm1;   //   (128 B x 128-row boxes, 64 for QKV layouts)
  uint32_t tok_begin;       // first slot in the token list / output rows
  uint32_t count;           // 1..8 tokens
  uint32_t expert;          // expert id (diagnostics)
  uint32_t pad;
};

struct GemvArgs {
  const GemvGroup *groups;
  const uint32_t *n_groups_dev;  // device group count (nullptr: use n_groups)
  uint32_t n_groups;             // host group count (upper bound if n_groups_dev)
  uint32_t rows;                 // output rows per group (multiple of 64)
  uint32_t K;                    // input columns (multiple of 128, <= 4096)
  uint32_t scale_cols;           // columns of the weight scale grid (K / 128)
  uint32_t layout;               // PW_LAYOUT_*
  const uint32_t *tok_list;      // activation row of token slot i (nullptr: i)
  const uint8_t *x_codes;        // e4m3 activations [*, K] (quantized kernels)
  const float *x_scales;         // [*, K/128]
  const float *x_f32;            // f32 activations [*, K] (readable kernel)
  float *out;                    // out[(tok_begin + t) * out_stride + row] (may be null for kind 2)
  uint32_t out_stride;
  uint8_t *q_codes;              // kind 2: dynamic-FP8 codes of the SwiGLU output [*, rows]
  float *q_scales;               //   and its per-128-row scales [*, rows / 128]
  uint32_t round_bf16;           // bf16-round the f32 result on store
  uint32_t *flags;
  uint32_t early_weights;        // PDL: weights and groups are ready before the predecessor
                                 //   ends, so the producer may stream them before waiting
  uint16_t *gate_bf16;           // tcgen05 kind 2: bf16(gate) and bf16(up) [*, rows], the
  uint16_t *up_bf16;             //   staged SwiGLU's inputs (k_swiglu_quant finishes it)
  uint16_t *out_bf16;            // tcgen05 kind 0 with round_bf16: the rounded result as bf16 bits
                                 //   [*, out_stride] instead of f32 in out
  uint8_t *const *peer_base;     // tcgen05 kind 0, expert parallelism: bf16 row p goes to
  uint64_t peer_off;             //   peer_base[row_rank[p]] + peer_off + row_place[p] * 2 * out_stride
  const uint32_t *row_rank;      //   (another GPU's window, plain 16-byte stores over NVLink)
  const uint32_t *row_place;
  uint32_t max_count;            // largest group token count (readable GEMV width bucket; 0: up to 8)
  uint32_t splits;               // GEMV split-K over the 8-leaf K tree: 1, 2, 4 or 8
  float *split_ws;               //   partial sums [tile][split][mats][128 rows][8 tokens]
  uint32_t *split_cnt;           //   per-tile arrival counters (zero; reset by the last CTA)
  const GemvGroup *l2_next;      // optional: the next kernel's groups (same count); CTAs with
  uint32_t l2_rows, l2_cols;     //   no unit of their own prefetch those groups' w0 [rows, cols]
                                 //   into L2 while the others stream
};

// Wide-width grouped GEMM (tcgen05): the GEMV arguments plus TMA maps of the
// activation codes [rows, K] (view {128 B, rows, K/128}); map i has a box of
// {128, 32 (i + 1) tokens, 2} so that a group loads only its own 32-token chunks.
struct GemmArgs {
  GemvArgs g;
  CUtensorMap xmap[4];
};
// Tokens per group (TN) of the tcgen05 GEMM (128 for every kind).
int gemm_tc_tokens(int kind);
cudaError_t launch_gemm_tc(int kind, const GemmArgs &args, int grid, cudaStream_t stream);
bool encode_act_maps(CUtensorMap (&out)[4], const void *base, uint32_t rows, uint32_t cols);
cudaError_t launch_gather_rows(const uint8_t *codes, const float *scales, const uint32_t *idx, uint32_t n,
                               uint32_t K, uint8_t *out_codes, float *out_scales, cudaStream_t stream);

// Kernel launchers (pw_kernels.cu).  All enqueue on `stream` and return the
// launch status.
// rows_dev (optional): the row count lives on the device; `rows` bounds it.
// zero (optional): n_zero words cleared by the kernel before anything after it
// in a PDL chain reads them (the chain's split-K counters).
cudaError_t launch_quantize(const float *x, uint32_t rows, uint32_t cols, uint8_t *codes, float *scales,
                            uint32_t *flags, cudaStream_t stream, const uint32_t *rows_dev = nullptr,
                            uint32_t *zero = nullptr, uint32_t n_zero = 0);
// kind: 0 = block-scaled (quantized x) over each group's w0/s0, 1 = readable
// (f32 x), 2 = fused gate/up SwiGLU over w0/s0 and w1/s1, 3 = block-scaled
// over w1/s1 (the unfused up projection)
cudaError_t launch_gemv(int kind, const GemvArgs &args, int grid, cudaStream_t stream);
int gemv_max_ctas(int num_sms);
cudaError_t launch_gemv_mma(int kind, const GemvArgs &args, int grid, cudaStream_t stream);
// The same kinds on tcgen05 / TMEM for PW_LAYOUT_PLAIN weights (pw_gemv_tc.cu).
cudaError_t launch_gemv_tc(int kind, const GemvArgs &args, int grid, cudaStream_t stream);
cudaError_t launch_round_bf16(float *v, uint32_t n, uint32_t *flags, cudaStream_t stream);
// Router logits (or, from 64 tokens, their per-slice sums) into `scratch`
// (router_scratch_floats floats), then the sigmoid no-aux top-8.
size_t router_scratch_floats(uint32_t tokens, uint32_t experts, uint32_t hidden);
// w: [experts, hidden] router weight, f32 or bf16 bits (w_dtype = PW_ROUTER_*).
// work: two words, zero before the first launch; the kernels leave them zero.
// q_codes / q_scales (optional, only where router_fuses_quantize(tokens)):
// the router's logits kernel also writes x's dynamic FP8 codes and scales,
// byte-identical to launch_quantize.
bool router_fuses_quantize(uint32_t tokens);
cudaError_t launch_router(const float *x, uint32_t tokens, const void *w, uint32_t w_dtype, const float *bias,
                          uint32_t experts, uint32_t hidden, float *scratch, uint32_t *selected, float *weights,
                          uint32_t *tie_rows, uint32_t *flags, uint32_t *work, int num_sms, cudaStream_t stream,
                          uint8_t *q_codes = nullptr, float *q_scales = nullptr);

// Device-side schedule for a routed layer: from selected [tokens, 8] build
// placements ordered by (expert asc, position asc) and the GEMV groups.
struct ScheduleOut {
  uint32_t *offsets;        // [experts + 1]
  uint32_t *placement_tok;  // [tokens*8] token position of placement p
  float *placement_w;       // [tokens*8] route weight of placement p
  uint32_t *slot_place;     // [tokens*8] placement index of (token, slot), slots in ascending expert
  GemvGroup *gu_groups;     // gate/up groups (<= tokens*8 + experts)
  GemvGroup *dn_groups;     // down groups
  uint32_t *n_groups;       // [1] number of groups
  uint32_t *counters;       // [4] unique experts, placements, max count, tie rows (stats)
  uint32_t *work;           // [schedule_work_words(experts)] scratch
};
size_t schedule_work_words(uint32_t experts);
struct BankTable {
  const uint8_t *const *gate_w;
  const float *const *gate_s;
  const uint8_t *const *up_w;
  const float *const *up_s;
  const uint8_t *const *down_w;
  const float *const *down_s;
  const CUtensorMap *gate_tm;  // [experts] each
  const CUtensorMap *up_tm;
  const CUtensorMap *down_tm;
};

// Host: encode the 2-D TMA map of one row-major e4m3 matrix [rows, cols]
// (box 128 B x box_rows, 128B swizzle).  row_stride (bytes, 0 = cols) lets the
// map cover a column slice of a wider matrix.  Returns false on failure.
bool encode_weight_map(CUtensorMap *out, const void *base, uint32_t rows, uint32_t cols, uint32_t box_rows,
                       uint32_t box_kb = 0, uint32_t row_stride = 0);
// y[i] = (bf16-rounded if round) sum over the n_parts partials p[k * n + i],
// added in k order.
cudaError_t launch_sum_partials(const float *p, uint32_t n_parts, uint64_t n, float *y, uint32_t round,
                                uint32_t *flags, cudaStream_t stream);
uint32_t map_box_rows(uint32_t layout);
// chunk: tokens per GEMV/GEMM group (8 for the GEMV, gemm_tc_tokens(2) for the GEMM);
// one launch up to 256 tokens, three above (schedule_launches)
uint32_t schedule_launches(uint32_t tokens);
cudaError_t launch_schedule(const uint32_t *selected, const float *weights, uint32_t tokens, uint32_t experts,
                            const BankTable &bank, const ScheduleOut &out, uint32_t *flags, uint32_t chunk,
                            cudaStream_t stream);
// residual (optional, [tokens, hidden]): y = bf16(residual + bf16(sum)), the
// decoder layer's residual add, instead of y = bf16(sum).
cudaError_t launch_combine(const float *down, const uint32_t *slot_place, const float *placement_w,
                           uint32_t tokens, uint32_t hidden, float *y, uint32_t *flags, cudaStream_t stream,
                           const float *residual = nullptr);
// The same combine over bf16 down rows (the expert-parallel return path; the
// rows are bf16-rounded, so the result is identical).
cudaError_t launch_combine_bf16(const uint16_t *down, const uint32_t *slot_place, const float *placement_w,
                                uint32_t tokens, uint32_t hidden, float *y, uint32_t *flags, cudaStream_t stream,
                                const float *residual = nullptr);
// RMSNorm (src/text_endpoint.rs:2939) of x [rows, cols] fused with the dynamic
// FP8 quantization of its output: xn (optional) receives the normalized f32
// rows, codes/scales (optional) their per-128 FP8 encoding, inv (optional)
// each row's inverse RMS.  cols % 256 == 0, cols <= 16384; w_dtype PW_NORM_*.
cudaError_t launch_rms_quantize(const float *x, uint32_t rows, uint32_t cols, const void *weight, uint32_t w_dtype,
                                float eps, float *xn, uint8_t *codes, float *scales, float *inv, uint32_t *flags,
                                cudaStream_t stream);
// out[idx[j]] = bf16 bits of rows[j] (rows already bf16-rounded), j < n.
cudaError_t launch_scatter_rows_bf16(const float *rows, const uint32_t *idx, uint32_t n, uint32_t cols,
                                     uint16_t *out, cudaStream_t stream);
// Staged SwiGLU of bf16 gate/up [rows, cols] followed by the hidden's dynamic
// FP8 quantization (per 128 values); h (f32, optional) receives the SwiGLU.
// silu_lut: 65536 bf16 staged-silu values (build_silu_lut).
cudaError_t launch_swiglu_quant(const uint16_t *gate, const uint16_t *up, uint32_t rows, uint32_t cols, float *h,
                                uint8_t *codes, float *scales, uint32_t *flags, const uint16_t *silu_lut,
                                int num_sms, cudaStream_t stream, const uint32_t *rows_dev = nullptr);
cudaError_t build_silu_lut(uint16_t *lut, cudaStream_t stream);
// n = rows * row_len elements; rows_dev (optional) caps the rows on the device
cudaError_t launch_swiglu(const float *gate, const float *up, float *h, uint32_t n, uint32_t *flags,
                          cudaStream_t stream, const uint32_t *rows_dev = nullptr, uint32_t row_len = 1);
cudaError_t launch_validate_fp8(const uint8_t *w, uint64_t n, const float *s, uint64_t ns,
                                unsigned long long *first_bad, uint32_t *flags, cudaStream_t stream);

// Expert-parallel window of one rank (byte offsets from its base): flags
// written by peers (ready for an epoch, data sent, rows returned), the
// mailbox (per-source per-local-expert counts and the source's placement
// index of its first row for this owner), the receive
// slots (source s: rows [s * slot_rows, (s + 1) * slot_rows)) and the
// returned bf16 rows of this rank's own placements.
struct EpWindow {
  uint64_t flag_ready, flag_data, flag_ret, mail_cnt, mail_base, recv_codes, recv_scales, ret_rows, total;
  uint32_t G, L, H, slot_rows;
};

struct EpArgs {
  uint8_t *const *peers;  // device array: each rank's window base (this rank's too)
  EpWindow w;
  uint32_t rank, epoch;
  uint32_t *flags;
  uint64_t deadline_ns;
};

cudaError_t launch_ep_dispatch(const EpArgs &e, const uint32_t *offsets, const uint8_t *codes, const float *scales,
                               uint32_t P, uint32_t *ctr, int grid, cudaStream_t stream);
cudaError_t launch_ep_plan(const EpArgs &e, const BankTable &bank, uint32_t chunk, uint32_t cap, uint32_t *perm,
                           uint32_t *src_rank, uint32_t *src_place, GemvGroup *gu, GemvGroup *dn, uint32_t *n_groups,
                           uint32_t *p_recv, cudaStream_t stream);
cudaError_t launch_ep_gather(const EpArgs &e, const uint32_t *perm, const uint32_t *p_recv, uint8_t *codes,
                             float *scales, int grid, cudaStream_t stream);
// After a down GEMM that stored its rows into the peers' windows: make them
// visible system-wide and release flag_ret[rank] = epoch in every window.
cudaError_t launch_ep_release(const EpArgs &e, cudaStream_t stream);
cudaError_t launch_ep_return(const EpArgs &e, const float *down, const uint32_t *src_rank, const uint32_t *src_place,
                             const uint32_t *p_recv, uint32_t *ctr, int grid, cudaStream_t stream);
cudaError_t launch_ep_wait_returns(const EpArgs &e, cudaStream_t stream);

// NCCL, dlopen'ed on first use (pw_nccl.cu).  Every call that can wait takes
// a deadline in seconds; ncclInProgress past it means "abort the comm".
namespace nccl {
struct Transfer {
  const void *ptr;
  size_t bytes;
  int peer;
};
bool load(std::string &err);
const char *error_string(ncclResult_t r);
ncclResult_t unique_id(ncclUniqueId *id);
ncclResult_t init_rank(ncclComm_t *comm, int world, const ncclUniqueId &id, int rank, double deadline_s);
ncclResult_t async_error(ncclComm_t comm);
void abort_comm(ncclComm_t comm);
ncclResult_t destroy(ncclComm_t comm, double deadline_s);
ncclResult_t all_gather(const void *send, void *recv, size_t count, ncclDataType_t t, ncclComm_t comm,
                        cudaStream_t s, double deadline_s);
// One grouped round of point-to-point byte transfers.
ncclResult_t exchange(const Transfer *sends, int n_sends, const Transfer *recvs, int n_recvs, ncclComm_t comm,
                      cudaStream_t s, double deadline_s);
}  // namespace nccl

}  // namespace pw
