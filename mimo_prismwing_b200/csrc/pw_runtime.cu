// pw_runtime.cu -- the C ABI (include/pw_cuda.h): argument validation, the
// runtime object (stream, scratch arena, error-flag word), host<->device
// staging and the kernel sequences of each entry point.
//
// Host-side orchestration mirrors the reference's WideMetalMoeRuntime
// (src/wide_metal_moe.rs:165-1316): validate shapes before dispatch, run the
// whole call as one stream of kernels, then fail closed on any device error
// bit or non-finite output.  Unlike the reference, nothing is gathered or
// scheduled on the host for pw_moe_layer: routing, scheduling and combine all
// run on the device.
#include <chrono>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <new>
#include <string>
#include <thread>
#include <unordered_map>
#include <vector>

#include <cuda.h>
#include <cuda_runtime.h>

#include "pw_cuda.h"
#include "pw_internal.h"

using namespace pw;

// ------------------------------------------------------------ TMA maps
namespace pw {
typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void *p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

uint32_t map_box_rows(uint32_t layout) { return layout == PW_LAYOUT_PLAIN ? 128u : 64u; }

// Activation codes [rows, cols] for the tcgen05 GEMM: view {128 B, rows,
// k-blocks}, boxes {128, 32 / 64 / 96 / 128 tokens, 2 k-blocks}; rows past the
// end of the buffer read as zeros.
bool encode_act_maps(CUtensorMap (&out)[4], const void *base, uint32_t rows, uint32_t cols) {
  EncodeTiledFn fn = encode_fn();
  if (!fn || cols % 128u || rows == 0) return false;
  cuuint64_t dims[3] = {128u, rows, cols / 128u};
  cuuint64_t strides[2] = {cols, 128u};
  cuuint32_t estr[3] = {1u, 1u, 1u};
  for (uint32_t i = 0; i < 4; ++i) {
    cuuint32_t box[3] = {128u, 32u * (i + 1u), 2u};
    if (fn(&out[i], CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void *>(base), dims, strides, box, estr,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return false;
  }
  return true;
}

// The weight is viewed as {128 B, rows, k-blocks} with strides {cols, 128}:
// a box of {128, box_rows, 256 / box_rows} is 32 KB and lands row-major in
// shared memory (one 128-byte line per row and k-block), 128B-swizzled.
// box_kb != 0 overrides the k-blocks per box (the tcgen05 GEMM's QKV tiles
// load {128, 64, 1} boxes).
bool encode_weight_map(CUtensorMap *out, const void *base, uint32_t rows, uint32_t cols, uint32_t box_rows,
                       uint32_t box_kb, uint32_t row_stride) {
  EncodeTiledFn fn = encode_fn();
  if (!fn || cols % 128u || (row_stride && (row_stride < cols || row_stride % 16u))) return false;
  cuuint64_t dims[3] = {128u, rows, cols / 128u};
  cuuint64_t strides[2] = {row_stride ? row_stride : cols, 128u};
  cuuint32_t box[3] = {128u, box_rows, box_kb ? box_kb : 256u / box_rows};
  cuuint32_t estr[3] = {1u, 1u, 1u};
  return fn(out, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void *>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}
}  // namespace pw

// Expert-parallel state of a runtime (pw_ep_init).
struct EpState {
  ncclComm_t comm = nullptr;
  int rank = 0, world = 1;
  double timeout_s = 60.0;
  bool dead = false;                 // aborted after an error or timeout
  void *scratch = nullptr;           // receive-side buffers, sized per call
  size_t cap = 0;
  uint32_t *h_off = nullptr;         // pinned: every rank's expert offsets
  size_t h_off_cap = 0;
  void *h_plan = nullptr;            // pinned: row permutation + expert groups
  size_t h_plan_cap = 0;
  // peer-memory transport (default)
  bool p2p = true;
  uint32_t max_tokens = 2048;        // per rank and call; sizes the receive slots
  void *win = nullptr;               // this rank's window
  EpWindow w{};
  std::vector<void *> peer_win;      // IPC mappings of the other ranks' windows
  uint8_t **d_peers = nullptr;       // device array of every rank's window base
  uint32_t *d_ctr = nullptr;         // last-CTA counters of dispatch / return
  uint32_t epoch = 0;
};

struct pw_runtime {
  int device = 0;
  uint32_t flags = 0;
  int num_sms = 148;
  cudaStream_t own_stream = nullptr;
  cudaStream_t stream = nullptr;
  uint32_t *d_flags = nullptr;            // error-flag word
  unsigned long long *d_bad = nullptr;    // validation: first bad byte
  uint32_t *d_ties = nullptr;             // router tie rows
  uint32_t *d_router_work = nullptr;      // router unit counters (two words, left zero)
  void *scratch = nullptr;
  size_t scratch_cap = 0;
  cudaEvent_t ev0 = nullptr, ev1 = nullptr;
  // profiling: an event before and after each timed launch group
  static constexpr int kProfEvents = 32;
  bool profiling = false;
  cudaEvent_t pev[kProfEvents] = {};
  int pclass[kProfEvents / 2] = {};
  int pcount = 0;
  uint32_t launches = 0;
  pw_profile last_profile{};
  std::string err;
  EpState *ep = nullptr;
  float *split_ws = nullptr;      // GEMV split-K partial sums (allocated on first use)
  uint32_t *split_cnt = nullptr;  // and per-tile arrival counters
  uint16_t *silu_lut = nullptr;   // staged silu of every bf16 pattern (built on first use)
  // Device-resident launch descriptors (TMA maps + group records) of the
  // projections and experts called so far, keyed by what they are built
  // from, so a repeated call enqueues only its kernels.
  static constexpr uint32_t kDescSlots = 512, kDescSlotBytes = 4096;
  uint8_t *desc = nullptr;
  std::unordered_map<std::string, uint32_t> desc_index;
  std::vector<std::string> desc_key;
  uint32_t desc_next = 0;
};

namespace pw {
int runtime_device(const pw_runtime *rt, int *device) {
  if (!rt || !device) return PW_ERR_ARGUMENT;
  *device = rt->device;
  return PW_OK;
}
}  // namespace pw

namespace {
enum ProfClass { P_QUANT, P_ROUTER, P_SCHED, P_GATEUP, P_DOWN, P_COMBINE, P_PROJ };

// Opens a timed launch group of class c (no-op unless profiling).
struct ProfScope {
  pw_runtime *rt;
  int idx = -1;
  ProfScope(pw_runtime *r, int c, uint32_t n_launches) : rt(r) {
    rt->launches += n_launches;
    if (!rt->profiling || rt->pcount >= pw_runtime::kProfEvents / 2) return;
    idx = rt->pcount++;
    rt->pclass[idx] = c;
    cudaEventRecord(rt->pev[2 * idx], rt->stream);
  }
  ~ProfScope() {
    if (idx >= 0) cudaEventRecord(rt->pev[2 * idx + 1], rt->stream);
  }
};
}  // namespace

struct pw_expert_bank {
  pw_runtime *rt = nullptr;
  void *owned = nullptr;  // weights uploaded by pw_bank_load (freed with the bank)
  uint32_t n = 0;
  uint32_t hidden = 0, inter = 0;
  void *d_table = nullptr;  // 6 arrays of n pointers
  CUtensorMap *d_maps = nullptr;  // 3 arrays of n TMA maps (gate, up, down)
  BankTable table{};
  std::vector<pw_expert_weights> host;
};

namespace pw {
void bank_adopt_memory(pw_expert_bank *bank, void *device_block) {
  if (bank) bank->owned = device_block;
}
}  // namespace pw

namespace {

int fail(pw_runtime *rt, int code, const char *fmt, ...) {
  if (rt) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    rt->err = buf;
  }
  return code;
}

#define CK(expr)                                                                               \
  do {                                                                                         \
    cudaError_t e_ = (expr);                                                                   \
    if (e_ != cudaSuccess) return fail(rt, PW_ERR_CUDA, "%s: %s", #expr, cudaGetErrorString(e_)); \
  } while (0)

// Bump allocator over the runtime's scratch buffer.  Sizes are computed in a
// first pass (dry run) so one cudaMalloc covers the whole call.
struct Arena {
  char *base = nullptr;
  size_t off = 0;
  template <class T>
  T *take(size_t count) {
    off = (off + 255) & ~size_t(255);
    T *p = reinterpret_cast<T *>(base ? base + off : nullptr);
    off += count * sizeof(T);
    return p;
  }
};

int ensure_scratch(pw_runtime *rt, size_t bytes) {
  if (bytes <= rt->scratch_cap) return PW_OK;
  size_t cap = rt->scratch_cap ? rt->scratch_cap : (size_t)1 << 20;
  while (cap < bytes) cap *= 2;
  CK(cudaStreamSynchronize(rt->stream));
  if (rt->scratch) CK(cudaFree(rt->scratch));
  rt->scratch = nullptr;
  rt->scratch_cap = 0;
  CK(cudaMalloc(&rt->scratch, cap));
  rt->scratch_cap = cap;
  return PW_OK;
}

double now_ms() {
  return std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now().time_since_epoch()).count();
}

bool tensor_ok(const pw_fp8_tensor *w) {
  return w && w->weight && w->scale && w->rows && w->cols && w->cols % 128u == 0;
}

// Shape contract of a projection under a layout (src/lib.rs:1217 for PLAIN,
// src/wide_metal_moe.rs:248-257 for the QKV layouts).
int check_projection(pw_runtime *rt, const pw_fp8_tensor *w, uint32_t layout) {
  if (!tensor_ok(w)) return fail(rt, PW_ERR_ARGUMENT, "FP8 tensor descriptor is null or empty");
  if (w->cols > 4096u) return fail(rt, PW_ERR_UNSUPPORTED, "input columns above 4096 are not supported");
  if (layout == PW_LAYOUT_PLAIN) {
    if (w->rows % 128u) return fail(rt, PW_ERR_SHAPE, "FP8 GEMV dimensions must be nonzero multiples of 128");
    if (w->scale_rows != w->rows / 128u || w->scale_cols != w->cols / 128u)
      return fail(rt, PW_ERR_SHAPE, "FP8 GEMV scale grid mismatch");
  } else if (layout == PW_LAYOUT_FULL_QKV) {
    if (w->rows != 13568u || w->cols != 4096u || w->scale_rows != 108u || w->scale_cols != 32u)
      return fail(rt, PW_ERR_SHAPE, "wide full-QKV layout mismatch");
  } else if (layout == PW_LAYOUT_SWA_QKV) {
    if (w->rows != 14848u || w->cols != 4096u || w->scale_rows != 116u || w->scale_cols != 32u)
      return fail(rt, PW_ERR_SHAPE, "wide SWA-QKV layout mismatch");
  } else {
    return fail(rt, PW_ERR_ARGUMENT, "unknown projection layout %u", layout);
  }
  return PW_OK;
}

int check_expert(pw_runtime *rt, const pw_expert_weights *w) {
  if (!w) return fail(rt, PW_ERR_ARGUMENT, "expert weights are null");
  int s;
  if ((s = check_projection(rt, &w->gate, PW_LAYOUT_PLAIN)) != PW_OK) return s;
  if ((s = check_projection(rt, &w->up, PW_LAYOUT_PLAIN)) != PW_OK) return s;
  if ((s = check_projection(rt, &w->down, PW_LAYOUT_PLAIN)) != PW_OK) return s;
  const uint32_t I = w->gate.rows, H = w->gate.cols;
  if (w->up.rows != I || w->up.cols != H || w->down.rows != H || w->down.cols != I)
    return fail(rt, PW_ERR_SHAPE, "expert gate/up/down shapes disagree");
  return PW_OK;
}

// Common call frame: host I/O staging, flag reset, events, final checks.
struct Call {
  pw_runtime *rt;
  uint32_t mem;
  pw_stats *stats;
  double t0;
  bool host() const { return (mem & PW_MEM_HOST) != 0; }
  bool async() const { return (mem & PW_MEM_ASYNC) != 0 && !host(); }

  int begin() {
    t0 = now_ms();
    rt->pcount = 0;
    rt->launches = 0;
    if (stats) memset(stats, 0, sizeof *stats);
    if (async() && stats) return fail(rt, PW_ERR_ARGUMENT, "stats cannot be returned by an asynchronous call");
    if (!async()) CK(cudaMemsetAsync(rt->d_flags, 0, sizeof(uint32_t), rt->stream));
    if (stats) CK(cudaEventRecord(rt->ev0, rt->stream));
    return PW_OK;
  }

  int stage_in(void *dst_dev, const void *src, size_t bytes) {
    if (bytes) CK(cudaMemcpyAsync(dst_dev, src, bytes, cudaMemcpyHostToDevice, rt->stream));
    return PW_OK;
  }

  int stage_out(void *dst_host, const void *src_dev, size_t bytes) {
    if (bytes) CK(cudaMemcpyAsync(dst_host, src_dev, bytes, cudaMemcpyDeviceToHost, rt->stream));
    return PW_OK;
  }

  // Wait, read the flag word and map it to a status.
  int finish(uint64_t weight_bytes) {
    if (stats) CK(cudaEventRecord(rt->ev1, rt->stream));
    if (async()) return PW_OK;
    uint32_t flags = 0;
    CK(cudaMemcpyAsync(&flags, rt->d_flags, sizeof flags, cudaMemcpyDeviceToHost, rt->stream));
    CK(cudaStreamSynchronize(rt->stream));
    if (stats) {
      stats->wall_ms = now_ms() - t0;
      CK(cudaEventElapsedTime(&stats->device_ms, rt->ev0, rt->ev1));
      stats->error_flags = flags;
      stats->weight_bytes = weight_bytes;
    }
    pw_profile prof{};
    for (int i = 0; i < rt->pcount; ++i) {
      float ms = 0.0f;
      CK(cudaEventElapsedTime(&ms, rt->pev[2 * i], rt->pev[2 * i + 1]));
      float *slot[] = {&prof.quantize_ms, &prof.router_ms, &prof.schedule_ms, &prof.gate_up_ms,
                       &prof.down_ms,     &prof.combine_ms, &prof.projection_ms};
      *slot[rt->pclass[i]] += ms;
    }
    prof.launches = rt->launches;
    rt->last_profile = prof;
    if (flags & PW_FLAG_WAIT_TIMEOUT) return fail(rt, PW_ERR_TIMEOUT, "a bounded device wait gave up (flags %u)", flags);
    if (flags & (PW_FLAG_NONFINITE_INPUT))
      return fail(rt, PW_ERR_NONFINITE, "non-finite input (device flags %u)", flags);
    if (flags & (PW_FLAG_NONFINITE_ROUND | PW_FLAG_NONFINITE_COMBINE | PW_FLAG_NONFINITE_FUSED |
                 PW_FLAG_NONFINITE_SWIGLU | PW_FLAG_BAD_WEIGHT))
      return fail(rt, PW_ERR_NONFINITE, "non-finite output (device flags %u)", flags);
    if (flags & (PW_FLAG_BAD_EXPERT_COUNT | PW_FLAG_ROUTE_WEIGHTS))
      return fail(rt, PW_ERR_SCHEDULE, "invalid routing on the device (flags %u)", flags);
    if (flags) return fail(rt, PW_ERR_DEVICE_FLAGS, "device error flags %u", flags);
    return PW_OK;
  }
};

// Projection groups for `width` tokens over one weight set (<= 8 per group).
std::vector<GemvGroup> width_groups(uint32_t width, const pw_fp8_tensor &a, const pw_fp8_tensor *b,
                                    const CUtensorMap *ma = nullptr, const CUtensorMap *mb = nullptr,
                                    uint32_t chunk = 8) {
  std::vector<GemvGroup> gs;
  for (uint32_t t = 0; t < width; t += chunk) {
    GemvGroup g{};
    g.w0 = a.weight;
    g.s0 = a.scale;
    g.w1 = b ? b->weight : nullptr;
    g.s1 = b ? b->scale : nullptr;
    g.tm0 = ma;
    g.tm1 = mb;
    g.tok_begin = t;
    g.count = width - t < chunk ? width - t : chunk;
    gs.push_back(g);
  }
  return gs;
}

GemvArgs gemv_args(const pw_runtime *rt, const GemvGroup *groups, uint32_t n_groups, uint32_t rows, uint32_t K,
                   uint32_t layout) {
  GemvArgs a{};
  a.groups = groups;
  a.n_groups = n_groups;
  a.rows = rows;
  a.K = K;
  a.scale_cols = K / 128u;
  a.layout = layout;
  a.flags = rt->d_flags;
  return a;
}

// Encode the maps of `n` matrices on the host into `host`; false on failure.
bool encode_maps(pw_runtime *rt, const pw_fp8_tensor *const *ts, size_t n, uint32_t layout, CUtensorMap *host) {
  for (size_t i = 0; i < n; ++i) {
    if (!encode_weight_map(&host[i], ts[i]->weight, ts[i]->rows, ts[i]->cols, map_box_rows(layout))) {
      fail(rt, PW_ERR_CUDA, "cuTensorMapEncodeTiled failed for a [%u, %u] weight", ts[i]->rows, ts[i]->cols);
      return false;
    }
  }
  return true;
}

// Width thresholds for the tcgen05 grouped GEMM: at or above these widths the
// weights are read once per group of up to 64-128 tokens instead of once per
// 8 tokens.
constexpr uint32_t kWideProjection = 32;   // pw_fp8_linear / pw_expert_forward widths
constexpr uint32_t kWideLayerTokens = 256; // routed-layer tokens (8 x tokens / experts >= 8)

int grid_for(const pw_runtime *rt, uint64_t units) {
  const uint64_t g = units < (uint64_t)rt->num_sms ? units : (uint64_t)rt->num_sms;
  return g ? (int)g : 1;
}

// GEMV split-K: with fewer 128-row tiles than SMs (a lone expert), spread
// each tile's K tree over 2, 4 or 8 CTAs.  Cost model per CTA: its units x
// (1/S of a tile's streaming time + a fixed ~3 us per unit for staging the
// activations and scales, publishing the partial sums and the last CTA's
// reduction), a tile streaming at ~40 GB/s per SM.  Results do not depend on
// the count (the GEMV adds K in a fixed 8-leaf tree).
constexpr size_t kSplitWsBytes = (size_t)16 << 20;
constexpr uint32_t kSplitCounters = 1024;
// next-kernel weights the decode GEMV may prefetch into L2 (126 MB) at once
constexpr uint64_t kL2PrefetchBytes = (uint64_t)72 << 20;

uint32_t gemv_splits(const pw_runtime *rt, uint64_t tiles, uint32_t K, uint32_t layout, int mats) {
  const uint32_t kbs = layout == PW_LAYOUT_PLAIN ? 2u : 4u;
  const uint32_t kcs = (K / 128u + kbs - 1u) / kbs;
  const uint64_t sms = (uint64_t)rt->num_sms;
  if (kcs % 8u || tiles == 0 || tiles >= sms) return 1u;
  const double tile_us = 128.0 * K * mats / 40e3;  // bytes / (40 GB/s) in us
  const double ovh = 3.0 / tile_us;                 // per-unit overhead, in tiles
  auto cost = [&](uint32_t S) { return (double)((tiles * S + sms - 1u) / sms) * (1.0 / S + ovh); };
  uint32_t bs = 1u;
  for (uint32_t S = 2u; S <= 8u; S *= 2u)
    if (cost(S) < cost(bs)) bs = S;
  return bs;
}

// Set up a GEMV launch over `tiles` (group, row-tile) pairs: split-K state
// and the grid.
int ensure_split_ws(pw_runtime *rt) {
  if (!rt->split_ws) {
    CK(cudaMalloc(&rt->split_ws, kSplitWsBytes));
    CK(cudaMalloc(&rt->split_cnt, kSplitCounters * sizeof(uint32_t)));
    CK(cudaMemset(rt->split_cnt, 0, kSplitCounters * sizeof(uint32_t)));
  }
  return PW_OK;
}

// counters_cleared: an earlier kernel of the same chain zeroes the counters
// (launch_quantize's `zero`), so no memset breaks the PDL chain here.
int gemv_launch_setup(pw_runtime *rt, GemvArgs &a, uint64_t tiles, int mats, int &grid,
                      bool counters_cleared = false) {
  const uint32_t S = gemv_splits(rt, tiles, a.K, a.layout, mats);
  grid = grid_for(rt, tiles * S);
  if (S == 1u) return PW_OK;
  if ((size_t)tiles * S * mats * 4096u > kSplitWsBytes || tiles > kSplitCounters) {
    grid = grid_for(rt, tiles);
    return PW_OK;
  }
  int s;
  if ((s = ensure_split_ws(rt)) != PW_OK) return s;
  // the last CTA of every tile resets its counter; clear them anyway in case
  // an earlier call was cut short
  if (!counters_cleared) CK(cudaMemsetAsync(rt->split_cnt, 0, tiles * sizeof(uint32_t), rt->stream));
  a.splits = S;
  a.split_ws = rt->split_ws;
  a.split_cnt = rt->split_cnt;
  return PW_OK;
}

// Launch descriptors of a projection (one matrix) or an expert (gate, up,
// down) at a given width: TMA maps first, then the group records, whose map
// pointers point at the maps in the same device slot.
struct Descs {
  const CUtensorMap *maps = nullptr;
  const GemvGroup *gu = nullptr, *dn = nullptr;  // dn: the expert's down groups
  uint32_t n_gu = 0, n_dn = 0;
};

// Looks up (or builds and uploads) the descriptors.  `b` (optional) is the
// second matrix of a fused pair (up), `c` (optional) an expert's down
// projection.  Maps use `box_rows` rows (and `box_kb` k-blocks when nonzero).
// Falls back to false when they do not fit a slot; a miss while the stream
// is being captured is an error (warm the call up first).
int get_descs(pw_runtime *rt, uint32_t tag, uint32_t width, uint32_t chunk, const pw_fp8_tensor &a,
              const pw_fp8_tensor *b, const pw_fp8_tensor *c, uint32_t box_rows, uint32_t box_kb, Descs &out,
              bool &cached) {
  cached = false;
  const uint32_t nmaps = 1u + (b ? 1u : 0u) + (c ? 1u : 0u);
  const uint32_t ng = (width + chunk - 1u) / chunk;
  const size_t bytes = nmaps * sizeof(CUtensorMap) + (size_t)ng * (c ? 2u : 1u) * sizeof(GemvGroup);
  if (bytes > pw_runtime::kDescSlotBytes) return PW_OK;
  std::string key(reinterpret_cast<const char *>(&tag), 4);
  auto put = [&key](const void *p, size_t n) { key.append(static_cast<const char *>(p), n); };
  put(&width, 4);
  put(&chunk, 4);
  put(&box_rows, 4);
  put(&box_kb, 4);
  for (const pw_fp8_tensor *t : {&a, b, c}) {
    if (t) put(t, sizeof *t);
    else key.append(sizeof(pw_fp8_tensor), '\0');
  }
  auto fill = [&](uint8_t *base) {
    const CUtensorMap *m = reinterpret_cast<const CUtensorMap *>(base);
    out.maps = m;
    const GemvGroup *g = reinterpret_cast<const GemvGroup *>(base + nmaps * sizeof(CUtensorMap));
    out.gu = g;
    out.n_gu = ng;
    out.dn = c ? g + ng : nullptr;
    out.n_dn = c ? ng : 0u;
  };
  auto it = rt->desc_index.find(key);
  if (it != rt->desc_index.end()) {
    fill(rt->desc + (size_t)it->second * pw_runtime::kDescSlotBytes);
    cached = true;
    return PW_OK;
  }
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  CK(cudaStreamIsCapturing(rt->stream, &cap));
  if (cap != cudaStreamCaptureStatusNone)
    return fail(rt, PW_ERR_ARGUMENT, "first call of this shape inside a stream capture: call it once before capturing");
  if (!rt->desc) {
    CK(cudaMalloc(&rt->desc, (size_t)pw_runtime::kDescSlots * pw_runtime::kDescSlotBytes));
    rt->desc_key.assign(pw_runtime::kDescSlots, std::string());
  }
  const uint32_t slot = rt->desc_next;
  rt->desc_next = (rt->desc_next + 1u) % pw_runtime::kDescSlots;
  if (!rt->desc_key[slot].empty()) {
    // evicting: kernels enqueued earlier may still read this slot
    CK(cudaStreamSynchronize(rt->stream));
    rt->desc_index.erase(rt->desc_key[slot]);
  }
  uint8_t *base = rt->desc + (size_t)slot * pw_runtime::kDescSlotBytes;
  std::vector<uint8_t> host(bytes);
  CUtensorMap *hm = reinterpret_cast<CUtensorMap *>(host.data());
  const pw_fp8_tensor *ts[3] = {&a, b ? b : c, b ? c : nullptr};
  for (uint32_t i = 0; i < nmaps; ++i)
    if (!encode_weight_map(&hm[i], ts[i]->weight, ts[i]->rows, ts[i]->cols, box_rows, box_kb))
      return fail(rt, PW_ERR_CUDA, "cuTensorMapEncodeTiled failed for a [%u, %u] weight", ts[i]->rows, ts[i]->cols);
  const CUtensorMap *dm = reinterpret_cast<const CUtensorMap *>(base);
  std::vector<GemvGroup> g1 = width_groups(width, a, b, dm, b ? dm + 1 : nullptr, chunk);
  memcpy(host.data() + nmaps * sizeof(CUtensorMap), g1.data(), g1.size() * sizeof(GemvGroup));
  if (c) {
    std::vector<GemvGroup> g2 = width_groups(width, *c, nullptr, dm + nmaps - 1u, nullptr, chunk);
    memcpy(host.data() + nmaps * sizeof(CUtensorMap) + ng * sizeof(GemvGroup), g2.data(),
           g2.size() * sizeof(GemvGroup));
  }
  // synchronous: the host buffer is temporary; a miss is a one-time cost
  CK(cudaStreamSynchronize(rt->stream));
  CK(cudaMemcpy(base, host.data(), bytes, cudaMemcpyHostToDevice));
  rt->desc_index[key] = slot;
  rt->desc_key[slot] = key;
  fill(base);
  cached = true;
  return PW_OK;
}

}  // namespace

// =================================================================== C ABI
extern "C" {

int pw_abi_version(void) { return PW_ABI_VERSION; }

int pw_runtime_create(int device, uint32_t flags, pw_runtime **out) {
  if (!out) return PW_ERR_ARGUMENT;
  *out = nullptr;
  pw_runtime *rt = new (std::nothrow) pw_runtime();
  if (!rt) return PW_ERR_ARGUMENT;
  rt->device = device;
  rt->flags = flags;
  auto bail = [&](cudaError_t) {
    pw_runtime_destroy(rt);
    return PW_ERR_CUDA;
  };
  cudaError_t e;
  if ((e = cudaSetDevice(device)) != cudaSuccess) return bail(e);
  cudaDeviceProp prop;
  if ((e = cudaGetDeviceProperties(&prop, device)) != cudaSuccess) return bail(e);
  if (prop.major < 10) {
    pw_runtime_destroy(rt);
    return PW_ERR_UNSUPPORTED;  // sm_100a only
  }
  rt->num_sms = prop.multiProcessorCount;
  if ((e = cudaStreamCreateWithFlags(&rt->own_stream, cudaStreamNonBlocking)) != cudaSuccess) return bail(e);
  rt->stream = rt->own_stream;
  if ((e = cudaMalloc(&rt->d_flags, 256)) != cudaSuccess) return bail(e);
  rt->d_bad = reinterpret_cast<unsigned long long *>(reinterpret_cast<char *>(rt->d_flags) + 64);
  rt->d_ties = reinterpret_cast<uint32_t *>(reinterpret_cast<char *>(rt->d_flags) + 128);
  rt->d_router_work = reinterpret_cast<uint32_t *>(reinterpret_cast<char *>(rt->d_flags) + 192);
  if ((e = cudaMemset(rt->d_flags, 0, 256)) != cudaSuccess) return bail(e);
  if ((e = cudaEventCreate(&rt->ev0)) != cudaSuccess) return bail(e);
  if ((e = cudaEventCreate(&rt->ev1)) != cudaSuccess) return bail(e);
  for (int i = 0; i < pw_runtime::kProfEvents; ++i)
    if ((e = cudaEventCreate(&rt->pev[i])) != cudaSuccess) return bail(e);
  *out = rt;
  return PW_OK;
}

void pw_runtime_destroy(pw_runtime *rt) {
  if (!rt) return;
  cudaSetDevice(rt->device);
  if (rt->stream) cudaStreamSynchronize(rt->stream);
  if (rt->ep) {
    // an aborted communicator (ep->comm cleared) is never finalized or destroyed
    if (rt->ep->comm) pw::nccl::destroy(rt->ep->comm, rt->ep->timeout_s);
    if (rt->ep->scratch) cudaFree(rt->ep->scratch);
    if (rt->ep->h_off) cudaFreeHost(rt->ep->h_off);
    if (rt->ep->h_plan) cudaFreeHost(rt->ep->h_plan);
    for (size_t g = 0; g < rt->ep->peer_win.size(); ++g)
      if (rt->ep->peer_win[g] && rt->ep->peer_win[g] != rt->ep->win) cudaIpcCloseMemHandle(rt->ep->peer_win[g]);
    if (rt->ep->win) cudaFree(rt->ep->win);
    if (rt->ep->d_peers) cudaFree(rt->ep->d_peers);
    if (rt->ep->d_ctr) cudaFree(rt->ep->d_ctr);
    delete rt->ep;
  }
  if (rt->scratch) cudaFree(rt->scratch);
  if (rt->split_ws) cudaFree(rt->split_ws);
  if (rt->split_cnt) cudaFree(rt->split_cnt);
  if (rt->silu_lut) cudaFree(rt->silu_lut);
  if (rt->desc) cudaFree(rt->desc);
  if (rt->d_flags) cudaFree(rt->d_flags);
  if (rt->ev0) cudaEventDestroy(rt->ev0);
  if (rt->ev1) cudaEventDestroy(rt->ev1);
  for (int i = 0; i < pw_runtime::kProfEvents; ++i)
    if (rt->pev[i]) cudaEventDestroy(rt->pev[i]);
  if (rt->own_stream) cudaStreamDestroy(rt->own_stream);
  delete rt;
}

const char *pw_last_error(const pw_runtime *rt) { return rt ? rt->err.c_str() : "null runtime"; }

int pw_set_stream(pw_runtime *rt, void *cuda_stream) {
  if (!rt) return PW_ERR_ARGUMENT;
  rt->stream = cuda_stream ? reinterpret_cast<cudaStream_t>(cuda_stream) : rt->own_stream;
  return PW_OK;
}

int pw_synchronize(pw_runtime *rt) {
  if (!rt) return PW_ERR_ARGUMENT;
  CK(cudaStreamSynchronize(rt->stream));
  return PW_OK;
}

int pw_set_profiling(pw_runtime *rt, int enable) {
  if (!rt) return PW_ERR_ARGUMENT;
  rt->profiling = enable != 0;
  return PW_OK;
}

int pw_last_profile(pw_runtime *rt, pw_profile *out) {
  if (!rt || !out) return PW_ERR_ARGUMENT;
  *out = rt->last_profile;
  return PW_OK;
}

int pw_read_error_flags(pw_runtime *rt, uint32_t *flags) {
  if (!rt || !flags) return PW_ERR_ARGUMENT;
  CK(cudaMemcpyAsync(flags, rt->d_flags, sizeof *flags, cudaMemcpyDeviceToHost, rt->stream));
  CK(cudaStreamSynchronize(rt->stream));
  return PW_OK;
}

// ------------------------------------------------------------------ quantize
int pw_quantize_fp8(pw_runtime *rt, const float *x, uint32_t rows, uint32_t cols, uint8_t *codes, float *scales,
                    uint32_t mem) {
  if (!rt || !x || !codes || !scales) return fail(rt, PW_ERR_ARGUMENT, "null argument");
  if (rows == 0 || cols == 0 || cols % 128u)
    return fail(rt, PW_ERR_SHAPE, "dynamic FP8 activation shape or value mismatch");
  CK(cudaSetDevice(rt->device));
  Call call{rt, mem, nullptr, 0};
  int s;
  if ((s = call.begin()) != PW_OK) return s;
  const size_t n = (size_t)rows * cols, ng = n / 128u;
  Arena ar;
  if (call.host()) {
    ar.take<float>(n);
    ar.take<uint8_t>(n);
    ar.take<float>(ng);
    if ((s = ensure_scratch(rt, ar.off)) != PW_OK) return s;
    ar = Arena{static_cast<char *>(rt->scratch), 0};
    float *dx = ar.take<float>(n);
    uint8_t *dc = ar.take<uint8_t>(n);
    float *ds = ar.take<float>(ng);
    if ((s = call.stage_in(dx, x, n * 4)) != PW_OK) return s;
    {
      ProfScope ps(rt, P_QUANT, 1);
      CK(launch_quantize(dx, rows, cols, dc, ds, rt->d_flags, rt->stream));
    }
    if ((s = call.stage_out(codes, dc, n)) != PW_OK) return s;
    if ((s = call.stage_out(scales, ds, ng * 4)) != PW_OK) return s;
  } else {
    ProfScope ps(rt, P_QUANT, 1);
    CK(launch_quantize(x, rows, cols, codes, scales, rt->d_flags, rt->stream));
  }
  return call.finish(0);
}

// ------------------------------------------------------------------ rms norm
static int check_norm(pw_runtime *rt, const pw_norm *n, uint32_t hidden) {
  if (!n || !n->weight) return fail(rt, PW_ERR_ARGUMENT, "norm descriptor is null");
  if (n->weight_dtype != PW_NORM_F32 && n->weight_dtype != PW_NORM_BF16)
    return fail(rt, PW_ERR_ARGUMENT, "norm weight_dtype must be PW_NORM_F32 or PW_NORM_BF16");
  if (!std::isfinite(n->epsilon) || n->epsilon <= 0.0f)
    return fail(rt, PW_ERR_ARGUMENT, "invalid RMSNorm epsilon");
  if (n->hidden != hidden || hidden == 0 || hidden % 256u || hidden > 16384u)
    return fail(rt, PW_ERR_SHAPE, "RMSNorm shape mismatch (hidden %u, a multiple of 256 up to 16384)", n->hidden);
  return PW_OK;
}

int pw_rms_norm(pw_runtime *rt, const pw_norm *norm, const float *x, uint32_t rows, float *y, float *inverse,
                uint32_t mem, pw_stats *stats) {
  if (!rt) return PW_ERR_ARGUMENT;
  if (!x || !y) return fail(rt, PW_ERR_ARGUMENT, "null argument");
  int s;
  if (!norm) return fail(rt, PW_ERR_ARGUMENT, "norm descriptor is null");
  if ((s = check_norm(rt, norm, norm->hidden)) != PW_OK) return s;
  if (rows == 0) return fail(rt, PW_ERR_SHAPE, "RMSNorm needs at least one row");
  CK(cudaSetDevice(rt->device));
  const uint32_t H = norm->hidden;
  const size_t n = (size_t)rows * H;
  Call call{rt, mem, stats, 0};
  if ((s = call.begin()) != PW_OK) return s;
  Arena ar;
  for (int pass = 0; pass < 2; ++pass) {
    if (pass == 1) {
      if ((s = ensure_scratch(rt, ar.off)) != PW_OK) return s;
      ar = Arena{static_cast<char *>(rt->scratch), 0};
    }
    float *dx = call.host() ? ar.take<float>(n) : const_cast<float *>(x);
    float *dy = call.host() ? ar.take<float>(n) : y;
    float *dinv = inverse && call.host() ? ar.take<float>(rows) : inverse;
    if (pass == 0) continue;
    if (call.host() && (s = call.stage_in(dx, x, n * 4)) != PW_OK) return s;
    {
      ProfScope ps(rt, P_QUANT, 1);
      CK(launch_rms_quantize(dx, rows, H, norm->weight, norm->weight_dtype, norm->epsilon, dy, nullptr, nullptr,
                             dinv, rt->d_flags, rt->stream));
    }
    if (call.host()) {
      if ((s = call.stage_out(y, dy, n * 4)) != PW_OK) return s;
      if (inverse && (s = call.stage_out(inverse, dinv, (size_t)rows * 4)) != PW_OK) return s;
    }
  }
  return call.finish((uint64_t)H * (norm->weight_dtype == PW_NORM_F32 ? 4u : 2u));
}

// ------------------------------------------------------------------ validate
int pw_validate_fp8(pw_runtime *rt, const pw_fp8_tensor *w, uint64_t *bad_offset) {
  if (!rt || !tensor_ok(w)) return fail(rt, PW_ERR_ARGUMENT, "FP8 tensor descriptor is null or empty");
  CK(cudaSetDevice(rt->device));
  Call call{rt, PW_MEM_DEVICE, nullptr, 0};
  int s;
  if ((s = call.begin()) != PW_OK) return s;
  CK(cudaMemsetAsync(rt->d_bad, 0xff, sizeof(unsigned long long), rt->stream));
  CK(launch_validate_fp8(w->weight, (uint64_t)w->rows * w->cols, w->scale, (uint64_t)w->scale_rows * w->scale_cols,
                         rt->d_bad, rt->d_flags, rt->stream));
  unsigned long long bad = ~0ull;
  CK(cudaMemcpyAsync(&bad, rt->d_bad, sizeof bad, cudaMemcpyDeviceToHost, rt->stream));
  s = call.finish(0);
  if (bad_offset) *bad_offset = bad;
  if (s == PW_ERR_NONFINITE) {
    if (bad != ~0ull) return fail(rt, PW_ERR_NONFINITE, "non-finite FP8 weight at byte offset %llu", bad);
    return fail(rt, PW_ERR_NONFINITE, "FP8 GEMV scale is non-finite");
  }
  return s;
}

// ------------------------------------------------------------ projections
// kind 0: block-scaled + bf16 round; 4: block-scaled, f32 output; 1: readable.
static int projection(pw_runtime *rt, int kind, const pw_fp8_tensor *w, uint32_t layout, const float *x,
                      uint32_t width, float *y, uint32_t mem, pw_stats *stats) {
  if (!rt) return PW_ERR_ARGUMENT;
  const uint32_t round = kind == 0 ? 1u : 0u;
  if (kind == 4) kind = 0;
  if (!x || !y) return fail(rt, PW_ERR_ARGUMENT, "null activation pointer");
  int s;
  if ((s = check_projection(rt, w, layout)) != PW_OK) return s;
  if (width == 0) return fail(rt, PW_ERR_SHAPE, "wide row count must be at least one");
  if (kind == 1 && width > 8u) return fail(rt, PW_ERR_SHAPE, "readable GEMV width must be 1..=8");
  CK(cudaSetDevice(rt->device));
  const uint32_t K = w->cols, N = w->rows;
  const size_t nx = (size_t)width * K, ny = (size_t)width * N;
  // wide block-scaled projections run on the tcgen05 GEMM (all layouts; the
  // QKV layouts load each 128-row tile as two 64-row source runs)
  const bool wide = kind != 1 && width >= kWideProjection;
  const uint32_t chunk = wide ? (uint32_t)gemm_tc_tokens(0) : 8u;
  const uint32_t box_rows = wide && layout != PW_LAYOUT_PLAIN ? 64u : map_box_rows(layout);
  const uint32_t box_kb = wide && layout != PW_LAYOUT_PLAIN ? 1u : 0u;
  // device-resident map and groups (built on the first call of this shape)
  Descs D;
  bool cached = false;
  if ((s = get_descs(rt, 2u + (uint32_t)kind, width, chunk, *w, nullptr, nullptr, box_rows, box_kb, D, cached)) !=
      PW_OK)
    return s;
  CUtensorMap hmap;
  if (!cached && !encode_weight_map(&hmap, w->weight, w->rows, w->cols, box_rows, box_kb))
    return fail(rt, PW_ERR_CUDA, "cuTensorMapEncodeTiled failed for a [%u, %u] weight", w->rows, w->cols);
  Call call{rt, mem, stats, 0};
  if ((s = call.begin()) != PW_OK) return s;
  // Narrow projections run as a programmatic-dependent-launch chain: the
  // GEMV streams its weights while the quantizer (or the previous call's
  // kernel) finishes, and the quantizer clears the split-K counters.
  const bool chain = !wide && !rt->profiling;
  if (chain && kind != 1 && (s = ensure_split_ws(rt)) != PW_OK) return s;
  PdlScope pdl(chain);
  Arena ar;
  for (int pass = 0; pass < 2; ++pass) {
    if (pass == 1) {
      if ((s = ensure_scratch(rt, ar.off)) != PW_OK) return s;
      ar = Arena{static_cast<char *>(rt->scratch), 0};
    }
    float *dx = call.host() ? ar.take<float>(nx) : const_cast<float *>(x);
    float *dy = call.host() ? ar.take<float>(ny) : y;
    uint8_t *dc = kind == 1 ? nullptr : ar.take<uint8_t>(nx);
    float *ds = kind == 1 ? nullptr : ar.take<float>(nx / 128u);
    CUtensorMap *dm = cached ? nullptr : ar.take<CUtensorMap>(1);
    std::vector<GemvGroup> groups;
    const GemvGroup *dg = D.gu;
    if (!cached) {
      groups = width_groups(width, *w, nullptr, dm, nullptr, chunk);
      dg = ar.take<GemvGroup>(groups.size());
    }
    const uint32_t n_groups = cached ? D.n_gu : (uint32_t)groups.size();
    if (pass == 0) continue;
    if (call.host() && (s = call.stage_in(dx, x, nx * 4)) != PW_OK) return s;
    if (!cached) {
      CK(cudaMemcpyAsync(dm, &hmap, sizeof hmap, cudaMemcpyHostToDevice, rt->stream));
      CK(cudaMemcpyAsync(const_cast<GemvGroup *>(dg), groups.data(), groups.size() * sizeof(GemvGroup),
                         cudaMemcpyHostToDevice, rt->stream));
    }
    GemvArgs a = gemv_args(rt, dg, n_groups, N, K, layout);
    a.out = dy;
    a.out_stride = N;
    if (kind == 1) {
      a.x_f32 = dx;
      a.round_bf16 = 0;
      a.max_count = width < 8u ? width : 8u;
    } else {
      ProfScope ps(rt, P_QUANT, 1);
      CK(launch_quantize(dx, width, K, dc, ds, rt->d_flags, rt->stream, nullptr, chain ? rt->split_cnt : nullptr,
                         chain ? kSplitCounters : 0u));
      a.x_codes = dc;
      a.x_scales = ds;
      a.round_bf16 = round;
      // the groups (cached, or copied in above) and the weights are final
      a.early_weights = chain ? 1u : 0u;
    }
    {
      ProfScope ps(rt, P_PROJ, 1);
      int grid = grid_for(rt, (uint64_t)n_groups * (N / (kind == 1 ? 64u : 128u)));
      if (!wide && kind != 1 &&
          (s = gemv_launch_setup(rt, a, (uint64_t)n_groups * (N / 128u), 1, grid, chain)) != PW_OK)
        return s;
      if (wide) {
        GemmArgs A{};
        A.g = a;
        if (!encode_act_maps(A.xmap, dc, width, K))
          return fail(rt, PW_ERR_CUDA, "cuTensorMapEncodeTiled failed for the activations");
        CK(launch_gemm_tc(0, A, grid, rt->stream));
      } else {
        CK(launch_gemv(kind, a, grid, rt->stream));
      }
    }
    if (call.host() && (s = call.stage_out(y, dy, ny * 4)) != PW_OK) return s;
  }
  return call.finish((uint64_t)N * K + (uint64_t)w->scale_rows * w->scale_cols * 4u);
}

int pw_fp8_gemv(pw_runtime *rt, const pw_fp8_tensor *w, const float *x, uint32_t width, float *y, uint32_t mem,
                pw_stats *stats) {
  return projection(rt, 1, w, PW_LAYOUT_PLAIN, x, width, y, mem, stats);
}

int pw_fp8_linear(pw_runtime *rt, const pw_fp8_tensor *w, uint32_t layout, const float *x, uint32_t width, float *y,
                  uint32_t mem, pw_stats *stats) {
  return projection(rt, (layout & PW_OUTPUT_F32) ? 4 : 0, w, layout & ~PW_OUTPUT_F32, x, width, y, mem, stats);
}

}  // extern "C"

// ------------------------------------------------------------------ expert
// Enqueue gate/up(+SwiGLU) -> quantize hidden -> down for `groups` whose
// token slots index rows of (xc, xs) through tok_list (nullptr: identity);
// hidden/down rows are indexed by slot.  Shared by the single expert and the
// host-scheduled layer.
static int enqueue_expert_chain(pw_runtime *rt, const GemvGroup *gu, const GemvGroup *dn, uint32_t n_groups,
                                const uint32_t *n_groups_dev, uint32_t slots, uint32_t H, uint32_t I,
                                const uint32_t *tok_list, const uint8_t *xc, const float *xs, float *hidden,
                                float *gate_tmp, float *up_tmp, uint8_t *hc, float *hs, float *down,
                                uint32_t down_round, uint64_t units_hint, const uint32_t *slots_dev = nullptr,
                                bool early = false) {
  const bool fused = (rt->flags & PW_RUNTIME_FUSED_GATE_UP) != 0;
  int s = PW_OK, grid_gu = 0;
  {
  ProfScope ps(rt, P_GATEUP, fused ? 1 : 3);
  if (fused) {
    // gate/up + SwiGLU + the hidden's dynamic FP8 quantization in one kernel
    GemvArgs a = gemv_args(rt, gu, n_groups, I, H, PW_LAYOUT_PLAIN);
    a.n_groups_dev = n_groups_dev;
    a.tok_list = tok_list;
    a.x_codes = xc;
    a.x_scales = xs;
    a.out = hidden;  // may be null
    a.out_stride = I;
    a.q_codes = hc;
    a.q_scales = hs;
    // early: the weights and groups were final before the chain started, so
    // under PDL the producer streams weights while the quantizer still runs
    a.early_weights = early && pdl_enabled() ? 1u : 0u;
    if ((s = gemv_launch_setup(rt, a, units_hint * (I / 128u), 2, grid_gu, early)) != PW_OK) return s;
    // few experts (a one-token decode layer): the gate/up CTAs that get no
    // tile prefetch the down weights into L2 while the others stream
    if (dn && a.splits <= 1u && (uint64_t)n_groups * H * I <= kL2PrefetchBytes) {
      a.l2_next = dn;
      a.l2_rows = H;
      a.l2_cols = I;
    }
    CK(launch_gemv(2, a, grid_gu, rt->stream));
  } else {
    // gate and up as two block-scaled projections, then the staged SwiGLU
    // (the reference's unfused schedule, src/wide_metal_moe.rs:1163-1187).
    GemvArgs a = gemv_args(rt, gu, n_groups, I, H, PW_LAYOUT_PLAIN);
    a.n_groups_dev = n_groups_dev;
    a.tok_list = tok_list;
    a.x_codes = xc;
    a.x_scales = xs;
    a.out_stride = I;
    a.out = gate_tmp;
    // gate and up take the same split, so the pair is bit-identical to the fused kernel
    if ((s = gemv_launch_setup(rt, a, units_hint * (I / 128u), 1, grid_gu)) != PW_OK) return s;
    CK(launch_gemv(0, a, grid_gu, rt->stream));
    // kind 3 is the same projection over each group's second matrix (up)
    GemvArgs b = a;
    b.out = up_tmp;
    CK(launch_gemv(3, b, grid_gu, rt->stream));
    CK(launch_swiglu(gate_tmp, up_tmp, hidden, slots * I, rt->d_flags, rt->stream, slots_dev, I));
  }
  }
  if (!fused) {
    ProfScope ps(rt, P_QUANT, 1);
    CK(launch_quantize(hidden, slots, I, hc, hs, rt->d_flags, rt->stream, slots_dev));
  }
  if (!dn) return PW_OK;  // the caller runs the down projection itself
  GemvArgs d = gemv_args(rt, dn, n_groups, H, I, PW_LAYOUT_PLAIN);
  d.n_groups_dev = n_groups_dev;
  d.x_codes = hc;
  d.x_scales = hs;
  d.out = down;
  d.out_stride = H;
  d.round_bf16 = down_round;
  // groups and weights were final before gate/up ran; with PDL the down
  // kernel's producer streams weights during gate/up's last wave
  d.early_weights = (pdl_enabled() && fused) ? 1u : 0u;
  int grid_dn = 0;
  if ((s = gemv_launch_setup(rt, d, units_hint * (H / 128u), 1, grid_dn, early && fused)) != PW_OK) return s;
  ProfScope ps(rt, P_DOWN, 1);
  CK(launch_gemv(0, d, grid_dn, rt->stream));
  return PW_OK;
}


// The expert chain on the tcgen05 GEMM.  xg / xsg are the gate/up input codes
// and scales laid out by group (tok_begin indexes rows directly).
// Expert parallelism: the down projection's bf16 rows go straight to the
// source ranks' windows (row p -> base[rank[p]] + off + place[p] * 2H).
struct PeerRows {
  uint8_t *const *base;
  uint64_t off;
  const uint32_t *rank, *place;
};

static int enqueue_expert_chain_wide(pw_runtime *rt, const GemvGroup *gu, const GemvGroup *dn, uint32_t n_groups,
                                     const uint32_t *n_groups_dev, uint32_t slots, uint32_t H, uint32_t I,
                                     const uint8_t *xg, const float *xsg, float *hidden, float *gate_tmp,
                                     float *up_tmp, uint8_t *hc, float *hs, float *down, uint32_t down_round,
                                     uint64_t units_hint, const uint32_t *slots_dev = nullptr,
                                     uint16_t *down16 = nullptr, const PeerRows *peer = nullptr) {
  const int grid_gu = grid_for(rt, units_hint * (I / 128u));
  const bool fused = (rt->flags & PW_RUNTIME_FUSED_GATE_UP) != 0;
  if (fused && !rt->silu_lut) {
    CK(cudaMalloc(&rt->silu_lut, 65536u * sizeof(uint16_t)));
    CK(build_silu_lut(rt->silu_lut, rt->stream));
  }
  {
    ProfScope ps(rt, P_GATEUP, fused ? 1 : 3);
    GemmArgs A{};
    A.g = gemv_args(rt, gu, n_groups, I, H, PW_LAYOUT_PLAIN);
    A.g.n_groups_dev = n_groups_dev;
    A.g.x_codes = xg;
    A.g.x_scales = xsg;
    A.g.out_stride = I;
    if (fused) {
      // gate and up in one kernel over shared activation tiles, bf16 out; the
      // staged SwiGLU + the hidden's quantization follow at full occupancy
      if (!encode_act_maps(A.xmap, xg, slots, H))
        return fail(rt, PW_ERR_CUDA, "cuTensorMapEncodeTiled failed for the activations");
      A.g.gate_bf16 = reinterpret_cast<uint16_t *>(gate_tmp);
      A.g.up_bf16 = reinterpret_cast<uint16_t *>(up_tmp);
      CK(launch_gemm_tc(2, A, grid_gu, rt->stream));
    } else {
      if (!encode_act_maps(A.xmap, xg, slots, H))
        return fail(rt, PW_ERR_CUDA, "cuTensorMapEncodeTiled failed for the activations");
      A.g.out = gate_tmp;
      CK(launch_gemm_tc(0, A, grid_gu, rt->stream));
      GemmArgs B = A;
      B.g.out = up_tmp;
      CK(launch_gemm_tc(3, B, grid_gu, rt->stream));
      CK(launch_swiglu(gate_tmp, up_tmp, hidden, slots * I, rt->d_flags, rt->stream, slots_dev, I));
    }
  }
  {
    ProfScope ps(rt, P_QUANT, 1);
    if (fused)
      CK(launch_swiglu_quant(reinterpret_cast<const uint16_t *>(gate_tmp), reinterpret_cast<const uint16_t *>(up_tmp),
                             slots, I, hidden, hc, hs, rt->d_flags, rt->silu_lut, rt->num_sms, rt->stream,
                             slots_dev));
    else
      CK(launch_quantize(hidden, slots, I, hc, hs, rt->d_flags, rt->stream, slots_dev));
  }
  if (!dn) return PW_OK;  // the caller runs the down projection itself
  GemmArgs D{};
  D.g = gemv_args(rt, dn, n_groups, H, I, PW_LAYOUT_PLAIN);
  D.g.n_groups_dev = n_groups_dev;
  D.g.x_codes = hc;
  D.g.x_scales = hs;
  D.g.out = down;
  D.g.out_stride = H;
  D.g.round_bf16 = down_round;
  if (down16 && down_round) D.g.out_bf16 = down16;  // bf16 rows: half the bytes for the combine
  if (peer && down_round) {
    D.g.peer_base = peer->base;
    D.g.peer_off = peer->off;
    D.g.row_rank = peer->rank;
    D.g.row_place = peer->place;
  }
  if (!encode_act_maps(D.xmap, hc, slots, I))
    return fail(rt, PW_ERR_CUDA, "cuTensorMapEncodeTiled failed for the hidden codes");
  ProfScope ps(rt, P_DOWN, 1);
  CK(launch_gemm_tc(0, D, grid_for(rt, units_hint * (H / 128u)), rt->stream));
  return PW_OK;
}

extern "C" {

int pw_expert_forward(pw_runtime *rt, const pw_expert_weights *w, const float *x, uint32_t width, float *y,
                      uint32_t mem, pw_stats *stats) {
  if (!rt) return PW_ERR_ARGUMENT;
  if (!x || !y) return fail(rt, PW_ERR_ARGUMENT, "null activation pointer");
  int s;
  if ((s = check_expert(rt, w)) != PW_OK) return s;
  if (width == 0) return fail(rt, PW_ERR_SHAPE, "expert width must be at least one");
  CK(cudaSetDevice(rt->device));
  const uint32_t H = w->gate.cols, I = w->gate.rows;
  const bool fused = (rt->flags & PW_RUNTIME_FUSED_GATE_UP) != 0;
  const bool wide = width >= kWideProjection;
  const uint32_t chunk = wide ? (uint32_t)gemm_tc_tokens(2) : 8u;
  // device-resident maps and groups (built on the first call of this shape)
  Descs D;
  bool cached = false;
  if ((s = get_descs(rt, 1u, width, chunk, w->gate, &w->up, &w->down, 128u, 0u, D, cached)) != PW_OK) return s;
  CUtensorMap hmaps[3];
  if (!cached) {
    const pw_fp8_tensor *ts[3] = {&w->gate, &w->up, &w->down};
    if (!encode_maps(rt, ts, 3, PW_LAYOUT_PLAIN, hmaps)) return PW_ERR_CUDA;
  }
  Call call{rt, mem, stats, 0};
  if ((s = call.begin()) != PW_OK) return s;
  Arena ar;
  for (int pass = 0; pass < 2; ++pass) {
    if (pass == 1) {
      if ((s = ensure_scratch(rt, ar.off)) != PW_OK) return s;
      ar = Arena{static_cast<char *>(rt->scratch), 0};
    }
    float *dx = call.host() ? ar.take<float>((size_t)width * H) : const_cast<float *>(x);
    float *dy = call.host() ? ar.take<float>((size_t)width * H) : y;
    uint8_t *xc = ar.take<uint8_t>((size_t)width * H);
    float *xs = ar.take<float>((size_t)width * H / 128u);
    float *hid = fused ? nullptr : ar.take<float>((size_t)width * I);
    // the wide fused chain stages bf16 gate/up here
    float *gt = fused && !wide ? nullptr : ar.take<float>((size_t)width * I);
    float *ut = fused && !wide ? nullptr : ar.take<float>((size_t)width * I);
    uint8_t *hc = ar.take<uint8_t>((size_t)width * I);
    float *hs = ar.take<float>((size_t)width * I / 128u);
    const GemvGroup *dgu = D.gu, *ddn = D.dn;
    std::vector<GemvGroup> gu, dn;
    CUtensorMap *dm = nullptr;
    if (!cached) {
      dm = ar.take<CUtensorMap>(3);
      gu = width_groups(width, w->gate, &w->up, dm, dm ? dm + 1 : nullptr, chunk);
      dn = width_groups(width, w->down, nullptr, dm ? dm + 2 : nullptr, nullptr, chunk);
      dgu = ar.take<GemvGroup>(gu.size());
      ddn = ar.take<GemvGroup>(dn.size());
    }
    const uint32_t n_groups = cached ? D.n_gu : (uint32_t)gu.size();
    if (pass == 0) continue;
    if (call.host() && (s = call.stage_in(dx, x, (size_t)width * H * 4)) != PW_OK) return s;
    if (!cached) {
      CK(cudaMemcpyAsync(dm, hmaps, sizeof hmaps, cudaMemcpyHostToDevice, rt->stream));
      CK(cudaMemcpyAsync(const_cast<GemvGroup *>(dgu), gu.data(), gu.size() * sizeof(GemvGroup),
                         cudaMemcpyHostToDevice, rt->stream));
      CK(cudaMemcpyAsync(const_cast<GemvGroup *>(ddn), dn.data(), dn.size() * sizeof(GemvGroup),
                         cudaMemcpyHostToDevice, rt->stream));
    }
    // quantize -> gate/up -> down as one PDL chain: the quantizer clears the
    // GEMVs' split-K counters, and each GEMV's producer streams its weights
    // while the kernel before it finishes
    const bool chain = !wide && fused && !rt->profiling;
    if (chain && (s = ensure_split_ws(rt)) != PW_OK) return s;
    PdlScope pdl(chain);
    {
      ProfScope ps(rt, P_QUANT, 1);
      CK(launch_quantize(dx, width, H, xc, xs, rt->d_flags, rt->stream, nullptr, chain ? rt->split_cnt : nullptr,
                         chain ? kSplitCounters : 0u));
    }
    if (wide)
      s = enqueue_expert_chain_wide(rt, dgu, ddn, n_groups, nullptr, width, H, I, xc, xs, hid, gt, ut, hc, hs, dy, 1,
                                    n_groups);
    else
      s = enqueue_expert_chain(rt, dgu, ddn, n_groups, nullptr, width, H, I, nullptr, xc, xs, hid, gt, ut, hc, hs, dy,
                               1, n_groups, nullptr, chain);
    if (s != PW_OK) return s;
    if (call.host() && (s = call.stage_out(y, dy, (size_t)width * H * 4)) != PW_OK) return s;
  }
  const uint64_t wb = 3ull * H * I + 4ull * (w->gate.scale_rows * w->gate.scale_cols * 2u +
                                             w->down.scale_rows * w->down.scale_cols);
  return call.finish(wb);
}

// --------------------------------------------------------------- dense MLP
// Reference: dense_mlp src/text_endpoint.rs:4266 (layer 0: gate and up
// [16384, 4096], staged SwiGLU, down [4096, 16384], each an fp8_linear).  The
// same chain as a routed expert at weight 1; an intermediate size above 4096
// runs the down projection over 4096-column slices of its K axis (the
// hidden's codes for a slice are copied contiguous, the weight slice is read
// in place through a strided TMA map) and adds the slice sums in slice order
// before the bf16 round.
constexpr uint32_t kDenseSlice = 4096;

int pw_dense_mlp(pw_runtime *rt, const pw_expert_weights *w, const float *x, uint32_t rows, float *y, uint32_t mem,
                 pw_stats *stats) {
  if (!rt) return PW_ERR_ARGUMENT;
  if (!x || !y || !w) return fail(rt, PW_ERR_ARGUMENT, "null argument");
  int s;
  if ((s = check_projection(rt, &w->gate, PW_LAYOUT_PLAIN)) != PW_OK) return s;
  if ((s = check_projection(rt, &w->up, PW_LAYOUT_PLAIN)) != PW_OK) return s;
  const uint32_t H = w->gate.cols, I = w->gate.rows;
  if (w->up.rows != I || w->up.cols != H) return fail(rt, PW_ERR_SHAPE, "gate and up shapes disagree");
  const pw_fp8_tensor &dw = w->down;
  if (!tensor_ok(&dw) || dw.rows != H || dw.cols != I || H % 128u || dw.scale_rows != H / 128u ||
      dw.scale_cols != I / 128u)
    return fail(rt, PW_ERR_SHAPE, "down projection must be [%u, %u] with a [%u, %u] scale grid", H, I, H / 128u,
                I / 128u);
  if (I > 65536u) return fail(rt, PW_ERR_UNSUPPORTED, "intermediate sizes above 65536 are not supported");
  if (rows == 0) return fail(rt, PW_ERR_SHAPE, "dense MLP needs at least one row");
  if (I <= kDenseSlice) return pw_expert_forward(rt, w, x, rows, y, mem, stats);
  CK(cudaSetDevice(rt->device));
  const uint32_t nsl = (I + kDenseSlice - 1u) / kDenseSlice;
  std::vector<CUtensorMap> hmaps(2 + nsl);
  {
    const pw_fp8_tensor *ts[2] = {&w->gate, &w->up};
    if (!encode_maps(rt, ts, 2, PW_LAYOUT_PLAIN, hmaps.data())) return PW_ERR_CUDA;
    for (uint32_t c = 0; c < nsl; ++c) {
      const uint32_t Kc = I - c * kDenseSlice < kDenseSlice ? I - c * kDenseSlice : kDenseSlice;
      if (!encode_weight_map(&hmaps[2 + c], dw.weight + (size_t)c * kDenseSlice, H, Kc, 128u, 0u, I))
        return fail(rt, PW_ERR_CUDA, "cuTensorMapEncodeTiled failed for a down-projection slice");
    }
  }
  const bool fused = (rt->flags & PW_RUNTIME_FUSED_GATE_UP) != 0;
  const bool wide = rows >= kWideProjection;
  Call call{rt, mem, stats, 0};
  if ((s = call.begin()) != PW_OK) return s;
  Arena ar;
  for (int pass = 0; pass < 2; ++pass) {
    if (pass == 1) {
      if ((s = ensure_scratch(rt, ar.off)) != PW_OK) return s;
      ar = Arena{static_cast<char *>(rt->scratch), 0};
    }
    float *dx = call.host() ? ar.take<float>((size_t)rows * H) : const_cast<float *>(x);
    float *dy = call.host() ? ar.take<float>((size_t)rows * H) : y;
    uint8_t *xc = ar.take<uint8_t>((size_t)rows * H);
    float *xs = ar.take<float>((size_t)rows * H / 128u);
    float *hid = fused ? nullptr : ar.take<float>((size_t)rows * I);
    float *gt = fused && !wide ? nullptr : ar.take<float>((size_t)rows * I);
    float *ut = fused && !wide ? nullptr : ar.take<float>((size_t)rows * I);
    uint8_t *hc = ar.take<uint8_t>((size_t)rows * I);
    float *hs = ar.take<float>((size_t)rows * I / 128u);
    uint8_t *hcc = ar.take<uint8_t>((size_t)rows * kDenseSlice);
    float *hsc = ar.take<float>((size_t)rows * kDenseSlice / 128u);
    float *part = ar.take<float>((size_t)nsl * rows * H);
    CUtensorMap *dm = ar.take<CUtensorMap>(2 + nsl);
    const uint32_t chunk = wide ? (uint32_t)gemm_tc_tokens(2) : 8u;
    std::vector<GemvGroup> gu = width_groups(rows, w->gate, &w->up, dm, dm ? dm + 1 : nullptr, chunk);
    std::vector<std::vector<GemvGroup>> dn(nsl);
    for (uint32_t c = 0; c < nsl; ++c) {
      pw_fp8_tensor sl = dw;
      sl.weight = dw.weight + (size_t)c * kDenseSlice;
      sl.scale = dw.scale + (size_t)c * (kDenseSlice / 128u);
      dn[c] = width_groups(rows, sl, nullptr, dm ? dm + 2 + c : nullptr, nullptr,
                           wide ? (uint32_t)gemm_tc_tokens(0) : 8u);
    }
    GemvGroup *dgu = ar.take<GemvGroup>(gu.size());
    std::vector<GemvGroup *> ddn(nsl);
    for (uint32_t c = 0; c < nsl; ++c) ddn[c] = ar.take<GemvGroup>(dn[c].size());
    if (pass == 0) continue;
    if (call.host() && (s = call.stage_in(dx, x, (size_t)rows * H * 4)) != PW_OK) return s;
    CK(cudaMemcpyAsync(dm, hmaps.data(), hmaps.size() * sizeof(CUtensorMap), cudaMemcpyHostToDevice, rt->stream));
    CK(cudaMemcpyAsync(dgu, gu.data(), gu.size() * sizeof(GemvGroup), cudaMemcpyHostToDevice, rt->stream));
    for (uint32_t c = 0; c < nsl; ++c)
      CK(cudaMemcpyAsync(ddn[c], dn[c].data(), dn[c].size() * sizeof(GemvGroup), cudaMemcpyHostToDevice,
                         rt->stream));
    {
      ProfScope ps(rt, P_QUANT, 1);
      CK(launch_quantize(dx, rows, H, xc, xs, rt->d_flags, rt->stream));
    }
    // gate/up, staged SwiGLU and the hidden's FP8 codes (no down projection)
    if (wide)
      s = enqueue_expert_chain_wide(rt, dgu, nullptr, (uint32_t)gu.size(), nullptr, rows, H, I, xc, xs, hid, gt, ut,
                                    hc, hs, nullptr, 1, gu.size());
    else
      s = enqueue_expert_chain(rt, dgu, nullptr, (uint32_t)gu.size(), nullptr, rows, H, I, nullptr, xc, xs, hid, gt,
                               ut, hc, hs, nullptr, 1, gu.size());
    if (s != PW_OK) return s;
    for (uint32_t c = 0; c < nsl; ++c) {
      const uint32_t Kc = I - c * kDenseSlice < kDenseSlice ? I - c * kDenseSlice : kDenseSlice;
      CK(cudaMemcpy2DAsync(hcc, Kc, hc + (size_t)c * kDenseSlice, I, Kc, rows, cudaMemcpyDeviceToDevice,
                           rt->stream));
      CK(cudaMemcpy2DAsync(hsc, (Kc / 128u) * 4u, hs + (size_t)c * (kDenseSlice / 128u), (I / 128u) * 4u,
                           (Kc / 128u) * 4u, rows, cudaMemcpyDeviceToDevice, rt->stream));
      GemvArgs d = gemv_args(rt, ddn[c], (uint32_t)dn[c].size(), H, Kc, PW_LAYOUT_PLAIN);
      d.scale_cols = I / 128u;  // the slice's scales are columns of the full grid
      d.x_codes = hcc;
      d.x_scales = hsc;
      d.out = part + (size_t)c * rows * H;
      d.out_stride = H;
      d.round_bf16 = 0;
      ProfScope ps(rt, P_DOWN, 1);
      if (wide) {
        GemmArgs D{};
        D.g = d;
        if (!encode_act_maps(D.xmap, hcc, rows, Kc))
          return fail(rt, PW_ERR_CUDA, "cuTensorMapEncodeTiled failed for the hidden codes");
        CK(launch_gemm_tc(0, D, grid_for(rt, (uint64_t)dn[c].size() * (H / 128u)), rt->stream));
      } else {
        int grid = 0;
        if ((s = gemv_launch_setup(rt, d, (uint64_t)dn[c].size() * (H / 128u), 1, grid)) != PW_OK) return s;
        CK(launch_gemv(0, d, grid, rt->stream));
      }
    }
    {
      ProfScope ps(rt, P_COMBINE, 1);
      CK(launch_sum_partials(part, nsl, (uint64_t)rows * H, dy, 1u, rt->d_flags, rt->stream));
    }
    if (call.host() && (s = call.stage_out(y, dy, (size_t)rows * H * 4)) != PW_OK) return s;
  }
  const uint64_t wb = 3ull * H * I + 4ull * (w->gate.scale_rows * w->gate.scale_cols * 2u + dw.scale_rows * dw.scale_cols);
  return call.finish(wb);
}

// ------------------------------------------------------------------- router
static uint64_t router_bytes(const pw_router *r) {
  return (uint64_t)r->experts * r->hidden * (r->weight_dtype == PW_ROUTER_F32 ? 4u : 2u) + r->experts * 4u;
}

static int check_router(pw_runtime *rt, const pw_router *r) {
  if (!r || !r->weight || !r->bias) return fail(rt, PW_ERR_ARGUMENT, "router descriptor is null");
  if (r->weight_dtype != PW_ROUTER_F32 && r->weight_dtype != PW_ROUTER_BF16)
    return fail(rt, PW_ERR_ARGUMENT, "router weight_dtype must be PW_ROUTER_F32 or PW_ROUTER_BF16");
  if (r->top_k != 8) return fail(rt, PW_ERR_UNSUPPORTED, "top_k must be 8");
  if (r->experts <= 8 || r->experts > 256 || r->hidden == 0 || r->hidden % 512u || r->hidden > 16384u)
    return fail(rt, PW_ERR_SHAPE, "router shape mismatch (experts 9..256, hidden a multiple of 512 up to 16384)");
  return PW_OK;
}

int pw_route(pw_runtime *rt, const pw_router *router, const float *x, uint32_t tokens, uint32_t *selected,
             float *weights, uint32_t mem, pw_stats *stats) {
  if (!rt) return PW_ERR_ARGUMENT;
  if (!x || !selected || !weights) return fail(rt, PW_ERR_ARGUMENT, "null argument");
  int s;
  if ((s = check_router(rt, router)) != PW_OK) return s;
  if (tokens == 0) return fail(rt, PW_ERR_SHAPE, "router needs at least one token");
  CK(cudaSetDevice(rt->device));
  const uint32_t E = router->experts, H = router->hidden;
  Call call{rt, mem, stats, 0};
  if ((s = call.begin()) != PW_OK) return s;
  Arena ar;
  for (int pass = 0; pass < 2; ++pass) {
    if (pass == 1) {
      if ((s = ensure_scratch(rt, ar.off)) != PW_OK) return s;
      ar = Arena{static_cast<char *>(rt->scratch), 0};
    }
    float *dx = call.host() ? ar.take<float>((size_t)tokens * H) : const_cast<float *>(x);
    uint32_t *dsel = call.host() ? ar.take<uint32_t>((size_t)tokens * 8) : selected;
    float *dw = call.host() ? ar.take<float>((size_t)tokens * 8) : weights;
    float *logits = ar.take<float>(router_scratch_floats(tokens, E, H));
    if (pass == 0) continue;
    if (call.host() && (s = call.stage_in(dx, x, (size_t)tokens * H * 4)) != PW_OK) return s;
    CK(cudaMemsetAsync(rt->d_ties, 0, 4, rt->stream));
    {
      ProfScope ps(rt, P_ROUTER, 2);
      CK(launch_router(dx, tokens, router->weight, router->weight_dtype, router->bias, E, H, logits, dsel, dw,
                       rt->d_ties, rt->d_flags, rt->d_router_work, rt->num_sms, rt->stream));
    }
    if (call.host()) {
      if ((s = call.stage_out(selected, dsel, (size_t)tokens * 32)) != PW_OK) return s;
      if ((s = call.stage_out(weights, dw, (size_t)tokens * 32)) != PW_OK) return s;
    }
  }
  uint32_t ties = 0;
  if (stats) CK(cudaMemcpyAsync(&ties, rt->d_ties, 4, cudaMemcpyDeviceToHost, rt->stream));
  s = call.finish(router_bytes(router));
  if (stats) stats->boundary_tie_rows = ties;
  return s;
}

// ------------------------------------------------- host-scheduled layer
int pw_moe_execute(pw_runtime *rt, const float *x, uint32_t rows, const pw_expert_binding *experts,
                   uint32_t n_experts, float *y, uint32_t mem, pw_stats *stats) {
  if (!rt) return PW_ERR_ARGUMENT;
  if (!x || !y || !experts || n_experts == 0) return fail(rt, PW_ERR_ARGUMENT, "wide MoE input or schedule mismatch");
  if (rows == 0) return fail(rt, PW_ERR_SHAPE, "wide row count must be at least one");
  int s;
  // schedule validation (src/wide_metal_moe.rs:858-868, 919-935)
  uint64_t total = 0;
  uint32_t max_count = 0;
  for (uint32_t i = 0; i < n_experts; ++i) {
    total += experts[i].count;
    max_count = experts[i].count > max_count ? experts[i].count : max_count;
  }
  if (total != (uint64_t)rows * 8u) return fail(rt, PW_ERR_SCHEDULE, "wide MoE input or schedule mismatch");
  // experts with many placements run on the tcgen05 GEMM (groups of up to 64)
  const bool wide = max_count > 16u;
  const uint32_t chunk = wide ? (uint32_t)gemm_tc_tokens(2) : 8u;
  const uint32_t H = experts[0].weights.gate.cols, I = experts[0].weights.gate.rows;
  std::vector<uint32_t> per_token(rows, 0);
  std::vector<uint32_t> placement_tok, slot_place((size_t)rows * 8u);
  std::vector<float> placement_w;
  std::vector<GemvGroup> gu, dn;
  std::vector<uint32_t> uniq;
  std::vector<CUtensorMap> hmaps((size_t)n_experts * 3);
  std::vector<size_t> group_binding;
  for (uint32_t i = 0; i < n_experts; ++i) {
    const pw_expert_binding &b = experts[i];
    if ((s = check_expert(rt, &b.weights)) != PW_OK) return s;
    if (b.weights.gate.cols != H || b.weights.gate.rows != I)
      return fail(rt, PW_ERR_SHAPE, "wide MoE expert %u identity mismatch", b.expert);
    if (b.count == 0 || !b.positions || !b.route_weights)
      return fail(rt, PW_ERR_SCHEDULE, "wide MoE expert %u identity mismatch", b.expert);
    bool seen = false;
    for (uint32_t u : uniq) seen = seen || u == b.expert;
    if (!seen) uniq.push_back(b.expert);
    const uint32_t begin = (uint32_t)placement_tok.size();
    for (uint32_t j = 0; j < b.count; ++j) {
      const uint32_t pos = b.positions[j];
      const float wt = b.route_weights[j];
      if (pos >= rows || !(wt == wt) || wt - wt != 0.0f)
        return fail(rt, PW_ERR_SCHEDULE, "wide MoE expert %u identity mismatch", b.expert);
      if (per_token[pos] >= 8u) return fail(rt, PW_ERR_SCHEDULE, "position %u has more than 8 placements", pos);
      slot_place[(size_t)pos * 8u + per_token[pos]++] = (uint32_t)placement_tok.size();
      placement_tok.push_back(pos);
      placement_w.push_back(wt);
    }
    for (uint32_t j = 0; j < b.count; j += chunk) {
      GemvGroup g{};
      g.w0 = b.weights.gate.weight;
      g.s0 = b.weights.gate.scale;
      g.w1 = b.weights.up.weight;
      g.s1 = b.weights.up.scale;
      g.tok_begin = begin + j;
      g.count = b.count - j < chunk ? b.count - j : chunk;
      g.expert = b.expert;
      gu.push_back(g);
      group_binding.push_back(i);
      GemvGroup d = g;
      d.w0 = b.weights.down.weight;
      d.s0 = b.weights.down.scale;
      d.w1 = nullptr;
      d.s1 = nullptr;
      dn.push_back(d);
    }
  }
  for (uint32_t t = 0; t < rows; ++t)
    if (per_token[t] != 8u) return fail(rt, PW_ERR_SCHEDULE, "position %u has %u placements, expected 8", t, per_token[t]);
  for (uint32_t i = 0; i < n_experts; ++i) {
    const pw_fp8_tensor *ts[3] = {&experts[i].weights.gate, &experts[i].weights.up, &experts[i].weights.down};
    if (!encode_maps(rt, ts, 3, PW_LAYOUT_PLAIN, &hmaps[(size_t)i * 3])) return PW_ERR_CUDA;
  }
  CK(cudaSetDevice(rt->device));
  const bool fused = (rt->flags & PW_RUNTIME_FUSED_GATE_UP) != 0;
  const uint32_t P = rows * 8u;
  Call call{rt, mem, stats, 0};
  if ((s = call.begin()) != PW_OK) return s;
  Arena ar;
  for (int pass = 0; pass < 2; ++pass) {
    if (pass == 1) {
      if ((s = ensure_scratch(rt, ar.off)) != PW_OK) return s;
      ar = Arena{static_cast<char *>(rt->scratch), 0};
    }
    float *dx = call.host() ? ar.take<float>((size_t)rows * H) : const_cast<float *>(x);
    float *dy = call.host() ? ar.take<float>((size_t)rows * H) : y;
    uint8_t *xc = ar.take<uint8_t>((size_t)rows * H);
    float *xs = ar.take<float>((size_t)rows * H / 128u);
    uint32_t *dtok = ar.take<uint32_t>(P);
    float *dpw = ar.take<float>(P);
    uint32_t *dslot = ar.take<uint32_t>(P);
    CUtensorMap *dm = ar.take<CUtensorMap>(hmaps.size());
    GemvGroup *dgu = ar.take<GemvGroup>(gu.size());
    GemvGroup *ddn = ar.take<GemvGroup>(dn.size());
    if (pass == 1) {
      for (size_t k = 0; k < gu.size(); ++k) {
        gu[k].tm0 = dm + group_binding[k] * 3;
        gu[k].tm1 = dm + group_binding[k] * 3 + 1;
        dn[k].tm0 = dm + group_binding[k] * 3 + 2;
        dn[k].tm1 = nullptr;
      }
    }
    float *hid = fused ? nullptr : ar.take<float>((size_t)P * I);
    float *gt = fused && !wide ? nullptr : ar.take<float>((size_t)P * I);
    float *ut = fused && !wide ? nullptr : ar.take<float>((size_t)P * I);
    uint8_t *hc = ar.take<uint8_t>((size_t)P * I);
    float *hs = ar.take<float>((size_t)P * I / 128u);
    float *down = ar.take<float>((size_t)P * H);
    uint8_t *xg = wide ? ar.take<uint8_t>((size_t)P * H) : nullptr;
    float *xsg = wide ? ar.take<float>((size_t)P * H / 128u) : nullptr;
    if (pass == 0) continue;
    if (call.host() && (s = call.stage_in(dx, x, (size_t)rows * H * 4)) != PW_OK) return s;
    CK(cudaMemcpyAsync(dm, hmaps.data(), hmaps.size() * sizeof(CUtensorMap), cudaMemcpyHostToDevice, rt->stream));
    CK(cudaMemcpyAsync(dtok, placement_tok.data(), P * 4u, cudaMemcpyHostToDevice, rt->stream));
    CK(cudaMemcpyAsync(dpw, placement_w.data(), P * 4u, cudaMemcpyHostToDevice, rt->stream));
    CK(cudaMemcpyAsync(dslot, slot_place.data(), P * 4u, cudaMemcpyHostToDevice, rt->stream));
    CK(cudaMemcpyAsync(dgu, gu.data(), gu.size() * sizeof(GemvGroup), cudaMemcpyHostToDevice, rt->stream));
    CK(cudaMemcpyAsync(ddn, dn.data(), dn.size() * sizeof(GemvGroup), cudaMemcpyHostToDevice, rt->stream));
    {
      ProfScope ps(rt, P_QUANT, 1);
      CK(launch_quantize(dx, rows, H, xc, xs, rt->d_flags, rt->stream));
    }
    if (wide) {
      {
        ProfScope ps(rt, P_QUANT, 1);
        CK(launch_gather_rows(xc, xs, dtok, P, H, xg, xsg, rt->stream));
      }
      s = enqueue_expert_chain_wide(rt, dgu, ddn, (uint32_t)gu.size(), nullptr, P, H, I, xg, xsg, hid, gt, ut, hc, hs,
                                    down, 1, gu.size(), nullptr, reinterpret_cast<uint16_t *>(down));
    } else {
      s = enqueue_expert_chain(rt, dgu, ddn, (uint32_t)gu.size(), nullptr, P, H, I, dtok, xc, xs, hid, gt, ut, hc, hs,
                               down, 1, gu.size());
    }
    if (s != PW_OK) return s;
    {
      ProfScope ps(rt, P_COMBINE, 1);
      if (wide)
        CK(launch_combine_bf16(reinterpret_cast<const uint16_t *>(down), dslot, dpw, rows, H, dy, rt->d_flags,
                               rt->stream));
      else
        CK(launch_combine(down, dslot, dpw, rows, H, dy, rt->d_flags, rt->stream));
    }
    if (call.host() && (s = call.stage_out(y, dy, (size_t)rows * H * 4)) != PW_OK) return s;
  }
  const pw_expert_weights &w0 = experts[0].weights;
  const uint64_t per_expert = 3ull * H * I + 4ull * (w0.gate.scale_rows * w0.gate.scale_cols * 2u +
                                                     w0.down.scale_rows * w0.down.scale_cols);
  s = call.finish(per_expert * uniq.size());
  if (stats) {
    stats->unique_experts = (uint32_t)uniq.size();
    stats->expert_rows = P;
  }
  return s;
}

// ---------------------------------------------------------------- banks
int pw_bank_create(pw_runtime *rt, const pw_expert_weights *experts, uint32_t n_experts, pw_expert_bank **out) {
  if (!rt) return PW_ERR_ARGUMENT;
  if (!experts || !out || n_experts == 0) return fail(rt, PW_ERR_ARGUMENT, "null bank argument");
  *out = nullptr;
  int s;
  for (uint32_t e = 0; e < n_experts; ++e) {
    if ((s = check_expert(rt, &experts[e])) != PW_OK) return s;
    if (experts[e].gate.rows != experts[0].gate.rows || experts[e].gate.cols != experts[0].gate.cols)
      return fail(rt, PW_ERR_SHAPE, "expert %u shape differs from expert 0", e);
  }
  CK(cudaSetDevice(rt->device));
  pw_expert_bank *bank = new (std::nothrow) pw_expert_bank();
  if (!bank) return fail(rt, PW_ERR_ARGUMENT, "out of host memory");
  bank->rt = rt;
  bank->n = n_experts;
  bank->hidden = experts[0].gate.cols;
  bank->inter = experts[0].gate.rows;
  bank->host.assign(experts, experts + n_experts);
  std::vector<const void *> table((size_t)n_experts * 6);
  for (uint32_t e = 0; e < n_experts; ++e) {
    table[0 * n_experts + e] = experts[e].gate.weight;
    table[1 * n_experts + e] = experts[e].gate.scale;
    table[2 * n_experts + e] = experts[e].up.weight;
    table[3 * n_experts + e] = experts[e].up.scale;
    table[4 * n_experts + e] = experts[e].down.weight;
    table[5 * n_experts + e] = experts[e].down.scale;
  }
  cudaError_t err = cudaMalloc(&bank->d_table, table.size() * sizeof(void *));
  if (err == cudaSuccess)
    err = cudaMemcpy(bank->d_table, table.data(), table.size() * sizeof(void *), cudaMemcpyHostToDevice);
  if (err != cudaSuccess) {
    pw_bank_destroy(bank);
    return fail(rt, PW_ERR_CUDA, "bank table: %s", cudaGetErrorString(err));
  }
  {
    std::vector<CUtensorMap> maps((size_t)n_experts * 3);
    for (uint32_t e = 0; e < n_experts; ++e) {
      const pw_fp8_tensor *ts[3] = {&experts[e].gate, &experts[e].up, &experts[e].down};
      for (int k = 0; k < 3; ++k) {
        if (!encode_weight_map(&maps[(size_t)k * n_experts + e], ts[k]->weight, ts[k]->rows, ts[k]->cols, 128u)) {
          pw_bank_destroy(bank);
          return fail(rt, PW_ERR_CUDA, "cuTensorMapEncodeTiled failed for expert %u", e);
        }
      }
    }
    err = cudaMalloc(&bank->d_maps, maps.size() * sizeof(CUtensorMap));
    if (err == cudaSuccess)
      err = cudaMemcpy(bank->d_maps, maps.data(), maps.size() * sizeof(CUtensorMap), cudaMemcpyHostToDevice);
    if (err != cudaSuccess) {
      pw_bank_destroy(bank);
      return fail(rt, PW_ERR_CUDA, "bank maps: %s", cudaGetErrorString(err));
    }
    bank->table.gate_tm = bank->d_maps;
    bank->table.up_tm = bank->d_maps + n_experts;
    bank->table.down_tm = bank->d_maps + 2 * (size_t)n_experts;
  }
  const void **d = static_cast<const void **>(bank->d_table);
  bank->table.gate_w = reinterpret_cast<const uint8_t *const *>(d + 0 * n_experts);
  bank->table.gate_s = reinterpret_cast<const float *const *>(d + 1 * n_experts);
  bank->table.up_w = reinterpret_cast<const uint8_t *const *>(d + 2 * n_experts);
  bank->table.up_s = reinterpret_cast<const float *const *>(d + 3 * n_experts);
  bank->table.down_w = reinterpret_cast<const uint8_t *const *>(d + 4 * n_experts);
  bank->table.down_s = reinterpret_cast<const float *const *>(d + 5 * n_experts);
  // fail-closed validation of every weight byte and scale, once
  for (uint32_t e = 0; e < n_experts; ++e) {
    const pw_fp8_tensor *ts[3] = {&experts[e].gate, &experts[e].up, &experts[e].down};
    for (const pw_fp8_tensor *t : ts) {
      uint64_t bad = ~0ull;
      if ((s = pw_validate_fp8(rt, t, &bad)) != PW_OK) {
        pw_bank_destroy(bank);
        return fail(rt, s, "expert %u: %s", e, rt->err.c_str());
      }
    }
  }
  *out = bank;
  return PW_OK;
}

void pw_bank_destroy(pw_expert_bank *bank) {
  if (!bank) return;
  if (bank->d_table || bank->d_maps || bank->owned) {
    cudaSetDevice(bank->rt->device);
    if (bank->d_table) cudaFree(bank->d_table);
    if (bank->d_maps) cudaFree(bank->d_maps);
    if (bank->owned) cudaFree(bank->owned);
  }
  delete bank;
}

// ------------------------------------------------------ device-routed layer
// The routed layer, optionally as the MoE half of a decoder layer: with
// `norm`, x is the post-attention residual stream, the layer's input is
// rms_norm(x) (fused with its FP8 quantization) and y = bf16(x + layer).
static int moe_layer_impl(pw_runtime *rt, const pw_norm *norm, const pw_router *router, const pw_expert_bank *bank,
                          const float *x, uint32_t tokens, float *y, uint32_t *selected, float *weights, uint32_t mem,
                          pw_stats *stats) {
  if (!rt) return PW_ERR_ARGUMENT;
  if (!x || !y || !bank) return fail(rt, PW_ERR_ARGUMENT, "null argument");
  int s;
  if ((s = check_router(rt, router)) != PW_OK) return s;
  if (bank->n != router->experts || bank->hidden != router->hidden)
    return fail(rt, PW_ERR_SHAPE, "router and expert bank disagree");
  if (norm && (s = check_norm(rt, norm, bank->hidden)) != PW_OK) return s;
  if (norm && x == y) return fail(rt, PW_ERR_ARGUMENT, "the block's output may not alias its residual input");
  if (tokens == 0) return fail(rt, PW_ERR_SHAPE, "routed layer needs at least one token");
  if (tokens > 2048u) return fail(rt, PW_ERR_UNSUPPORTED, "routed layer supports at most 2048 tokens per call");
  CK(cudaSetDevice(rt->device));
  const uint32_t H = bank->hidden, I = bank->inter, E = bank->n, P = tokens * 8u;
  // wide layers (prefill) run the experts on the tcgen05 GEMM in groups of up
  // to 64 placements; decode widths on the GEMV in groups of up to 8
  const bool wide = tokens >= kWideLayerTokens;
  const uint32_t chunk = wide ? (uint32_t)gemm_tc_tokens(2) : 8u;
  const uint32_t max_groups = P / chunk + E;  // >= sum over experts of ceil(count / chunk)
  const bool fused = (rt->flags & PW_RUNTIME_FUSED_GATE_UP) != 0;
  Call call{rt, mem, stats, 0};
  if ((s = call.begin()) != PW_OK) return s;
  Arena ar;
  uint32_t *counters = nullptr;
  for (int pass = 0; pass < 2; ++pass) {
    if (pass == 1) {
      if ((s = ensure_scratch(rt, ar.off)) != PW_OK) return s;
      ar = Arena{static_cast<char *>(rt->scratch), 0};
    }
    float *dx = call.host() ? ar.take<float>((size_t)tokens * H) : const_cast<float *>(x);
    float *dy = call.host() ? ar.take<float>((size_t)tokens * H) : y;
    float *dn = norm ? ar.take<float>((size_t)tokens * H) : dx;  // the layer input the router reads
    uint8_t *xc = ar.take<uint8_t>((size_t)tokens * H);
    float *xs = ar.take<float>((size_t)tokens * H / 128u);
    float *logits = ar.take<float>(router_scratch_floats(tokens, E, H));
    uint32_t *sel = ar.take<uint32_t>(P);
    float *wts = ar.take<float>(P);
    ScheduleOut so{};
    so.offsets = ar.take<uint32_t>(E + 1);
    so.placement_tok = ar.take<uint32_t>(P);
    so.placement_w = ar.take<float>(P);
    so.slot_place = ar.take<uint32_t>(P);
    so.gu_groups = ar.take<GemvGroup>(max_groups);
    so.dn_groups = ar.take<GemvGroup>(max_groups);
    so.n_groups = ar.take<uint32_t>(1);
    so.counters = ar.take<uint32_t>(4);
    so.work = ar.take<uint32_t>(schedule_work_words(E));
    float *hid = fused ? nullptr : ar.take<float>((size_t)P * I);
    float *gt = fused && !wide ? nullptr : ar.take<float>((size_t)P * I);
    float *ut = fused && !wide ? nullptr : ar.take<float>((size_t)P * I);
    uint8_t *hc = ar.take<uint8_t>((size_t)P * I);
    float *hs = ar.take<float>((size_t)P * I / 128u);
    float *down = ar.take<float>((size_t)P * H);
    uint8_t *xg = wide ? ar.take<uint8_t>((size_t)P * H) : nullptr;
    float *xsg = wide ? ar.take<float>((size_t)P * H / 128u) : nullptr;
    if (pass == 0) continue;
    counters = so.counters;
    if (call.host() && (s = call.stage_in(dx, x, (size_t)tokens * H * 4)) != PW_OK) return s;
    CK(cudaMemsetAsync(rt->d_ties, 0, 4, rt->stream));
    // the kernel chain below runs with programmatic dependent launch
    PdlScope pdl(!rt->profiling);
    // decode widths without a norm: the router's logits kernel quantizes x
    // for the experts too (one launch fewer on the chain's critical path)
    const bool fuse_quant = !norm && router_fuses_quantize(tokens);
    if (!fuse_quant) {
      ProfScope ps(rt, P_QUANT, 1);
      if (norm)
        CK(launch_rms_quantize(dx, tokens, H, norm->weight, norm->weight_dtype, norm->epsilon, dn, xc, xs, nullptr,
                               rt->d_flags, rt->stream));
      else
        CK(launch_quantize(dx, tokens, H, xc, xs, rt->d_flags, rt->stream));
    }
    {
      ProfScope ps(rt, P_ROUTER, 2);
      CK(launch_router(dn, tokens, router->weight, router->weight_dtype, router->bias, E, H, logits, sel, wts,
                       rt->d_ties, rt->d_flags, rt->d_router_work, rt->num_sms, rt->stream, fuse_quant ? xc : nullptr,
                       fuse_quant ? xs : nullptr));
    }
    {
      ProfScope ps(rt, P_SCHED, schedule_launches(tokens));
      CK(launch_schedule(sel, wts, tokens, E, bank->table, so, rt->d_flags, chunk, rt->stream));
    }
    // the grid covers the worst case; CTAs read the real group count
    if (wide) {
      {
        ProfScope ps(rt, P_QUANT, 1);
        CK(launch_gather_rows(xc, xs, so.placement_tok, P, H, xg, xsg, rt->stream));
      }
      s = enqueue_expert_chain_wide(rt, so.gu_groups, so.dn_groups, max_groups, so.n_groups, P, H, I, xg, xsg, hid,
                                    gt, ut, hc, hs, down, 1, max_groups, nullptr, reinterpret_cast<uint16_t *>(down));
    } else {
      s = enqueue_expert_chain(rt, so.gu_groups, so.dn_groups, max_groups, so.n_groups, P, H, I, so.placement_tok, xc,
                               xs, hid, gt, ut, hc, hs, down, 1, max_groups);
    }
    if (s != PW_OK) return s;
    {
      ProfScope ps(rt, P_COMBINE, 1);
      const float *residual = norm ? dx : nullptr;
      if (wide)
        CK(launch_combine_bf16(reinterpret_cast<const uint16_t *>(down), so.slot_place, so.placement_w, tokens, H, dy,
                               rt->d_flags, rt->stream, residual));
      else
        CK(launch_combine(down, so.slot_place, so.placement_w, tokens, H, dy, rt->d_flags, rt->stream, residual));
    }
    if (call.host()) {
      if ((s = call.stage_out(y, dy, (size_t)tokens * H * 4)) != PW_OK) return s;
      if (selected && (s = call.stage_out(selected, sel, (size_t)P * 4)) != PW_OK) return s;
      if (weights && (s = call.stage_out(weights, wts, (size_t)P * 4)) != PW_OK) return s;
    } else {
      if (selected) CK(cudaMemcpyAsync(selected, sel, (size_t)P * 4, cudaMemcpyDeviceToDevice, rt->stream));
      if (weights) CK(cudaMemcpyAsync(weights, wts, (size_t)P * 4, cudaMemcpyDeviceToDevice, rt->stream));
    }
  }
  uint32_t cnt[4] = {0, 0, 0, 0};
  uint32_t ties = 0;
  if (stats) {
    CK(cudaMemcpyAsync(cnt, counters, sizeof cnt, cudaMemcpyDeviceToHost, rt->stream));
    CK(cudaMemcpyAsync(&ties, rt->d_ties, 4, cudaMemcpyDeviceToHost, rt->stream));
  }
  const pw_expert_weights &w0 = bank->host[0];
  const uint64_t per_expert = 3ull * H * I + 4ull * (w0.gate.scale_rows * w0.gate.scale_cols * 2u +
                                                     w0.down.scale_rows * w0.down.scale_cols);
  s = call.finish(0);
  if (stats) {
    stats->unique_experts = cnt[0];
    stats->expert_rows = cnt[1];
    stats->boundary_tie_rows = ties;
    stats->weight_bytes = per_expert * cnt[0] + router_bytes(router);
  }
  return s;
}

int pw_moe_layer(pw_runtime *rt, const pw_router *router, const pw_expert_bank *bank, const float *x, uint32_t tokens,
                 float *y, uint32_t *selected, float *weights, uint32_t mem, pw_stats *stats) {
  return moe_layer_impl(rt, nullptr, router, bank, x, tokens, y, selected, weights, mem, stats);
}

int pw_moe_block(pw_runtime *rt, const pw_norm *post_norm, const pw_router *router, const pw_expert_bank *bank,
                 const float *residual, uint32_t tokens, float *out, uint32_t *selected, float *weights,
                 uint32_t mem, pw_stats *stats) {
  if (rt && !post_norm) return fail(rt, PW_ERR_ARGUMENT, "norm descriptor is null");
  return moe_layer_impl(rt, post_norm, router, bank, residual, tokens, out, selected, weights, mem, stats);
}

}  // extern "C"

// ======================================================= expert parallelism
// One process per GPU; rank g holds experts [g L, (g + 1) L) of the layer's
// E = L x world (src/text_endpoint.rs:4750 runs all 256 on one device; the
// partition is this build's).  Every rank routes its own tokens, and every
// rank takes the same collective steps in the same order:
//   1. quantize + route + schedule all E experts (expert-major placements,
//      so the rows for rank g are one contiguous block), gather the codes;
//   2. all-gather the per-expert placement offsets (E + 1 words per rank)
//      and wait for them: from here on every rank knows every transfer size;
//   3. grouped send/recv of FP8 codes and per-128 scales (quantizing before
//      dispatch is exact: an expert's first step is that quantization);
//   4. permute the received rows into expert order, run the local experts
//      (tcgen05 GEMM, or the GEMV for <= 16 rows per expert), and scatter the
//      bf16-rounded down rows back into received order as bf16;
//   5. grouped send/recv of the bf16 rows back to their source ranks;
//   6. the weighted combine in ascending expert order, as on one GPU, so the
//      layer is bit-identical to pw_moe_layer on the same tokens.
namespace {

int ep_dead(pw_runtime *rt, int code, const char *what, ncclResult_t r) {
  pw::nccl::abort_comm(rt->ep->comm);
  rt->ep->comm = nullptr;
  rt->ep->dead = true;
  return fail(rt, code, "%s: %s (communicator aborted)", what,
              r == ncclInProgress ? "deadline passed" : pw::nccl::error_string(r));
}

#define NK(expr, what)                                                                         \
  do {                                                                                         \
    ncclResult_t r_ = (expr);                                                                  \
    if (r_ != ncclSuccess) return ep_dead(rt, r_ == ncclInProgress ? PW_ERR_TIMEOUT : PW_ERR_NCCL, what, r_); \
  } while (0)

// Bounded wait for the runtime's stream; the deadline aborts the
// communicator (which also ends its kernels).  Only the stream and the clock
// are polled here: a communicator query can wait on NCCL's own background
// work, which is exactly what may be stuck when a peer is gone.
int ep_wait(pw_runtime *rt) {
  const double t0 = now_ms();
  for (;;) {
    const cudaError_t q = cudaStreamQuery(rt->stream);
    if (q == cudaSuccess) return PW_OK;
    if (q != cudaErrorNotReady) return fail(rt, PW_ERR_CUDA, "stream: %s", cudaGetErrorString(q));
    const double el = now_ms() - t0;
    if (el > rt->ep->timeout_s * 1e3)
      return ep_dead(rt, PW_ERR_TIMEOUT, "expert-parallel exchange", ncclInProgress);
    // spin for the first 2 ms (a sleep costs tens of microseconds of timer
    // slack, per layer), then back off
    if (el > 2.0) std::this_thread::sleep_for(std::chrono::microseconds(50));
    else std::this_thread::yield();
  }
}

// The transfer plan of rank r from every rank's expert offsets
// (all_off[g * (E + 1) + e] = first placement of expert e on rank g; rank r
// owns experts [r L, (r + 1) L), L = E / G):
//   n_send[g]    rows r sends to g (its placements of g's experts),
//   n_recv[g]    rows r receives from g, landing at recv_base[g] (G + 1 words),
//   perm[j]      received row of the j-th row in expert order (expert, then
//                source rank, then the source's placement order),
//   e_begin[le]  first expert-order row of local expert le (L + 1 words).
void ep_plan(const uint32_t *all_off, uint32_t G, uint32_t r, uint32_t E, uint32_t *n_send, uint32_t *n_recv,
             uint32_t *recv_base, uint32_t *perm, uint32_t *e_begin) {
  const uint32_t L = E / G;
  auto off = [&](uint32_t g, uint32_t e) { return all_off[(size_t)g * (E + 1) + e]; };
  recv_base[0] = 0;
  for (uint32_t g = 0; g < G; ++g) {
    n_send[g] = off(r, (g + 1) * L) - off(r, g * L);
    n_recv[g] = off(g, (r + 1) * L) - off(g, r * L);
    recv_base[g + 1] = recv_base[g] + n_recv[g];
  }
  uint32_t j = 0;
  e_begin[0] = 0;
  for (uint32_t le = 0; le < L; ++le) {
    const uint32_t e = r * L + le;
    for (uint32_t g = 0; g < G; ++g) {
      const uint32_t base = recv_base[g] + (off(g, e) - off(g, r * L));
      for (uint32_t k = 0; k < off(g, e + 1) - off(g, e); ++k) perm[j++] = base + k;
    }
    e_begin[le + 1] = j;
  }
}

template <class T>
int ep_pinned(pw_runtime *rt, T *&buf, size_t &cap, size_t bytes) {
  if (bytes <= cap) return PW_OK;
  if (buf) CK(cudaFreeHost(buf));
  buf = nullptr;
  cap = 0;
  void *p = nullptr;
  CK(cudaMallocHost(&p, bytes));
  buf = static_cast<T *>(p);
  cap = bytes;
  return PW_OK;
}

// Builds this rank's window for L local experts of hidden H and maps every
// other rank's (collective: IPC handles and geometry go through one
// all-gather, and a second one orders every rank's zeroed, mapped window
// before any peer stores into it).
int ep_window_setup(pw_runtime *rt, uint32_t L, uint32_t H) {
  EpState *ep = rt->ep;
  const uint32_t G = (uint32_t)ep->world, r = (uint32_t)ep->rank;
  CK(cudaStreamSynchronize(rt->stream));
  for (size_t g = 0; g < ep->peer_win.size(); ++g)
    if (ep->peer_win[g] && ep->peer_win[g] != ep->win) CK(cudaIpcCloseMemHandle(ep->peer_win[g]));
  ep->peer_win.clear();
  if (ep->win) CK(cudaFree(ep->win));
  if (ep->d_peers) CK(cudaFree(ep->d_peers));
  if (ep->d_ctr) CK(cudaFree(ep->d_ctr));
  ep->win = nullptr;
  ep->d_peers = nullptr;
  ep->d_ctr = nullptr;
  EpWindow w{};
  w.G = G;
  w.L = L;
  w.H = H;
  w.slot_rows = ep->max_tokens * 8u;
  uint64_t off = 0;
  auto take = [&](uint64_t bytes) {
    const uint64_t o = off;
    off += (bytes + 255u) & ~uint64_t(255);
    return o;
  };
  w.flag_ready = take(G * 4u);
  w.flag_data = take(G * 4u);
  w.flag_ret = take(G * 4u);
  w.mail_cnt = take((uint64_t)G * L * 4u);
  w.mail_base = take(G * 4u);
  w.recv_codes = take((uint64_t)G * w.slot_rows * H);
  w.recv_scales = take((uint64_t)G * w.slot_rows * (H / 128u) * 4u);
  w.ret_rows = take((uint64_t)w.slot_rows * H * 2u);
  w.total = off;
  CK(cudaMalloc(&ep->win, w.total));
  CK(cudaMemset(ep->win, 0, w.total));
  struct Rec {
    cudaIpcMemHandle_t h;
    uint32_t L, H, slot_rows, pad;
  };
  Rec mine{};
  if (G > 1) CK(cudaIpcGetMemHandle(&mine.h, ep->win));
  mine.L = L;
  mine.H = H;
  mine.slot_rows = w.slot_rows;
  std::vector<Rec> recs(G);
  Rec *d_rec = nullptr;
  CK(cudaMalloc(&d_rec, sizeof(Rec) * (G + 1)));
  CK(cudaMemcpy(d_rec + G, &mine, sizeof(Rec), cudaMemcpyHostToDevice));
  NK(pw::nccl::all_gather(d_rec + G, d_rec, sizeof(Rec), ncclUint8, ep->comm, rt->stream, ep->timeout_s),
     "window handle exchange");
  CK(cudaMemcpyAsync(recs.data(), d_rec, sizeof(Rec) * G, cudaMemcpyDeviceToHost, rt->stream));
  int s = ep_wait(rt);
  cudaFree(d_rec);
  if (s != PW_OK) return s;
  for (uint32_t g = 0; g < G; ++g)
    if (recs[g].L != L || recs[g].H != H || recs[g].slot_rows != w.slot_rows)
      return ep_dead(rt, PW_ERR_SHAPE, "ranks disagree on experts per rank, hidden size or max_tokens", ncclInvalidUsage);
  ep->peer_win.assign(G, nullptr);
  ep->peer_win[r] = ep->win;
  for (uint32_t g = 0; g < G; ++g)
    if (g != r) CK(cudaIpcOpenMemHandle(&ep->peer_win[g], recs[g].h, cudaIpcMemLazyEnablePeerAccess));
  CK(cudaMalloc(&ep->d_peers, G * sizeof(uint8_t *)));
  CK(cudaMemcpy(ep->d_peers, ep->peer_win.data(), G * sizeof(void *), cudaMemcpyHostToDevice));
  CK(cudaMalloc(&ep->d_ctr, 4 * sizeof(uint32_t)));
  CK(cudaMemset(ep->d_ctr, 0, 4 * sizeof(uint32_t)));
  ep->w = w;
  ep->epoch = 0;
  // barrier: no rank stores into a window before its owner has mapped all
  uint32_t *d_b = nullptr;
  CK(cudaMalloc(&d_b, (G + 1) * sizeof(uint32_t)));
  CK(cudaMemset(d_b, 0, (G + 1) * sizeof(uint32_t)));
  NK(pw::nccl::all_gather(d_b + G, d_b, 1, ncclUint32, ep->comm, rt->stream, ep->timeout_s), "window barrier");
  s = ep_wait(rt);
  cudaFree(d_b);
  return s;
}

// Rest of a routed layer on the peer-memory transport: everything after the
// local routing and the gathered send rows stays on the device.
int ep_layer_p2p(pw_runtime *rt, Call &call, const pw_expert_bank *bank, uint32_t tokens,
                 float *y, uint32_t *selected, float *weights, const ScheduleOut &so, float *dy, uint32_t *sel,
                 float *wts, const uint8_t *xsend, const float *ssend, const float *residual) {
  EpState *ep = rt->ep;
  const EpWindow &w = ep->w;
  const uint32_t G = w.G, L = w.L, H = bank->hidden, I = bank->inter, P = tokens * 8u;
  const uint32_t cap = G * w.slot_rows;  // rows this rank can receive
  // the tcgen05 GEMM when the layer is wide (judged from this rank's tokens:
  // the owners' row counts are known only on the device)
  const bool wide = (uint64_t)G * tokens >= kWideLayerTokens;
  const bool fuse_return = wide;  // see the down projection below
  const uint32_t chunk = wide ? (uint32_t)gemm_tc_tokens(2) : 8u;
  const uint32_t max_groups = cap / chunk + L;
  const bool fused = (rt->flags & PW_RUNTIME_FUSED_GATE_UP) != 0;
  int s;
  Arena br;
  uint32_t *perm = nullptr, *src_rank = nullptr, *src_place = nullptr, *n_groups = nullptr, *p_recv = nullptr;
  GemvGroup *gu = nullptr, *dn = nullptr;
  uint8_t *xg = nullptr, *hc = nullptr;
  float *xsg = nullptr, *hid = nullptr, *gt = nullptr, *ut = nullptr, *hs = nullptr, *down = nullptr;
  for (int pass = 0; pass < 2; ++pass) {
    if (pass == 1 && br.off > ep->cap) {
      CK(cudaStreamSynchronize(rt->stream));
      if (ep->scratch) CK(cudaFree(ep->scratch));
      ep->scratch = nullptr;
      ep->cap = 0;
      size_t c = (size_t)1 << 20;
      while (c < br.off) c *= 2;
      CK(cudaMalloc(&ep->scratch, c));
      ep->cap = c;
    }
    if (pass == 1) br = Arena{static_cast<char *>(ep->scratch), 0};
    perm = br.take<uint32_t>(cap);
    src_rank = br.take<uint32_t>(cap);
    src_place = br.take<uint32_t>(cap);
    gu = br.take<GemvGroup>(max_groups);
    dn = br.take<GemvGroup>(max_groups);
    n_groups = br.take<uint32_t>(3);  // [n_groups, p_recv, experts used], read back together
    p_recv = n_groups ? n_groups + 1 : nullptr;
    xg = wide ? br.take<uint8_t>((size_t)cap * H) : nullptr;
    xsg = wide ? br.take<float>((size_t)cap * (H / 128u)) : nullptr;
    hid = fused ? nullptr : br.take<float>((size_t)cap * I);
    gt = fused && !wide ? nullptr : br.take<float>((size_t)cap * I);
    ut = fused && !wide ? nullptr : br.take<float>((size_t)cap * I);
    hc = br.take<uint8_t>((size_t)cap * I);
    hs = br.take<float>((size_t)cap * (I / 128u));
    down = br.take<float>((size_t)cap * H);
  }
  const uint32_t epoch = ++ep->epoch;
  const EpArgs ea{ep->d_peers, w, (uint32_t)ep->rank, epoch, rt->d_flags, (uint64_t)(ep->timeout_s * 1e9)};
  uint8_t *mine = static_cast<uint8_t *>(ep->win);
  {
    ProfScope ps(rt, P_SCHED, 2);
    CK(launch_ep_dispatch(ea, so.offsets, xsend, ssend, P, ep->d_ctr, grid_for(rt, P / 4u), rt->stream));
    CK(launch_ep_plan(ea, bank->table, chunk, cap, perm, src_rank, src_place, gu, dn, n_groups, p_recv, rt->stream));
  }
  if (wide) {
    {
      ProfScope ps(rt, P_QUANT, 1);
      CK(launch_ep_gather(ea, perm, p_recv, xg, xsg, rt->num_sms, rt->stream));
    }
    // fused return: the down GEMM's epilogue stores each bf16 row into its
    // source's window (8 rows x 64 B per store instruction, through the
    // staging rows).  Measured at 4 GPUs: down 117 -> 131 us, return + wait +
    // combine 76 -> 30 us, 69-72k -> 75-76k tok/s against a separate return
    // kernel.  (With per-thread 16-byte row stores the fused form lost at 4
    // GPUs: down 133 -> 200 us.)
    const PeerRows pr{ep->d_peers, w.ret_rows, src_rank, src_place};
    s = enqueue_expert_chain_wide(rt, gu, dn, max_groups, n_groups, cap, H, I, xg, xsg, hid, gt, ut, hc, hs, down, 1,
                                  max_groups, p_recv, nullptr, fuse_return ? &pr : nullptr);
  } else {
    s = enqueue_expert_chain(rt, gu, dn, max_groups, n_groups, cap, H, I, perm,
                             reinterpret_cast<const uint8_t *>(mine + w.recv_codes),
                             reinterpret_cast<const float *>(mine + w.recv_scales), hid, gt, ut, hc, hs, down, 1,
                             max_groups, p_recv);
  }
  if (s != PW_OK) return s;
  {
    ProfScope ps(rt, P_COMBINE, 3);
    if (fuse_return)
      CK(launch_ep_release(ea, rt->stream));
    else
      CK(launch_ep_return(ea, down, src_rank, src_place, p_recv, ep->d_ctr + 1, rt->num_sms, rt->stream));
    CK(launch_ep_wait_returns(ea, rt->stream));
    if (tokens)
      CK(launch_combine_bf16(reinterpret_cast<const uint16_t *>(mine + w.ret_rows), so.slot_place, so.placement_w,
                             tokens, H, dy, rt->d_flags, rt->stream, residual));
  }
  if (tokens) {
    if (call.host()) {
      if ((s = call.stage_out(y, dy, (size_t)tokens * H * 4)) != PW_OK) return s;
      if (selected && (s = call.stage_out(selected, sel, (size_t)P * 4)) != PW_OK) return s;
      if (weights && (s = call.stage_out(weights, wts, (size_t)P * 4)) != PW_OK) return s;
    } else {
      if (selected) CK(cudaMemcpyAsync(selected, sel, (size_t)P * 4, cudaMemcpyDeviceToDevice, rt->stream));
      if (weights) CK(cudaMemcpyAsync(weights, wts, (size_t)P * 4, cudaMemcpyDeviceToDevice, rt->stream));
    }
  }
  if (!call.async() && (s = ep_wait(rt)) != PW_OK) return s;
  uint32_t got[3] = {0, 0, 0};
  if (call.stats) {
    CK(cudaMemcpyAsync(got, n_groups, 3 * sizeof(uint32_t), cudaMemcpyDeviceToHost, rt->stream));
    CK(cudaStreamSynchronize(rt->stream));
  }
  const pw_expert_weights &w0 = bank->host[0];
  const uint64_t per_expert = 3ull * H * I + 4ull * (w0.gate.scale_rows * w0.gate.scale_cols * 2u +
                                                     w0.down.scale_rows * w0.down.scale_cols);
  s = call.finish(per_expert * got[2]);
  if (call.stats) {
    call.stats->expert_rows = got[1];
    call.stats->unique_experts = got[2];
  }
  // a wait that ran out leaves the windows of this epoch unusable
  if (s == PW_ERR_TIMEOUT) ep_dead(rt, PW_ERR_TIMEOUT, "expert-parallel exchange", ncclInProgress);
  return s;
}

}  // namespace

extern "C" {

int pw_ep_unique_id(void *id, uint32_t bytes) {
  if (!id || bytes < sizeof(ncclUniqueId)) return PW_ERR_ARGUMENT;
  std::string err;
  if (!pw::nccl::load(err)) return PW_ERR_UNSUPPORTED;
  ncclUniqueId u;
  if (pw::nccl::unique_id(&u) != ncclSuccess) return PW_ERR_NCCL;
  memcpy(id, &u, sizeof u);
  return PW_OK;
}

int pw_ep_init(pw_runtime *rt, int rank, int world, const void *id, uint32_t bytes, uint32_t timeout_ms,
               uint32_t max_tokens, uint32_t hidden, uint32_t local_experts, uint32_t flags) {
  if (!rt) return PW_ERR_ARGUMENT;
  if (!id || bytes < sizeof(ncclUniqueId)) return fail(rt, PW_ERR_ARGUMENT, "NCCL unique id must be %zu bytes",
                                                       sizeof(ncclUniqueId));
  if (world < 1 || rank < 0 || rank >= world) return fail(rt, PW_ERR_ARGUMENT, "rank %d of %d", rank, world);
  if (rt->ep) return fail(rt, PW_ERR_ARGUMENT, "expert parallelism is already initialised on this runtime");
  std::string err;
  if (!pw::nccl::load(err)) return fail(rt, PW_ERR_UNSUPPORTED, "%s", err.c_str());
  CK(cudaSetDevice(rt->device));
  EpState *ep = new (std::nothrow) EpState();
  if (!ep) return fail(rt, PW_ERR_ARGUMENT, "out of host memory");
  ep->rank = rank;
  ep->world = world;
  ep->timeout_s = timeout_ms ? timeout_ms / 1e3 : 60.0;
  if (max_tokens > 2048u) {
    delete ep;
    return fail(rt, PW_ERR_UNSUPPORTED, "at most 2048 tokens per rank and call");
  }
  ep->max_tokens = max_tokens ? max_tokens : 2048u;
  ep->p2p = (flags & PW_EP_NCCL_TRANSPORT) == 0u;
  ncclUniqueId u;
  memcpy(&u, id, sizeof u);
  ncclComm_t comm = nullptr;
  const ncclResult_t r = pw::nccl::init_rank(&comm, world, u, rank, ep->timeout_s);
  if (r != ncclSuccess) {
    pw::nccl::abort_comm(comm);
    delete ep;
    return fail(rt, r == ncclInProgress ? PW_ERR_TIMEOUT : PW_ERR_NCCL, "ncclCommInitRank (rank %d of %d): %s", rank,
                world, r == ncclInProgress ? "peers did not join before the deadline" : pw::nccl::error_string(r));
  }
  ep->comm = comm;
  rt->ep = ep;
  // Establish every connection now, while all ranks are here: one all-gather
  // and one send/recv with each peer.  NCCL connects lazily on a
  // communicator's first use, and that handshake runs on the calling thread;
  // a peer lost later can then only stall kernels, which the bounded stream
  // wait and the abort end.
  uint32_t *probe = nullptr;
  CK(cudaMalloc(&probe, (size_t)world * 3 * sizeof(uint32_t)));
  CK(cudaMemsetAsync(probe, 0, (size_t)world * 3 * sizeof(uint32_t), rt->stream));
  int s = PW_OK;
  NK(pw::nccl::all_gather(probe, probe + world, 1, ncclUint32, ep->comm, rt->stream, ep->timeout_s),
     "connection warm-up (all-gather)");
  std::vector<pw::nccl::Transfer> sends, recvs;
  for (int g = 0; g < world; ++g) {
    sends.push_back({probe, sizeof(uint32_t), g});
    recvs.push_back({probe + 2 * world + g, sizeof(uint32_t), g});
  }
  NK(pw::nccl::exchange(sends.data(), (int)sends.size(), recvs.data(), (int)recvs.size(), ep->comm, rt->stream,
                        ep->timeout_s),
     "connection warm-up (send/recv)");
  s = ep_wait(rt);
  cudaFree(probe);
  if (s != PW_OK) return s;
  // the peer-memory windows are mapped now, while every rank is here
  if (ep->p2p && hidden && local_experts) {
    if (hidden % 512u || local_experts > 256u) return fail(rt, PW_ERR_SHAPE, "hidden must be a multiple of 512");
    s = ep_window_setup(rt, local_experts, hidden);
  }
  return s;
}

// With `norm` (pw_ep_moe_block) x is the residual stream: the RMSNorm runs
// fused with the input quantization and the combine adds the residual.
static int ep_moe_layer_impl(pw_runtime *rt, const pw_norm *norm, const pw_router *router, const pw_expert_bank *bank,
                             const float *x, uint32_t tokens, float *y, uint32_t *selected, float *weights,
                             uint32_t mem, pw_stats *stats) {
  if (!rt) return PW_ERR_ARGUMENT;
  EpState *ep = rt->ep;
  if (!ep || !ep->comm)
    return fail(rt, PW_ERR_ARGUMENT, ep ? "the expert-parallel communicator was aborted" : "pw_ep_init was not called");
  if (!bank || (tokens && (!x || !y))) return fail(rt, PW_ERR_ARGUMENT, "null argument");
  int s;
  if ((s = check_router(rt, router)) != PW_OK) return s;
  if (norm && (s = check_norm(rt, norm, bank->hidden)) != PW_OK) return s;
  if (norm && tokens && x == y) return fail(rt, PW_ERR_ARGUMENT, "the block's output may not alias its residual input");
  const uint32_t G = (uint32_t)ep->world, r = (uint32_t)ep->rank;
  const uint32_t L = bank->n, E = router->experts, H = bank->hidden, I = bank->inter;
  if (E != L * G) return fail(rt, PW_ERR_SHAPE, "router has %u experts; %u ranks x %u local experts", E, G, L);
  if (bank->hidden != router->hidden) return fail(rt, PW_ERR_SHAPE, "router and expert bank disagree");
  if (tokens > 2048u) return fail(rt, PW_ERR_UNSUPPORTED, "at most 2048 tokens per rank and call");
  if ((mem & PW_MEM_ASYNC) && (mem & PW_MEM_HOST))
    return fail(rt, PW_ERR_ARGUMENT, "asynchronous expert-parallel calls need device I/O");
  if (ep->p2p && tokens > ep->max_tokens)
    return fail(rt, PW_ERR_UNSUPPORTED, "%u tokens exceed this rank's max_tokens %u", tokens, ep->max_tokens);
  CK(cudaSetDevice(rt->device));
  if (ep->p2p && (!ep->win || ep->w.L != L || ep->w.H != H))
    if ((s = ep_window_setup(rt, L, H)) != PW_OK) return s;
  const uint32_t P = tokens * 8u, Hs = H / 128u, Is = I / 128u;
  Call call{rt, mem, stats, 0};
  if ((s = call.begin()) != PW_OK) return s;

  // ---- phase 1: local routing, schedule, send rows (runtime scratch)
  Arena ar;
  float *dx = nullptr, *dy = nullptr, *dnorm = nullptr;
  uint32_t *sel = nullptr, *alloff = nullptr;
  float *wts = nullptr;
  uint8_t *xsend = nullptr;
  float *ssend = nullptr;
  uint16_t *ret = nullptr;
  ScheduleOut so{};
  for (int pass = 0; pass < 2; ++pass) {
    if (pass == 1) {
      if ((s = ensure_scratch(rt, ar.off)) != PW_OK) return s;
      ar = Arena{static_cast<char *>(rt->scratch), 0};
    }
    dx = call.host() ? ar.take<float>((size_t)tokens * H) : const_cast<float *>(x);
    dy = call.host() ? ar.take<float>((size_t)tokens * H) : y;
    dnorm = norm ? ar.take<float>((size_t)tokens * H) : dx;  // the layer input the router reads
    uint8_t *xc = ar.take<uint8_t>((size_t)tokens * H);
    float *xs = ar.take<float>((size_t)tokens * Hs);
    float *logits = ar.take<float>(router_scratch_floats(tokens, E, H));
    sel = ar.take<uint32_t>(P);
    wts = ar.take<float>(P);
    so = ScheduleOut{};
    so.offsets = ar.take<uint32_t>(E + 1);
    so.placement_tok = ar.take<uint32_t>(P);
    so.placement_w = ar.take<float>(P);
    so.slot_place = ar.take<uint32_t>(P);
    so.counters = ar.take<uint32_t>(4);
    so.work = ar.take<uint32_t>(schedule_work_words(E));
    xsend = ar.take<uint8_t>((size_t)P * H);
    ssend = ar.take<float>((size_t)P * Hs);
    ret = ar.take<uint16_t>((size_t)P * H);
    alloff = ar.take<uint32_t>((size_t)G * (E + 1));
    if (pass == 0) continue;
    if (tokens == 0) {
      CK(cudaMemsetAsync(so.offsets, 0, (E + 1) * sizeof(uint32_t), rt->stream));
      break;
    }
    if (call.host() && (s = call.stage_in(dx, x, (size_t)tokens * H * 4)) != PW_OK) return s;
    CK(cudaMemsetAsync(rt->d_ties, 0, 4, rt->stream));
    {
      ProfScope ps(rt, P_QUANT, 1);
      if (norm)
        CK(launch_rms_quantize(dx, tokens, H, norm->weight, norm->weight_dtype, norm->epsilon, dnorm, xc, xs,
                               nullptr, rt->d_flags, rt->stream));
      else
        CK(launch_quantize(dx, tokens, H, xc, xs, rt->d_flags, rt->stream));
    }
    {
      ProfScope ps(rt, P_ROUTER, 2);
      CK(launch_router(dnorm, tokens, router->weight, router->weight_dtype, router->bias, E, H, logits, sel, wts,
                       rt->d_ties, rt->d_flags, rt->d_router_work, rt->num_sms, rt->stream));
    }
    {
      ProfScope ps(rt, P_SCHED, 4);
      CK(launch_schedule(sel, wts, tokens, E, BankTable{}, so, rt->d_flags, 1u, rt->stream));
      CK(launch_gather_rows(xc, xs, so.placement_tok, P, H, xsend, ssend, rt->stream));
    }
  }
  const float *residual = norm ? dx : nullptr;
  if (ep->p2p)
    return ep_layer_p2p(rt, call, bank, tokens, y, selected, weights, so, dy, sel, wts, xsend, ssend, residual);
  if ((s = ep_pinned(rt, ep->h_off, ep->h_off_cap, (size_t)G * (E + 1) * 4)) != PW_OK) return s;
  NK(pw::nccl::all_gather(so.offsets, alloff, E + 1, ncclUint32, ep->comm, rt->stream, ep->timeout_s),
     "ncclAllGather of expert offsets");
  CK(cudaMemcpyAsync(ep->h_off, alloff, (size_t)G * (E + 1) * 4, cudaMemcpyDeviceToHost, rt->stream));
  if ((s = ep_wait(rt)) != PW_OK) return s;

  // ---- plan (host): transfer sizes, expert-order permutation, groups
  std::vector<uint32_t> offs(ep->h_off, ep->h_off + (size_t)G * (E + 1));
  auto off = [&](uint32_t rank, uint32_t e) { return offs[(size_t)rank * (E + 1) + e]; };
  std::vector<uint32_t> n_send(G), n_recv(G), recv_base(G + 1, 0), e_begin(L + 1, 0);
  uint32_t P_recv = 0;
  for (uint32_t g = 0; g < G; ++g) P_recv += off(g, (r + 1) * L) - off(g, r * L);
  std::vector<uint32_t> perm(P_recv);
  ep_plan(offs.data(), G, r, E, n_send.data(), n_recv.data(), recv_base.data(), perm.data(), e_begin.data());
  uint32_t max_count = 0, local_used = 0;
  for (uint32_t le = 0; le < L; ++le) {
    const uint32_t c = e_begin[le + 1] - e_begin[le];
    max_count = c > max_count ? c : max_count;
    local_used += c ? 1u : 0u;
  }
  const bool wide = max_count > 16u;
  const uint32_t chunk = wide ? (uint32_t)gemm_tc_tokens(2) : 8u;
  std::vector<GemvGroup> gu, dn;
  for (uint32_t le = 0; le < L; ++le) {
    const pw_expert_weights &w = bank->host[le];
    for (uint32_t b = e_begin[le]; b < e_begin[le + 1]; b += chunk) {
      GemvGroup g{};
      g.tok_begin = b;
      g.count = std::min(chunk, e_begin[le + 1] - b);
      g.expert = r * L + le;
      g.w0 = w.gate.weight;
      g.s0 = w.gate.scale;
      g.w1 = w.up.weight;
      g.s1 = w.up.scale;
      g.tm0 = bank->d_maps + le;
      g.tm1 = bank->d_maps + L + le;
      gu.push_back(g);
      GemvGroup d = g;
      d.w0 = w.down.weight;
      d.s0 = w.down.scale;
      d.w1 = nullptr;
      d.s1 = nullptr;
      d.tm0 = bank->d_maps + 2 * (size_t)L + le;
      d.tm1 = nullptr;
      dn.push_back(d);
    }
  }
  const uint32_t ng = (uint32_t)gu.size();
  const bool fused = (rt->flags & PW_RUNTIME_FUSED_GATE_UP) != 0;

  // ---- phase 2 buffers (expert-parallel scratch, sized now)
  Arena br;
  uint8_t *rcodes = nullptr, *xg = nullptr, *hc = nullptr;
  float *rscales = nullptr, *xsg = nullptr, *hid = nullptr, *gt = nullptr, *ut = nullptr, *hs = nullptr,
        *down = nullptr;
  uint32_t *perm_d = nullptr;
  GemvGroup *gu_d = nullptr, *dn_d = nullptr;
  uint16_t *ret_send = nullptr;
  for (int pass = 0; pass < 2; ++pass) {
    if (pass == 1 && br.off > ep->cap) {
      if (ep->scratch) CK(cudaFree(ep->scratch));
      ep->scratch = nullptr;
      ep->cap = 0;
      size_t cap = (size_t)1 << 20;
      while (cap < br.off) cap *= 2;
      CK(cudaMalloc(&ep->scratch, cap));
      ep->cap = cap;
    }
    if (pass == 1) br = Arena{static_cast<char *>(ep->scratch), 0};
    rcodes = br.take<uint8_t>((size_t)P_recv * H);
    rscales = br.take<float>((size_t)P_recv * Hs);
    perm_d = br.take<uint32_t>(P_recv);
    gu_d = br.take<GemvGroup>(ng);
    dn_d = br.take<GemvGroup>(ng);
    xg = wide ? br.take<uint8_t>((size_t)P_recv * H) : nullptr;
    xsg = wide ? br.take<float>((size_t)P_recv * Hs) : nullptr;
    hid = fused ? nullptr : br.take<float>((size_t)P_recv * I);
    gt = fused && !wide ? nullptr : br.take<float>((size_t)P_recv * I);
    ut = fused && !wide ? nullptr : br.take<float>((size_t)P_recv * I);
    hc = br.take<uint8_t>((size_t)P_recv * I);
    hs = br.take<float>((size_t)P_recv * Is);
    down = br.take<float>((size_t)P_recv * H);
    ret_send = br.take<uint16_t>((size_t)P_recv * H);
  }
  // plan upload through pinned staging (the call waits before returning)
  const size_t plan_bytes = (size_t)P_recv * 4 + 2 * (size_t)ng * sizeof(GemvGroup);
  if ((s = ep_pinned(rt, ep->h_plan, ep->h_plan_cap, plan_bytes + 16)) != PW_OK) return s;
  {
    char *hp = static_cast<char *>(ep->h_plan);
    if (P_recv) memcpy(hp, perm.data(), (size_t)P_recv * 4);
    if (ng) {
      memcpy(hp + (size_t)P_recv * 4, gu.data(), ng * sizeof(GemvGroup));
      memcpy(hp + (size_t)P_recv * 4 + ng * sizeof(GemvGroup), dn.data(), ng * sizeof(GemvGroup));
      CK(cudaMemcpyAsync(gu_d, hp + (size_t)P_recv * 4, ng * sizeof(GemvGroup), cudaMemcpyHostToDevice, rt->stream));
      CK(cudaMemcpyAsync(dn_d, hp + (size_t)P_recv * 4 + ng * sizeof(GemvGroup), ng * sizeof(GemvGroup),
                         cudaMemcpyHostToDevice, rt->stream));
    }
    if (P_recv) CK(cudaMemcpyAsync(perm_d, hp, (size_t)P_recv * 4, cudaMemcpyHostToDevice, rt->stream));
  }

  // ---- dispatch: codes and scales to the expert owners
  std::vector<pw::nccl::Transfer> sends, recvs;
  for (uint32_t g = 0; g < G; ++g) {
    const size_t b = off(r, g * L);
    sends.push_back({xsend + b * H, (size_t)n_send[g] * H, (int)g});
    sends.push_back({ssend + b * Hs, (size_t)n_send[g] * Hs * 4, (int)g});
    recvs.push_back({rcodes + (size_t)recv_base[g] * H, (size_t)n_recv[g] * H, (int)g});
    recvs.push_back({rscales + (size_t)recv_base[g] * Hs, (size_t)n_recv[g] * Hs * 4, (int)g});
  }
  NK(pw::nccl::exchange(sends.data(), (int)sends.size(), recvs.data(), (int)recvs.size(), ep->comm, rt->stream,
                        ep->timeout_s),
     "dispatch send/recv");

  // ---- local experts on the received rows
  if (P_recv) {
    if (wide) {
      {
        ProfScope ps(rt, P_QUANT, 1);
        CK(launch_gather_rows(rcodes, rscales, perm_d, P_recv, H, xg, xsg, rt->stream));
      }
      s = enqueue_expert_chain_wide(rt, gu_d, dn_d, ng, nullptr, P_recv, H, I, xg, xsg, hid, gt, ut, hc, hs, down, 1,
                                    ng);
    } else {
      s = enqueue_expert_chain(rt, gu_d, dn_d, ng, nullptr, P_recv, H, I, perm_d, rcodes, rscales, hid, gt, ut, hc,
                               hs, down, 1, ng);
    }
    if (s != PW_OK) return s;
    ProfScope ps(rt, P_COMBINE, 1);
    CK(launch_scatter_rows_bf16(down, perm_d, P_recv, H, ret_send, rt->stream));
  }

  // ---- return: bf16 down rows to their source ranks
  sends.clear();
  recvs.clear();
  for (uint32_t g = 0; g < G; ++g) {
    sends.push_back({ret_send + (size_t)recv_base[g] * H, (size_t)n_recv[g] * H * 2, (int)g});
    recvs.push_back({ret + (size_t)off(r, g * L) * H, (size_t)n_send[g] * H * 2, (int)g});
  }
  NK(pw::nccl::exchange(sends.data(), (int)sends.size(), recvs.data(), (int)recvs.size(), ep->comm, rt->stream,
                        ep->timeout_s),
     "combine send/recv");

  // ---- weighted combine in ascending expert order
  if (tokens) {
    {
      ProfScope ps(rt, P_COMBINE, 1);
      CK(launch_combine_bf16(ret, so.slot_place, so.placement_w, tokens, H, dy, rt->d_flags, rt->stream, residual));
    }
    if (call.host()) {
      if ((s = call.stage_out(y, dy, (size_t)tokens * H * 4)) != PW_OK) return s;
      if (selected && (s = call.stage_out(selected, sel, (size_t)P * 4)) != PW_OK) return s;
      if (weights && (s = call.stage_out(weights, wts, (size_t)P * 4)) != PW_OK) return s;
    } else {
      if (selected) CK(cudaMemcpyAsync(selected, sel, (size_t)P * 4, cudaMemcpyDeviceToDevice, rt->stream));
      if (weights) CK(cudaMemcpyAsync(weights, wts, (size_t)P * 4, cudaMemcpyDeviceToDevice, rt->stream));
    }
  }
  // PW_MEM_ASYNC: return with the dispatch, the experts, the return trip and
  // the combine enqueued; the next expert-parallel call's offset wait covers
  // them, and every buffer this call used is rewritten only after that wait.
  if (!call.async() && (s = ep_wait(rt)) != PW_OK) return s;
  const pw_expert_weights &w0 = bank->host[0];
  const uint64_t per_expert = 3ull * H * I + 4ull * (w0.gate.scale_rows * w0.gate.scale_cols * 2u +
                                                     w0.down.scale_rows * w0.down.scale_cols);
  s = call.finish(per_expert * local_used);
  if (stats) {
    stats->unique_experts = local_used;
    stats->expert_rows = P_recv;
  }
  return s;
}

int pw_ep_moe_layer(pw_runtime *rt, const pw_router *router, const pw_expert_bank *bank, const float *x,
                    uint32_t tokens, float *y, uint32_t *selected, float *weights, uint32_t mem, pw_stats *stats) {
  return ep_moe_layer_impl(rt, nullptr, router, bank, x, tokens, y, selected, weights, mem, stats);
}

int pw_ep_moe_block(pw_runtime *rt, const pw_norm *post_norm, const pw_router *router, const pw_expert_bank *bank,
                    const float *residual, uint32_t tokens, float *out, uint32_t *selected, float *weights,
                    uint32_t mem, pw_stats *stats) {
  if (rt && !post_norm) return fail(rt, PW_ERR_ARGUMENT, "norm descriptor is null");
  return ep_moe_layer_impl(rt, post_norm, router, bank, residual, tokens, out, selected, weights, mem, stats);
}

int pw_ep_plan(const uint32_t *all_offsets, uint32_t world, uint32_t rank, uint32_t experts, uint32_t *n_send,
               uint32_t *n_recv, uint32_t *recv_base, uint32_t *perm, uint32_t *expert_begin) {
  if (!all_offsets || !n_send || !n_recv || !recv_base || !expert_begin || world == 0 || rank >= world ||
      experts % world)
    return PW_ERR_ARGUMENT;
  const uint32_t L = experts / world;
  for (uint32_t g = 0; g < world; ++g)
    for (uint32_t e = 0; e < experts; ++e)
      if (all_offsets[(size_t)g * (experts + 1) + e + 1] < all_offsets[(size_t)g * (experts + 1) + e])
        return PW_ERR_SCHEDULE;
  uint32_t rows = 0;
  for (uint32_t g = 0; g < world; ++g)
    rows += all_offsets[(size_t)g * (experts + 1) + (rank + 1) * L] - all_offsets[(size_t)g * (experts + 1) + rank * L];
  if (rows && !perm) return PW_ERR_ARGUMENT;
  ep_plan(all_offsets, world, rank, experts, n_send, n_recv, recv_base, perm, expert_begin);
  return PW_OK;
}

int pw_ep_rank(const pw_runtime *rt, int *rank, int *world) {
  if (!rt || !rank || !world) return PW_ERR_ARGUMENT;
  if (!rt->ep || !rt->ep->comm) return PW_ERR_ARGUMENT;
  *rank = rt->ep->rank;
  *world = rt->ep->world;
  return PW_OK;
}

}  // extern "C"
