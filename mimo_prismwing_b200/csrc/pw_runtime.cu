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
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <new>
#include <string>
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
bool encode_weight_map(CUtensorMap *out, const void *base, uint32_t rows, uint32_t cols, uint32_t box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn || cols % 128u) return false;
  cuuint64_t dims[3] = {128u, rows, cols / 128u};
  cuuint64_t strides[2] = {cols, 128u};
  cuuint32_t box[3] = {128u, box_rows, 256u / box_rows};
  cuuint32_t estr[3] = {1u, 1u, 1u};
  return fn(out, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void *>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}
}  // namespace pw

struct pw_runtime {
  int device = 0;
  uint32_t flags = 0;
  int num_sms = 148;
  cudaStream_t own_stream = nullptr;
  cudaStream_t stream = nullptr;
  uint32_t *d_flags = nullptr;            // error-flag word
  unsigned long long *d_bad = nullptr;    // validation: first bad byte
  uint32_t *d_ties = nullptr;             // router tie rows
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
};

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
  uint32_t n = 0;
  uint32_t hidden = 0, inter = 0;
  void *d_table = nullptr;  // 6 arrays of n pointers
  CUtensorMap *d_maps = nullptr;  // 3 arrays of n TMA maps (gate, up, down)
  BankTable table{};
  std::vector<pw_expert_weights> host;
};

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
  if (rt->scratch) cudaFree(rt->scratch);
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
  CUtensorMap hmap;
  if (kind != 1) {
    const pw_fp8_tensor *ts[1] = {w};
    if (!encode_maps(rt, ts, 1, layout, &hmap)) return PW_ERR_CUDA;
  }
  // wide block-scaled projections run on the tcgen05 GEMM (plain layout)
  const bool wide = kind != 1 && layout == PW_LAYOUT_PLAIN && width >= kWideProjection;
  Call call{rt, mem, stats, 0};
  if ((s = call.begin()) != PW_OK) return s;
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
    CUtensorMap *dm = ar.take<CUtensorMap>(1);
    std::vector<GemvGroup> groups =
        width_groups(width, *w, nullptr, kind == 1 ? nullptr : dm, nullptr, wide ? (uint32_t)gemm_tc_tokens(0) : 8u);
    GemvGroup *dg = ar.take<GemvGroup>(groups.size());
    if (pass == 0) continue;
    if (call.host() && (s = call.stage_in(dx, x, nx * 4)) != PW_OK) return s;
    if (kind != 1) CK(cudaMemcpyAsync(dm, &hmap, sizeof hmap, cudaMemcpyHostToDevice, rt->stream));
    CK(cudaMemcpyAsync(dg, groups.data(), groups.size() * sizeof(GemvGroup), cudaMemcpyHostToDevice, rt->stream));
    GemvArgs a = gemv_args(rt, dg, (uint32_t)groups.size(), N, K, layout);
    a.out = dy;
    a.out_stride = N;
    if (kind == 1) {
      a.x_f32 = dx;
      a.round_bf16 = 0;
    } else {
      ProfScope ps(rt, P_QUANT, 1);
      CK(launch_quantize(dx, width, K, dc, ds, rt->d_flags, rt->stream));
      a.x_codes = dc;
      a.x_scales = ds;
      a.round_bf16 = round;
    }
    {
      ProfScope ps(rt, P_PROJ, 1);
      const int grid = grid_for(rt, (uint64_t)groups.size() * (N / (kind == 1 ? 64u : 128u)));
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
                                uint32_t down_round, uint64_t units_hint) {
  const int grid_gu = grid_for(rt, units_hint * (I / 128u));
  const bool fused = (rt->flags & PW_RUNTIME_FUSED_GATE_UP) != 0;
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
    CK(launch_gemv(0, a, grid_gu, rt->stream));
    // kind 3 is the same projection over each group's second matrix (up)
    GemvArgs b = a;
    b.out = up_tmp;
    CK(launch_gemv(3, b, grid_gu, rt->stream));
    CK(launch_swiglu(gate_tmp, up_tmp, hidden, slots * I, rt->d_flags, rt->stream));
  }
  }
  if (!fused) {
    ProfScope ps(rt, P_QUANT, 1);
    CK(launch_quantize(hidden, slots, I, hc, hs, rt->d_flags, rt->stream));
  }
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
  ProfScope ps(rt, P_DOWN, 1);
  CK(launch_gemv(0, d, grid_for(rt, units_hint * (H / 128u)), rt->stream));
  return PW_OK;
}


// The expert chain on the tcgen05 GEMM.  xg / xsg are the gate/up input codes
// and scales laid out by group (tok_begin indexes rows directly).
static int enqueue_expert_chain_wide(pw_runtime *rt, const GemvGroup *gu, const GemvGroup *dn, uint32_t n_groups,
                                     const uint32_t *n_groups_dev, uint32_t slots, uint32_t H, uint32_t I,
                                     const uint8_t *xg, const float *xsg, float *hidden, float *gate_tmp,
                                     float *up_tmp, uint8_t *hc, float *hs, float *down, uint32_t down_round,
                                     uint64_t units_hint) {
  const int grid_gu = grid_for(rt, units_hint * (I / 128u));
  const bool fused = (rt->flags & PW_RUNTIME_FUSED_GATE_UP) != 0;
  {
    ProfScope ps(rt, P_GATEUP, fused ? 2 : 3);
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
      CK(launch_swiglu_quant(A.g.gate_bf16, A.g.up_bf16, slots, I, hidden, hc, hs, rt->d_flags, rt->stream));
    } else {
      if (!encode_act_maps(A.xmap, xg, slots, H))
        return fail(rt, PW_ERR_CUDA, "cuTensorMapEncodeTiled failed for the activations");
      A.g.out = gate_tmp;
      CK(launch_gemm_tc(0, A, grid_gu, rt->stream));
      GemmArgs B = A;
      B.g.out = up_tmp;
      CK(launch_gemm_tc(3, B, grid_gu, rt->stream));
      CK(launch_swiglu(gate_tmp, up_tmp, hidden, slots * I, rt->d_flags, rt->stream));
    }
  }
  if (!fused) {
    ProfScope ps(rt, P_QUANT, 1);
    CK(launch_quantize(hidden, slots, I, hc, hs, rt->d_flags, rt->stream));
  }
  GemmArgs D{};
  D.g = gemv_args(rt, dn, n_groups, H, I, PW_LAYOUT_PLAIN);
  D.g.n_groups_dev = n_groups_dev;
  D.g.x_codes = hc;
  D.g.x_scales = hs;
  D.g.out = down;
  D.g.out_stride = H;
  D.g.round_bf16 = down_round;
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
  CUtensorMap hmaps[3];
  {
    const pw_fp8_tensor *ts[3] = {&w->gate, &w->up, &w->down};
    if (!encode_maps(rt, ts, 3, PW_LAYOUT_PLAIN, hmaps)) return PW_ERR_CUDA;
  }
  const bool fused = (rt->flags & PW_RUNTIME_FUSED_GATE_UP) != 0;
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
    const bool wide = width >= kWideProjection;
    float *hid = fused ? nullptr : ar.take<float>((size_t)width * I);
    // the wide fused chain stages bf16 gate/up here
    float *gt = fused && !wide ? nullptr : ar.take<float>((size_t)width * I);
    float *ut = fused && !wide ? nullptr : ar.take<float>((size_t)width * I);
    uint8_t *hc = ar.take<uint8_t>((size_t)width * I);
    float *hs = ar.take<float>((size_t)width * I / 128u);
    CUtensorMap *dm = ar.take<CUtensorMap>(3);
    const uint32_t chunk = wide ? (uint32_t)gemm_tc_tokens(2) : 8u;
    std::vector<GemvGroup> gu = width_groups(width, w->gate, &w->up, dm, dm ? dm + 1 : nullptr, chunk);
    std::vector<GemvGroup> dn = width_groups(width, w->down, nullptr, dm ? dm + 2 : nullptr, nullptr, chunk);
    GemvGroup *dgu = ar.take<GemvGroup>(gu.size());
    GemvGroup *ddn = ar.take<GemvGroup>(dn.size());
    if (pass == 0) continue;
    if (call.host() && (s = call.stage_in(dx, x, (size_t)width * H * 4)) != PW_OK) return s;
    CK(cudaMemcpyAsync(dm, hmaps, sizeof hmaps, cudaMemcpyHostToDevice, rt->stream));
    CK(cudaMemcpyAsync(dgu, gu.data(), gu.size() * sizeof(GemvGroup), cudaMemcpyHostToDevice, rt->stream));
    CK(cudaMemcpyAsync(ddn, dn.data(), dn.size() * sizeof(GemvGroup), cudaMemcpyHostToDevice, rt->stream));
    {
      ProfScope ps(rt, P_QUANT, 1);
      CK(launch_quantize(dx, width, H, xc, xs, rt->d_flags, rt->stream));
    }
    if (wide)
      s = enqueue_expert_chain_wide(rt, dgu, ddn, (uint32_t)gu.size(), nullptr, width, H, I, xc, xs, hid, gt, ut, hc,
                                    hs, dy, 1, gu.size());
    else
      s = enqueue_expert_chain(rt, dgu, ddn, (uint32_t)gu.size(), nullptr, width, H, I, nullptr, xc, xs, hid, gt, ut,
                               hc, hs, dy, 1, gu.size());
    if (s != PW_OK) return s;
    if (call.host() && (s = call.stage_out(y, dy, (size_t)width * H * 4)) != PW_OK) return s;
  }
  const uint64_t wb = 3ull * H * I + 4ull * (w->gate.scale_rows * w->gate.scale_cols * 2u +
                                             w->down.scale_rows * w->down.scale_cols);
  return call.finish(wb);
}

// ------------------------------------------------------------------- router
static int check_router(pw_runtime *rt, const pw_router *r) {
  if (!r || !r->weight_bf16 || !r->bias) return fail(rt, PW_ERR_ARGUMENT, "router descriptor is null");
  if (r->top_k != 8) return fail(rt, PW_ERR_UNSUPPORTED, "top_k must be 8");
  if (r->experts <= 8 || r->experts > 256 || r->hidden == 0 || r->hidden % 512u)
    return fail(rt, PW_ERR_SHAPE, "router shape mismatch (experts 9..256, hidden a multiple of 512)");
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
    float *logits = ar.take<float>((size_t)tokens * E);
    if (pass == 0) continue;
    if (call.host() && (s = call.stage_in(dx, x, (size_t)tokens * H * 4)) != PW_OK) return s;
    CK(cudaMemsetAsync(rt->d_ties, 0, 4, rt->stream));
    {
      ProfScope ps(rt, P_ROUTER, 2);
      CK(launch_router_logits(dx, tokens, router->weight_bf16, E, H, logits, rt->stream));
      CK(launch_router_topk(logits, router->bias, tokens, E, dsel, dw, rt->d_ties, rt->d_flags, rt->stream));
    }
    if (call.host()) {
      if ((s = call.stage_out(selected, dsel, (size_t)tokens * 32)) != PW_OK) return s;
      if ((s = call.stage_out(weights, dw, (size_t)tokens * 32)) != PW_OK) return s;
    }
  }
  uint32_t ties = 0;
  if (stats) CK(cudaMemcpyAsync(&ties, rt->d_ties, 4, cudaMemcpyDeviceToHost, rt->stream));
  s = call.finish((uint64_t)E * H * 2 + E * 4);
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
                                    down, 1, gu.size());
    } else {
      s = enqueue_expert_chain(rt, dgu, ddn, (uint32_t)gu.size(), nullptr, P, H, I, dtok, xc, xs, hid, gt, ut, hc, hs,
                               down, 1, gu.size());
    }
    if (s != PW_OK) return s;
    {
      ProfScope ps(rt, P_COMBINE, 1);
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
  if (bank->d_table || bank->d_maps) {
    cudaSetDevice(bank->rt->device);
    if (bank->d_table) cudaFree(bank->d_table);
    if (bank->d_maps) cudaFree(bank->d_maps);
  }
  delete bank;
}

// ------------------------------------------------------ device-routed layer
int pw_moe_layer(pw_runtime *rt, const pw_router *router, const pw_expert_bank *bank, const float *x, uint32_t tokens,
                 float *y, uint32_t *selected, float *weights, uint32_t mem, pw_stats *stats) {
  if (!rt) return PW_ERR_ARGUMENT;
  if (!x || !y || !bank) return fail(rt, PW_ERR_ARGUMENT, "null argument");
  int s;
  if ((s = check_router(rt, router)) != PW_OK) return s;
  if (bank->n != router->experts || bank->hidden != router->hidden)
    return fail(rt, PW_ERR_SHAPE, "router and expert bank disagree");
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
    uint8_t *xc = ar.take<uint8_t>((size_t)tokens * H);
    float *xs = ar.take<float>((size_t)tokens * H / 128u);
    float *logits = ar.take<float>((size_t)tokens * E);
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
    {
      ProfScope ps(rt, P_QUANT, 1);
      CK(launch_quantize(dx, tokens, H, xc, xs, rt->d_flags, rt->stream));
    }
    {
      ProfScope ps(rt, P_ROUTER, 2);
      CK(launch_router_logits(dx, tokens, router->weight_bf16, E, H, logits, rt->stream));
      CK(launch_router_topk(logits, router->bias, tokens, E, sel, wts, rt->d_ties, rt->d_flags, rt->stream));
    }
    {
      ProfScope ps(rt, P_SCHED, 1);
      CK(launch_schedule(sel, wts, tokens, E, bank->table, so, rt->d_flags, chunk, rt->stream));
    }
    // the grid covers the worst case; CTAs read the real group count
    if (wide) {
      {
        ProfScope ps(rt, P_QUANT, 1);
        CK(launch_gather_rows(xc, xs, so.placement_tok, P, H, xg, xsg, rt->stream));
      }
      s = enqueue_expert_chain_wide(rt, so.gu_groups, so.dn_groups, max_groups, so.n_groups, P, H, I, xg, xsg, hid,
                                    gt, ut, hc, hs, down, 1, max_groups);
    } else {
      s = enqueue_expert_chain(rt, so.gu_groups, so.dn_groups, max_groups, so.n_groups, P, H, I, so.placement_tok, xc,
                               xs, hid, gt, ut, hc, hs, down, 1, max_groups);
    }
    if (s != PW_OK) return s;
    {
      ProfScope ps(rt, P_COMBINE, 1);
      CK(launch_combine(down, so.slot_place, so.placement_w, tokens, H, dy, rt->d_flags, rt->stream));
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
    stats->weight_bytes = per_expert * cnt[0] + (uint64_t)E * H * 2 + E * 4;
  }
  return s;
}

}  // extern "C"
