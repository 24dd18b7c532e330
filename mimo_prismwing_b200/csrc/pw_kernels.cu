// pw_kernels.cu -- the small kernels around the GEMV: dynamic FP8 activation
// quantization, router logits + sigmoid no-aux top-8, the device-side expert
// schedule, the weighted combine, bf16 rounding and weight validation.
#include <cstdint>
#include <type_traits>
#include <cuda_runtime.h>

#include "pw_device.cuh"
#include "pw_internal.h"

namespace pw {

static thread_local bool t_pdl = false;
bool pdl_enabled() { return t_pdl; }
void set_pdl(bool on) { t_pdl = on; }

// ------------------------------------------------------------ quantization
// One warp per 128-value group (src/text_endpoint.rs:3008,
// kernels/block_fp8_gemv.metal:84): absmax, scale = max(absmax,1e-10)/448,
// code = RNE_e4m3(clamp(x/scale, +-448)).  The scale is an IEEE division and
// the quotients are correctly rounded (Fp8GroupScale), so the bytes match the
// reference's; lane l holds values 4l..4l+3.
__global__ void k_quantize(const float *__restrict__ x, uint64_t groups, uint8_t *__restrict__ codes,
                           float *__restrict__ scales, uint32_t *flags, const uint32_t *rows_dev,
                           uint32_t groups_per_row, uint32_t *zero, uint32_t n_zero) {
  pdl_wait();
  pdl_launch_dependents();
  // the first kernel of a chain clears the next kernels' split-K counters
  if (zero && blockIdx.x == 0)
    for (uint32_t i = threadIdx.x; i < n_zero; i += blockDim.x) zero[i] = 0u;
  if (rows_dev) groups = min(groups, (uint64_t)*rows_dev * groups_per_row);
  const uint64_t warp_global = ((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) / 32u;
  const uint32_t lane = threadIdx.x % 32u;
  const uint64_t nwarps = ((uint64_t)gridDim.x * blockDim.x) / 32u;
  for (uint64_t g = warp_global; g < groups; g += nwarps) {
    const float4 v = __ldg(reinterpret_cast<const float4 *>(x + g * 128u) + lane);
    const bool ok = finite(v.x) && finite(v.y) && finite(v.z) && finite(v.w);
    if (!ok) raise_flag(flags, PW_FLAG_NONFINITE_INPUT);
    float m = ok ? fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))) : 0.0f;
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    const Fp8GroupScale gs = Fp8GroupScale::of(m);
    const float scale = gs.scale;
    auto q = [&](float val) { return gs.quotient(val); };
    const uint32_t lo = encode2(q(v.x), q(v.y));
    const uint32_t hi = encode2(q(v.z), q(v.w));
    reinterpret_cast<uint32_t *>(codes + g * 128u)[lane] = lo | (hi << 16);
    if (lane == 0) scales[g] = scale;
  }
}

cudaError_t launch_quantize(const float *x, uint32_t rows, uint32_t cols, uint8_t *codes, float *scales,
                            uint32_t *flags, cudaStream_t stream, const uint32_t *rows_dev, uint32_t *zero,
                            uint32_t n_zero) {
  if (cols % 128u) return cudaErrorInvalidValue;
  const uint64_t groups = (uint64_t)rows * (cols / 128u);
  if (groups == 0 && !zero) return cudaSuccess;
  const int threads = 256;
  uint64_t blocks = (groups * 32u + threads - 1) / threads;
  if (blocks > 148u * 16u) blocks = 148u * 16u;
  if (blocks == 0) blocks = 1;
  return launch_kernel(k_quantize, dim3((unsigned)blocks), dim3(threads), 0, stream, x, groups, codes, scales, flags,
                       rows_dev, cols / 128u, zero, n_zero);
}

// ------------------------------------------------- RMSNorm + quantization
// The decoder layer's post-attention RMSNorm (src/text_endpoint.rs:2939
// rms_norm; stable_rms_inverse src/lib.rs:1890) fused with the dynamic FP8
// quantization of its output, the routed experts' first step.  One CTA per
// row.  The sum of squares follows PyTorch's vectorised cascade
// (pytorch_contiguous_inner_square_sum_f32, src/lib.rs:1905) exactly: with
// cols % 256 == 0 it is 16 accumulators j = 4 * register + lane, each summing
// the squares of columns c = j (mod 16); level 0 sums 16 steps of one 256-
// column block from zero and is added into level 1 after every block, level 1
// into level 2 when the step count is a multiple of 256, level 2 into level 3
// at multiples of 4096; then levels fold into level 0, registers into
// register 0, lanes into the result.  Here the 16 x (cols / 256) block sums
// run in parallel (one thread each) and 16 threads replay the level cascade.
// Products and sums round separately.  Then out = bf16(bf16(x * inv) * w[c])
// and its per-128 FP8 codes and scales (as k_quantize).
constexpr uint32_t kRmsMaxBlocks = 64;  // cols <= 16384

template <bool F32W>
__global__ void __launch_bounds__(256) k_rms_quantize(const float *__restrict__ x, uint32_t cols,
                                                      const void *__restrict__ weight, float eps,
                                                      float *__restrict__ xn, uint8_t *__restrict__ codes,
                                                      float *__restrict__ scales, float *__restrict__ inv_out,
                                                      uint32_t *flags) {
  pdl_wait();
  pdl_launch_dependents();
  __shared__ float blk[kRmsMaxBlocks][16];
  __shared__ float lvl[16];
  __shared__ float inv_s;
  const uint32_t row = blockIdx.x, tid = threadIdx.x, nb = cols / 256u;
  const float *xr = x + (size_t)row * cols;
  bool ok = true;
  for (uint32_t pr = tid; pr < nb * 16u; pr += blockDim.x) {
    const uint32_t b = pr / 16u, j = pr % 16u;
    float sacc = 0.0f;
#pragma unroll
    for (uint32_t i = 0; i < 16u; ++i) {
      const float v = __ldg(xr + 256u * b + 16u * i + j);
      ok = ok && finite(v);
      sacc = __fadd_rn(sacc, __fmul_rn(v, v));
    }
    blk[b][j] = sacc;
  }
  if (!ok) raise_flag(flags, PW_FLAG_NONFINITE_INPUT);
  __syncthreads();
  if (tid < 16u) {
    float a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
    for (uint32_t b = 0; b < nb; ++b) {
      const uint32_t index = 16u * (b + 1u);
      a1 = __fadd_rn(a1, blk[b][tid]);  // level 0 -> 1 (level 0 restarts from zero)
      if (index & (15u << 4)) continue;
      a2 = __fadd_rn(a2, a1);
      a1 = 0.0f;
      if (index & (15u << 8)) continue;
      a3 = __fadd_rn(a3, a2);
      a2 = 0.0f;
    }
    lvl[tid] = __fadd_rn(__fadd_rn(__fadd_rn(0.0f, a1), a2), a3);
  }
  __syncthreads();
  if (tid == 0) {
    float result = 0.0f;
#pragma unroll
    for (uint32_t l = 0; l < 4u; ++l) {
      const float t = __fadd_rn(__fadd_rn(__fadd_rn(lvl[l], lvl[4u + l]), lvl[8u + l]), lvl[12u + l]);
      result = __fadd_rn(result, t);
    }
    const float variance = __fdiv_rn(result, (float)cols);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(variance, eps)));
    inv_s = inv;
    if (inv_out) inv_out[row] = inv;
  }
  __syncthreads();
  const float inv = inv_s;
  const uint32_t lane = tid % 32u, warp = tid / 32u, nwarps = blockDim.x / 32u;
  for (uint32_t g = warp; g < cols / 128u; g += nwarps) {
    const uint32_t c0 = 128u * g + 4u * lane;
    const float4 v = __ldg(reinterpret_cast<const float4 *>(xr + c0));
    float wv[4];
    if (F32W) {
      const float4 w4 = __ldg(reinterpret_cast<const float4 *>(static_cast<const float *>(weight) + c0));
      wv[0] = w4.x, wv[1] = w4.y, wv[2] = w4.z, wv[3] = w4.w;
    } else {
      const uint2 w2 = __ldg(reinterpret_cast<const uint2 *>(static_cast<const uint16_t *>(weight) + c0));
      wv[0] = __uint_as_float(w2.x << 16), wv[1] = __uint_as_float(w2.x & 0xffff0000u);
      wv[2] = __uint_as_float(w2.y << 16), wv[3] = __uint_as_float(w2.y & 0xffff0000u);
    }
    const float xv[4] = {v.x, v.y, v.z, v.w};
    float o[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) o[k] = round_bf16(__fmul_rn(round_bf16(__fmul_rn(xv[k], inv)), wv[k]));
    if (xn) *reinterpret_cast<float4 *>(xn + (size_t)row * cols + c0) = make_float4(o[0], o[1], o[2], o[3]);
    float m = fmaxf(fmaxf(fabsf(o[0]), fabsf(o[1])), fmaxf(fabsf(o[2]), fabsf(o[3])));
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    const Fp8GroupScale gs = Fp8GroupScale::of(m);
    const float scale = gs.scale;
    auto q = [&](float val) { return gs.quotient(val); };
    const uint32_t lo = encode2(q(o[0]), q(o[1]));
    const uint32_t hi = encode2(q(o[2]), q(o[3]));
    if (codes) reinterpret_cast<uint32_t *>(codes + (size_t)row * cols + 128u * g)[lane] = lo | (hi << 16);
    if (scales && lane == 0) scales[(size_t)row * (cols / 128u) + g] = scale;
  }
}

cudaError_t launch_rms_quantize(const float *x, uint32_t rows, uint32_t cols, const void *weight, uint32_t w_dtype,
                                float eps, float *xn, uint8_t *codes, float *scales, float *inv, uint32_t *flags,
                                cudaStream_t stream) {
  if (cols == 0 || cols % 256u || cols / 256u > kRmsMaxBlocks || (w_dtype != PW_NORM_F32 && w_dtype != PW_NORM_BF16))
    return cudaErrorInvalidValue;
  if (rows == 0) return cudaSuccess;
  if (w_dtype == PW_NORM_F32)
    return launch_kernel(k_rms_quantize<true>, dim3(rows), dim3(256), 0, stream, x, cols, weight, eps, xn, codes,
                         scales, inv, flags);
  return launch_kernel(k_rms_quantize<false>, dim3(rows), dim3(256), 0, stream, x, cols, weight, eps, xn, codes, scales,
                       inv, flags);
}

// ---------------------------------------------------------- partial sums
// A projection computed over slices of its K axis (the dense MLP's 16384-wide
// down projection): the slice sums are added in slice order, then rounded.
__global__ void k_sum_partials(const float *__restrict__ p, uint32_t n_parts, uint64_t n, float *__restrict__ y,
                               uint32_t round, uint32_t *flags) {
  pdl_wait();
  pdl_launch_dependents();
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x) {
    float acc = p[i];
    for (uint32_t k = 1; k < n_parts; ++k) acc = __fadd_rn(acc, p[k * n + i]);
    if (round) acc = round_bf16(acc);
    if (!finite(acc)) raise_flag(flags, PW_FLAG_NONFINITE_ROUND);
    y[i] = acc;
  }
}

cudaError_t launch_sum_partials(const float *p, uint32_t n_parts, uint64_t n, float *y, uint32_t round,
                                uint32_t *flags, cudaStream_t stream) {
  if (n_parts == 0) return cudaErrorInvalidValue;
  if (n == 0) return cudaSuccess;
  uint64_t blocks = (n + 255u) / 256u;
  if (blocks > 148u * 8u) blocks = 148u * 8u;
  return launch_kernel(k_sum_partials, dim3((unsigned)blocks), dim3(256), 0, stream, p, n_parts, n, y, round, flags);
}

// --------------------------------------------------------------- bf16 round
__global__ void k_round_bf16(float *v, uint32_t n, uint32_t *flags) {
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const float r = round_bf16(v[i]);
    if (!finite(r)) raise_flag(flags, PW_FLAG_NONFINITE_ROUND);
    v[i] = r;
  }
}

cudaError_t launch_round_bf16(float *v, uint32_t n, uint32_t *flags, cudaStream_t stream) {
  if (n == 0) return cudaSuccess;
  unsigned blocks = (n + 255u) / 256u;
  if (blocks > 148u * 8u) blocks = 148u * 8u;
  k_round_bf16<<<blocks, 256, 0, stream>>>(v, n, flags);
  return cudaGetLastError();
}

// ------------------------------------------------------------ router logits
// logit[t,e] = sum_c x[t,c] * w[e,c] in f32 in a fixed order (the oracle's
// pwo_router_logits restates it; the reference's own logits are f32 too,
// from an SGEMM of unspecified order): the K axis is cut into 256-column
// slices; slice s's sum is a chain of fused multiply-adds from +0 over its
// columns in ascending order; the logit adds the slice sums in slice order
// starting from slice 0's.  bf16 weights widen to f32 exactly (a shift).
constexpr uint32_t kRouterSlice = 256;

__device__ __forceinline__ float bf16lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

// Decode widths: one CTA per (slice, 32 experts, 8 tokens) stages the
// slice's activation columns and weight rows in shared memory with coalesced
// loads; thread (token, expert) then runs its chain from shared memory (the
// warp shares a token: broadcast reads of x, consecutive experts' weights).
// The slice sums go to the same partials as the prefill kernel.  WT is the
// router weight's storage type: float (the checkpoint's F32 gate.weight) or
// uint16_t (bf16 bits, widened exactly); the f32 chain is the same.
// With q_codes, the CTAs of the first expert block also quantize the staged
// activation slice for the experts (its two 128-column groups per token, a
// warp per token, the same steps as k_quantize), so the decode chain has no
// separate quantize launch.
constexpr int kRouterTok = 8;
constexpr uint32_t kRouterMaxSlices = 64;  // hidden <= 16384

__device__ __forceinline__ float router_w(float v) { return v; }
__device__ __forceinline__ float router_w(uint16_t v) { return __uint_as_float((uint32_t)v << 16); }

template <typename WT>
__global__ void __launch_bounds__(256) k_router_slices_small(const float *__restrict__ x, uint32_t tokens,
                                                             const WT *__restrict__ w, uint32_t experts,
                                                             uint32_t hidden, float *__restrict__ part,
                                                             uint8_t *__restrict__ q_codes,
                                                             float *__restrict__ q_scales, uint32_t *flags) {
  constexpr uint32_t kPer = 16u / sizeof(WT);  // weight values per 16-byte load
  __shared__ __align__(16) float xs[kRouterTok][kRouterSlice];
  __shared__ __align__(16) WT ws[kRouterSlice][32];
  const uint32_t s = blockIdx.x, e0 = blockIdx.y * 32u, t0 = blockIdx.z * kRouterTok;
  const uint32_t tid = threadIdx.x, col0 = kRouterSlice * s;
  // every 16-byte load of the CTA is in flight before the first store (one
  // memory round trip instead of one per loop iteration)
  constexpr uint32_t kXLoads = (uint32_t)kRouterTok * kRouterSlice / 4u / 256u;
  constexpr uint32_t kWLoads = 32u * kRouterSlice / kPer / 256u;
  float4 xv[kXLoads];
  uint4 wv[kWLoads];
  // the router weight is not written by the kernels before this one, so
  // under programmatic dependent launch it is fetched before the wait
#pragma unroll
  for (uint32_t k = 0; k < kWLoads; ++k) {
    const uint32_t i = tid + 256u * k, el = i % 32u, cq = i / 32u;  // lanes: consecutive experts
    wv[k] = e0 + el < experts ? __ldg(reinterpret_cast<const uint4 *>(w + (size_t)(e0 + el) * hidden + col0) + cq)
                              : make_uint4(0u, 0u, 0u, 0u);
  }
  pdl_wait();
  pdl_launch_dependents();
#pragma unroll
  for (uint32_t k = 0; k < kXLoads; ++k) {
    const uint32_t i = tid + 256u * k, j = i / (kRouterSlice / 4u), c4 = i % (kRouterSlice / 4u);
    xv[k] = t0 + j < tokens ? __ldg(reinterpret_cast<const float4 *>(x + (size_t)(t0 + j) * hidden + col0) + c4)
                            : make_float4(0.f, 0.f, 0.f, 0.f);
  }
#pragma unroll
  for (uint32_t k = 0; k < kXLoads; ++k) {
    const uint32_t i = tid + 256u * k;
    reinterpret_cast<float4 *>(&xs[i / (kRouterSlice / 4u)][0])[i % (kRouterSlice / 4u)] = xv[k];
  }
#pragma unroll
  for (uint32_t k = 0; k < kWLoads; ++k) {
    const uint32_t i = tid + 256u * k, el = i % 32u, cq = i / 32u;  // conflict-free stores
    const WT *v = reinterpret_cast<const WT *>(&wv[k]);
#pragma unroll
    for (uint32_t q = 0; q < kPer; ++q) ws[kPer * cq + q][el] = v[q];
  }
  __syncthreads();
  const uint32_t el = tid % 32u, j = tid / 32u;
  float acc = 0.0f;
#pragma unroll 16
  for (uint32_t i = 0; i < kRouterSlice; ++i) acc = __fmaf_rn(xs[j][i], router_w(ws[i][el]), acc);
  if (t0 + j < tokens && e0 + el < experts) part[((size_t)s * tokens + t0 + j) * experts + e0 + el] = acc;
  if (q_codes && blockIdx.y == 0u && t0 + j < tokens) {
    // warp j: token t0 + j, groups 2 s and 2 s + 1 (lane l holds values 4l..4l+3)
#pragma unroll
    for (uint32_t g = 0; g < 2u; ++g) {
      const float4 v = reinterpret_cast<const float4 *>(&xs[j][g * 128u])[el];
      const bool ok = finite(v.x) && finite(v.y) && finite(v.z) && finite(v.w);
      if (!ok) raise_flag(flags, PW_FLAG_NONFINITE_INPUT);
      float m = ok ? fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))) : 0.0f;
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      const Fp8GroupScale gs = Fp8GroupScale::of(m);
      auto q = [&](float val) { return gs.quotient(val); };
      const uint32_t lo = encode2(q(v.x), q(v.y));
      const uint32_t hi = encode2(q(v.z), q(v.w));
      const size_t grp = (size_t)(t0 + j) * (hidden / 128u) + 2u * s + g;
      reinterpret_cast<uint32_t *>(q_codes + grp * 128u)[el] = lo | (hi << 16);
      if (el == 0) q_scales[grp] = gs.scale;
    }
  }
}

// Prefill widths: the slice chains as a register-tiled product.  Work unit:
// 64 tokens x EXPT experts (128, or 64 when 128-expert units would leave SMs
// idle: the expert-parallel ranks' few hundred tokens) x one slice (256
// columns, 8 stages of 32); thread (tg, eg) owns tokens 8tg..8tg+7 and
// experts 4eg..4eg+3 (+ 64 + the same for EXPT = 128), one f32 chain each
// (packed f32x2 FMAs over expert pairs; each lane of a pair rounds like
// fmaf).  Stages are double-buffered in shared memory and fetched one stage
// ahead into registers; persistent CTAs walk the units and store each unit's
// slice sums to partials [slice][token][expert], which k_router_topk adds in
// slice order.  The tile shape changes which thread computes a chain, never
// the chain.
namespace rp {
constexpr int kCols = 32, kThreads = 128;
constexpr uint32_t kStages = kRouterSlice / kCols;
template <int EXPT, int TOK>
struct Smem {
  float xs[2][kCols][TOK];   // activation [column][token]
  float ws[2][kCols][EXPT];  // router weight widened to f32 [column][expert]
};
}  // namespace rp

struct RouterUnits {
  uint32_t tokens, experts, hidden, slices, tiles_e, n_units, exp_tile, tok_tile;
};

struct RouterCursor {
  uint32_t u, st, s, t0, e0;
  __device__ __forceinline__ void decode(const RouterUnits &g) {
    if (u >= g.n_units) return;
    s = u % g.slices;
    const uint32_t tile = u / g.slices;
    e0 = (tile % g.tiles_e) * g.exp_tile;
    t0 = (tile / g.tiles_e) * g.tok_tile;
  }
  __device__ __forceinline__ bool valid(const RouterUnits &g) const { return u < g.n_units; }
  // one stage on; true when the unit is finished (the caller enters the next)
  __device__ __forceinline__ bool step() {
    if (++st < rp::kStages) return false;
    st = 0;
    return true;
  }
  __device__ __forceinline__ void enter(uint32_t unit, const RouterUnits &g) {
    u = unit;
    decode(g);
  }
  __device__ __forceinline__ uint32_t base() const { return kRouterSlice * s + rp::kCols * st; }
};

// One stage's global loads, fetched a stage ahead: TOK tokens x 32 columns of
// x and EXPT experts x 32 columns of the weight.
template <bool F32W, int EXPT, int TOK>
struct RouterStage {
  static constexpr int kX = TOK * rp::kCols / 4 / rp::kThreads;                      // float4 x loads
  static constexpr int kW = EXPT * rp::kCols * (F32W ? 4 : 2) / 16 / rp::kThreads;  // 16-byte weight loads
  float4 x[kX];
  uint4 w[kW];
};

// Shared-memory layout: xs[column][token] and ws[column][expert] (f32), read
// by the product as float4 runs of 4 tokens / 4 experts.  The global loads are
// row-wise coalesced: a warp loads 4 token rows x 128 B of x, and 8 expert rows
// x 64 B (bf16) or 4 x 128 B (f32) of the weight.  Storing them column-wise
// would put a warp's stores in few banks, so each row's float4 slots are
// permuted by an XOR with a function of the row (xs_slot / ws_slot): the
// stores become conflict-free and the product's float4 reads stay whole.
__device__ __forceinline__ uint32_t xs_slot(uint32_t col, uint32_t slot) { return slot ^ ((col >> 2) & 7u); }
template <bool F32W>
__device__ __forceinline__ uint32_t ws_slot(uint32_t col, uint32_t slot) {
  return F32W ? slot ^ ((col >> 2) & 7u) : slot ^ (2u * ((col >> 3) & 3u));
}

template <bool F32W, int EXPT, int TOK>
__device__ __forceinline__ void router_gload(const float *__restrict__ x, const void *__restrict__ wv,
                                             const RouterUnits &g, const RouterCursor &c,
                                             RouterStage<F32W, EXPT, TOK> &r) {
  const uint32_t base = c.base();
#pragma unroll
  for (int m = 0; m < RouterStage<F32W, EXPT, TOK>::kX; ++m) {
    const uint32_t i = threadIdx.x + rp::kThreads * m;
    const uint32_t tok = c.t0 + i / 8u, c4 = i % 8u;  // x: 8 lanes per token row
    r.x[m] = tok < g.tokens ? __ldg(reinterpret_cast<const float4 *>(x + (size_t)tok * g.hidden + base + 4u * c4))
                            : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  constexpr uint32_t kPer = F32W ? 4u : 8u;       // weight columns per 16-byte load
  constexpr uint32_t kLoadsRow = 32u / kPer;       // 16-byte loads per expert row of the stage
  const unsigned char *w = static_cast<const unsigned char *>(wv);
  const size_t esz = F32W ? 4u : 2u;
#pragma unroll
  for (int m = 0; m < RouterStage<F32W, EXPT, TOK>::kW; ++m) {
    const uint32_t i = threadIdx.x + rp::kThreads * m;
    const uint32_t e = c.e0 + i / kLoadsRow, cq = i % kLoadsRow;  // w: consecutive lanes along the row
    r.w[m] = e < g.experts ? __ldg(reinterpret_cast<const uint4 *>(w + ((size_t)e * g.hidden + base + kPer * cq) * esz))
                           : make_uint4(0u, 0u, 0u, 0u);
  }
}

template <bool F32W, int EXPT, int TOK>
__device__ __forceinline__ void router_sstore(rp::Smem<EXPT, TOK> &sm, int b, const RouterStage<F32W, EXPT, TOK> &r) {
#pragma unroll
  for (int m = 0; m < RouterStage<F32W, EXPT, TOK>::kX; ++m) {
    const uint32_t i = threadIdx.x + rp::kThreads * m;
    const uint32_t tok = i / 8u, c4 = i % 8u;
    const float v[4] = {r.x[m].x, r.x[m].y, r.x[m].z, r.x[m].w};
#pragma unroll
    for (uint32_t j = 0; j < 4u; ++j) {
      const uint32_t col = 4u * c4 + j;
      sm.xs[b][col][4u * xs_slot(col, tok / 4u) + tok % 4u] = v[j];
    }
  }
  constexpr uint32_t kLoadsRow = F32W ? 8u : 4u;
#pragma unroll
  for (int m = 0; m < RouterStage<F32W, EXPT, TOK>::kW; ++m) {
    const uint32_t i = threadIdx.x + rp::kThreads * m;
    const uint32_t e = i / kLoadsRow, cq = i % kLoadsRow;
    const uint32_t q[4] = {r.w[m].x, r.w[m].y, r.w[m].z, r.w[m].w};
#pragma unroll
    for (uint32_t j = 0; j < 4u; ++j) {
      if (F32W) {
        const uint32_t col = 4u * cq + j;
        sm.ws[b][col][4u * ws_slot<F32W>(col, e / 4u) + e % 4u] = __uint_as_float(q[j]);
      } else {
        const uint32_t c0 = 8u * cq + 2u * j, c1 = c0 + 1u;
        sm.ws[b][c0][4u * ws_slot<F32W>(c0, e / 4u) + e % 4u] = bf16lo(q[j]);
        sm.ws[b][c1][4u * ws_slot<F32W>(c1, e / 4u) + e % 4u] = bf16hi(q[j]);
      }
    }
  }
}

// Units (TOK tokens x EXPT experts x one 256-column slice) are handed out
// dynamically: each CTA starts on unit blockIdx.x and takes the next free one
// from work[0] when it finishes a unit, so the SMs finish together (a fixed
// round-robin left the last wave ~15% idle).  Results do not depend on which
// CTA runs a unit.  The last CTA to exit zeroes work[0..1] for the next launch.
// Thread (tg, eg) owns tokens TT tg .. TT tg + TT - 1 (TT = TOK / 8).
template <int EXPT, int TOK>
constexpr int router_ctas_per_sm() {
  return TOK == 64 ? 3 : 4;
}

template <bool F32W, int EXPT, int TOK>
__global__ void __launch_bounds__(rp::kThreads, router_ctas_per_sm<EXPT, TOK>())
    k_router_partials(const float *__restrict__ x, const void *__restrict__ w, RouterUnits g,
                      float *__restrict__ part, uint32_t *__restrict__ work) {
  constexpr int NP = EXPT / 32;  // f32x2 expert pairs per thread and token
  constexpr int TT = TOK / 8;    // tokens per thread
  pdl_wait();
  pdl_launch_dependents();
  extern __shared__ __align__(16) unsigned char router_smem[];
  __shared__ uint32_t next_unit;  // written by thread 0 one stage after each unit change
  rp::Smem<EXPT, TOK> &sm = *reinterpret_cast<rp::Smem<EXPT, TOK> *>(router_smem);
  const uint32_t lane = threadIdx.x % 32u, wp = threadIdx.x / 32u;
  const uint32_t eg = lane % 16u, tg = 2u * wp + lane / 16u;
  if (threadIdx.x == 0) next_unit = gridDim.x + atomicAdd(work, 1u);
  RouterCursor ld{blockIdx.x, 0, 0, 0, 0};
  ld.decode(g);
  RouterCursor cp = ld;
  RouterStage<F32W, EXPT, TOK> r;
  if (ld.valid(g)) router_gload(x, w, g, ld, r);
  __syncthreads();  // next_unit
  bool refresh = false;
  auto advance_ld = [&]() {
    if (ld.step()) {
      ld.enter(next_unit, g);
      refresh = true;
    }
  };
  if (ld.valid(g)) {
    advance_ld();
    router_sstore(sm, 0, r);
  }
  bool have = ld.valid(g);
  if (have) {
    router_gload(x, w, g, ld, r);
    advance_ld();
  }
  __syncthreads();

  float2 acc[TT][NP];
#pragma unroll
  for (int t = 0; t < TT; ++t)
#pragma unroll
    for (int p = 0; p < NP; ++p) acc[t][p] = make_float2(0.f, 0.f);
  int b = 0;
  while (cp.valid(g)) {
#pragma unroll 4
    for (int k = 0; k < rp::kCols; ++k) {
      float xv[TT];
#pragma unroll
      for (int q = 0; q < TT / 4; ++q) {
        const float4 xq = *reinterpret_cast<const float4 *>(&sm.xs[b][k][4u * xs_slot(k, (TT * tg) / 4u + q)]);
        xv[4 * q] = xq.x;
        xv[4 * q + 1] = xq.y;
        xv[4 * q + 2] = xq.z;
        xv[4 * q + 3] = xq.w;
      }
      float2 wv[NP];
#pragma unroll
      for (int h = 0; h < NP / 2; ++h) {
        const float4 wq = *reinterpret_cast<const float4 *>(&sm.ws[b][k][4u * ws_slot<F32W>(k, 16u * h + eg)]);
        wv[2 * h] = make_float2(wq.x, wq.y);
        wv[2 * h + 1] = make_float2(wq.z, wq.w);
      }
#pragma unroll
      for (int t = 0; t < TT; ++t) {
        const float2 xd = make_float2(xv[t], xv[t]);
#pragma unroll
        for (int p = 0; p < NP; ++p) acc[t][p] = __ffma2_rn(wv[p], xd, acc[t][p]);
      }
    }
    if (cp.st == rp::kStages - 1u) {  // the unit's slice chains are complete
      float *dst = part + (size_t)cp.s * g.tokens * g.experts;
#pragma unroll
      for (int t = 0; t < TT; ++t) {
        const uint32_t tok = cp.t0 + (uint32_t)(TT * tg + t);
        if (tok < g.tokens) {
          float *row = dst + (size_t)tok * g.experts;
#pragma unroll
          for (int hlf = 0; hlf < NP / 2; ++hlf) {
            const uint32_t e = cp.e0 + 64u * hlf + 4u * eg;
            const float v[4] = {acc[t][2 * hlf].x, acc[t][2 * hlf].y, acc[t][2 * hlf + 1].x, acc[t][2 * hlf + 1].y};
            if ((g.experts & 3u) == 0u && e + 3u < g.experts) {
              *reinterpret_cast<float4 *>(row + e) = make_float4(v[0], v[1], v[2], v[3]);
            } else {
#pragma unroll
              for (int j = 0; j < 4; ++j)
                if (e + j < g.experts) row[e + j] = v[j];
            }
          }
        }
#pragma unroll
        for (int p = 0; p < NP; ++p) acc[t][p] = make_float2(0.f, 0.f);
      }
    }
    if (have) router_sstore(sm, b ^ 1, r);
    have = ld.valid(g);
    if (have) {
      router_gload(x, w, g, ld, r);
      advance_ld();
    }
    __syncthreads();
    // every thread has read next_unit for the unit ld entered before this
    // barrier; the next read is a whole unit (8 stages, 8 barriers) away
    if (refresh) {
      if (threadIdx.x == 0) next_unit = gridDim.x + atomicAdd(work, 1u);
      refresh = false;
    }
    b ^= 1;
    // the loader runs two stages ahead and a unit has eight: the unit the
    // compute cursor enters is the one the loader is in
    if (cp.step()) cp.enter(ld.u, g);
  }
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(work + 1, 1u) == gridDim.x - 1u) {
      work[0] = 0u;
      work[1] = 0u;
    }
  }
}

static RouterUnits router_units(uint32_t tokens, uint32_t experts, uint32_t hidden, uint32_t exp_tile = 128u,
                                uint32_t tok_tile = 64u) {
  RouterUnits g{};
  g.tokens = tokens;
  g.experts = experts;
  g.hidden = hidden;
  g.slices = hidden / kRouterSlice;
  g.exp_tile = exp_tile;
  g.tok_tile = tok_tile;
  g.tiles_e = (experts + exp_tile - 1) / exp_tile;
  const uint32_t tiles_t = (tokens + tok_tile - 1) / tok_tile;
  g.n_units = tiles_t * g.tiles_e * g.slices;
  return g;
}

constexpr uint32_t kRouterPartialMinTokens = 64;  // below: k_router_slices_small
constexpr uint32_t kRouterTopkCtaMaxTokens = 256;  // below: k_router_topk_cta

size_t router_scratch_floats(uint32_t tokens, uint32_t experts, uint32_t hidden) {
  return (size_t)tokens * experts * (hidden / kRouterSlice);
}

// --------------------------------------------------------------- router top-k
// One warp per token (src/text_endpoint.rs:4394 pytorch_noaux_routes): the
// logit (read, or the slice sums added in slice order); score =
// SLEEF sigmoid(logit); corrected = score + bias; 9 rounds of warp argmax
// (ties -> lower index) give the 8 picks in canonical order and the first
// rejected value (boundary margin / tie detection).
// weight_k = score_k / (pairwise sum of the 8 + 1e-20) (src/text_endpoint.rs:4382).
__device__ __forceinline__ bool better(float va, uint32_t ia, float vb, uint32_t ib) {
  return va > vb || (va == vb && ia < ib);
}

__device__ __forceinline__ void argmax_shfl(float &bv, uint32_t &bi, float &bs) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
    const float os = __shfl_xor_sync(0xffffffffu, bs, o);
    if (better(ov, oi, bv, bi)) {
      bv = ov;
      bi = oi;
      bs = os;
    }
  }
}

// Token t's picks and weights by one warp (lane l holds experts l + 32 k):
// the logit (the slice sums added in slice order), score = SLEEF
// sigmoid(logit), corrected = score + bias; 9 rounds of warp argmax (ties ->
// lower index) give the 8 picks in canonical order and the first rejected
// value (boundary tie detection).
template <int NPL>
__device__ __forceinline__ void topk_token_warp(const float *__restrict__ src, uint32_t slices,
                                                const float (&bias_r)[NPL], uint32_t tokens, uint32_t experts,
                                                uint32_t t, uint32_t *selected, float *weights, uint32_t *tie_rows,
                                                uint32_t *flags) {
  const uint32_t lane = threadIdx.x % 32u;
  const float ninf = -__int_as_float(0x7f800000);
  const size_t plane = (size_t)tokens * experts;
  float score[NPL], corr[NPL];
  bool bad = false;
#pragma unroll
  for (int k = 0; k < NPL; ++k) {
    const uint32_t e = lane + 32u * k;
    score[k] = 0.0f;
    corr[k] = ninf;
    if (e < experts) {
      const float *p = src + (size_t)t * experts + e;
      float lg;
      if (slices <= 16u) {  // independent loads first, then the ordered sum
        float v[16];
#pragma unroll
        for (uint32_t q = 0; q < 16u; ++q) v[q] = q < slices ? __ldcs(p + q * plane) : 0.0f;
        lg = v[0];
#pragma unroll
        for (uint32_t q = 1; q < 16u; ++q)
          if (q < slices) lg = __fadd_rn(lg, v[q]);
      } else {
        lg = p[0];
        for (uint32_t q = 1; q < slices; ++q) lg = __fadd_rn(lg, p[q * plane]);
      }
      bad |= !finite(lg) || !finite(bias_r[k]);
      score[k] = sigmoid_sleef(lg);
      corr[k] = __fadd_rn(score[k], bias_r[k]);
    }
  }
  if (bad) raise_flag(flags, PW_FLAG_NONFINITE_INPUT);
  // 9 rounds of warp argmax (ties -> lower index): lane r keeps round r's
  // pick (corrected value, expert, unbiased score)
  uint32_t taken = 0;
  float my_v = ninf, my_s = 0.0f;
  uint32_t my_i = 0xffffffffu;
#pragma unroll 1
  for (uint32_t round = 0; round < 9u; ++round) {
    float bv = ninf, bs = 0.0f;
    uint32_t bi = 0xffffffffu;
#pragma unroll
    for (int k = 0; k < NPL; ++k) {
      const uint32_t e = lane + 32u * k;
      if (e < experts && !((taken >> k) & 1u) && better(corr[k], e, bv, bi)) {
        bv = corr[k];
        bi = e;
        bs = score[k];
      }
    }
    argmax_shfl(bv, bi, bs);
    if (lane == round) {
      my_v = bv;
      my_i = bi;
      my_s = bs;
    }
    if (round < 8u && bi != 0xffffffffu && bi % 32u == lane) taken |= 1u << (bi / 32u);
  }
  // weight_k = score_k / (pairwise sum of the 8 + 1e-20), src/text_endpoint.rs:4382
  const float s4 = __shfl_down_sync(0xffffffffu, my_s, 4);  // lane k < 4: score of pick k + 4
  const float lk = __fadd_rn(my_s, s4);                      // lane k < 4: l_k
  const float l0 = __shfl_sync(0xffffffffu, lk, 0), l1 = __shfl_sync(0xffffffffu, lk, 1);
  const float l2 = __shfl_sync(0xffffffffu, lk, 2), l3 = __shfl_sync(0xffffffffu, lk, 3);
  const float den = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(0.0f, l0), l1), l2), l3), 1.0e-20f);
  const float wk = __fdiv_rn(my_s, den);
  const bool ok_k = lane >= 8u || (finite(wk) && wk >= 0.0f && my_i < experts);
  float sum = 0.0f;
#pragma unroll
  for (int k = 0; k < 8; ++k) sum = __fadd_rn(sum, __shfl_sync(0xffffffffu, wk, k));
  const bool all_ok = __all_sync(0xffffffffu, ok_k);
  if (lane < 8u) {
    selected[(size_t)t * 8 + lane] = my_i;
    weights[(size_t)t * 8 + lane] = wk;
  }
  const float v7 = __shfl_sync(0xffffffffu, my_v, 7), v8 = __shfl_sync(0xffffffffu, my_v, 8);
  if (lane == 0) {
    if (!all_ok || fabsf(__fsub_rn(sum, 1.0f)) > 1.0e-6f) raise_flag(flags, PW_FLAG_ROUTE_WEIGHTS);
    if (v7 == v8 && tie_rows) atomicAdd(tie_rows, 1u);
  }
}

template <int NPL>
__global__ void __launch_bounds__(256) k_router_topk(const float *__restrict__ src, uint32_t slices,
                                                     const float *__restrict__ bias, uint32_t tokens,
                                                     uint32_t experts, uint32_t *__restrict__ selected,
                                                     float *__restrict__ weights, uint32_t *tie_rows,
                                                     uint32_t *flags) {
  // Persistent warps loop over tokens: the code stays hot in the instruction
  // cache (a warp per token and launch ran each instruction once, and stalled
  // on instruction fetch: ~22 us per call at any token count).
  const uint32_t lane = threadIdx.x % 32u;
  const uint32_t nwarps = gridDim.x * (blockDim.x / 32u);
  float bias_r[NPL];  // the bias is no kernel's output: fetched before the wait
#pragma unroll
  for (int k = 0; k < NPL; ++k) {
    const uint32_t e = lane + 32u * k;
    bias_r[k] = e < experts ? __ldg(bias + e) : 0.0f;
  }
  pdl_wait();
  pdl_launch_dependents();
  for (uint32_t t = blockIdx.x * (blockDim.x / 32u) + threadIdx.x / 32u; t < tokens; t += nwarps)
    topk_token_warp<NPL>(src, slices, bias_r, tokens, experts, t, selected, weights, tie_rows, flags);
}

// The same selection with a whole CTA per token (experts <= 256, one expert
// per thread): every thread loads its expert's slice sums at once, each warp
// keeps its 9 best (corrected value, expert) under the same total order
// (value descending, then expert ascending), and warp 0 picks the 9 best of
// those 72.  The top 9 of the union of per-warp top 9s is the top 9 overall,
// so picks, weights and the tie test equal k_router_topk's; the token's
// critical path is one round of loads and two 9-round selections instead of
// 8 expert columns per lane in sequence.  CTAs loop over tokens.
__global__ void __launch_bounds__(256) k_router_topk_cta(const float *__restrict__ src, uint32_t slices,
                                                         const float *__restrict__ bias, uint32_t tokens,
                                                         uint32_t experts, uint32_t *__restrict__ selected,
                                                         float *__restrict__ weights, uint32_t *tie_rows,
                                                         uint32_t *flags) {
  pdl_wait();
  pdl_launch_dependents();
  __shared__ float cv[8][9], cs[8][9];
  __shared__ uint32_t ci[8][9];
  const uint32_t tid = threadIdx.x, lane = tid % 32u, warp = tid / 32u;
  const float ninf = -__int_as_float(0x7f800000);
  const size_t plane = (size_t)tokens * experts;
  const uint32_t e = tid;
  const bool valid = e < experts;
  const float b = valid ? __ldg(bias + e) : 0.0f;
  for (uint32_t t = blockIdx.x; t < tokens; t += gridDim.x) {
    float score = 0.0f, corr = ninf;
    uint32_t idx = 0xffffffffu;
    if (valid) {
      const float *p = src + (size_t)t * experts + e;
      float lg;
      if (slices <= 16u) {  // independent loads first, then the ordered sum
        float v[16];
#pragma unroll
        for (uint32_t q = 0; q < 16u; ++q) v[q] = q < slices ? __ldcs(p + q * plane) : 0.0f;
        lg = v[0];
#pragma unroll
        for (uint32_t q = 1; q < 16u; ++q)
          if (q < slices) lg = __fadd_rn(lg, v[q]);
      } else {
        lg = p[0];
        for (uint32_t q = 1; q < slices; ++q) lg = __fadd_rn(lg, p[q * plane]);
      }
      if (!finite(lg) || !finite(b)) raise_flag(flags, PW_FLAG_NONFINITE_INPUT);
      score = sigmoid_sleef(lg);
      corr = __fadd_rn(score, b);
      idx = e;
    }
    // this warp's 9 best: lane r keeps round r's pick
    bool taken = false;
#pragma unroll 1
    for (uint32_t round = 0; round < 9u; ++round) {
      float bv = taken ? ninf : corr, bs = taken ? 0.0f : score;
      uint32_t bi = taken ? 0xffffffffu : idx;
      argmax_shfl(bv, bi, bs);
      if (lane == round) {
        cv[warp][round] = bv;
        ci[warp][round] = bi;
        cs[warp][round] = bs;
      }
      if (bi != 0xffffffffu && bi == idx) taken = true;
    }
    __syncthreads();
    if (warp == 0) {
      // 72 candidates, slots lane, lane + 32, lane + 64
      float v[3], sc[3];
      uint32_t ix[3];
#pragma unroll
      for (int k = 0; k < 3; ++k) {
        const uint32_t c = lane + 32u * (uint32_t)k;
        const bool in = c < 72u;
        v[k] = in ? cv[c / 9u][c % 9u] : ninf;
        ix[k] = in ? ci[c / 9u][c % 9u] : 0xffffffffu;
        sc[k] = in ? cs[c / 9u][c % 9u] : 0.0f;
      }
      uint32_t took = 0;
      float my_v = ninf, my_s = 0.0f;
      uint32_t my_i = 0xffffffffu;
#pragma unroll 1
      for (uint32_t round = 0; round < 9u; ++round) {
        float bv = ninf, bs = 0.0f;
        uint32_t bi = 0xffffffffu;
#pragma unroll
        for (int k = 0; k < 3; ++k)
          if (!((took >> k) & 1u) && ix[k] != 0xffffffffu && better(v[k], ix[k], bv, bi)) {
            bv = v[k];
            bi = ix[k];
            bs = sc[k];
          }
        argmax_shfl(bv, bi, bs);
        if (lane == round) {
          my_v = bv;
          my_i = bi;
          my_s = bs;
        }
#pragma unroll
        for (int k = 0; k < 3; ++k)
          if (bi != 0xffffffffu && ix[k] == bi) took |= 1u << k;
      }
      // weight_k = score_k / (pairwise sum of the 8 + 1e-20), src/text_endpoint.rs:4382
      const float s4 = __shfl_down_sync(0xffffffffu, my_s, 4);
      const float lk = __fadd_rn(my_s, s4);
      const float l0 = __shfl_sync(0xffffffffu, lk, 0), l1 = __shfl_sync(0xffffffffu, lk, 1);
      const float l2 = __shfl_sync(0xffffffffu, lk, 2), l3 = __shfl_sync(0xffffffffu, lk, 3);
      const float den = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(0.0f, l0), l1), l2), l3), 1.0e-20f);
      const float wk = __fdiv_rn(my_s, den);
      const bool ok_k = lane >= 8u || (finite(wk) && wk >= 0.0f && my_i < experts);
      float sum = 0.0f;
#pragma unroll
      for (int k = 0; k < 8; ++k) sum = __fadd_rn(sum, __shfl_sync(0xffffffffu, wk, k));
      const bool all_ok = __all_sync(0xffffffffu, ok_k);
      if (lane < 8u) {
        selected[(size_t)t * 8 + lane] = my_i;
        weights[(size_t)t * 8 + lane] = wk;
      }
      const float v7 = __shfl_sync(0xffffffffu, my_v, 7), v8 = __shfl_sync(0xffffffffu, my_v, 8);
      if (lane == 0) {
        if (!all_ok || fabsf(__fsub_rn(sum, 1.0f)) > 1.0e-6f) raise_flag(flags, PW_FLAG_ROUTE_WEIGHTS);
        if (v7 == v8 && tie_rows) atomicAdd(tie_rows, 1u);
      }
    }
    __syncthreads();  // the candidates are rewritten by the next token
  }
}

template <bool F32W, int EXPT, int TOK>
static cudaError_t launch_partials(const float *x, const void *w, const RouterUnits &g, float *scratch, uint32_t *work,
                                   int num_sms, cudaStream_t stream) {
  using Sm = rp::Smem<EXPT, TOK>;
  static bool configured = false;
  if (!configured) {
    const cudaError_t st = cudaFuncSetAttribute(k_router_partials<F32W, EXPT, TOK>,
                                                cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(Sm));
    if (st != cudaSuccess) return st;
    configured = true;
  }
  // three or four 4-warp CTAs per SM: with fewer warps per scheduler the FMA
  // pipe idled on every short dependency (one CTA: ~50% FMA-pipe activity,
  // two: 58%)
  const uint32_t slots = (uint32_t)router_ctas_per_sm<EXPT, TOK>() * (uint32_t)num_sms;
  const uint32_t grid = g.n_units < slots ? g.n_units : slots;
  return launch_kernel(k_router_partials<F32W, EXPT, TOK>, dim3(grid), dim3(rp::kThreads), sizeof(Sm), stream, x, w,
                       g, scratch, work);
}

bool router_fuses_quantize(uint32_t tokens) { return tokens < kRouterPartialMinTokens; }

template <bool F32W>
static cudaError_t launch_router_logits(const float *x, uint32_t tokens, const void *w, const RouterUnits &g,
                                        float *scratch, uint32_t *work, int num_sms, cudaStream_t stream,
                                        uint8_t *q_codes, float *q_scales, uint32_t *flags) {
  if (tokens >= kRouterPartialMinTokens) {
    if (q_codes) return cudaErrorInvalidValue;  // only the decode kernel quantizes
    // The largest unit that still gives every CTA slot two or more units:
    // 64 tokens x 128 experts, then 64 x 64, then 32 x 64.  With fewer units
    // most slots run one or two whole units and the smaller ones finish first
    // (measured per pw_route call: 2048 tokens, 145 us with 128-expert units
    // vs 182 with 64; 1024 tokens, 132 vs 100 vs 121 with 32-token units;
    // 512 tokens, 97 with 64 x 64 vs 84 with 32 x 64).
    const uint32_t sms = (uint32_t)num_sms;
    if (g.n_units >= 2u * (uint32_t)router_ctas_per_sm<128, 64>() * sms)
      return launch_partials<F32W, 128, 64>(x, w, g, scratch, work, num_sms, stream);
    const RouterUnits g64 = router_units(g.tokens, g.experts, g.hidden, 64u, 64u);
    if (g64.n_units >= 2u * (uint32_t)router_ctas_per_sm<64, 64>() * sms)
      return launch_partials<F32W, 64, 64>(x, w, g64, scratch, work, num_sms, stream);
    const RouterUnits g32 = router_units(g.tokens, g.experts, g.hidden, 64u, 32u);
    return launch_partials<F32W, 64, 32>(x, w, g32, scratch, work, num_sms, stream);
  }
  using WT = typename std::conditional<F32W, float, uint16_t>::type;
  return launch_kernel(k_router_slices_small<WT>,
                       dim3(g.slices, (g.experts + 31u) / 32u, (tokens + kRouterTok - 1) / kRouterTok), dim3(256), 0,
                       stream, x, tokens, static_cast<const WT *>(w), g.experts, g.hidden, scratch, q_codes, q_scales,
                       flags);
}

cudaError_t launch_router(const float *x, uint32_t tokens, const void *w, uint32_t w_dtype, const float *bias,
                          uint32_t experts, uint32_t hidden, float *scratch, uint32_t *selected, float *weights,
                          uint32_t *tie_rows, uint32_t *flags, uint32_t *work, int num_sms, cudaStream_t stream,
                          uint8_t *q_codes, float *q_scales) {
  if (hidden % 512u || hidden > kRouterSlice * kRouterMaxSlices || tokens == 0 || experts <= 8 || experts > 1024u ||
      (w_dtype != PW_ROUTER_BF16 && w_dtype != PW_ROUTER_F32))
    return cudaErrorInvalidValue;
  const RouterUnits g = router_units(tokens, experts, hidden);
  cudaError_t st = w_dtype == PW_ROUTER_F32
                       ? launch_router_logits<true>(x, tokens, w, g, scratch, work, num_sms, stream, q_codes, q_scales,
                                                    flags)
                       : launch_router_logits<false>(x, tokens, w, g, scratch, work, num_sms, stream, q_codes, q_scales,
                                                     flags);
  if (st != cudaSuccess) return st;
  if (experts <= 256u && tokens < kRouterTopkCtaMaxTokens) {
    // decode widths: a CTA per token (a shorter critical path per token; at
    // 2048 tokens the warp-per-token kernel is faster, 145 vs 170 us per call)
    return launch_kernel(k_router_topk_cta, dim3(tokens), dim3(256), 0, stream, (const float *)scratch, g.slices,
                         bias, tokens, experts, selected, weights, tie_rows, flags);
  }
  // persistent: up to two 8-warp CTAs per SM, each warp looping over tokens
  uint32_t blocks = (tokens + 7u) / 8u;
  if (blocks > 2u * (uint32_t)num_sms) blocks = 2u * (uint32_t)num_sms;
  const dim3 grid(blocks);
  if (experts <= 256u)
    return launch_kernel(k_router_topk<8>, grid, dim3(256), 0, stream, (const float *)scratch, g.slices, bias,
                         tokens, experts, selected, weights, tie_rows, flags);
  return launch_kernel(k_router_topk<32>, grid, dim3(256), 0, stream, (const float *)scratch, g.slices, bias,
                       tokens, experts, selected, weights, tie_rows, flags);
}

// ----------------------------------------------------------------- schedule
// Placements are ordered by (expert ascending, position ascending) -- the
// reference's BTreeMap<expert, [(position, weight)]>
// (src/text_endpoint.rs:4768-4776, src/text_endpoint.rs:5302-5310).  The rank
// of a token among an expert's placements comes from per-expert token
// bitmasks, so the order is deterministic without sorting.  Three launches:
//   k_sched_mask  (one CTA per 32 tokens): warp b ballots, for experts
//                 32b .. 32b+31, which of the 32 tokens chose them -> the mask
//                 word [expert][word]; rows are validated here;
//   k_sched_scan  (one CTA): per-expert prefix counts over the words, the
//                 scan over experts (placement and group offsets), the groups;
//   k_sched_place (one CTA per 32 tokens): each token's 8 placement indices,
//                 the placement lists and, through a sorting network, its
//                 placements in ascending expert order (the combine order).
// Scratch (ScheduleOut::work): mask [experts][64], base [experts][64]
// (placement index of each word's first token), 64 per-word error words and
// one summary word.
constexpr uint32_t kSchedMaxTokens = 2048;
constexpr uint32_t kSchedMaxExperts = 256;
constexpr uint32_t kSchedWords = kSchedMaxTokens / 32u;
constexpr uint32_t kSchedThreads = 1024;
static_assert(kSchedMaxExperts * 4u <= kSchedThreads, "four scan threads and one group writer per expert");

size_t schedule_work_words(uint32_t experts) { return 2u * (size_t)experts * kSchedWords + kSchedWords + 1u; }

__device__ __forceinline__ void cswap(uint32_t &ea, uint32_t &pa, uint32_t &eb, uint32_t &pb) {
  const bool sw = ea > eb;
  const uint32_t e0 = sw ? eb : ea, e1 = sw ? ea : eb, p0 = sw ? pb : pa, p1 = sw ? pa : pb;
  ea = e0;
  eb = e1;
  pa = p0;
  pb = p1;
}

__global__ void __launch_bounds__(256) k_sched_mask(const uint32_t *__restrict__ selected, uint32_t tokens,
                                                    uint32_t experts, uint32_t *__restrict__ work) {
  pdl_wait();
  pdl_launch_dependents();
  uint32_t *mask = work, *badw = work + 2u * experts * kSchedWords;
  const uint32_t w = blockIdx.x, lane = threadIdx.x % 32u, eb = threadIdx.x / 32u;
  const uint32_t t = 32u * w + lane;
  uint32_t sel[8];
  if (t < tokens) {
    const uint4 a = *reinterpret_cast<const uint4 *>(selected + (size_t)t * 8u);
    const uint4 b = *reinterpret_cast<const uint4 *>(selected + (size_t)t * 8u + 4u);
    sel[0] = a.x; sel[1] = a.y; sel[2] = a.z; sel[3] = a.w;
    sel[4] = b.x; sel[5] = b.y; sel[6] = b.z; sel[7] = b.w;
  } else {
#pragma unroll
    for (int k = 0; k < 8; ++k) sel[k] = 0xffffffffu;
  }
  if (eb == 0u) {  // validation: experts in range, no expert twice in a row
    bool bad = false;
    if (t < tokens) {
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        bad |= sel[k] >= experts;
#pragma unroll
        for (int j = k + 1; j < 8; ++j) bad |= sel[k] == sel[j];
      }
    }
    const uint32_t any = __ballot_sync(0xffffffffu, bad);
    if (lane == 0) badw[w] = any ? 1u : 0u;
  }
  if (32u * eb >= experts) return;
  uint32_t bits = 0;
#pragma unroll
  for (int k = 0; k < 8; ++k)
    if (sel[k] < experts && sel[k] / 32u == eb) bits |= 1u << (sel[k] % 32u);
  uint32_t mine = 0;
#pragma unroll
  for (uint32_t j = 0; j < 32u; ++j) {
    const uint32_t b = __ballot_sync(0xffffffffu, (bits >> j) & 1u);
    mine = lane == j ? b : mine;
  }
  const uint32_t e = 32u * eb + lane;
  if (e < experts) mask[e * kSchedWords + w] = mine;
}

__global__ void __launch_bounds__(kSchedThreads) k_sched_scan(uint32_t tokens, uint32_t experts, BankTable bank,
                                                              ScheduleOut out, uint32_t *flags, uint32_t chunk) {
  const uint32_t tid = threadIdx.x, lane = tid % 32u, warp = tid / 32u;
  // the bank table is final before the layer's kernels start, so its entries
  // are fetched before the programmatic-launch wait
  const bool has_bank = out.gu_groups && tid < experts;
  const uint8_t *bw[3] = {nullptr, nullptr, nullptr};
  const float *bs[3] = {nullptr, nullptr, nullptr};
  if (has_bank) {
    bw[0] = bank.gate_w[tid];
    bs[0] = bank.gate_s[tid];
    bw[1] = bank.up_w[tid];
    bs[1] = bank.up_s[tid];
    bw[2] = bank.down_w[tid];
    bs[2] = bank.down_s[tid];
  }
  pdl_wait();
  pdl_launch_dependents();
  const uint32_t *mask = out.work;
  uint32_t *base = out.work + experts * kSchedWords, *badw = base + experts * kSchedWords;
  uint32_t *summary = badw + kSchedWords;
  __shared__ uint32_t off[kSchedMaxExperts + 1], grp_off[kSchedMaxExperts + 1];
  __shared__ uint32_t uniq, maxc, wsum_c[kSchedThreads / 32], wsum_g[kSchedThreads / 32];
  const uint32_t words = (tokens + 31u) / 32u;
  if (tid == 0) {
    uniq = 0;
    maxc = 0;
  }
  // every other global load this kernel needs is issued up front, so its
  // latency is paid once: the per-word error flags and the mask words (four
  // threads per expert, experts <= 256, up to 16 words each)
  const uint32_t ex = tid / 4u, q = tid % 4u;
  const uint32_t per = (words + 3u) / 4u, w0 = min(words, q * per), w1 = min(words, w0 + per);
  const bool badword = tid < words && badw[tid] != 0u;
  uint32_t mw[kSchedWords / 4u];
#pragma unroll
  for (uint32_t k = 0; k < kSchedWords / 4u; ++k)
    mw[k] = ex < experts && w0 + k < w1 ? mask[ex * kSchedWords + w0 + k] : 0u;
  const int bad = __syncthreads_or(badword);
  if (bad) {
    if (tid == 0) {
      raise_flag(flags, PW_FLAG_BAD_EXPERT_COUNT);
      if (out.n_groups) *out.n_groups = 0;
      *summary = 1u;
    }
    return;
  }
  if (tid == 0) *summary = 0u;
  uint32_t local = 0;
#pragma unroll
  for (uint32_t k = 0; k < kSchedWords / 4u; ++k) local += __popc(mw[k]);
  uint32_t incl = local;
#pragma unroll
  for (uint32_t o = 1; o < 4u; o <<= 1) {
    const uint32_t v = __shfl_up_sync(0xffffffffu, incl, o, 4);
    if (q >= o) incl += v;
  }
  const uint32_t cnt_e = __shfl_sync(0xffffffffu, incl, 3, 4);
  if (q == 0u && ex < experts) off[ex] = cnt_e;
  __syncthreads();
  // scan over experts: thread e holds count c and group count g
  {
    const uint32_t e = tid;
    const uint32_t c = e < experts ? off[e] : 0u;
    const uint32_t g = (c + chunk - 1u) / chunk;
    uint32_t ic = c, ig = g;
#pragma unroll
    for (uint32_t o = 1; o < 32u; o <<= 1) {
      const uint32_t vc = __shfl_up_sync(0xffffffffu, ic, o), vg = __shfl_up_sync(0xffffffffu, ig, o);
      if (lane >= o) {
        ic += vc;
        ig += vg;
      }
    }
    if (lane == 31u) {
      wsum_c[warp] = ic;
      wsum_g[warp] = ig;
    }
    if (e < experts && c) {
      atomicAdd(&uniq, 1u);
      atomicMax(&maxc, c);
    }
    __syncthreads();  // every count read before off[] is overwritten
    uint32_t bc = 0, bg = 0;
    for (uint32_t k = 0; k < warp; ++k) {
      bc += wsum_c[k];
      bg += wsum_g[k];
    }
    if (e < experts) {
      off[e] = bc + ic - c;
      grp_off[e] = bg + ig - g;
      out.offsets[e] = bc + ic - c;
      if (e == experts - 1u) {
        off[experts] = bc + ic;
        grp_off[experts] = bg + ig;
        out.offsets[experts] = bc + ic;
        if (out.n_groups) *out.n_groups = bg + ig;
        out.counters[1] = bc + ic;
      }
    }
  }
  __syncthreads();
  if (tid == 0) {
    out.counters[0] = uniq;
    out.counters[2] = maxc;
  }
  // placement index of the first token of every (expert, word)
  if (ex < experts) {
    uint32_t run = off[ex] + incl - local;
#pragma unroll
    for (uint32_t k = 0; k < kSchedWords / 4u; ++k) {
      if (w0 + k < w1) base[ex * kSchedWords + w0 + k] = run;
      run += __popc(mw[k]);
    }
  }
  // GEMV/GEMM groups: each expert's placements in chunks of <= chunk tokens
  // (skipped when the caller runs the experts elsewhere: no group arrays);
  // thread e writes expert e's (experts <= kSchedMaxExperts <= threads)
  if (has_bank) {
    const uint32_t e = tid;
    const uint32_t c = off[e + 1] - off[e];
    for (uint32_t j = 0; j * chunk < c; ++j) {
      GemvGroup g;
      g.tok_begin = off[e] + chunk * j;
      g.count = min(chunk, c - chunk * j);
      g.expert = e;
      g.pad = 0;
      g.w0 = bw[0];
      g.s0 = bs[0];
      g.w1 = bw[1];
      g.s1 = bs[1];
      g.tm0 = bank.gate_tm + e;
      g.tm1 = bank.up_tm + e;
      out.gu_groups[grp_off[e] + j] = g;
      GemvGroup d = g;
      d.w0 = bw[2];
      d.s0 = bs[2];
      d.w1 = nullptr;
      d.s1 = nullptr;
      d.tm0 = bank.down_tm + e;
      d.tm1 = nullptr;
      out.dn_groups[grp_off[e] + j] = d;
    }
  }
}

__global__ void __launch_bounds__(32) k_sched_place(const uint32_t *__restrict__ selected,
                                                    const float *__restrict__ weights, uint32_t tokens,
                                                    uint32_t experts, ScheduleOut out) {
  pdl_wait();
  pdl_launch_dependents();
  const uint32_t *mask = out.work, *base = out.work + experts * kSchedWords;
  if (base[experts * kSchedWords + kSchedWords] != 0u) return;  // invalid rows: k_sched_scan flagged them
  const uint32_t w = blockIdx.x, t = 32u * w + threadIdx.x;
  if (t >= tokens) return;
  const uint4 sa = *reinterpret_cast<const uint4 *>(selected + (size_t)t * 8u);
  const uint4 sb = *reinterpret_cast<const uint4 *>(selected + (size_t)t * 8u + 4u);
  const float4 wa = *reinterpret_cast<const float4 *>(weights + (size_t)t * 8u);
  const float4 wb = *reinterpret_cast<const float4 *>(weights + (size_t)t * 8u + 4u);
  uint32_t ex[8] = {sa.x, sa.y, sa.z, sa.w, sb.x, sb.y, sb.z, sb.w};
  const float wt[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
  const uint32_t below = (1u << (t % 32u)) - 1u;
  uint32_t pl[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const uint32_t i = ex[k] * kSchedWords + w;
    pl[k] = base[i] + __popc(mask[i] & below);
    out.placement_tok[pl[k]] = t;
    out.placement_w[pl[k]] = wt[k];
  }
  // Batcher odd-even merge sort of 8 (experts of a row are distinct)
  cswap(ex[0], pl[0], ex[1], pl[1]); cswap(ex[2], pl[2], ex[3], pl[3]);
  cswap(ex[4], pl[4], ex[5], pl[5]); cswap(ex[6], pl[6], ex[7], pl[7]);
  cswap(ex[0], pl[0], ex[2], pl[2]); cswap(ex[1], pl[1], ex[3], pl[3]);
  cswap(ex[4], pl[4], ex[6], pl[6]); cswap(ex[5], pl[5], ex[7], pl[7]);
  cswap(ex[1], pl[1], ex[2], pl[2]); cswap(ex[5], pl[5], ex[6], pl[6]);
  cswap(ex[0], pl[0], ex[4], pl[4]); cswap(ex[1], pl[1], ex[5], pl[5]);
  cswap(ex[2], pl[2], ex[6], pl[6]); cswap(ex[3], pl[3], ex[7], pl[7]);
  cswap(ex[2], pl[2], ex[4], pl[4]); cswap(ex[3], pl[3], ex[5], pl[5]);
  cswap(ex[1], pl[1], ex[2], pl[2]); cswap(ex[3], pl[3], ex[4], pl[4]);
  cswap(ex[5], pl[5], ex[6], pl[6]);
  uint4 *sp = reinterpret_cast<uint4 *>(out.slot_place + (size_t)t * 8u);
  sp[0] = make_uint4(pl[0], pl[1], pl[2], pl[3]);
  sp[1] = make_uint4(pl[4], pl[5], pl[6], pl[7]);
}

// Decode widths (<= 256 tokens): everything in one CTA, the bitmasks built
// with shared-memory atomics; the same placements as the three-launch path.
constexpr uint32_t kSchedSmallTokens = 256;
constexpr uint32_t kSchedSmallWords = kSchedSmallTokens / 32u;

// Bank entries of expert `e` (final before the layer's kernels start, so they
// are fetched before the programmatic-launch wait).
struct BankEntry {
  const uint8_t *w[3];
  const float *s[3];
  __device__ __forceinline__ void fetch(const BankTable &bank, uint32_t e) {
    w[0] = bank.gate_w[e];
    s[0] = bank.gate_s[e];
    w[1] = bank.up_w[e];
    s[1] = bank.up_s[e];
    w[2] = bank.down_w[e];
    s[2] = bank.down_s[e];
  }
};

// The one-CTA schedule; `be` holds expert threadIdx.x's bank entries when
// has_bank.  `selected` / `weights` carry no restrict or read-only
// qualifiers: the fused route + schedule kernel writes them earlier in the
// same launch.
__device__ __forceinline__ void schedule_small_body(const uint32_t *selected, const float *weights, uint32_t tokens,
                                                    uint32_t experts, const BankTable &bank, const ScheduleOut &out,
                                                    uint32_t *flags, uint32_t chunk, bool has_bank,
                                                    const BankEntry &be) {
  extern __shared__ uint32_t sm[];
  uint32_t *mask = sm;                                                            // [experts][kSchedSmallWords]
  uint16_t *prefix = reinterpret_cast<uint16_t *>(mask + experts * kSchedSmallWords);  // [experts][kSchedSmallWords]
  uint32_t *off = reinterpret_cast<uint32_t *>(prefix + experts * kSchedSmallWords);   // [experts + 1]
  uint32_t *grp_off = off + experts + 1;                                          // [experts + 1]
  __shared__ uint32_t bad, uniq, maxc, wsum_c[kSchedThreads / 32], wsum_g[kSchedThreads / 32];
  const uint32_t words = (tokens + 31u) / 32u;
  const uint32_t tid = threadIdx.x, lane = tid % 32u, warp = tid / 32u;
  if (tid == 0) {
    bad = 0;
    uniq = 0;
    maxc = 0;
  }
  for (uint32_t i = tid; i < experts * words; i += kSchedThreads) mask[(i / words) * kSchedSmallWords + i % words] = 0;
  __syncthreads();
  // 1. bitmasks
  for (uint32_t i = tid; i < tokens * 8u; i += kSchedThreads) {
    const uint32_t e = selected[i];
    const uint32_t t = i / 8u;
    if (e >= experts) {
      bad = 1;
      continue;
    }
    const uint32_t prev = atomicOr(&mask[e * kSchedSmallWords + t / 32u], 1u << (t % 32u));
    if (prev & (1u << (t % 32u))) bad = 1;  // duplicate expert in one row
  }
  __syncthreads();
  if (bad) {
    if (tid == 0) raise_flag(flags, PW_FLAG_BAD_EXPERT_COUNT);
    if (tid == 0 && out.n_groups) *out.n_groups = 0;
    return;
  }
  // 2. word prefixes, four threads per expert (experts <= 256)
  uint32_t cnt = 0;
  {
    const uint32_t e = tid / 4u, q = tid % 4u;
    const uint32_t per = (words + 3u) / 4u, w0 = min(words, q * per), w1 = min(words, w0 + per);
    uint32_t local = 0;
    if (e < experts)
      for (uint32_t wi = w0; wi < w1; ++wi) local += __popc(mask[e * kSchedSmallWords + wi]);
    // exclusive scan over the 4 lanes of this expert (lanes 4k..4k+3 of a warp)
    uint32_t incl = local;
#pragma unroll
    for (uint32_t o = 1; o < 4u; o <<= 1) {
      const uint32_t v = __shfl_up_sync(0xffffffffu, incl, o, 4);
      if (q >= o) incl += v;
    }
    uint32_t run = incl - local;
    if (e < experts)
      for (uint32_t wi = w0; wi < w1; ++wi) {
        prefix[e * kSchedSmallWords + wi] = (uint16_t)run;
        run += __popc(mask[e * kSchedSmallWords + wi]);
      }
    cnt = __shfl_sync(0xffffffffu, incl, 3, 4);  // the expert's total
  }
  __syncthreads();
  // 3. offsets: thread e (< experts) holds count c and group count g
  {
    const uint32_t e = tid;
    uint32_t c = 0;
    // counts live in lanes 4e..4e+3 of step 2; gather them through shared memory
    if (tid % 4u == 0u && tid / 4u < experts) off[tid / 4u] = cnt;
    __syncthreads();
    if (e < experts) c = off[e];
    const uint32_t g = (c + chunk - 1u) / chunk;
    uint32_t ic = c, ig = g;
#pragma unroll
    for (uint32_t o = 1; o < 32u; o <<= 1) {
      const uint32_t vc = __shfl_up_sync(0xffffffffu, ic, o), vg = __shfl_up_sync(0xffffffffu, ig, o);
      if (lane >= o) {
        ic += vc;
        ig += vg;
      }
    }
    if (lane == 31u) {
      wsum_c[warp] = ic;
      wsum_g[warp] = ig;
    }
    if (e < experts && c) {
      atomicAdd(&uniq, 1u);
      atomicMax(&maxc, c);
    }
    __syncthreads();  // everyone has read off[] (counts) before it is overwritten
    uint32_t bc = 0, bg = 0;
    for (uint32_t k = 0; k < warp; ++k) {
      bc += wsum_c[k];
      bg += wsum_g[k];
    }
    if (e < experts) {
      off[e] = bc + ic - c;
      grp_off[e] = bg + ig - g;
      out.offsets[e] = bc + ic - c;
      if (e == experts - 1u) {
        const uint32_t total = bc + ic, gtotal = bg + ig;
        off[experts] = total;
        grp_off[experts] = gtotal;
        out.offsets[experts] = total;
        if (out.n_groups) *out.n_groups = gtotal;
        out.counters[1] = total;
      }
    }
  }
  __syncthreads();
  if (tid == 0) {
    out.counters[0] = uniq;
    out.counters[2] = maxc;
  }
  // 4. per token: placements, placement lists and the combine order
  for (uint32_t t = tid; t < tokens; t += kSchedThreads) {
    const uint4 sa = *reinterpret_cast<const uint4 *>(selected + (size_t)t * 8u);
    const uint4 sb = *reinterpret_cast<const uint4 *>(selected + (size_t)t * 8u + 4u);
    const float4 wa = *reinterpret_cast<const float4 *>(weights + (size_t)t * 8u);
    const float4 wb = *reinterpret_cast<const float4 *>(weights + (size_t)t * 8u + 4u);
    uint32_t ex[8] = {sa.x, sa.y, sa.z, sa.w, sb.x, sb.y, sb.z, sb.w};
    const float wt[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
    const uint32_t wi = t / 32u, below_mask = (1u << (t % 32u)) - 1u;
    uint32_t pl[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const uint32_t e = ex[k];
      pl[k] = off[e] + prefix[e * kSchedSmallWords + wi] + __popc(mask[e * kSchedSmallWords + wi] & below_mask);
      out.placement_tok[pl[k]] = t;
      out.placement_w[pl[k]] = wt[k];
    }
    // Batcher odd-even merge sort of 8 (experts of a row are distinct)
    cswap(ex[0], pl[0], ex[1], pl[1]); cswap(ex[2], pl[2], ex[3], pl[3]);
    cswap(ex[4], pl[4], ex[5], pl[5]); cswap(ex[6], pl[6], ex[7], pl[7]);
    cswap(ex[0], pl[0], ex[2], pl[2]); cswap(ex[1], pl[1], ex[3], pl[3]);
    cswap(ex[4], pl[4], ex[6], pl[6]); cswap(ex[5], pl[5], ex[7], pl[7]);
    cswap(ex[1], pl[1], ex[2], pl[2]); cswap(ex[5], pl[5], ex[6], pl[6]);
    cswap(ex[0], pl[0], ex[4], pl[4]); cswap(ex[1], pl[1], ex[5], pl[5]);
    cswap(ex[2], pl[2], ex[6], pl[6]); cswap(ex[3], pl[3], ex[7], pl[7]);
    cswap(ex[2], pl[2], ex[4], pl[4]); cswap(ex[3], pl[3], ex[5], pl[5]);
    cswap(ex[1], pl[1], ex[2], pl[2]); cswap(ex[3], pl[3], ex[4], pl[4]);
    cswap(ex[5], pl[5], ex[6], pl[6]);
    uint4 *sp = reinterpret_cast<uint4 *>(out.slot_place + (size_t)t * 8u);
    sp[0] = make_uint4(pl[0], pl[1], pl[2], pl[3]);
    sp[1] = make_uint4(pl[4], pl[5], pl[6], pl[7]);
  }
  // 5. GEMV/GEMM groups: each expert's placements in chunks of <= chunk tokens
  // (skipped when the caller runs the experts elsewhere: no group arrays)
  if (has_bank) {
    const uint32_t e = tid;
    const uint32_t c = off[e + 1] - off[e];
    for (uint32_t j = 0; j * chunk < c; ++j) {
      GemvGroup g;
      g.tok_begin = off[e] + chunk * j;
      g.count = min(chunk, c - chunk * j);
      g.expert = e;
      g.pad = 0;
      g.w0 = be.w[0];
      g.s0 = be.s[0];
      g.w1 = be.w[1];
      g.s1 = be.s[1];
      g.tm0 = bank.gate_tm + e;
      g.tm1 = bank.up_tm + e;
      out.gu_groups[grp_off[e] + j] = g;
      GemvGroup d = g;
      d.w0 = be.w[2];
      d.s0 = be.s[2];
      d.w1 = nullptr;
      d.s1 = nullptr;
      d.tm0 = bank.down_tm + e;
      d.tm1 = nullptr;
      out.dn_groups[grp_off[e] + j] = d;
    }
  }
}


__global__ void __launch_bounds__(kSchedThreads) k_schedule_small(const uint32_t *__restrict__ selected,
                                                            const float *__restrict__ weights, uint32_t tokens,
                                                            uint32_t experts, BankTable bank, ScheduleOut out,
                                                            uint32_t *flags, uint32_t chunk) {
  // thread e writes expert e's groups; its bank entries before the wait
  const bool has_bank = out.gu_groups && threadIdx.x < experts;
  BankEntry be{};
  if (has_bank) be.fetch(bank, threadIdx.x);
  pdl_wait();
  pdl_launch_dependents();
  schedule_small_body(selected, weights, tokens, experts, bank, out, flags, chunk, has_bank, be);
}

uint32_t schedule_launches(uint32_t tokens) { return tokens <= kSchedSmallTokens ? 1u : 3u; }

cudaError_t launch_schedule(const uint32_t *selected, const float *weights, uint32_t tokens, uint32_t experts,
                            const BankTable &bank, const ScheduleOut &out, uint32_t *flags, uint32_t chunk,
                            cudaStream_t stream) {
  if (tokens == 0 || tokens > kSchedMaxTokens || experts > kSchedMaxExperts || experts < 8 || chunk == 0 ||
      !out.work)
    return cudaErrorInvalidValue;
  if (tokens <= kSchedSmallTokens) {
    const size_t smem = (size_t)experts * kSchedSmallWords * 6 + (size_t)(experts + 1) * 8;
    return launch_kernel(k_schedule_small, dim3(1), dim3(kSchedThreads), smem, stream, selected, weights, tokens,
                         experts, bank, out, flags, chunk);
  }
  const uint32_t words = (tokens + 31u) / 32u;
  cudaError_t e = launch_kernel(k_sched_mask, dim3(words), dim3(256), 0, stream, selected, tokens, experts, out.work);
  if (e != cudaSuccess) return e;
  e = launch_kernel(k_sched_scan, dim3(1), dim3(kSchedThreads), 0, stream, tokens, experts, bank, out, flags, chunk);
  if (e != cudaSuccess) return e;
  return launch_kernel(k_sched_place, dim3(words), dim3(32), 0, stream, selected, weights, tokens, experts, out);
}

// ------------------------------------------------------------------ combine
// y[t, c] = bf16( sum over t's 8 placements in ascending expert order of
//                 down[p, c] * w_p )   -- product rounded, then added, from 0
// (src/text_endpoint.rs:5365-5373; the down rows are already bf16-rounded).
__device__ __forceinline__ float4 load4(const float *row, uint32_t c4) {
  return __ldg(reinterpret_cast<const float4 *>(row) + c4);
}
__device__ __forceinline__ float4 load4(const uint16_t *row, uint32_t c4) {
  const uint2 q = __ldg(reinterpret_cast<const uint2 *>(row) + c4);
  return make_float4(__uint_as_float(q.x << 16), __uint_as_float(q.x & 0xffff0000u), __uint_as_float(q.y << 16),
                     __uint_as_float(q.y & 0xffff0000u));
}

template <typename T>
__global__ void k_combine(const T *__restrict__ down, const uint32_t *__restrict__ slot_place,
                          const float *__restrict__ placement_w, uint32_t tokens, uint32_t hidden,
                          const float *__restrict__ residual, float *__restrict__ y, uint32_t *flags) {
  pdl_wait();
  pdl_launch_dependents();
  const uint32_t t = blockIdx.y;
  __shared__ uint32_t pl[8];
  if (threadIdx.x < 8) pl[threadIdx.x] = slot_place[t * 8u + threadIdx.x];
  __syncthreads();
  // two 4-column groups per thread: all 16 row loads in flight together,
  // and the 8 route weights (L1 broadcasts) in the same round trip
  for (uint32_t c8 = blockIdx.x * blockDim.x + threadIdx.x; c8 < hidden / 8u; c8 += gridDim.x * blockDim.x) {
    float4 d[2][8];
    float wt[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      d[0][k] = load4(down + (size_t)pl[k] * hidden, 2u * c8);
      d[1][k] = load4(down + (size_t)pl[k] * hidden, 2u * c8 + 1u);
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) wt[k] = __ldg(placement_w + pl[k]);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        acc.x = __fadd_rn(acc.x, __fmul_rn(d[h][k].x, wt[k]));
        acc.y = __fadd_rn(acc.y, __fmul_rn(d[h][k].y, wt[k]));
        acc.z = __fadd_rn(acc.z, __fmul_rn(d[h][k].z, wt[k]));
        acc.w = __fadd_rn(acc.w, __fmul_rn(d[h][k].w, wt[k]));
      }
      acc = round_bf16x4(acc);
      if (!finite(acc.x) || !finite(acc.y) || !finite(acc.z) || !finite(acc.w))
        raise_flag(flags, PW_FLAG_NONFINITE_COMBINE);
      if (residual) {  // the decoder layer's residual add: bf16(residual + mlp) (src/text_endpoint.rs:5576-5580)
        const float4 r = __ldg(reinterpret_cast<const float4 *>(residual + (size_t)t * hidden) + 2u * c8 + h);
        acc = round_bf16x4(make_float4(__fadd_rn(r.x, acc.x), __fadd_rn(r.y, acc.y), __fadd_rn(r.z, acc.z),
                                       __fadd_rn(r.w, acc.w)));
      }
      reinterpret_cast<float4 *>(y + (size_t)t * hidden)[2u * c8 + h] = acc;
    }
  }
}

cudaError_t launch_combine(const float *down, const uint32_t *slot_place, const float *placement_w,
                           uint32_t tokens, uint32_t hidden, float *y, uint32_t *flags, cudaStream_t stream,
                           const float *residual) {
  if (hidden % 8u || tokens == 0) return cudaErrorInvalidValue;
  dim3 grid((hidden / 8u + 255u) / 256u, tokens);
  return launch_kernel(k_combine<float>, grid, dim3(256), 0, stream, down, slot_place, placement_w, tokens, hidden,
                       residual, y, flags);
}

cudaError_t launch_combine_bf16(const uint16_t *down, const uint32_t *slot_place, const float *placement_w,
                                uint32_t tokens, uint32_t hidden, float *y, uint32_t *flags, cudaStream_t stream,
                                const float *residual) {
  if (hidden % 8u || tokens == 0) return cudaErrorInvalidValue;
  dim3 grid((hidden / 8u + 255u) / 256u, tokens);
  return launch_kernel(k_combine<uint16_t>, grid, dim3(256), 0, stream, down, slot_place, placement_w, tokens,
                       hidden, residual, y, flags);
}

// ------------------------------------------------------ bf16 row scatter
// out[idx[j]] = bf16 bits of rows[j]: puts the expert-parallel down rows
// (computed in expert order) back in received order for the return trip.
__global__ void k_scatter_rows_bf16(const float *__restrict__ rows, const uint32_t *__restrict__ idx, uint32_t n,
                                    uint32_t cols, uint16_t *__restrict__ out) {
  pdl_wait();
  pdl_launch_dependents();
  const uint32_t per_row = cols / 4u;
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < (uint64_t)n * per_row;
       i += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t j = (uint32_t)(i / per_row), c4 = (uint32_t)(i % per_row);
    const float4 v = __ldg(reinterpret_cast<const float4 *>(rows + (size_t)j * cols) + c4);
    const uint2 q = make_uint2((__float_as_uint(v.x) >> 16) | (__float_as_uint(v.y) & 0xffff0000u),
                               (__float_as_uint(v.z) >> 16) | (__float_as_uint(v.w) & 0xffff0000u));
    reinterpret_cast<uint2 *>(out + (size_t)idx[j] * cols)[c4] = q;
  }
}

cudaError_t launch_scatter_rows_bf16(const float *rows, const uint32_t *idx, uint32_t n, uint32_t cols,
                                     uint16_t *out, cudaStream_t stream) {
  if (cols % 4u) return cudaErrorInvalidValue;
  if (n == 0) return cudaSuccess;
  uint64_t blocks = ((uint64_t)n * (cols / 4u) + 255u) / 256u;
  if (blocks > 148u * 8u) blocks = 148u * 8u;
  return launch_kernel(k_scatter_rows_bf16, dim3((unsigned)blocks), dim3(256), 0, stream, rows, idx, n, cols, out);
}

// --------------------------------------------------------------- row gather
// dst row i = src row idx[i] (codes and their per-128 scales): lays the
// routed tokens out in placement order so a TMA box can read an expert's
// tokens as one contiguous block.
__global__ void k_gather_rows(const uint8_t *__restrict__ codes, const float *__restrict__ scales,
                              const uint32_t *__restrict__ idx, uint32_t n, uint32_t K, uint8_t *__restrict__ out_codes,
                              float *__restrict__ out_scales) {
  pdl_wait();
  pdl_launch_dependents();
  const uint32_t row = blockIdx.x;
  if (row >= n) return;
  const uint32_t src = idx[row];
  const uint4 *s = reinterpret_cast<const uint4 *>(codes + (size_t)src * K);
  uint4 *d = reinterpret_cast<uint4 *>(out_codes + (size_t)row * K);
  for (uint32_t i = threadIdx.x; i < K / 16u; i += blockDim.x) d[i] = __ldg(s + i);
  for (uint32_t i = threadIdx.x; i < K / 128u; i += blockDim.x)
    out_scales[(size_t)row * (K / 128u) + i] = __ldg(scales + (size_t)src * (K / 128u) + i);
}

cudaError_t launch_gather_rows(const uint8_t *codes, const float *scales, const uint32_t *idx, uint32_t n,
                               uint32_t K, uint8_t *out_codes, float *out_scales, cudaStream_t stream) {
  if (n == 0) return cudaSuccess;
  if (K % 128u) return cudaErrorInvalidValue;
  return launch_kernel(k_gather_rows, dim3(n), dim3(128), 0, stream, codes, scales, idx, n, K, out_codes, out_scales);
}

// ------------------------------------------------------- weight validation
// src/lib.rs:1217: every weight byte must not be 0x7f/0xff and every scale
// must be finite.  first_bad receives the smallest bad byte offset.
__global__ void k_validate(const uint8_t *__restrict__ w, uint64_t n, const float *__restrict__ s, uint64_t ns,
                           unsigned long long *first_bad, uint32_t *flags) {
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  const uint64_t n16 = n / 16u;
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n16; i += stride) {
    const uint4 q = __ldg(reinterpret_cast<const uint4 *>(w) + i);
    const uint32_t v[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      for (int b = 0; b < 4; ++b) {
        if (((v[k] >> (8 * b)) & 0x7fu) == 0x7fu) {  // 0x7f or 0xff
          atomicMin(first_bad, (unsigned long long)(i * 16u + k * 4u + b));
          raise_flag(flags, PW_FLAG_BAD_WEIGHT);
        }
      }
    }
  }
  for (uint64_t i = n16 * 16u + (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    if ((w[i] & 0x7fu) == 0x7fu) {
      atomicMin(first_bad, (unsigned long long)i);
      raise_flag(flags, PW_FLAG_BAD_WEIGHT);
    }
  }
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < ns; i += stride)
    if (!finite(s[i])) raise_flag(flags, PW_FLAG_BAD_WEIGHT);
}

cudaError_t launch_validate_fp8(const uint8_t *w, uint64_t n, const float *s, uint64_t ns,
                                unsigned long long *first_bad, uint32_t *flags, cudaStream_t stream) {
  k_validate<<<148u * 4u, 256, 0, stream>>>(w, n, s, ns, first_bad, flags);
  return cudaGetLastError();
}

// ----------------------------------------------------- unfused staged SwiGLU
// kernels/block_fp8_gemv.metal:139 bf16_staged_swiglu (the non-fused runtime).
__global__ void k_swiglu(const float *__restrict__ gate, const float *__restrict__ up, float *__restrict__ h,
                         uint32_t n, uint32_t *flags, const uint32_t *rows_dev, uint32_t row_len) {
  if (rows_dev) n = min(n, *rows_dev * row_len);
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const float r = staged_swiglu(gate[i], up[i]);
    if (!finite(r)) raise_flag(flags, PW_FLAG_NONFINITE_SWIGLU);
    h[i] = r;
  }
}

cudaError_t launch_swiglu(const float *gate, const float *up, float *h, uint32_t n, uint32_t *flags,
                          cudaStream_t stream, const uint32_t *rows_dev, uint32_t row_len) {
  if (n == 0) return cudaSuccess;
  unsigned blocks = (n + 255u) / 256u;
  if (blocks > 148u * 8u) blocks = 148u * 8u;
  k_swiglu<<<blocks, 256, 0, stream>>>(gate, up, h, n, flags, rows_dev, row_len);
  return cudaGetLastError();
}

// ------------------------------------- staged SwiGLU + hidden quantization
// The wide (tcgen05) gate/up kernel stores bf16(gate) and bf16(up), the first
// two roundings of the staged SwiGLU; this pass finishes it:
// h = bf16(bf16(g / (1 + exp(-g))) * u) (kernels/block_fp8_gemv.metal:139),
// then the down input's dynamic FP8 quantization exactly as k_quantize.
// g is a bf16, so silu(g) is a function of 16 bits: a 64 Ki-entry table of
// staged_silu over every bf16 pattern (built once on the device by the same
// code) replaces the exponential and the division.  The table sits in
// shared memory (loaded before the programmatic-launch wait, so it overlaps
// the GEMM's tail); each thread owns 8 consecutive values, a half-warp one
// 128-value group, a warp two groups per step, two steps in flight.
constexpr uint32_t kSiluLutEntries = 65536;

__global__ void k_build_silu_lut(uint16_t *lut) {
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < kSiluLutEntries) lut[i] = (uint16_t)(__float_as_uint(staged_silu(__uint_as_float(i << 16))) >> 16);
}

cudaError_t build_silu_lut(uint16_t *lut, cudaStream_t stream) {
  k_build_silu_lut<<<kSiluLutEntries / 256u, 256, 0, stream>>>(lut);
  return cudaGetLastError();
}

namespace {
struct SwigluChunk {
  uint4 g, u;
};

__device__ __forceinline__ void swiglu_chunk_load(const uint16_t *__restrict__ gate, const uint16_t *__restrict__ up,
                                                  uint64_t chunk, bool ok, SwigluChunk &c) {
  if (ok) {
    c.g = __ldcs(reinterpret_cast<const uint4 *>(gate) + chunk);
    c.u = __ldcs(reinterpret_cast<const uint4 *>(up) + chunk);
  } else {
    c.g = make_uint4(0u, 0u, 0u, 0u);
    c.u = c.g;
  }
}

__device__ __forceinline__ void swiglu_chunk_finish(const SwigluChunk &c, const uint16_t *slut, uint64_t chunk,
                                                    bool ok, float *__restrict__ h, uint8_t *__restrict__ codes,
                                                    float *__restrict__ scales, uint32_t *flags) {
  const uint32_t gw[4] = {c.g.x, c.g.y, c.g.z, c.g.w}, uw[4] = {c.u.x, c.u.y, c.u.z, c.u.w};
  float v[8];
  bool fin = true;
  float m = 0.0f;
#pragma unroll
  for (int k = 0; k < 8; k += 2) {
    // h = bf16(silu * u); u is already a bf16 value, so its own rounding is
    // the identity (a NaN anywhere is an error)
    float p[2];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const uint32_t gb = ((k + j) & 1) ? (gw[(k + j) / 2] >> 16) : (gw[(k + j) / 2] & 0xffffu);
      const float silu = __uint_as_float((uint32_t)slut[gb] << 16);
      const float u = __uint_as_float(((k + j) & 1) ? (uw[(k + j) / 2] & 0xffff0000u) : (uw[(k + j) / 2] << 16));
      p[j] = __fmul_rn(silu, u);
    }
    const uint32_t hb = pack_bf16x2_rn(p[0], p[1]);
    v[k] = __uint_as_float(hb << 16);
    v[k + 1] = __uint_as_float(hb & 0xffff0000u);
    fin = fin && finite(v[k]) && finite(v[k + 1]);
    m = fmaxf(m, fmaxf(fabsf(v[k]), fabsf(v[k + 1])));
  }
  if (ok && !fin) raise_flag(flags, PW_FLAG_NONFINITE_FUSED);
#pragma unroll
  for (int o = 8; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if (!ok) return;
  if (h) {
    float4 *hp = reinterpret_cast<float4 *>(h) + 2u * chunk;
    hp[0] = make_float4(v[0], v[1], v[2], v[3]);
    hp[1] = make_float4(v[4], v[5], v[6], v[7]);
  }
  const Fp8GroupScale gs = Fp8GroupScale::of(m);
  const float scale = gs.scale;
  auto q = [&](float val) { return gs.quotient(val); };
  const uint32_t w0 = encode2(q(v[0]), q(v[1])) | (encode2(q(v[2]), q(v[3])) << 16);
  const uint32_t w1 = encode2(q(v[4]), q(v[5])) | (encode2(q(v[6]), q(v[7])) << 16);
  reinterpret_cast<uint2 *>(codes)[chunk] = make_uint2(w0, w1);
  if ((threadIdx.x & 15u) == 0u) scales[chunk / 16u] = scale;
}
}  // namespace

__global__ void __launch_bounds__(1024, 1)
    k_swiglu_quant(const uint16_t *__restrict__ gate, const uint16_t *__restrict__ up, uint64_t groups,
                   float *__restrict__ h, uint8_t *__restrict__ codes, float *__restrict__ scales, uint32_t *flags,
                   const uint32_t *rows_dev, uint32_t groups_per_row, const uint16_t *__restrict__ lut) {
  extern __shared__ __align__(16) uint16_t slut[];
  for (uint32_t i = threadIdx.x; i < kSiluLutEntries / 8u; i += blockDim.x)
    reinterpret_cast<uint4 *>(slut)[i] = __ldg(reinterpret_cast<const uint4 *>(lut) + i);
  __syncthreads();
  pdl_wait();
  pdl_launch_dependents();
  if (rows_dev) groups = min(groups, (uint64_t)*rows_dev * groups_per_row);
  const uint64_t chunks = groups * 16u;  // 8 values per chunk
  const uint64_t warp_global = ((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) / 32u;
  const uint64_t nwarps = ((uint64_t)gridDim.x * blockDim.x) / 32u;
  const uint32_t lane = threadIdx.x % 32u;
  // warp step s covers chunks [64 s, 64 s + 64): lane l takes chunk 64 s + l
  // and 64 s + 32 + l (two groups per 32 lanes)
  for (uint64_t s = warp_global; 64u * s < chunks; s += 2u * nwarps) {
    const uint64_t s2 = s + nwarps;
    const uint64_t c0 = 64u * s + lane, c1 = c0 + 32u, c2 = 64u * s2 + lane, c3 = c2 + 32u;
    const bool second = 64u * s2 < chunks;  // uniform across the warp
    SwigluChunk a, b, c, d;
    swiglu_chunk_load(gate, up, c0, c0 < chunks, a);
    swiglu_chunk_load(gate, up, c1, c1 < chunks, b);
    if (second) {
      swiglu_chunk_load(gate, up, c2, c2 < chunks, c);
      swiglu_chunk_load(gate, up, c3, c3 < chunks, d);
    }
    swiglu_chunk_finish(a, slut, c0, c0 < chunks, h, codes, scales, flags);
    swiglu_chunk_finish(b, slut, c1, c1 < chunks, h, codes, scales, flags);
    if (second) {
      swiglu_chunk_finish(c, slut, c2, c2 < chunks, h, codes, scales, flags);
      swiglu_chunk_finish(d, slut, c3, c3 < chunks, h, codes, scales, flags);
    }
  }
}

cudaError_t launch_swiglu_quant(const uint16_t *gate, const uint16_t *up, uint32_t rows, uint32_t cols, float *h,
                                uint8_t *codes, float *scales, uint32_t *flags, const uint16_t *silu_lut,
                                int num_sms, cudaStream_t stream, const uint32_t *rows_dev) {
  if (cols % 128u || !silu_lut) return cudaErrorInvalidValue;
  const uint64_t groups = (uint64_t)rows * (cols / 128u);
  if (groups == 0) return cudaSuccess;
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(k_swiglu_quant, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)(kSiluLutEntries * 2u));
    if (e != cudaSuccess) return e;
    configured = true;
  }
  // one 1024-thread CTA per SM; fewer when there is little work
  const uint64_t steps = (groups * 16u + 63u) / 64u;  // warp steps
  uint64_t blocks = (steps + 31u) / 32u;
  if (blocks > (uint64_t)num_sms) blocks = (uint64_t)num_sms;
  return launch_kernel(k_swiglu_quant, dim3((unsigned)blocks), dim3(1024), (size_t)kSiluLutEntries * 2u, stream,
                       gate, up, groups, h, codes, scales, flags, rows_dev, cols / 128u, silu_lut);
}

}  // namespace pw
