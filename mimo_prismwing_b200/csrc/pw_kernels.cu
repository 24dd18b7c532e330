// pw_kernels.cu -- the small kernels around the GEMV: dynamic FP8 activation
// quantization, router logits + sigmoid no-aux top-8, the device-side expert
// schedule, the weighted combine, bf16 rounding and weight validation.
#include <cstdint>
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
// code = RNE_e4m3(clamp(x/scale, +-448)).  IEEE divisions (__fdiv_rn) keep it
// bit-exact with the reference; lane l holds values 4l..4l+3.
__global__ void k_quantize(const float *__restrict__ x, uint64_t groups, uint8_t *__restrict__ codes,
                           float *__restrict__ scales, uint32_t *flags, const uint32_t *rows_dev,
                           uint32_t groups_per_row) {
  pdl_wait();
  pdl_launch_dependents();
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
    const float scale = __fdiv_rn(fmaxf(m, 1.0e-10f), 448.0f);
    auto q = [&](float val) { return fminf(fmaxf(__fdiv_rn(val, scale), -448.0f), 448.0f); };
    const uint32_t lo = encode2(q(v.x), q(v.y));
    const uint32_t hi = encode2(q(v.z), q(v.w));
    reinterpret_cast<uint32_t *>(codes + g * 128u)[lane] = lo | (hi << 16);
    if (lane == 0) scales[g] = scale;
  }
}

cudaError_t launch_quantize(const float *x, uint32_t rows, uint32_t cols, uint8_t *codes, float *scales,
                            uint32_t *flags, cudaStream_t stream, const uint32_t *rows_dev) {
  if (cols % 128u) return cudaErrorInvalidValue;
  const uint64_t groups = (uint64_t)rows * (cols / 128u);
  if (groups == 0) return cudaSuccess;
  const int threads = 256;
  uint64_t blocks = (groups * 32u + threads - 1) / threads;
  if (blocks > 148u * 16u) blocks = 148u * 16u;
  return launch_kernel(k_quantize, dim3((unsigned)blocks), dim3(threads), 0, stream, x, groups, codes, scales, flags,
                       rows_dev, cols / 128u);
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
// pwo_router_logits restates it; the reference's own logits are f32 too):
//   the K axis is cut into 512-column slices; warp w (of 8) owns slices
//   s = w, w+8, ...; lane l accumulates, for each owned slice in ascending
//   order, the 8-column chunks at 512s + 8l and 512s + 8l + 256, column by
//   column, with fused multiply-adds; an xor butterfly (16, 8, 4, 2, 1) adds
//   the lanes; the CTA then adds the 8 warp partials in warp order starting
//   from warp 0's.  bf16 weights widen to f32 exactly (a shift).
// Decode widths: one CTA per (expert, 8 tokens).
constexpr int kRouterTok = 8;

__device__ __forceinline__ float bf16lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

__global__ void __launch_bounds__(256) k_router_logits(const float *__restrict__ x, uint32_t tokens,
                                                       const uint16_t *__restrict__ w, uint32_t experts,
                                                       uint32_t hidden, float *__restrict__ logits) {
  pdl_wait();
  pdl_launch_dependents();
  __shared__ float part[8][kRouterTok];
  const uint32_t lane = threadIdx.x % 32u, warp = threadIdx.x / 32u;
  const uint32_t e = blockIdx.x;
  const uint32_t t0 = blockIdx.y * kRouterTok;
  float acc[kRouterTok];
#pragma unroll
  for (int t = 0; t < kRouterTok; ++t) acc[t] = 0.0f;
  const uint16_t *wrow = w + (size_t)e * hidden;
  const uint32_t slices = hidden / 512u;
  for (uint32_t sl = warp; sl < slices; sl += 8u) {
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const uint32_t c0 = 512u * sl + 8u * lane + 256u * j;
      const uint4 wq = __ldg(reinterpret_cast<const uint4 *>(wrow + c0));
      const float wf[8] = {bf16lo(wq.x), bf16hi(wq.x), bf16lo(wq.y), bf16hi(wq.y),
                           bf16lo(wq.z), bf16hi(wq.z), bf16lo(wq.w), bf16hi(wq.w)};
#pragma unroll
      for (int t = 0; t < kRouterTok; ++t) {
        if (t0 + t < tokens) {
          const float4 *xp = reinterpret_cast<const float4 *>(x + (size_t)(t0 + t) * hidden + c0);
          const float4 a = __ldg(xp), b = __ldg(xp + 1);
          const float xv[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
          for (int i = 0; i < 8; ++i) acc[t] = __fmaf_rn(xv[i], wf[i], acc[t]);
        }
      }
    }
  }
#pragma unroll
  for (int t = 0; t < kRouterTok; ++t) {
    float v = acc[t];
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (lane == 0) part[warp][t] = v;
  }
  __syncthreads();
  if (threadIdx.x < kRouterTok && t0 + threadIdx.x < tokens) {
    float s = part[0][threadIdx.x];
#pragma unroll
    for (int k = 1; k < 8; ++k) s = __fadd_rn(s, part[k][threadIdx.x]);
    logits[(size_t)(t0 + threadIdx.x) * experts + e] = s;
  }
}

// Prefill-width router logits: the same per-(token, expert) order as
// k_router_logits, for a tile of 8 tokens x 16 experts per CTA so that each
// activation and weight value loaded feeds 16 (resp. 8) chains.  Thread
// (warp w, lane l) runs the 128 lane chains of its columns four columns at a
// time, two tokens per packed f32x2 FMA (each lane of the pair rounds like
// fmaf).  The 32-lane xor tree is evaluated as a transpose-reduce (at each
// level lane l adds its xor partner's value for the half of the pairs it
// keeps): every pair gets the same tree of commutative additions as the
// butterfly, in 124 exchanges instead of 640.  Lane l ends with pairs
// 4l..4l+3; the 8 warp sums are then added in warp order.
constexpr int kTileTok = 8, kTileExp = 16;

__global__ void __launch_bounds__(256) k_router_logits_tiled(const float *__restrict__ x, uint32_t tokens,
                                                             const uint16_t *__restrict__ w, uint32_t experts,
                                                             uint32_t hidden, float *__restrict__ logits) {
  pdl_wait();
  pdl_launch_dependents();
  constexpr int NP = kTileTok * kTileExp;  // pairs, index p = e * kTileTok + t
  __shared__ float part[8][NP];
  const uint32_t lane = threadIdx.x % 32u, warp = threadIdx.x / 32u;
  const uint32_t e0 = blockIdx.x * kTileExp, t0 = blockIdx.y * kTileTok;
  float2 acc[kTileExp][kTileTok / 2];  // acc[e][tp] = tokens 2tp, 2tp+1
#pragma unroll
  for (int e = 0; e < kTileExp; ++e)
#pragma unroll
    for (int tp = 0; tp < kTileTok / 2; ++tp) acc[e][tp] = make_float2(0.0f, 0.0f);
  const uint32_t slices = hidden / 512u;
  for (uint32_t sl = warp; sl < slices; sl += 8u) {
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const uint32_t c0 = 512u * sl + 8u * lane + 256u * (uint32_t)j;
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        float4 xq[kTileTok];
#pragma unroll
        for (int t = 0; t < kTileTok; ++t)
          xq[t] = t0 + t < tokens ? __ldg(reinterpret_cast<const float4 *>(x + (size_t)(t0 + t) * hidden + c0) + hf)
                                  : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int e = 0; e < kTileExp; ++e) {
          const uint2 wq = e0 + e < experts
                               ? __ldg(reinterpret_cast<const uint2 *>(w + (size_t)(e0 + e) * hidden + c0) + hf)
                               : make_uint2(0u, 0u);
          const float wf[4] = {bf16lo(wq.x), bf16hi(wq.x), bf16lo(wq.y), bf16hi(wq.y)};
#pragma unroll
          for (int tp = 0; tp < kTileTok / 2; ++tp) {
            const float4 a = xq[2 * tp], b = xq[2 * tp + 1];
            acc[e][tp] = __ffma2_rn(make_float2(a.x, b.x), make_float2(wf[0], wf[0]), acc[e][tp]);
            acc[e][tp] = __ffma2_rn(make_float2(a.y, b.y), make_float2(wf[1], wf[1]), acc[e][tp]);
            acc[e][tp] = __ffma2_rn(make_float2(a.z, b.z), make_float2(wf[2], wf[2]), acc[e][tp]);
            acc[e][tp] = __ffma2_rn(make_float2(a.w, b.w), make_float2(wf[3], wf[3]), acc[e][tp]);
          }
        }
      }
    }
  }
  // flatten: v[e * 8 + t]
  float v[NP];
#pragma unroll
  for (int e = 0; e < kTileExp; ++e)
#pragma unroll
    for (int tp = 0; tp < kTileTok / 2; ++tp) {
      v[e * kTileTok + 2 * tp] = acc[e][tp].x;
      v[e * kTileTok + 2 * tp + 1] = acc[e][tp].y;
    }
  // transpose-reduce over the 32 lanes: 128 pairs -> 4 per lane
#pragma unroll
  for (int o = 16, n = NP / 2; o >= 1; o >>= 1, n >>= 1) {
    const bool upper = (lane & (uint32_t)o) != 0u;
#pragma unroll
    for (int i = 0; i < n; ++i) {
      const float send = upper ? v[i] : v[i + n];
      const float keep = upper ? v[i + n] : v[i];
      v[i] = __fadd_rn(keep, __shfl_xor_sync(0xffffffffu, send, o));
    }
  }
#pragma unroll
  for (int k = 0; k < NP / 32; ++k) part[warp][(NP / 32) * lane + k] = v[k];
  __syncthreads();
  if (threadIdx.x < (unsigned)NP) {
    const uint32_t p = threadIdx.x, e = p / kTileTok, t = p % kTileTok;
    if (t0 + t < tokens && e0 + e < experts) {
      float s = part[0][p];
#pragma unroll
      for (int k = 1; k < 8; ++k) s = __fadd_rn(s, part[k][p]);
      logits[(size_t)(t0 + t) * experts + e0 + e] = s;
    }
  }
}

cudaError_t launch_router_logits(const float *x, uint32_t tokens, const uint16_t *w, uint32_t experts,
                                 uint32_t hidden, float *logits, cudaStream_t stream) {
  if (hidden % 512u || tokens == 0) return cudaErrorInvalidValue;
  if (tokens >= 64u) {
    dim3 grid((experts + kTileExp - 1) / kTileExp, (tokens + kTileTok - 1) / kTileTok);
    return launch_kernel(k_router_logits_tiled, grid, dim3(256), 0, stream, x, tokens, w, experts, hidden, logits);
  }
  dim3 grid(experts, (tokens + kRouterTok - 1) / kRouterTok);
  return launch_kernel(k_router_logits, grid, dim3(256), 0, stream, x, tokens, w, experts, hidden, logits);
}

// --------------------------------------------------------------- router top-k
// One CTA per token (src/text_endpoint.rs:4394 pytorch_noaux_routes):
// score = SLEEF sigmoid(logit); corrected = score + bias; 9 rounds of
// block-wide argmax (ties -> lower index) give the 8 picks in canonical order
// and the first rejected value (boundary margin / tie detection).
// weight_k = score_k / (pairwise sum of the 8 + 1e-20) (src/text_endpoint.rs:4382).
constexpr int kTopkPer = 4;  // experts per thread: up to 1024 experts

__device__ __forceinline__ bool better(float va, uint32_t ia, float vb, uint32_t ib) {
  return va > vb || (va == vb && ia < ib);
}

__device__ __forceinline__ void argmax_shfl(float &bv, uint32_t &bi, float &bs, int width) {
  for (int o = width / 2; o >= 1; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o, width);
    const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, o, width);
    const float os = __shfl_xor_sync(0xffffffffu, bs, o, width);
    if (better(ov, oi, bv, bi)) {
      bv = ov;
      bi = oi;
      bs = os;
    }
  }
}

__global__ void __launch_bounds__(256) k_router_topk(const float *__restrict__ logits, const float *__restrict__ bias,
                                                     uint32_t tokens, uint32_t experts, uint32_t *__restrict__ selected,
                                                     float *__restrict__ weights, uint32_t *tie_rows, uint32_t *flags) {
  pdl_wait();
  pdl_launch_dependents();
  __shared__ float cv[8], cs[8];
  __shared__ uint32_t ci[8];
  __shared__ float pick_s[9], pick_v[9];
  __shared__ uint32_t pick_i[9];
  const uint32_t t = blockIdx.x;
  const uint32_t tid = threadIdx.x, lane = tid % 32u, warp = tid / 32u;
  float score[kTopkPer], corr[kTopkPer];
  uint32_t taken = 0;
#pragma unroll
  for (int k = 0; k < kTopkPer; ++k) {
    const uint32_t e = tid + 256u * k;
    score[k] = 0.0f;
    corr[k] = -__int_as_float(0x7f800000);
    if (e < experts) {
      const float lg = logits[(size_t)t * experts + e];
      const float b = __ldg(bias + e);
      if (!finite(lg) || !finite(b)) raise_flag(flags, PW_FLAG_NONFINITE_INPUT);
      score[k] = sigmoid_sleef(lg);
      corr[k] = __fadd_rn(score[k], b);
    }
  }
  for (int round = 0; round < 9; ++round) {
    float bv = -__int_as_float(0x7f800000), bs = 0.0f;
    uint32_t bi = 0xffffffffu;
#pragma unroll
    for (int k = 0; k < kTopkPer; ++k) {
      const uint32_t e = tid + 256u * k;
      if (e < experts && !(taken & (1u << k)) && better(corr[k], e, bv, bi)) {
        bv = corr[k];
        bi = e;
        bs = score[k];
      }
    }
    argmax_shfl(bv, bi, bs, 32);
    if (lane == 0) {
      cv[warp] = bv;
      ci[warp] = bi;
      cs[warp] = bs;
    }
    __syncthreads();
    if (warp == 0) {
      bv = lane < 8u ? cv[lane] : -__int_as_float(0x7f800000);
      bi = lane < 8u ? ci[lane] : 0xffffffffu;
      bs = lane < 8u ? cs[lane] : 0.0f;
      argmax_shfl(bv, bi, bs, 32);
      if (lane == 0) {
        pick_v[round] = bv;
        pick_i[round] = bi;
        pick_s[round] = bs;
      }
    }
    __syncthreads();
    const uint32_t w = pick_i[round];
    if (round < 8 && w != 0xffffffffu && w % 256u == tid) taken |= 1u << (w / 256u);
  }
  if (tid == 0) {
    const float l0 = __fadd_rn(pick_s[0], pick_s[4]);
    const float l1 = __fadd_rn(pick_s[1], pick_s[5]);
    const float l2 = __fadd_rn(pick_s[2], pick_s[6]);
    const float l3 = __fadd_rn(pick_s[3], pick_s[7]);
    const float den = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(0.0f, l0), l1), l2), l3), 1.0e-20f);
    float sum = 0.0f;
    bool ok = true;
    for (int k = 0; k < 8; ++k) {
      const float wk = __fdiv_rn(pick_s[k], den);
      ok = ok && finite(wk) && wk >= 0.0f && pick_i[k] < experts;
      sum = __fadd_rn(sum, wk);
      selected[(size_t)t * 8 + k] = pick_i[k];
      weights[(size_t)t * 8 + k] = wk;
    }
    if (!ok || fabsf(__fsub_rn(sum, 1.0f)) > 1.0e-6f) raise_flag(flags, PW_FLAG_ROUTE_WEIGHTS);
    if (pick_v[7] == pick_v[8] && tie_rows) atomicAdd(tie_rows, 1u);
  }
}

cudaError_t launch_router_topk(const float *logits, const float *bias, uint32_t tokens, uint32_t experts,
                               uint32_t *selected, float *weights, uint32_t *tie_rows, uint32_t *flags,
                               cudaStream_t stream) {
  if (experts <= 8 || experts > 256u * kTopkPer || tokens == 0) return cudaErrorInvalidValue;
  return launch_kernel(k_router_topk, dim3(tokens), dim3(256), 0, stream, logits, bias, tokens, experts, selected,
                       weights, tie_rows, flags);
}

// ----------------------------------------------------------------- schedule
// Single CTA.  Placements are ordered by (expert ascending, position
// ascending) -- the reference's BTreeMap<expert, [(position, weight)]>
// (src/text_endpoint.rs:4768-4776, src/text_endpoint.rs:5302-5310).  The rank
// of a token among an expert's placements comes from per-expert token
// bitmasks, so the order is deterministic without sorting.
constexpr uint32_t kSchedMaxTokens = 2048;
constexpr uint32_t kSchedMaxExperts = 256;
constexpr uint32_t kSchedWords = kSchedMaxTokens / 32u;

__global__ void __launch_bounds__(1024) k_schedule(const uint32_t *__restrict__ selected,
                                                   const float *__restrict__ weights, uint32_t tokens,
                                                   uint32_t experts, BankTable bank, ScheduleOut out,
                                                   uint32_t *flags, uint32_t chunk) {
  pdl_wait();
  pdl_launch_dependents();
  extern __shared__ uint32_t sm[];
  uint32_t *mask = sm;                                      // [experts][words]
  uint16_t *prefix = reinterpret_cast<uint16_t *>(mask + experts * kSchedWords);  // [experts][words]
  uint32_t *cnt = reinterpret_cast<uint32_t *>(prefix + experts * kSchedWords);   // [experts + 1]
  uint32_t *grp_off = cnt + experts + 1;                    // [experts + 1]
  __shared__ uint32_t bad;
  const uint32_t words = (tokens + 31u) / 32u;
  const uint32_t tid = threadIdx.x, nt = blockDim.x;
  if (tid == 0) bad = 0;
  for (uint32_t i = tid; i < experts * words; i += nt) mask[(i / words) * kSchedWords + i % words] = 0;
  __syncthreads();
  for (uint32_t i = tid; i < tokens * 8u; i += nt) {
    const uint32_t e = selected[i];
    const uint32_t t = i / 8u;
    if (e >= experts) {
      bad = 1;
      continue;
    }
    const uint32_t prev = atomicOr(&mask[e * kSchedWords + t / 32u], 1u << (t % 32u));
    if (prev & (1u << (t % 32u))) bad = 1;  // duplicate expert in one row
  }
  __syncthreads();
  if (bad) {
    if (tid == 0) raise_flag(flags, PW_FLAG_BAD_EXPERT_COUNT);
    if (tid == 0 && out.n_groups) *out.n_groups = 0;
    return;
  }
  // per-expert counts and word prefixes (thread per expert)
  for (uint32_t e = tid; e < experts; e += nt) {
    uint32_t run = 0;
    for (uint32_t wi = 0; wi < words; ++wi) {
      prefix[e * kSchedWords + wi] = (uint16_t)run;
      run += __popc(mask[e * kSchedWords + wi]);
    }
    cnt[e] = run;
  }
  __syncthreads();
  if (tid == 0) {
    uint32_t off = 0, goff = 0, uniq = 0, maxc = 0;
    for (uint32_t e = 0; e < experts; ++e) {
      const uint32_t c = cnt[e];
      out.offsets[e] = off;
      grp_off[e] = goff;
      off += c;
      goff += (c + chunk - 1u) / chunk;
      uniq += c ? 1u : 0u;
      maxc = c > maxc ? c : maxc;
    }
    out.offsets[experts] = off;
    grp_off[experts] = goff;
    if (out.n_groups) *out.n_groups = goff;
    out.counters[0] = uniq;
    out.counters[1] = off;
    out.counters[2] = maxc;
  }
  __syncthreads();
  // placement index of every (token, slot)
  for (uint32_t i = tid; i < tokens * 8u; i += nt) {
    const uint32_t e = selected[i];
    const uint32_t t = i / 8u;
    const uint32_t wi = t / 32u;
    const uint32_t below = mask[e * kSchedWords + wi] & ((1u << (t % 32u)) - 1u);
    const uint32_t p = out.offsets[e] + prefix[e * kSchedWords + wi] + __popc(below);
    out.placement_tok[p] = t;
    out.placement_w[p] = weights[i];
  }
  // per token: its 8 placements in ascending expert order (combine order)
  for (uint32_t t = tid; t < tokens; t += nt) {
    uint32_t ex[8], pl[8];
    for (int k = 0; k < 8; ++k) {
      const uint32_t e = selected[t * 8u + k];
      const uint32_t wi = t / 32u;
      const uint32_t below = mask[e * kSchedWords + wi] & ((1u << (t % 32u)) - 1u);
      ex[k] = e;
      pl[k] = out.offsets[e] + prefix[e * kSchedWords + wi] + __popc(below);
    }
    for (int a = 1; a < 8; ++a) {
      const uint32_t ke = ex[a], kp = pl[a];
      int b = a - 1;
      while (b >= 0 && ex[b] > ke) {
        ex[b + 1] = ex[b];
        pl[b + 1] = pl[b];
        --b;
      }
      ex[b + 1] = ke;
      pl[b + 1] = kp;
    }
    for (int k = 0; k < 8; ++k) out.slot_place[t * 8u + k] = pl[k];
  }
  // GEMV/GEMM groups: each expert's placements in chunks of <= chunk tokens
  // (skipped when the caller runs the experts elsewhere: no group arrays)
  for (uint32_t e = tid; e < experts && out.gu_groups; e += nt) {
    const uint32_t c = cnt[e];
    for (uint32_t j = 0; j * chunk < c; ++j) {
      GemvGroup g;
      g.tok_begin = out.offsets[e] + chunk * j;
      g.count = min(chunk, c - chunk * j);
      g.expert = e;
      g.pad = 0;
      g.w0 = bank.gate_w[e];
      g.s0 = bank.gate_s[e];
      g.w1 = bank.up_w[e];
      g.s1 = bank.up_s[e];
      g.tm0 = bank.gate_tm + e;
      g.tm1 = bank.up_tm + e;
      out.gu_groups[grp_off[e] + j] = g;
      GemvGroup d = g;
      d.w0 = bank.down_w[e];
      d.s0 = bank.down_s[e];
      d.w1 = nullptr;
      d.s1 = nullptr;
      d.tm0 = bank.down_tm + e;
      d.tm1 = nullptr;
      out.dn_groups[grp_off[e] + j] = d;
    }
  }
}

cudaError_t launch_schedule(const uint32_t *selected, const float *weights, uint32_t tokens, uint32_t experts,
                            const BankTable &bank, const ScheduleOut &out, uint32_t *flags, uint32_t chunk,
                            cudaStream_t stream) {
  if (tokens == 0 || tokens > kSchedMaxTokens || experts > kSchedMaxExperts || experts < 8 || chunk == 0)
    return cudaErrorInvalidValue;
  const size_t smem = (size_t)experts * kSchedWords * 4 + (size_t)experts * kSchedWords * 2 +
                      (size_t)(experts + 1) * 8;
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(k_schedule, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)((size_t)kSchedMaxExperts * kSchedWords * 6 +
                                               (size_t)(kSchedMaxExperts + 1) * 8));
    if (e != cudaSuccess) return e;
    configured = true;
  }
  return launch_kernel(k_schedule, dim3(1), dim3(1024), smem, stream, selected, weights, tokens, experts, bank, out,
                       flags, chunk);
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
                          float *__restrict__ y, uint32_t *flags) {
  pdl_wait();
  pdl_launch_dependents();
  const uint32_t t = blockIdx.y;
  __shared__ uint32_t pl[8];
  __shared__ float wt[8];
  if (threadIdx.x < 8) {
    pl[threadIdx.x] = slot_place[t * 8u + threadIdx.x];
    wt[threadIdx.x] = placement_w[pl[threadIdx.x]];
  }
  __syncthreads();
  for (uint32_t c4 = blockIdx.x * blockDim.x + threadIdx.x; c4 < hidden / 4u; c4 += gridDim.x * blockDim.x) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float4 d = load4(down + (size_t)pl[k] * hidden, c4);
      acc.x = __fadd_rn(acc.x, __fmul_rn(d.x, wt[k]));
      acc.y = __fadd_rn(acc.y, __fmul_rn(d.y, wt[k]));
      acc.z = __fadd_rn(acc.z, __fmul_rn(d.z, wt[k]));
      acc.w = __fadd_rn(acc.w, __fmul_rn(d.w, wt[k]));
    }
    acc.x = round_bf16(acc.x);
    acc.y = round_bf16(acc.y);
    acc.z = round_bf16(acc.z);
    acc.w = round_bf16(acc.w);
    if (!finite(acc.x) || !finite(acc.y) || !finite(acc.z) || !finite(acc.w))
      raise_flag(flags, PW_FLAG_NONFINITE_COMBINE);
    reinterpret_cast<float4 *>(y + (size_t)t * hidden)[c4] = acc;
  }
}

cudaError_t launch_combine(const float *down, const uint32_t *slot_place, const float *placement_w,
                           uint32_t tokens, uint32_t hidden, float *y, uint32_t *flags, cudaStream_t stream) {
  if (hidden % 4u || tokens == 0) return cudaErrorInvalidValue;
  dim3 grid((hidden / 4u + 255u) / 256u, tokens);
  return launch_kernel(k_combine<float>, grid, dim3(256), 0, stream, down, slot_place, placement_w, tokens, hidden,
                       y, flags);
}

cudaError_t launch_combine_bf16(const uint16_t *down, const uint32_t *slot_place, const float *placement_w,
                                uint32_t tokens, uint32_t hidden, float *y, uint32_t *flags, cudaStream_t stream) {
  if (hidden % 4u || tokens == 0) return cudaErrorInvalidValue;
  dim3 grid((hidden / 4u + 255u) / 256u, tokens);
  return launch_kernel(k_combine<uint16_t>, grid, dim3(256), 0, stream, down, slot_place, placement_w, tokens,
                       hidden, y, flags);
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
// two roundings of the staged SwiGLU; this pass finishes it at full occupancy:
// h = bf16(bf16(g / (1 + exp(-g))) * u) (kernels/block_fp8_gemv.metal:139),
// then the down input's dynamic FP8 quantization exactly as k_quantize.  One
// warp per 128-value group; lane l holds values 4l..4l+3.
__global__ void k_swiglu_quant(const uint16_t *__restrict__ gate, const uint16_t *__restrict__ up, uint64_t groups,
                               float *__restrict__ h, uint8_t *__restrict__ codes, float *__restrict__ scales,
                               uint32_t *flags, const uint32_t *rows_dev, uint32_t groups_per_row) {
  pdl_wait();
  pdl_launch_dependents();
  if (rows_dev) groups = min(groups, (uint64_t)*rows_dev * groups_per_row);
  const uint64_t warp_global = ((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) / 32u;
  const uint32_t lane = threadIdx.x % 32u;
  const uint64_t nwarps = ((uint64_t)gridDim.x * blockDim.x) / 32u;
  for (uint64_t grp = warp_global; grp < groups; grp += nwarps) {
    const uint2 gq = __ldg(reinterpret_cast<const uint2 *>(gate + grp * 128u) + lane);
    const uint2 uq = __ldg(reinterpret_cast<const uint2 *>(up + grp * 128u) + lane);
    const uint32_t gw[2] = {gq.x, gq.y}, uw[2] = {uq.x, uq.y};
    float v[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float g = __uint_as_float((k & 1) ? (gw[k / 2] & 0xffff0000u) : (gw[k / 2] << 16));
      const float u = __uint_as_float((k & 1) ? (uw[k / 2] & 0xffff0000u) : (uw[k / 2] << 16));
      v[k] = staged_swiglu(g, u);
    }
    const bool ok = finite(v[0]) && finite(v[1]) && finite(v[2]) && finite(v[3]);
    if (!ok) raise_flag(flags, PW_FLAG_NONFINITE_FUSED);
    if (h) reinterpret_cast<float4 *>(h + grp * 128u)[lane] = make_float4(v[0], v[1], v[2], v[3]);
    float m = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    const float scale = __fdiv_rn(fmaxf(m, 1.0e-10f), 448.0f);
    auto q = [&](float val) { return fminf(fmaxf(__fdiv_rn(val, scale), -448.0f), 448.0f); };
    const uint32_t lo = encode2(q(v[0]), q(v[1]));
    const uint32_t hi = encode2(q(v[2]), q(v[3]));
    reinterpret_cast<uint32_t *>(codes + grp * 128u)[lane] = lo | (hi << 16);
    if (lane == 0) scales[grp] = scale;
  }
}

cudaError_t launch_swiglu_quant(const uint16_t *gate, const uint16_t *up, uint32_t rows, uint32_t cols, float *h,
                                uint8_t *codes, float *scales, uint32_t *flags, cudaStream_t stream,
                                const uint32_t *rows_dev) {
  if (cols % 128u) return cudaErrorInvalidValue;
  const uint64_t groups = (uint64_t)rows * (cols / 128u);
  if (groups == 0) return cudaSuccess;
  const int threads = 256;
  uint64_t blocks = (groups * 32u + threads - 1) / threads;
  if (blocks > 148u * 8u) blocks = 148u * 8u;
  return launch_kernel(k_swiglu_quant, dim3((unsigned)blocks), dim3(threads), 0, stream, gate, up, groups, h, codes,
                       scales, flags, rows_dev, cols / 128u);
}

}  // namespace pw
