// pw_gemv.cu -- the readable block-FP8 GEMV for sm_100a (widths 1..8).
//
// Computes, for every group g of <= 8 tokens sharing one e4m3 weight matrix,
//   y[t, r] = sum_kb ( sum_{c in kb} dec(W[r, c]) * x_t[c] ) * S[r/128, kb]
// with x an unquantized f32 activation: the reference's readable projection
// (mapped_fp8_gemv src/lib.rs:1272, block_fp8_gemv src/lib.rs:7469).  The
// block-scaled kinds (quantized x) run on the FP8 tensor-core GEMV in
// pw_gemv_mma.cu.
//
// B200 design.  A [2048 x 4096] projection is 8.4 MB: a weight stream whose
// whole HBM time is ~1.3 us, so the kernel must put every SM to work at once
// and keep tens of KB in flight per SM from the first cycle:
//  * one warp per output row, 8 rows per CTA, grid = rows / 8 per group
//    (256 CTAs for 2048 rows, several resident per SM);
//  * each lane issues all its 16-byte weight loads of the row (K / 512 of
//    them, 8 for K = 4096) before using any, so a CTA has its 32 KB of weight
//    reads in flight at once; the activation slices come from L1 (every warp
//    of the CTA reads the same x);
//  * lane l covers columns 512 i + 16 l .. + 15: its 16-term dot per token
//    (two interleaved chains of 8 fused multiply-adds) is scaled by that
//    block's S and added into the token's accumulator; a butterfly over the
//    32 lanes gives the row's sums.
// The code is small and branch-free per width bucket (the previous design, 8
// warps per CTA over 64-row units, had 32 CTAs for this shape and stalled on
// instruction fetch).
#include <cstdint>
#include <cuda_runtime.h>

#include "pw_device.cuh"
#include "pw_internal.h"

namespace pw {

constexpr int kRowsPerCta = 8;  // one warp per row
constexpr uint32_t kMaxKSteps = 8;  // K <= 4096: 512 columns per step

template <int CMAX>
__global__ void __launch_bounds__(kRowsPerCta * 32) k_gemv_readable(const GemvArgs a) {
  const uint32_t lane = threadIdx.x % 32u, warp = threadIdx.x / 32u;
  const uint32_t n_groups = a.n_groups_dev ? min(*a.n_groups_dev, a.n_groups) : a.n_groups;
  const uint32_t tiles = a.rows / kRowsPerCta;
  const uint32_t gi = blockIdx.x / tiles;
  if (gi >= n_groups) return;
  const GemvGroup grp = a.groups[gi];
  const uint32_t r = (blockIdx.x % tiles) * kRowsPerCta + warp;
  const uint32_t count = min(grp.count, (uint32_t)CMAX);
  const uint32_t steps = (a.K + 511u) / 512u;
  const uint8_t *wrow = grp.w0 + (size_t)r * a.K;
  const float *srow = grp.s0 + (size_t)(r / 128u) * a.scale_cols;
  // all of this lane's weight loads first.  Under programmatic dependent
  // launch they are issued before the wait: the weights and the group record
  // are no kernel's output (the record is cached or copied in before the
  // launch), so the stream overlaps the previous kernel's tail; x and y wait.
  // The next kernel is released only once this one's sums are done, so at
  // most two of these kernels hold SMs at a time.
  uint4 q[kMaxKSteps];
#pragma unroll
  for (uint32_t i = 0; i < kMaxKSteps; ++i) {
    const uint32_t c = 512u * i + 16u * lane;
    q[i] = (i < steps && c < a.K) ? __ldg(reinterpret_cast<const uint4 *>(wrow + c)) : make_uint4(0u, 0u, 0u, 0u);
  }
  pdl_wait();
  float acc[CMAX];
#pragma unroll
  for (int t = 0; t < CMAX; ++t) acc[t] = 0.0f;
#pragma unroll
  for (uint32_t i = 0; i < kMaxKSteps; ++i) {
    const uint32_t c = 512u * i + 16u * lane;
    if (i < steps && c < a.K) {
      float wf[16];
      decode16(q[i], wf);
      const float s = __ldg(srow + c / 128u);
#pragma unroll
      for (int t = 0; t < CMAX; ++t) {
        if (t < (int)count) {
          const uint32_t slot = grp.tok_begin + (uint32_t)t;
          const uint32_t xrow = a.tok_list ? __ldg(a.tok_list + slot) : slot;
          const float4 *xp = reinterpret_cast<const float4 *>(a.x_f32 + (size_t)xrow * a.K + c);
          float d0 = 0.0f, d1 = 0.0f;
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            const float4 xv = __ldg(xp + v);
            d0 = fmaf(wf[4 * v + 0], xv.x, d0);
            d1 = fmaf(wf[4 * v + 1], xv.y, d1);
            d0 = fmaf(wf[4 * v + 2], xv.z, d0);
            d1 = fmaf(wf[4 * v + 3], xv.w, d1);
          }
          acc[t] = fmaf(d0 + d1, s, acc[t]);
        }
      }
    }
  }
  pdl_launch_dependents();
#pragma unroll
  for (int t = 0; t < CMAX; ++t) {
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) acc[t] += __shfl_xor_sync(0xffffffffu, acc[t], o);
  }
  if (lane < count) {
    float v = acc[0];
#pragma unroll
    for (int t = 1; t < CMAX; ++t)
      if ((int)lane == t) v = acc[t];
    const float out = a.round_bf16 ? round_bf16(v) : v;
    if (!finite(out)) raise_flag(a.flags, PW_FLAG_NONFINITE_ROUND);
    a.out[(size_t)(grp.tok_begin + lane) * a.out_stride + r] = out;
  }
}

cudaError_t launch_gemv(int kind, const GemvArgs &a, int grid, cudaStream_t stream) {
  if (a.K == 0 || a.K % 128u || a.K > 4096u || a.rows % 64u || grid <= 0) return cudaErrorInvalidValue;
  switch (kind) {
    case 1: {
      if (a.layout != PW_LAYOUT_PLAIN || !a.x_f32) return cudaErrorInvalidValue;
      const dim3 g(a.n_groups * (a.rows / kRowsPerCta));
      const uint32_t w = a.max_count ? a.max_count : 8u;
      if (w <= 1u) return launch_kernel(k_gemv_readable<1>, g, dim3(kRowsPerCta * 32), 0, stream, a);
      if (w <= 2u) return launch_kernel(k_gemv_readable<2>, g, dim3(kRowsPerCta * 32), 0, stream, a);
      if (w <= 4u) return launch_kernel(k_gemv_readable<4>, g, dim3(kRowsPerCta * 32), 0, stream, a);
      return launch_kernel(k_gemv_readable<8>, g, dim3(kRowsPerCta * 32), 0, stream, a);
    }
    case 0:
    case 2:
    case 3:
      // Plain row-major weights, whole-K units: the tcgen05 GEMV (decode
      // layer at width 8: 282 -> 264 us).  Fused-QKV shard maps (64-row
      // boxes) and split-K launches (a lone expert: 1/8-tile units, where the
      // tcgen05 pipeline's fill latency cost 19 -> 24 us) keep the
      // warp-level MMA kernel.
      return a.layout == PW_LAYOUT_PLAIN && a.splits <= 1u ? launch_gemv_tc(kind, a, grid, stream)
                                                           : launch_gemv_mma(kind, a, grid, stream);
    default: return cudaErrorInvalidValue;
  }
}

int gemv_max_ctas(int num_sms) { return num_sms; }

}  // namespace pw
