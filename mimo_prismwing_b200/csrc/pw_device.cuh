// pw_device.cuh -- device helpers for the sm_100a block-FP8 routed-MoE path.
//
// Number formats follow the reference bit for bit:
//   e4m3fn decode          src/lib.rs:7456 (hardware cvt e4m3x2 -> f16x2 is exact)
//   bf16 round (RNE, NaN)  src/text_endpoint.rs:2960
//   e4m3fn encode (RNE)    src/text_endpoint.rs:2985 (nearest code, ties to even
//                          code == cvt.rn.satfinite after the +-448 clamp)
//   SLEEF expf_u10         src/text_endpoint.rs:4511 (SLEEF's published method)
// Arithmetic whose bits the oracle pins uses explicit __f*_rn intrinsics so
// that nvcc's FMA contraction cannot change the result.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#include "pw_cuda.h"

namespace pw {

// ------------------------------------------------------------ number formats
// Branch-free (selects): an unrolled epilogue stays one basic block.
__device__ __forceinline__ float round_bf16(float v) {
  const uint32_t bits = __float_as_uint(v);
  const uint32_t rn = (bits + 0x7fffu + ((bits >> 16) & 1u)) & 0xffff0000u;  // finite: RNE
  const uint32_t qnan = (bits | 0x00400000u) & 0xffff0000u;                  // NaN: quiet, payload kept
  const uint32_t a = bits & 0x7fffffffu;
  return __uint_as_float(a > 0x7f800000u ? qnan : (a == 0x7f800000u ? bits : rn));
}

// bf16(lo) | bf16(hi) << 16 with one conversion instruction, round to nearest
// even: for every non-NaN input the same bits as round_bf16 (a NaN becomes
// the canonical quiet NaN; callers treat any NaN as an error).
__device__ __forceinline__ uint32_t pack_bf16x2_rn(float lo, float hi) {
  uint32_t d;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
  return d;
}

// Four values bf16-rounded (as f32) by two conversion instructions.
__device__ __forceinline__ float4 round_bf16x4(float4 v) {
  const uint32_t a = pack_bf16x2_rn(v.x, v.y), b = pack_bf16x2_rn(v.z, v.w);
  return make_float4(__uint_as_float(a << 16), __uint_as_float(a & 0xffff0000u), __uint_as_float(b << 16),
                     __uint_as_float(b & 0xffff0000u));
}

// Smallest |f32| bit pattern that bf16 rounding turns into an infinity: the
// halfway point above the largest finite bf16 (0x7f7f, odd), where round to
// nearest even goes up to 0x7f80.
constexpr uint32_t kBf16OverflowBits = 0x7f7f8000u;

// Dynamic FP8 quantization of a 128-value group (src/text_endpoint.rs:3008):
// scale = max(absmax, 1e-10) / 448 and code = e4m3(clamp(value / scale)).
// The quotients are correctly rounded without a division per value, by
// Markstein's method (P. Markstein, IBM J. Res. Dev. 34(1), 1990; the division
// theorem in Muller et al., Handbook of Floating-Point Arithmetic): with
// rcp = RN(1/scale), q1 = q0 + (value - q0 scale) rcp is a faithful quotient,
// and one more correction from the exact FMA remainder of a faithful quotient
// gives RN(value / scale).  In range: |value| <= 448 scale (no overflow), and
// quotients small enough to meet underflow (< 2^-10) encode to zero either way.
// The sign is the value's (scale > 0): the corrections can turn -0 into +0.
struct Fp8GroupScale {
  float scale, rcp;
  __device__ __forceinline__ static Fp8GroupScale of(float absmax) {
    Fp8GroupScale g;
    g.scale = __fdiv_rn(fmaxf(absmax, 1.0e-10f), 448.0f);
    g.rcp = __frcp_rn(g.scale);
    return g;
  }
  // clamp(RN(value / scale), -448, 448)
  __device__ __forceinline__ float quotient(float value) const {
    const float q0 = __fmul_rn(value, rcp);
    const float q1 = __fmaf_rn(__fmaf_rn(-q0, scale, value), rcp, q0);
    const float q = copysignf(__fmaf_rn(__fmaf_rn(-q1, scale, value), rcp, q1), value);
    return fminf(fmaxf(q, -448.0f), 448.0f);
  }
};

// 4 packed e4m3 bytes -> 4 floats (byte 0 -> out[0]).  Exact.
__device__ __forceinline__ void decode4(uint32_t w, float &o0, float &o1, float &o2, float &o3) {
  uint32_t h01, h23;
  asm("{\n\t.reg .b16 lo, hi;\n\t"
      "mov.b32 {lo, hi}, %2;\n\t"
      "cvt.rn.f16x2.e4m3x2 %0, lo;\n\t"
      "cvt.rn.f16x2.e4m3x2 %1, hi;\n\t}"
      : "=r"(h01), "=r"(h23)
      : "r"(w));
  asm("{\n\t.reg .f16 a, b;\n\t"
      "mov.b32 {a, b}, %2;\n\t"
      "cvt.f32.f16 %0, a;\n\t"
      "cvt.f32.f16 %1, b;\n\t}"
      : "=f"(o0), "=f"(o1)
      : "r"(h01));
  asm("{\n\t.reg .f16 a, b;\n\t"
      "mov.b32 {a, b}, %2;\n\t"
      "cvt.f32.f16 %0, a;\n\t"
      "cvt.f32.f16 %1, b;\n\t}"
      : "=f"(o2), "=f"(o3)
      : "r"(h23));
}

__device__ __forceinline__ void decode16(const uint4 &q, float (&f)[16]) {
  decode4(q.x, f[0], f[1], f[2], f[3]);
  decode4(q.y, f[4], f[5], f[6], f[7]);
  decode4(q.z, f[8], f[9], f[10], f[11]);
  decode4(q.w, f[12], f[13], f[14], f[15]);
}

// Two floats -> two e4m3 bytes packed in the low 16 bits (lo -> byte 0).
// Round-to-nearest-even with saturation; inputs are already clamped to
// [-448, 448] so saturation never triggers.
__device__ __forceinline__ uint32_t encode2(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return (uint32_t)r;
}

// SLEEF expf_u10 (Cody-Waite reduction + degree-6 minimax polynomial), the
// method the reference restates at src/text_endpoint.rs:4511.
__device__ __forceinline__ float sleef_expf_u10(float d) {
  if (d < -104.0f) return 0.0f;
  if (d > 100.0f) return __int_as_float(0x7f800000);
  const float qf = rintf(__fmul_rn(d, 1.442695040888963407359924681001892137f));
  const int q = (int)qf;
  float s = __fmaf_rn(qf, -0.693145751953125f, d);
  s = __fmaf_rn(qf, -1.428606765330187045e-06f, s);
  float u = 0.000198527617612853646278381f;
  u = __fmaf_rn(u, s, 0.00139304355252534151077271f);
  u = __fmaf_rn(u, s, 0.00833336077630519866943359f);
  u = __fmaf_rn(u, s, 0.0416664853692054748535156f);
  u = __fmaf_rn(u, s, 0.166666671633720397949219f);
  u = __fmaf_rn(u, s, 0.5f);
  u = __fadd_rn(__fmaf_rn(__fmul_rn(s, s), u, s), 1.0f);
  const int q1 = q >> 1;
  const int q2 = q - q1;
  return __fmul_rn(__fmul_rn(u, __int_as_float((q1 + 127) << 23)), __int_as_float((q2 + 127) << 23));
}

__device__ __forceinline__ float sigmoid_sleef(float logit) {
  return __fdiv_rn(1.0f, __fadd_rn(1.0f, sleef_expf_u10(-logit)));
}

// Staged bf16 SwiGLU (src/text_endpoint.rs:5336-5342,
// kernels/block_fp8_gemv.metal:139): bf16 boundaries on g, u, silu and h.
__device__ __forceinline__ float staged_silu(float gate) {
  const float g = round_bf16(gate);
  return round_bf16(__fdiv_rn(g, __fadd_rn(1.0f, sleef_expf_u10(-g))));
}
__device__ __forceinline__ float staged_swiglu(float gate, float up) {
  const float silu = staged_silu(gate);
  const float u = round_bf16(up);
  return round_bf16(__fmul_rn(silu, u));
}

// Programmatic dependent launch: a kernel launched behind another may start
// early; it must wait for its predecessor's completion (and memory) before
// touching anything the predecessor, or any earlier kernel, writes.  Both are
// no-ops for a normal launch.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ bool finite(float v) { return (__float_as_uint(v) & 0x7f800000u) != 0x7f800000u; }

__device__ __forceinline__ void raise_flag(uint32_t *flags, uint32_t bit) {
  if (flags) atomicOr(flags, bit);
}

// -------------------------------------------------------- mbarrier / bulk copy
__device__ __forceinline__ uint32_t smem_addr(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.b32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Every wait in this library is bounded: after ~1 s of wall time the wait
// gives up, the caller raises PW_FLAG_WAIT_TIMEOUT and unwinds.
constexpr uint64_t kWaitLimitNs = 1000000000ull;

__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t start = global_timer_ns();
  for (;;) {
    if (mbar_try_wait(bar, parity)) return true;
    if (global_timer_ns() - start > kWaitLimitNs) return false;
  }
}

// 1-D bulk copy global -> shared, completing `bytes` of transaction count on
// `bar`.  src, dst 16-byte aligned; bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

__device__ __forceinline__ void named_bar_sync(uint32_t id, uint32_t threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// ------------------------------------------------------------- row mappings
// Fused-QKV row maps (src/text_endpoint.rs:3174 full_qkv_source_row, :3200
// swa_qkv_source_row, :3227 full_qkv_scale_row).  Logical rows are global
// Q, K, V; the checkpoint stores 4 tensor-parallel shards.
__device__ __host__ __forceinline__ uint32_t full_qkv_source_row(uint32_t r) {
  if (r < 12288u) return (r / 3072u) * 3392u + r % 3072u;
  if (r < 13056u) {
    const uint32_t l = r - 12288u;
    return (l / 192u) * 3392u + 3072u + l % 192u;
  }
  const uint32_t l = r - 13056u;
  return (l / 128u) * 3392u + 3264u + l % 128u;
}

__device__ __host__ __forceinline__ uint32_t full_qkv_scale_row_of_source(uint32_t src) {
  const uint32_t shard = src / 3392u, local = src % 3392u;
  if (local < 3072u) return shard * 27u + local / 128u;
  if (local < 3264u) return shard * 27u + 24u + (local - 3072u) / 128u;
  return shard * 27u + 26u;
}

__device__ __host__ __forceinline__ uint32_t swa_qkv_source_row(uint32_t r) {
  if (r < 12288u) return (r / 3072u) * 3712u + r % 3072u;
  if (r < 13824u) {
    const uint32_t l = r - 12288u;
    return (l / 384u) * 3712u + 3072u + l % 384u;
  }
  const uint32_t l = r - 13824u;
  return (l / 256u) * 3712u + 3456u + l % 256u;
}

// (source row, scale row) of a logical row.  Rows inside one aligned tile of
// <= 64 logical rows map to consecutive source rows with one scale row.
__device__ __host__ __forceinline__ void map_row(uint32_t layout, uint32_t logical, uint32_t &src,
                                                 uint32_t &scale_row) {
  if (layout == PW_LAYOUT_FULL_QKV) {
    src = full_qkv_source_row(logical);
    scale_row = full_qkv_scale_row_of_source(src);
  } else if (layout == PW_LAYOUT_SWA_QKV) {
    src = swa_qkv_source_row(logical);
    scale_row = src / 128u;
  } else {
    src = logical;
    scale_row = logical / 128u;
  }
}

}  // namespace pw
