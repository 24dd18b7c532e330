// pw_gemm_tc.cu -- grouped block-scaled FP8 GEMM on tcgen05 / TMEM (wide widths).
//
// For prefill-width groups (tens to hundreds of tokens per weight matrix) the
// same equation as the GEMV (src/wide_metal_moe.rs:404-423)
//   y[t, r] = sum_kb ( sum_{c in kb} dec(W[r, c]) * dec(code[t, c]) ) * S[r/128, kb] * xs[t, kb]
// runs on the 5th-generation tensor cores:
//  * A = 128 weight rows x 32 columns, B = TN token rows x 32 columns, both
//    K-major e4m3 in shared memory (128B swizzle, written by TMA);
//  * one elected thread issues tcgen05.mma.kind::f8f6f4 into a TMEM
//    accumulator; every 128-column block gets a fresh accumulator (the
//    checkpoint's f32 block scales are not power-of-two UE8M0 scales, so the
//    hardware block-scaled MMA cannot apply them);
//  * four epilogue warps tcgen05.ld each block's result, promote it with
//    S[r/128, kb] * xs[t, kb] into f32 registers (one thread per row), while
//    the MMA of the next block fills the other TMEM buffer;
//  * a producer warp streams stages of {128 rows x 2 blocks} weights (one
//    32 KB 3-D TMA box) and {TN tokens x 2 blocks} activation codes; in the
//    fused kernel all gate stages of a tile come first, then all up stages,
//    and the finished gate sums wait in spare TMEM columns so only one set of
//    accumulators occupies registers.
// Work: persistent CTAs over (group, 128-row tile); a group is <= TN tokens
// of one weight matrix (an expert's placements, or a chunk of a projection).
// The fused variant alternates gate and up stages and finishes with the
// staged bf16 SwiGLU and the hidden's dynamic FP8 quantization, exactly as
// the GEMV does.
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

#include "pw_device.cuh"
#include "pw_internal.h"

namespace pw {
namespace tc {

constexpr int kProducerWarp = 0;
constexpr int kMmaWarp = 1;
constexpr int kEpiWarp0 = 2;
constexpr int kEpiThreads = 128;
constexpr int kThreads = 6 * 32;
constexpr int kTileRows = 128;
constexpr int kWBox = 32 * 1024;  // weights: 128 rows x 2 k-blocks x 128 B

template <int KIND, int TN>
struct Cfg {
  static constexpr bool FUSED = KIND == 2;
  static constexpr int MATS = FUSED ? 2 : 1;
  static constexpr int XBOX = TN * 256;  // activations: TN rows x 2 k-blocks x 128 B
  static constexpr int STAGE = kWBox + XBOX;
  static constexpr int NST = (200 * 1024) / STAGE;
  // 2 k-blocks x 2 buffers x TN f32 columns, plus TN columns for the gate
  // sums of the fused kernel; allocations are powers of two
  static constexpr int TMEM_USED = 4 * TN + (FUSED ? TN : 0);
  static constexpr int TMEM_COLS = TMEM_USED <= 128 ? 128 : TMEM_USED <= 256 ? 256 : 512;
  static constexpr int RING = NST * STAGE;
  static constexpr int XS = RING;                     // token scales [TN][32] f32
  static constexpr int WS = XS + TN * 32 * 4;         // weight scales [2][32] f32
  static constexpr int AMAX = WS + 2 * 32 * 4;        // [4 warps][TN] f32
  static constexpr int BARS = AMAX + 4 * TN * 4;      // mbarriers
  static constexpr int NBARS = 2 * NST + 4;           // full, empty, tfull[2], tempty[2]
  static constexpr int MISC = BARS + NBARS * 8;       // tmem base, abort
  static constexpr int SMEM = MISC + 16 + 1024;       // + alignment slack
  static_assert(TMEM_COLS <= 512, "TMEM holds 512 columns");
  static_assert(SMEM <= 227 * 1024, "shared memory");
};

// ------------------------------------------------------------------ PTX
__device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *map, int x, int y, int z, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(
          smem_addr(dst)),
      "l"(map), "r"(x), "r"(y), "r"(z), "r"(smem_addr(bar))
      : "memory");
}

__device__ __forceinline__ void tensormap_acquire(const CUtensorMap *map) {
  asm volatile("fence.proxy.tensormap::generic.acquire.gpu [%0], 128;" ::"l"(map) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// K-major operand, 128B swizzle: rows are 128-byte lines, 8-row groups 1024 B
// apart (SBO), LBO unused (1), version 1, base offset 0 (1024-aligned tiles).
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3fffu);        // start address
  d |= (uint64_t)1u << 16;                         // leading byte offset (unused for SW128 K-major)
  d |= (uint64_t)(1024u >> 4) << 32;               // stride byte offset
  d |= (uint64_t)1u << 46;                         // descriptor version (sm_100)
  d |= (uint64_t)2u << 61;                         // SWIZZLE_128B
  return d;
}

// kind::f8f6f4 instruction descriptor: D f32, A/B e4m3, both K-major, M=128, N=TN.
template <int TN>
__device__ __forceinline__ uint32_t instr_desc() {
  return (1u << 4)                   // c_format F32
         | (0u << 7) | (0u << 10)    // a, b: E4M3
         | (0u << 15) | (0u << 16)   // K-major
         | ((uint32_t)(TN >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}

__device__ __forceinline__ void mma_f8(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(accum), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
      : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
               : "memory");
}

// 32 lanes x 32 consecutive f32 columns (one per register) of the warp's lane quarter.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 32 lanes x 32 consecutive f32 columns from registers into TMEM.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float *v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7]), "f"(v[8]), "f"(v[9]),
      "f"(v[10]), "f"(v[11]), "f"(v[12]), "f"(v[13]), "f"(v[14]), "f"(v[15]), "f"(v[16]), "f"(v[17]), "f"(v[18]),
      "f"(v[19]), "f"(v[20]), "f"(v[21]), "f"(v[22]), "f"(v[23]), "f"(v[24]), "f"(v[25]), "f"(v[26]), "f"(v[27]),
      "f"(v[28]), "f"(v[29]), "f"(v[30]), "f"(v[31])
      : "memory");
}

__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

struct Shared {
  uint8_t *ring;
  float *xs;
  float *ws;
  float *amax;
  uint64_t *full, *empty, *tfull, *tempty;
  uint32_t *tmem_base;
  volatile int *abort;
};

__device__ __forceinline__ bool bwait(const Shared &sh, uint64_t *bar, uint32_t parity, uint32_t *flags) {
  if (*sh.abort) return false;
  if (mbar_wait(bar, parity)) return true;
  *sh.abort = 1;
  raise_flag(flags, PW_FLAG_WAIT_TIMEOUT);
  return false;
}

template <int KIND, int TN>
__global__ void __launch_bounds__(kThreads, 1) k_gemm_tc(const __grid_constant__ GemmArgs A) {
  using C = Cfg<KIND, TN>;
  constexpr int MATS = C::MATS;
  const GemvArgs &a = A.g;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Shared sh;
  sh.ring = smem;
  sh.xs = reinterpret_cast<float *>(smem + C::XS);
  sh.ws = reinterpret_cast<float *>(smem + C::WS);
  sh.amax = reinterpret_cast<float *>(smem + C::AMAX);
  sh.full = reinterpret_cast<uint64_t *>(smem + C::BARS);
  sh.empty = sh.full + C::NST;
  sh.tfull = sh.empty + C::NST;
  sh.tempty = sh.tfull + 2;
  sh.tmem_base = reinterpret_cast<uint32_t *>(smem + C::MISC);
  sh.abort = reinterpret_cast<volatile int *>(smem + C::MISC + 4);

  const uint32_t warp = threadIdx.x / 32u, lane = threadIdx.x % 32u;
  if (threadIdx.x == 0) {
    for (int i = 0; i < C::NST; ++i) {
      mbar_init(&sh.full[i], 1);
      mbar_init(&sh.empty[i], 1);  // arrived by the MMA warp's tcgen05.commit
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sh.tfull[i], 1);                // tcgen05.commit after a stage's MMAs
      mbar_init(&sh.tempty[i], kEpiThreads / 32);  // one arrive per epilogue warp
    }
    *sh.abort = 0;
    mbar_fence_init();
  }
  if (warp == kMmaWarp) {
    // allocate the accumulator columns (whole warp), then let other CTAs allocate
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(sh.tmem_base)),
                 "r"((uint32_t)C::TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pdl_wait();
  pdl_launch_dependents();

  const uint32_t tmem = *sh.tmem_base;
  const uint32_t n_groups = a.n_groups_dev ? min(*a.n_groups_dev, a.n_groups) : a.n_groups;
  const uint32_t tpg = a.rows / kTileRows;
  const uint64_t total = (uint64_t)n_groups * tpg;
  const uint32_t u_begin = (uint32_t)(total * blockIdx.x / gridDim.x);
  const uint32_t u_end = (uint32_t)(total * (blockIdx.x + 1) / gridDim.x);
  const uint32_t kblocks = a.K / 128u;
  const uint32_t kcs = (kblocks + 1u) / 2u;          // stages per matrix per tile
  const uint32_t per_tile = kcs * (uint32_t)MATS;   // stages per tile

  if (warp == kProducerWarp) {
    if (lane == 0) {
      uint32_t slot = 0, phase = 0, issued = 0, parity = 0;
      for (uint32_t u = u_begin; u < u_end; ++u) {
        const GemvGroup &g = a.groups[u / tpg];
        const CUtensorMap *m0 = KIND == 3 ? g.tm1 : g.tm0;
        tensormap_acquire(m0);
        if (MATS == 2) tensormap_acquire(g.tm1);
        const uint32_t row0 = (u % tpg) * kTileRows;
        for (uint32_t st = 0; st < per_tile; ++st) {
          const uint32_t m = st / kcs, kc = st % kcs;
          if (bwait(sh, &sh.empty[slot], phase ^ 1u, a.flags)) {
            uint8_t *dst = sh.ring + slot * C::STAGE;
            mbar_arrive_expect_tx(&sh.full[slot], C::STAGE);
            tma_load_3d(dst, m == 0 ? m0 : g.tm1, 0, (int)row0, (int)(kc * 2u), &sh.full[slot]);
            tma_load_3d(dst + kWBox, &A.xmap, 0, (int)g.tok_begin, (int)(kc * 2u), &sh.full[slot]);
            issued |= 1u << slot;
            parity = (parity & ~(1u << slot)) | (phase << slot);
          }
          if (++slot == (uint32_t)C::NST) {
            slot = 0;
            phase ^= 1u;
          }
        }
      }
      for (int i = 0; i < C::NST; ++i)
        if (issued & (1u << i))
          if (!mbar_wait(&sh.full[i], (parity >> i) & 1u)) raise_flag(a.flags, PW_FLAG_WAIT_TIMEOUT);
    }
  } else if (warp == kMmaWarp) {
    if (lane == 0) {
      const uint32_t idesc = instr_desc<TN>();
      const uint32_t ring = smem_addr(sh.ring);
      uint32_t slot = 0, phase = 0, buf = 0, bphase = 0;
      bool committed = false;
      uint32_t last_buf = 0, last_phase = 0;
      for (uint32_t u = u_begin; u < u_end; ++u) {
        for (uint32_t st = 0; st < per_tile; ++st) {
          const bool ok_full = bwait(sh, &sh.full[slot], phase, a.flags);
          const bool ok_buf = bwait(sh, &sh.tempty[buf], bphase ^ 1u, a.flags);
          tc_fence_after();
          if (ok_full && ok_buf) {
            const uint32_t kc = st % kcs;
            const uint32_t wbase = ring + slot * C::STAGE;
            const uint32_t xbase = wbase + kWBox;
#pragma unroll
            for (uint32_t j = 0; j < 2; ++j) {
              if (kc * 2u + j >= kblocks) break;
              const uint32_t d = tmem + buf * (2u * TN) + j * TN;
#pragma unroll
              for (uint32_t s = 0; s < 4; ++s) {
                const uint64_t ad = smem_desc_sw128(wbase + j * (kTileRows * 128u) + s * 32u);
                const uint64_t bd = smem_desc_sw128(xbase + j * (TN * 128u) + s * 32u);
                mma_f8(d, ad, bd, idesc, s > 0 ? 1u : 0u);
              }
            }
          }
          mma_commit(&sh.empty[slot]);   // stage reusable once these MMAs are done
          mma_commit(&sh.tfull[buf]);    // accumulators ready for the epilogue
          committed = true;
          last_buf = buf;
          last_phase = bphase;
          if (++slot == (uint32_t)C::NST) {
            slot = 0;
            phase ^= 1u;
          }
          if (++buf == 2u) {
            buf = 0;
            bphase ^= 1u;
          }
        }
      }
      // every MMA must be complete before the columns are freed
      if (committed)
        if (!mbar_wait(&sh.tfull[last_buf], last_phase)) raise_flag(a.flags, PW_FLAG_WAIT_TIMEOUT);
    }
  } else {
    // ---------------------------------------------------------- epilogue
    const uint32_t ew = warp - kEpiWarp0;         // 0..3
    const uint32_t quarter = warp % 4u;           // TMEM lane quarter this warp may access
    const uint32_t r_local = quarter * 32u + lane;  // tile row owned by this thread
    const uint32_t etid = ew * 32u + lane;
    uint32_t buf = 0, bphase = 0;
    for (uint32_t u = u_begin; u < u_end; ++u) {
      const GemvGroup grp = a.groups[u / tpg];
      const uint32_t row0 = (u % tpg) * kTileRows;
      // token scales and this tile's weight-scale row
      named_bar_sync(1, kEpiThreads);
      for (uint32_t i = etid; i < (uint32_t)TN * kblocks; i += kEpiThreads) {
        const uint32_t t = i / kblocks, kb = i % kblocks;
        sh.xs[t * 32u + kb] = t < grp.count ? __ldg(a.x_scales + (size_t)(grp.tok_begin + t) * kblocks + kb) : 0.0f;
      }
      {
        const uint32_t srow = row0 / 128u;
        const float *s0 = (KIND == 3 ? grp.s1 : grp.s0) + (size_t)srow * a.scale_cols;
        for (uint32_t i = etid; i < kblocks; i += kEpiThreads) {
          sh.ws[i] = __ldg(s0 + i);
          if (MATS == 2) sh.ws[32u + i] = __ldg(grp.s1 + (size_t)srow * a.scale_cols + i);
        }
      }
      named_bar_sync(1, kEpiThreads);

      float acc[TN];
#pragma unroll
      for (int t = 0; t < TN; ++t) acc[t] = 0.0f;
      const uint32_t lane_base = (quarter * 32u) << 16;
      const uint32_t stash = tmem + lane_base + 4u * TN;  // gate sums (fused)

      for (uint32_t st = 0; st < per_tile; ++st) {
        const uint32_t m = st / kcs, kc = st % kcs;
        if (MATS == 2 && st == kcs) {
          // gate finished: park its sums in TMEM and start the up sums
#pragma unroll
          for (int c = 0; c < TN; c += 32) tmem_st32(stash + c, &acc[c]);
          tmem_wait_st();
#pragma unroll
          for (int t = 0; t < TN; ++t) acc[t] = 0.0f;
        }
        const bool ok = bwait(sh, &sh.tfull[buf], bphase, a.flags);
        tc_fence_after();
        if (ok) {
#pragma unroll
          for (uint32_t j = 0; j < 2; ++j) {
            const uint32_t kb = kc * 2u + j;
            if (kb >= kblocks) break;
            const float ws = sh.ws[m * 32u + kb];
#pragma unroll
            for (int c = 0; c < TN; c += 32) {
              float v[32];
              tmem_ld32(tmem + lane_base + buf * (2u * TN) + j * TN + c, v);
              tmem_wait_ld();
#pragma unroll
              for (int i = 0; i < 32; ++i) acc[c + i] = fmaf(v[i], ws * sh.xs[(c + i) * 32u + kb], acc[c + i]);
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sh.tempty[buf]);
        if (++buf == 2u) {
          buf = 0;
          bphase ^= 1u;
        }
      }

      // outputs: thread owns row row0 + r_local, all TN token columns
      const uint32_t r = row0 + r_local;
      if (KIND != 2) {
#pragma unroll
        for (int t = 0; t < TN; ++t) {
          if ((uint32_t)t < grp.count) {
            const float out = a.round_bf16 ? round_bf16(acc[t]) : acc[t];
            if (!finite(out)) raise_flag(a.flags, PW_FLAG_NONFINITE_ROUND);
            a.out[(size_t)(grp.tok_begin + t) * a.out_stride + r] = out;
          }
        }
      } else {
        // staged SwiGLU (gate sums back from TMEM, up sums in registers), then
        // the hidden's dynamic FP8 quantization over this tile's 128 rows
        // (one quantization group of the down input)
#pragma unroll
        for (int c = 0; c < TN; c += 32) {
          float g[32];
          tmem_ld32(stash + c, g);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int t = c + i;
            const float h = (uint32_t)t < grp.count ? staged_swiglu(g[i], acc[t]) : 0.0f;
            if (!finite(h)) raise_flag(a.flags, PW_FLAG_NONFINITE_FUSED);
            acc[t] = h;
            if (a.out && (uint32_t)t < grp.count) a.out[(size_t)(grp.tok_begin + t) * a.out_stride + r] = h;
            float mx = fabsf(h);
#pragma unroll
            for (int o = 16; o >= 1; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
            if (lane == 0) sh.amax[ew * TN + t] = mx;
          }
        }
        named_bar_sync(1, kEpiThreads);
        const uint32_t I = a.rows;
#pragma unroll
        for (int t = 0; t < TN; ++t) {
          if ((uint32_t)t < grp.count) {
            const float M = fmaxf(fmaxf(sh.amax[t], sh.amax[TN + t]), fmaxf(sh.amax[2 * TN + t], sh.amax[3 * TN + t]));
            const float sc = __fdiv_rn(fmaxf(M, 1.0e-10f), 448.0f);
            const float q = fminf(fmaxf(__fdiv_rn(acc[t], sc), -448.0f), 448.0f);
            a.q_codes[(size_t)(grp.tok_begin + t) * I + r] = (uint8_t)(encode2(q, 0.0f) & 0xffu);
            if (r_local == 0) a.q_scales[(size_t)(grp.tok_begin + t) * (I / 128u) + row0 / 128u] = sc;
          }
        }
      }
    }
  }

  // free the accumulator columns once every role is done with them
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == kMmaWarp)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)C::TMEM_COLS)
                 : "memory");
}

template <int KIND, int TN>
static cudaError_t launch_one(const GemmArgs &a, int grid, cudaStream_t stream) {
  using C = Cfg<KIND, TN>;
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(k_gemm_tc<KIND, TN>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  return launch_kernel(k_gemm_tc<KIND, TN>, dim3(grid), dim3(kThreads), C::SMEM, stream, a);
}

}  // namespace tc

int gemm_tc_tokens(int kind) { return kind == 2 ? 64 : 128; }

cudaError_t launch_gemm_tc(int kind, const GemmArgs &a, int grid, cudaStream_t stream) {
  const GemvArgs &g = a.g;
  if (g.K == 0 || g.K % 128u || g.K > 4096u || g.rows % tc::kTileRows || grid <= 0 || g.layout != PW_LAYOUT_PLAIN)
    return cudaErrorInvalidValue;
  switch (kind) {
    case 0: return tc::launch_one<0, 128>(a, grid, stream);
    case 2: return tc::launch_one<2, 64>(a, grid, stream);
    case 3: return tc::launch_one<3, 128>(a, grid, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace pw
