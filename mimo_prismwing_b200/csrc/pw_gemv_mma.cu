// pw_gemv_mma.cu -- block-scaled FP8 GEMV on the FP8 tensor-core MMA (widths 1..8).
//
// Equation (src/wide_metal_moe.rs:404-423, kernels/block_fp8_gemv.metal:935-1046):
//   y[t, r] = sum_kb ( sum_{c in kb} dec(W[src(r), c]) * dec(code[t, c]) ) * S[srow(r), kb] * xs[t, kb]
// Each 128-column block dot runs as four m16n8k32 e4m3 x e4m3 -> f32 MMAs
// (A = 16 weight rows x 32 columns straight from the e4m3 bytes, B = the 8
// token slots' activation codes); its result is scaled by S * xs and added
// to f32 accumulators in increasing block order.
//
// B200 design.  At decode widths the kernel is a weight stream that has to
// run at HBM rate (~6.5 TB/s, ~22 B/clk per SM).  Measured on this part with
// one CTA per SM: achieved bandwidth tracks the bytes in flight and drops with
// the number of copies per byte (16 x 1 KB copies per stage: 2.0 TB/s; one
// 16 KB copy: 5.6 TB/s; 32 KB: 6.6 TB/s).  So:
//  * a CTA owns a 128-row tile of one weight matrix for the whole K; warp w
//    owns rows 16w..16w+15 of it, so there is no cross-warp reduction;
//  * a stage is one 128-column block of the tile: one 2-D TMA box of
//    128 rows x 128 B (two 64-row boxes when the rows come from a QKV shard
//    map), 128B-swizzled so ldmatrix reads are bank-conflict-free;
//  * a ~176 KB ring (11 stages, 5 for gate+up) keeps ~160 KB in flight per SM;
//  * lane 0 of warp 0 issues the TMA copies NST-1 stages ahead (a separate
//    producer warp would cap registers); the 8 token slots' codes and scales
//    sit in shared memory for the tile (rows padded to K+16 bytes).
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

#include "pw_device.cuh"
#include "pw_internal.h"

namespace pw {
namespace mma {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kTileRows = 128;
constexpr int kBoxBytes = kTileRows * 128;  // one matrix, one 128-column block
constexpr int kRingBytes = 176 * 1024;
constexpr int kMaxK = 4096;
constexpr int kXStride = kMaxK + 16;        // padded activation row in smem

template <int KIND>
struct Cfg {
  static constexpr bool FUSED = KIND == 2;
  static constexpr int MATS = FUSED ? 2 : 1;
  static constexpr int SLOT = kBoxBytes * MATS;
  static constexpr int NST = kRingBytes / SLOT;  // 11 or 5
  static constexpr int RING = NST * SLOT;
  static constexpr int XOFF = RING;                       // x codes [8][kXStride]
  static constexpr int SOFF = XOFF + 8 * kXStride;        // x scales [8][32]
  static constexpr int BOFF = SOFF + 8 * 32 * 4;          // barriers
  static constexpr int SMEM = BOFF + 2 * NST * 8 + 16 + 1024;  // + alignment slack
};

struct Ring {
  uint32_t slot = 0, phase = 0, issued = 0, parity = 0;
  __device__ __forceinline__ void advance(int nst) {
    if (++slot == (uint32_t)nst) {
      slot = 0;
      phase ^= 1u;
    }
  }
};

struct Shared {
  uint8_t *ring;
  uint8_t *x;
  float *xs;
  uint64_t *full;
  uint64_t *empty;
  volatile int *abort;
};

__device__ __forceinline__ bool ring_wait(const Shared &sh, uint64_t *bar, uint32_t parity, uint32_t *flags) {
  if (*sh.abort) return false;
  if (mbar_wait(bar, parity)) return true;
  *sh.abort = 1;
  raise_flag(flags, PW_FLAG_WAIT_TIMEOUT);
  return false;
}

__device__ __forceinline__ void ldmatrix_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

// D = A(16x32 e4m3, row) * B(32x8 e4m3, col) + D, f32 accumulate.
__device__ __forceinline__ void mma_e4m3(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.f32.e4m3.e4m3.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// 2-D TMA tile load: box at (x = column byte, y = row) of the tensor map.
// x is always a multiple of 128 (16-byte rule of the tiled copy).
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_addr(dst)),
      "l"(map), "r"(x), "r"(y), "r"(smem_addr(bar))
      : "memory");
}

__device__ __forceinline__ void tensormap_acquire(const CUtensorMap *map) {
  asm volatile("fence.proxy.tensormap::generic.acquire.gpu [%0], 128;" ::"l"(map) : "memory");
}

// Producer: walks (tile, k-block) exactly as the consumers do and issues one
// stage per call.  Lives in lane 0 of warp 0.
template <int KIND>
struct Producer {
  using C = Cfg<KIND>;
  uint32_t u, u_end, tpg, kb, kblocks;
  const CUtensorMap *m0;
  const CUtensorMap *m1;
  uint32_t src_lo, src_hi;  // source rows of the tile's two 64-row halves
  Ring ring;

  __device__ __forceinline__ void enter_tile(const GemvArgs &a) {
    if (u >= u_end) return;
    const GemvGroup &g = a.groups[u / tpg];
    m0 = KIND == 3 ? g.tm1 : g.tm0;
    m1 = g.tm1;
    // the maps were written through the generic proxy (host copy or bank
    // build); make those writes visible to the TMA unit before first use
    tensormap_acquire(m0);
    if (C::FUSED) tensormap_acquire(m1);
    const uint32_t row0 = (u % tpg) * kTileRows;
    uint32_t s;
    map_row(a.layout, row0, src_lo, s);
    map_row(a.layout, row0 + 64u, src_hi, s);
    kb = 0;
  }

  __device__ __forceinline__ void init(const GemvArgs &a, uint32_t ub, uint32_t ue, uint32_t tpg_) {
    u = ub;
    u_end = ue;
    tpg = tpg_;
    kblocks = a.K / 128u;
    enter_tile(a);
  }

  __device__ __forceinline__ void issue_next(const GemvArgs &a, const Shared &sh) {
    if (u >= u_end) return;
    if (ring_wait(sh, &sh.empty[ring.slot], ring.phase ^ 1u, a.flags)) {
      uint8_t *dst = sh.ring + ring.slot * C::SLOT;
      mbar_arrive_expect_tx(&sh.full[ring.slot], kBoxBytes * C::MATS);
      const int x = (int)(kb * 128u);
#pragma unroll
      for (int m = 0; m < C::MATS; ++m) {
        const CUtensorMap *map = m == 0 ? m0 : m1;
        if (a.layout == PW_LAYOUT_PLAIN) {
          tma_load_2d(dst + m * kBoxBytes, map, x, (int)src_lo, &sh.full[ring.slot]);
        } else {
          tma_load_2d(dst + m * kBoxBytes, map, x, (int)src_lo, &sh.full[ring.slot]);
          tma_load_2d(dst + m * kBoxBytes + kBoxBytes / 2, map, x, (int)src_hi, &sh.full[ring.slot]);
        }
      }
      ring.issued |= 1u << ring.slot;
      ring.parity = (ring.parity & ~(1u << ring.slot)) | (ring.phase << ring.slot);
    }
    ring.advance(C::NST);
    if (++kb == kblocks) {
      ++u;
      enter_tile(a);
    }
  }

  __device__ __forceinline__ void drain(const GemvArgs &a, const Shared &sh) {
    for (int i = 0; i < C::NST; ++i)
      if (ring.issued & (1u << i))
        if (!mbar_wait(&sh.full[i], (ring.parity >> i) & 1u)) raise_flag(a.flags, PW_FLAG_WAIT_TIMEOUT);
  }
};

template <int KIND>
__global__ void __launch_bounds__(kThreads, 1) k_gemv_mma(const GemvArgs a) {
  using C = Cfg<KIND>;
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte alignment for the 128B swizzle pattern of the TMA boxes
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Shared sh;
  sh.ring = smem;
  sh.x = smem + C::XOFF;
  sh.xs = reinterpret_cast<float *>(smem + C::SOFF);
  sh.full = reinterpret_cast<uint64_t *>(smem + C::BOFF);
  sh.empty = sh.full + C::NST;
  sh.abort = reinterpret_cast<volatile int *>(sh.empty + C::NST);

  const uint32_t warp = threadIdx.x / 32u, lane = threadIdx.x % 32u;
  const uint32_t gid = lane / 4u, tig = lane % 4u;
  if (threadIdx.x == 0) {
    for (int i = 0; i < C::NST; ++i) {
      mbar_init(&sh.full[i], 1);
      mbar_init(&sh.empty[i], kWarps);
    }
    *sh.abort = 0;
    mbar_fence_init();
  }
  __syncthreads();

  const uint32_t n_groups = a.n_groups_dev ? min(*a.n_groups_dev, a.n_groups) : a.n_groups;
  const uint32_t tpg = a.rows / kTileRows;
  const uint64_t total = (uint64_t)n_groups * tpg;
  const uint32_t u_begin = (uint32_t)(total * blockIdx.x / gridDim.x);
  const uint32_t u_end = (uint32_t)(total * (blockIdx.x + 1) / gridDim.x);
  const uint32_t kblocks = a.K / 128u;

  Producer<KIND> prod;
  if (warp == 0 && lane == 0) {
    prod.init(a, u_begin, u_end, tpg);
    for (int i = 0; i < C::NST - 1; ++i) prod.issue_next(a, sh);
  }
  __syncwarp();

  Ring ring;
  // ldmatrix lane -> (row within the warp's 16, 16-byte half of a 32-byte k-step)
  const uint32_t arow = warp * 16u + (lane & 7u) + ((lane >> 3) & 1u) * 8u;
  const uint32_t ahalf = lane >> 4;
  const uint32_t aswz = arow & 7u;
  const uint32_t ring_base = smem_addr(sh.ring);
  // B: lane -> (token row, which of {b0(j), b1(j), b0(j+1), b1(j+1)})
  const uint32_t x_lane = smem_addr(sh.x) + (lane & 7u) * kXStride + (lane >> 3) * 16u;
  uint32_t cur_group = 0xffffffffu;

  for (uint32_t u = u_begin; u < u_end; ++u) {
    const uint32_t gi = u / tpg;
    const GemvGroup grp = a.groups[gi];
    const uint32_t row0 = (u % tpg) * kTileRows;
    if (gi != cur_group) {
      // restage this group's activation codes and scales once every warp is
      // done with the previous group's
      if (cur_group != 0xffffffffu) named_bar_sync(1, kThreads);
      const uint32_t vec_per_row = a.K / 16u;
      for (uint32_t i = threadIdx.x; i < grp.count * vec_per_row; i += kThreads) {
        const uint32_t t = i / vec_per_row, v = i % vec_per_row;
        const uint32_t xrow = a.tok_list ? __ldg(a.tok_list + grp.tok_begin + t) : grp.tok_begin + t;
        *reinterpret_cast<uint4 *>(sh.x + t * kXStride + v * 16u) =
            __ldg(reinterpret_cast<const uint4 *>(a.x_codes + (size_t)xrow * a.K) + v);
      }
      for (uint32_t i = threadIdx.x; i < 8u * kblocks; i += kThreads) {
        const uint32_t t = i / kblocks, kbi = i % kblocks;
        float v = 0.0f;
        if (t < grp.count) {
          const uint32_t xrow = a.tok_list ? __ldg(a.tok_list + grp.tok_begin + t) : grp.tok_begin + t;
          v = __ldg(a.x_scales + (size_t)xrow * kblocks + kbi);
        }
        sh.xs[t * 32u + kbi] = v;
      }
      cur_group = gi;
      named_bar_sync(1, kThreads);
    }
    // scale row of this warp's 16 rows (one 128-row block, or one QKV segment block)
    uint32_t wsrc, wsrow;
    map_row(a.layout, row0 + warp * 16u, wsrc, wsrow);
    const float *s0 = (KIND == 3 ? grp.s1 : grp.s0) + (size_t)wsrow * a.scale_cols;
    const float *s1 = grp.s1 + (size_t)wsrow * a.scale_cols;

    float acc[C::MATS][4];
#pragma unroll
    for (int m = 0; m < C::MATS; ++m)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[m][i] = 0.0f;

#pragma unroll 1
    for (uint32_t kb = 0; kb < kblocks; ++kb) {
      if (warp == 0 && lane == 0) prod.issue_next(a, sh);
      __syncwarp();
      const bool ok = ring_wait(sh, &sh.full[ring.slot], ring.phase, a.flags);
      if (ok) {
        uint32_t b[4][2];
        ldmatrix_x4(x_lane + kb * 128u, b[0][0], b[0][1], b[1][0], b[1][1]);
        ldmatrix_x4(x_lane + kb * 128u + 64u, b[2][0], b[2][1], b[3][0], b[3][1]);
        const float xs0 = sh.xs[(tig * 2u) * 32u + kb], xs1 = sh.xs[(tig * 2u + 1u) * 32u + kb];
        const uint32_t tile = ring_base + ring.slot * C::SLOT + arow * 128u;
#pragma unroll
        for (int m = 0; m < C::MATS; ++m) {
          float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint32_t chunk = (2u * j + ahalf) ^ aswz;
            uint32_t a0, a1, a2, a3;
            ldmatrix_x4(tile + m * kBoxBytes + chunk * 16u, a0, a1, a2, a3);
            mma_e4m3(d, a0, a1, a2, a3, b[j][0], b[j][1]);
          }
          const float ws = __ldg((m == 0 ? s0 : s1) + kb);
          const float c0 = ws * xs0, c1 = ws * xs1;
          acc[m][0] = fmaf(d[0], c0, acc[m][0]);
          acc[m][1] = fmaf(d[1], c1, acc[m][1]);
          acc[m][2] = fmaf(d[2], c0, acc[m][2]);
          acc[m][3] = fmaf(d[3], c1, acc[m][3]);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&sh.empty[ring.slot]);
      ring.advance(C::NST);
    }

    // epilogue: thread holds rows (gid, gid+8) x tokens (2 tig, 2 tig + 1)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t r = row0 + warp * 16u + gid + (i >= 2 ? 8u : 0u);
      const uint32_t t = tig * 2u + (i & 1u);
      if (t < grp.count) {
        float out;
        if (C::FUSED) {
          out = staged_swiglu(acc[0][i], acc[C::MATS - 1][i]);
          if (!finite(out)) raise_flag(a.flags, PW_FLAG_NONFINITE_FUSED);
        } else {
          out = a.round_bf16 ? round_bf16(acc[0][i]) : acc[0][i];
          if (!finite(out)) raise_flag(a.flags, PW_FLAG_NONFINITE_ROUND);
        }
        a.out[(size_t)(grp.tok_begin + t) * a.out_stride + r] = out;
      }
    }
  }
  if (warp == 0 && lane == 0) prod.drain(a, sh);
}

template <int KIND>
static cudaError_t launch_one(const GemvArgs &a, int grid, cudaStream_t stream) {
  using C = Cfg<KIND>;
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(k_gemv_mma<KIND>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  k_gemv_mma<KIND><<<grid, kThreads, C::SMEM, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace mma

cudaError_t launch_gemv_mma(int kind, const GemvArgs &a, int grid, cudaStream_t stream) {
  if (a.K == 0 || a.K % 128u || a.K > (uint32_t)mma::kMaxK || a.rows % mma::kTileRows || grid <= 0)
    return cudaErrorInvalidValue;
  switch (kind) {
    case 0: return mma::launch_one<0>(a, grid, stream);
    case 2: return mma::launch_one<2>(a, grid, stream);
    case 3: return mma::launch_one<3>(a, grid, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace pw
