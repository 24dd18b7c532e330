// pw_gemv_mma.cu -- block-scaled FP8 GEMV on the warp-level FP8 MMA (widths 1..8).
//
// Used where the tcgen05 GEMV (pw_gemv_tc.cu) is not: fused-QKV shard maps
// (64-row TMA boxes) and split-K launches (a lone expert's 1/8-tile units,
// whose short pipelines this kernel fills faster).
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
// one CTA per SM streaming through a shared-memory ring: every 16 KB TMA
// operation shape tops out near 4.4 TB/s, while 32 KB operations reach
// 6.5-6.9 TB/s.  So:
//  * a CTA owns a 128-row tile of one weight matrix for the whole K; warp w
//    owns rows 16w..16w+15, so no cross-warp reduction is needed;
//  * one stage = one 32 KB 3-D TMA box over the view {128 B, rows, k-block}
//    (strides {K, 128}) of the row-major matrix: 128 rows x 2 k-blocks, or
//    64 rows x 4 k-blocks when a QKV shard map splits the tile into two
//    contiguous 64-row halves.  Rows land in consecutive 128-byte lines, so
//    the 128B swizzle makes the ldmatrix reads of 8 rows bank-conflict-free;
//  * gate and up are separate stages of one ring (fused kernel);
//  * a ninth warp is the producer: one lane waits for free ring slots and
//    issues the copies, decoupled from the consumer warps' progress; the 8
//    token slots' codes and scales and each consumer warp's weight-scale row
//    sit in shared memory for the tile;
//  * when K allows (its stages divide into 8 equal leaves), the block sums are
//    added per leaf and the 8 leaf sums in a fixed pairwise tree
//    ((l0+l1)+(l2+l3))+((l4+l5)+(l6+l7)).  With few tiles (a lone expert, a
//    narrow QKV) the runtime splits each tile's K over 2, 4 or 8 CTAs, each
//    evaluating a complete subtree; the last to arrive adds the partials with
//    the same tree and runs the epilogue, so the result does not depend on
//    the split.
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

#include "pw_device.cuh"
#include "pw_internal.h"

namespace pw {
namespace mma {

constexpr int kWarps = 8;                    // consumer warps
constexpr int kThreads = (kWarps + 1) * 32;  // + one producer warp
constexpr int kConsumerThreads = kWarps * 32;
constexpr int kTileRows = 128;
constexpr int kStageBytes = 32 * 1024;   // one 3-D box: 256 lines of 128 B
constexpr int kMaxK = 4096;
constexpr int kMaxStages = 8;
constexpr uint32_t kLeaves = 8;  // K tree leaves

// Shared-memory carve-up (runtime: the activation tile depends on K).
struct Layout {
  uint32_t nst, xstride, x, xs, ws, amax, bars, total;
};

__host__ __device__ inline Layout make_layout(uint32_t K, uint32_t nst) {
  Layout l;
  l.nst = nst;
  l.xstride = K + 16u;  // padded activation row: conflict-free ldmatrix
  l.x = nst * kStageBytes;
  l.xs = l.x + 8u * l.xstride;            // x scales [8][32]
  l.ws = l.xs + 8u * 32u * 4u;            // weight scales [8 warps][2][32]
  l.amax = l.ws + 8u * 2u * 32u * 4u;     // [8 warps][8 tokens]
  l.bars = l.amax + 8u * 8u * 4u;         // full[nst], empty[nst], abort
  l.total = l.bars + 2u * nst * 8u + 16u;
  return l;
}

struct Ring {
  uint32_t slot = 0, phase = 0, issued = 0, parity = 0;
  __device__ __forceinline__ void advance(uint32_t nst) {
    if (++slot == nst) {
      slot = 0;
      phase ^= 1u;
    }
  }
};

struct Shared {
  uint8_t *ring;
  uint8_t *x;
  float *xs;
  float *ws;
  float *amax;
  uint64_t *full;
  uint64_t *empty;
  volatile int *abort;
  volatile int *last;  // this CTA finishes the tile (split-K)
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

// 3-D TMA box load at (x = 0, y = row, z = k-block) of the {128 B, rows,
// k-blocks} view.  The innermost coordinate is 0, so the 16-byte rule of the
// tiled copy holds trivially.
__device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *map, int row, int kblock, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(
          smem_addr(dst)),
      "l"(map), "r"(0), "r"(row), "r"(kblock), "r"(smem_addr(bar))
      : "memory");
}

__device__ __forceinline__ void tensormap_acquire(const CUtensorMap *map) {
  asm volatile("fence.proxy.tensormap::generic.acquire.gpu [%0], 128;" ::"l"(map) : "memory");
}

// Stage geometry of a tile: box rows BR (128, or 64 for QKV maps), k-blocks
// per box KBS = 256 / BR, halves = 128 / BR; stages run kc-major, then half,
// then matrix.
struct Geo {
  uint32_t br, kbs, halves, kcs, per_kc, splits, leaves, leaf_kc;
};

__device__ __forceinline__ Geo make_geo(const GemvArgs &a, int mats) {
  Geo g;
  g.br = a.layout == PW_LAYOUT_PLAIN ? 128u : 64u;
  g.kbs = 256u / g.br;
  g.halves = 128u / g.br;
  const uint32_t kblocks = a.K / 128u;
  g.kcs = (kblocks + g.kbs - 1u) / g.kbs;
  g.per_kc = g.halves * (uint32_t)mats;  // stages per kc
  const bool tree = g.kcs % kLeaves == 0u;
  g.splits = tree && a.splits > 1u ? a.splits : 1u;
  g.leaves = tree ? kLeaves / g.splits : 1u;    // leaves per unit
  g.leaf_kc = tree ? g.kcs / kLeaves : g.kcs;   // kc per leaf
  return g;
}

// first kc of split s of a tile
__device__ __forceinline__ uint32_t kc_first(const Geo &g, uint32_t split) { return split * g.leaves * g.leaf_kc; }

// Producer: walks (tile, stage) exactly as the consumers do and issues one
// stage per call.  Lives in lane 0 of warp 0.
template <int KIND>
struct Producer {
  static constexpr int MATS = KIND == 2 ? 2 : 1;
  uint32_t u, u_end, tpg, st, nst;
  Geo geo;
  const CUtensorMap *m0;
  const CUtensorMap *m1;
  uint32_t src0, src1;  // source rows of the tile's two 64-row halves
  Ring ring;

  uint32_t kc0, per_unit;

  __device__ __forceinline__ void enter_tile(const GemvArgs &a) {
    if (u >= u_end) return;
    const uint32_t tile = u / geo.splits;
    kc0 = kc_first(geo, u % geo.splits);
    per_unit = geo.leaves * geo.leaf_kc * geo.per_kc;
    const GemvGroup &g = a.groups[tile / tpg];
    m0 = KIND == 3 ? g.tm1 : g.tm0;
    m1 = g.tm1;
    // the maps were written through the generic proxy (host copy or bank
    // build); make those writes visible to the TMA unit before first use
    tensormap_acquire(m0);
    if (MATS == 2) tensormap_acquire(m1);
    const uint32_t row0 = (tile % tpg) * kTileRows;
    uint32_t s;
    map_row(a.layout, row0, src0, s);
    map_row(a.layout, row0 + 64u, src1, s);
    st = 0;
  }

  __device__ __forceinline__ void init(const GemvArgs &a, uint32_t ub, uint32_t ue, uint32_t tpg_, uint32_t nst_) {
    u = ub;
    u_end = ue;
    tpg = tpg_;
    nst = nst_;
    geo = make_geo(a, MATS);
    enter_tile(a);
  }

  __device__ __forceinline__ void issue_next(const GemvArgs &a, const Shared &sh) {
    if (u >= u_end) return;
    if (ring_wait(sh, &sh.empty[ring.slot], ring.phase ^ 1u, a.flags)) {
      const uint32_t m = st % MATS, h = (st / MATS) % geo.halves, kc = kc0 + st / (MATS * geo.halves);
      mbar_arrive_expect_tx(&sh.full[ring.slot], kStageBytes);
      tma_load_3d(sh.ring + ring.slot * kStageBytes, m == 0 ? m0 : m1, (int)(h ? src1 : src0), (int)(kc * geo.kbs),
                  &sh.full[ring.slot]);
      ring.issued |= 1u << ring.slot;
      ring.parity = (ring.parity & ~(1u << ring.slot)) | (ring.phase << ring.slot);
    }
    ring.advance(nst);
    if (++st == per_unit) {
      ++u;
      enter_tile(a);
    }
  }

  __device__ __forceinline__ void drain(const GemvArgs &a, const Shared &sh) {
    for (uint32_t i = 0; i < nst; ++i)
      if (ring.issued & (1u << i))
        if (!mbar_wait(&sh.full[i], (ring.parity >> i) & 1u)) raise_flag(a.flags, PW_FLAG_WAIT_TIMEOUT);
  }
};

// K-tree helpers: dst = src, and acc = left + acc (left subtree first).
template <int MATS>
__device__ __forceinline__ void tree_copy(float (&dst)[MATS][4], const float (&src)[MATS][4]) {
#pragma unroll
  for (int m = 0; m < MATS; ++m)
#pragma unroll
    for (int i = 0; i < 4; ++i) dst[m][i] = src[m][i];
}

template <int MATS>
__device__ __forceinline__ void tree_add(float (&acc)[MATS][4], const float (&left)[MATS][4]) {
#pragma unroll
  for (int m = 0; m < MATS; ++m)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[m][i] = __fadd_rn(left[m][i], acc[m][i]);
}

template <int KIND>
__global__ void __launch_bounds__(kThreads, 1) k_gemv_mma(const GemvArgs a, const uint32_t nst) {
  constexpr bool FUSED = KIND == 2;
  constexpr int MATS = FUSED ? 2 : 1;
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte alignment for the 128B swizzle pattern of the TMA boxes
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const Layout L = make_layout(a.K, nst);
  Shared sh;
  sh.ring = smem;
  sh.x = smem + L.x;
  sh.xs = reinterpret_cast<float *>(smem + L.xs);
  sh.ws = reinterpret_cast<float *>(smem + L.ws);
  sh.amax = reinterpret_cast<float *>(smem + L.amax);
  sh.full = reinterpret_cast<uint64_t *>(smem + L.bars);
  sh.empty = sh.full + nst;
  sh.abort = reinterpret_cast<volatile int *>(sh.empty + nst);
  sh.last = sh.abort + 1;

  const uint32_t warp = threadIdx.x / 32u, lane = threadIdx.x % 32u;
  const uint32_t gid = lane / 4u, tig = lane % 4u;
  if (threadIdx.x == 0) {
    for (uint32_t i = 0; i < nst; ++i) {
      mbar_init(&sh.full[i], 1);
      mbar_init(&sh.empty[i], kWarps);
    }
    *sh.abort = 0;
    mbar_fence_init();
  }
  __syncthreads();
  // Under programmatic dependent launch the previous kernel may still run.
  // With early_weights the groups and weights are already final (they come
  // from two launches back), so only the activations must wait: the producer
  // streams weights at once and the consumers wait before staging x.
  if (!a.early_weights) pdl_wait();
  pdl_launch_dependents();

  const uint32_t n_groups = a.n_groups_dev ? min(*a.n_groups_dev, a.n_groups) : a.n_groups;
  const uint32_t tpg = a.rows / kTileRows;
  const Geo geo = make_geo(a, MATS);
  const uint64_t total = (uint64_t)n_groups * tpg * geo.splits;  // units: (tile, split)
  const uint32_t u_begin = (uint32_t)(total * blockIdx.x / gridDim.x);
  const uint32_t u_end = (uint32_t)(total * (blockIdx.x + 1) / gridDim.x);
  const uint32_t kblocks = a.K / 128u;

  if (warp == kWarps) {
    // producer warp: stream every stage of this CTA's units into the ring
    if (lane == 0) {
      Producer<KIND> prod;
      prod.init(a, u_begin, u_end, tpg, nst);
      while (prod.u < u_end) prod.issue_next(a, sh);
      prod.drain(a, sh);
    }
    return;
  }

  if (a.early_weights) pdl_wait();
  Ring ring;
  // this warp's rows within its box half and the ldmatrix lane pattern:
  // lanes 0-7 rows 0-7 / bytes 0-15, 8-15 rows 8-15 / 0-15, 16-23 rows 0-7 /
  // 16-31, 24-31 rows 8-15 / 16-31 of a 32-byte k-step
  const uint32_t my_half = (warp * 16u) / geo.br;
  const uint32_t lrow = (warp * 16u - my_half * geo.br) + (lane & 7u) + ((lane >> 3) & 1u) * 8u;
  const uint32_t ahalf = lane >> 4;
  const uint32_t ring_base = smem_addr(sh.ring);
  // B: lane -> (token row, which of {b0(j), b1(j), b0(j+1), b1(j+1)})
  const uint32_t x_lane = smem_addr(sh.x) + (lane & 7u) * L.xstride + (lane >> 3) * 16u;
  float *my_ws = sh.ws + warp * 64u;
  uint32_t cur_group = 0xffffffffu;

  for (uint32_t u = u_begin; u < u_end; ++u) {
    const uint32_t tile = u / geo.splits, split = u % geo.splits;
    const uint32_t gi = tile / tpg;
    const GemvGroup grp = a.groups[gi];
    const uint32_t row0 = (tile % tpg) * kTileRows;
    const uint32_t kc0 = kc_first(geo, split);
    if (gi != cur_group) {
      // restage this group's activation codes and scales once every warp is
      // done with the previous group's
      if (cur_group != 0xffffffffu) named_bar_sync(1, kConsumerThreads);
      const uint32_t vec_per_row = a.K / 16u;
      for (uint32_t i = threadIdx.x; i < grp.count * vec_per_row; i += kConsumerThreads) {
        const uint32_t t = i / vec_per_row, v = i % vec_per_row;
        const uint32_t xrow = a.tok_list ? __ldg(a.tok_list + grp.tok_begin + t) : grp.tok_begin + t;
        *reinterpret_cast<uint4 *>(sh.x + t * L.xstride + v * 16u) =
            __ldg(reinterpret_cast<const uint4 *>(a.x_codes + (size_t)xrow * a.K) + v);
      }
      for (uint32_t i = threadIdx.x; i < 8u * kblocks; i += kConsumerThreads) {
        const uint32_t t = i / kblocks, kbi = i % kblocks;
        float v = 0.0f;
        if (t < grp.count) {
          const uint32_t xrow = a.tok_list ? __ldg(a.tok_list + grp.tok_begin + t) : grp.tok_begin + t;
          v = __ldg(a.x_scales + (size_t)xrow * kblocks + kbi);
        }
        sh.xs[t * 32u + kbi] = v;
      }
      cur_group = gi;
      named_bar_sync(1, kConsumerThreads);
    }
    {
      // this warp's weight-scale row (its 16 rows sit in one 128-row block,
      // or one QKV segment block)
      uint32_t wsrc, wsrow;
      map_row(a.layout, row0 + warp * 16u, wsrc, wsrow);
      const float *s0 = (KIND == 3 ? grp.s1 : grp.s0) + (size_t)wsrow * a.scale_cols;
      if (lane < kblocks) {
        my_ws[lane] = __ldg(s0 + lane);
        if (FUSED) my_ws[32 + lane] = __ldg(grp.s1 + (size_t)wsrow * a.scale_cols + lane);
      }
      __syncwarp();
    }

    float acc[MATS][4];                           // current leaf
    float s0[MATS][4], s1[MATS][4], s2[MATS][4];  // pending left subtrees (1, 2, 4 leaves)
    const uint32_t st_leaf = geo.leaf_kc * geo.per_kc;
#pragma unroll 1
    for (uint32_t leaf = 0; leaf < geo.leaves; ++leaf) {
#pragma unroll
    for (int m = 0; m < MATS; ++m)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[m][i] = 0.0f;
#pragma unroll 1
    for (uint32_t sl = 0; sl < st_leaf; ++sl) {
      const uint32_t st = leaf * st_leaf + sl;
      const uint32_t m = st % MATS, h = (st / MATS) % geo.halves, kc = kc0 + st / (MATS * geo.halves);
      const bool ok = ring_wait(sh, &sh.full[ring.slot], ring.phase, a.flags);
      if (ok && h == my_half) {
        const uint32_t box = ring_base + ring.slot * kStageBytes;
        for (uint32_t j = 0; j < geo.kbs; ++j) {
          const uint32_t kb = kc * geo.kbs + j;
          if (kb >= kblocks) break;
          uint32_t b[4][2];
          ldmatrix_x4(x_lane + kb * 128u, b[0][0], b[0][1], b[1][0], b[1][1]);
          ldmatrix_x4(x_lane + kb * 128u + 64u, b[2][0], b[2][1], b[3][0], b[3][1]);
          const uint32_t line = j * geo.br + lrow;
          const uint32_t lbase = box + line * 128u;
          const uint32_t swz = line & 7u;
          float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int s = 0; s < 4; ++s) {
            uint32_t a0, a1, a2, a3;
            ldmatrix_x4(lbase + (((2u * s + ahalf) ^ swz) << 4), a0, a1, a2, a3);
            mma_e4m3(d, a0, a1, a2, a3, b[s][0], b[s][1]);
          }
          const float ws = my_ws[m * 32u + kb];
          const float c0 = ws * sh.xs[(tig * 2u) * 32u + kb];
          const float c1 = ws * sh.xs[(tig * 2u + 1u) * 32u + kb];
          if (m == 0) {
            acc[0][0] = fmaf(d[0], c0, acc[0][0]);
            acc[0][1] = fmaf(d[1], c1, acc[0][1]);
            acc[0][2] = fmaf(d[2], c0, acc[0][2]);
            acc[0][3] = fmaf(d[3], c1, acc[0][3]);
          } else {
            acc[MATS - 1][0] = fmaf(d[0], c0, acc[MATS - 1][0]);
            acc[MATS - 1][1] = fmaf(d[1], c1, acc[MATS - 1][1]);
            acc[MATS - 1][2] = fmaf(d[2], c0, acc[MATS - 1][2]);
            acc[MATS - 1][3] = fmaf(d[3], c1, acc[MATS - 1][3]);
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&sh.empty[ring.slot]);
      ring.advance(nst);
    }
    // fold the leaf into the pairwise tree (left subtree + right, fixed order);
    // after the unit's last leaf acc holds its whole subtree
    if ((leaf & 1u) == 0u) {
      if (leaf + 1u < geo.leaves) tree_copy<MATS>(s0, acc);
    } else {
      tree_add<MATS>(acc, s0);
      if ((leaf & 2u) == 0u) {
        if (leaf + 1u < geo.leaves) tree_copy<MATS>(s1, acc);
      } else {
        tree_add<MATS>(acc, s1);
        if ((leaf & 4u) == 0u) {
          if (leaf + 1u < geo.leaves) tree_copy<MATS>(s2, acc);
        } else {
          tree_add<MATS>(acc, s2);
        }
      }
    }
    }

    if (geo.splits > 1u) {
      // split-K: publish this subtree; the last CTA of the tile adds all
      // subtrees in the same pairwise tree and runs the epilogue
      float *mine = a.split_ws + ((size_t)(tile * geo.splits + split) * MATS) * 1024u;
#pragma unroll
      for (int m = 0; m < MATS; ++m)
#pragma unroll
        for (int i = 0; i < 4; ++i)
          mine[m * 1024 + (warp * 16u + gid + (i >= 2 ? 8u : 0u)) * 8u + tig * 2u + (i & 1u)] = acc[m][i];
      __threadfence();
      named_bar_sync(1, kConsumerThreads);
      if (threadIdx.x == 0) *sh.last = atomicAdd(a.split_cnt + tile, 1u) == geo.splits - 1u;
      named_bar_sync(1, kConsumerThreads);
      if (!*sh.last) continue;
      __threadfence();
      // every other subtree in one round of loads, then the fixed pairwise
      // tree over the splits (each split is a whole subtree of the 8 leaves)
      float part[8][MATS][4];
#pragma unroll
      for (uint32_t sp = 0; sp < 8u; ++sp) {
        const float *src = a.split_ws + ((size_t)(tile * geo.splits + sp) * MATS) * 1024u;
#pragma unroll
        for (int m = 0; m < MATS; ++m)
#pragma unroll
          for (int i = 0; i < 4; ++i)
            part[sp][m][i] = sp == split ? acc[m][i]
                             : sp < geo.splits
                                 ? __ldcg(src + m * 1024 + (warp * 16u + gid + (i >= 2 ? 8u : 0u)) * 8u + tig * 2u +
                                          (i & 1u))
                                 : 0.0f;
      }
#pragma unroll
      for (int m = 0; m < MATS; ++m)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float p01 = __fadd_rn(part[0][m][i], part[1][m][i]);
          const float p23 = __fadd_rn(part[2][m][i], part[3][m][i]);
          const float p45 = __fadd_rn(part[4][m][i], part[5][m][i]);
          const float p67 = __fadd_rn(part[6][m][i], part[7][m][i]);
          acc[m][i] = geo.splits == 2u   ? p01
                      : geo.splits == 4u ? __fadd_rn(p01, p23)
                                         : __fadd_rn(__fadd_rn(p01, p23), __fadd_rn(p45, p67));
        }
      if (threadIdx.x == 0) a.split_cnt[tile] = 0u;  // ready for the next call
    }

    // epilogue: thread holds rows (gid, gid+8) x tokens (2 tig, 2 tig + 1)
    float outv[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t t = tig * 2u + (i & 1u);
      float out = 0.0f;
      if (t < grp.count) {
        if (FUSED) {
          out = staged_swiglu(acc[0][i], acc[MATS - 1][i]);
          if (!finite(out)) raise_flag(a.flags, PW_FLAG_NONFINITE_FUSED);
        } else {
          out = a.round_bf16 ? round_bf16(acc[0][i]) : acc[0][i];
          if (!finite(out)) raise_flag(a.flags, PW_FLAG_NONFINITE_ROUND);
        }
        if (a.out) a.out[(size_t)(grp.tok_begin + t) * a.out_stride + row0 + warp * 16u + gid + (i >= 2 ? 8u : 0u)] = out;
      }
      outv[i] = out;
    }
    if (FUSED && a.q_codes) {
      // The tile's 128 rows are exactly one 128-column group of the down
      // projection's input, so its dynamic FP8 quantization
      // (src/text_endpoint.rs:3008) is finished here: per-token absmax over the
      // 128 rows, scale = max(absmax, 1e-10) / 448, RNE e4m3 codes -- the
      // same IEEE steps as the stand-alone quantizer, so the bytes match it.
      float m0 = fmaxf(fabsf(outv[0]), fabsf(outv[2]));
      float m1 = fmaxf(fabsf(outv[1]), fabsf(outv[3]));
#pragma unroll
      for (int o = 4; o <= 16; o <<= 1) {
        m0 = fmaxf(m0, __shfl_xor_sync(0xffffffffu, m0, o));
        m1 = fmaxf(m1, __shfl_xor_sync(0xffffffffu, m1, o));
      }
      if (gid == 0) {
        sh.amax[warp * 8u + tig * 2u] = m0;
        sh.amax[warp * 8u + tig * 2u + 1u] = m1;
      }
      named_bar_sync(1, kConsumerThreads);
      float M0 = 0.0f, M1 = 0.0f;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) {
        M0 = fmaxf(M0, sh.amax[w * 8 + tig * 2u]);
        M1 = fmaxf(M1, sh.amax[w * 8 + tig * 2u + 1u]);
      }
      const Fp8GroupScale g0 = Fp8GroupScale::of(M0), g1 = Fp8GroupScale::of(M1);
      const float sc0 = g0.scale, sc1 = g1.scale;
      const uint32_t I = a.rows;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint32_t t = tig * 2u + (i & 1u);
        if (t < grp.count) {
          const float q = (i & 1) ? g1.quotient(outv[i]) : g0.quotient(outv[i]);
          const uint32_t r = row0 + warp * 16u + gid + (i >= 2 ? 8u : 0u);
          a.q_codes[(size_t)(grp.tok_begin + t) * I + r] = (uint8_t)(encode2(q, 0.0f) & 0xffu);
        }
      }
      if (warp == 0 && gid == 0) {
        const uint32_t t0 = tig * 2u, t1 = tig * 2u + 1u;
        if (t0 < grp.count) a.q_scales[(size_t)(grp.tok_begin + t0) * (I / 128u) + row0 / 128u] = sc0;
        if (t1 < grp.count) a.q_scales[(size_t)(grp.tok_begin + t1) * (I / 128u) + row0 / 128u] = sc1;
      }
      named_bar_sync(1, kConsumerThreads);  // amax is rewritten by the next tile
    }
  }
}

constexpr uint32_t kSmemLimit = 227u * 1024u;

template <int KIND>
static cudaError_t launch_one(const GemvArgs &a, int grid, cudaStream_t stream) {
  // deepest ring that fits next to this K's activation tile
  uint32_t nst = kMaxStages;
  while (nst > 2 && make_layout(a.K, nst).total + 1024u > kSmemLimit) --nst;
  const uint32_t smem = make_layout(a.K, nst).total + 1024u;
  static uint32_t configured = 0;
  if (smem > configured) {
    cudaError_t e = cudaFuncSetAttribute(k_gemv_mma<KIND>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemLimit);
    if (e != cudaSuccess) return e;
    configured = kSmemLimit;
  }
  return launch_kernel(k_gemv_mma<KIND>, dim3(grid), dim3(kThreads), smem, stream, a, nst);
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
