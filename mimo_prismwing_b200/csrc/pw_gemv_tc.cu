// pw_gemv_tc.cu -- block-scaled FP8 GEMV for decode widths (1..8 tokens) on
// tcgen05 / TMEM, for plain row-major weights (expert gate/up/down and
// unsharded projections).
//
// Equation and order (src/wide_metal_moe.rs:404-423,
// kernels/block_fp8_gemv.metal:935-1046), the same as pw_gemv_mma.cu:
//   y[t, r] = sum_kb ( sum_{c in kb} dec(W[r, c]) * dec(code[t, c]) ) * S[r/128, kb] * xs[t, kb]
// Each 128-column block dot is four K=32 e4m3 x e4m3 -> f32 MMAs; it is
// promoted as acc = fma(dot, S * xs, acc) in increasing block order within
// each of the 8 leaves of the K tree, and the leaves add in the fixed
// pairwise tree ((l0+l1)+(l2+l3))+((l4+l5)+(l6+l7)).
//
// Why tcgen05 at widths this narrow.  The weight stream has to run at HBM
// rate (~22 B/clk per SM).  With warp-level MMAs every consumer warp issued
// 8 ldmatrix + 8 mma.sync per 32 KB stage plus the promotion, and the stage
// stayed in the ring until all eight warps were done with it: consumers that
// skipped the math streamed the decode layer 15% faster (0.77 -> 0.89 of the
// measured HBM bandwidth at width 8).  Here one elected lane of an MMA warp
// issues per stage 2 k-blocks x 4 tcgen05.mma (M = 128 weight rows straight
// from the TMA box, N = 16: the 8 token slots plus 8 unused columns), and the
// stage returns to the producer as soon as those MMAs complete.  Eight
// epilogue warps promote each k-block's 128 x 8 block sums from TMEM (one
// 4-column tcgen05.ld and four FMAs per thread) out of 8 rotating 16-column
// accumulator slots, so promotion never holds a ring stage.
//
// Roles (320 threads, one CTA per SM):
//  * warps 0-7 (epilogue): warp w reads TMEM lane quarter w % 4, i.e. tile
//    rows 32 (w % 4) .. + 31 (one per lane), and owns token slots
//    4 (w / 4) .. + 3; they stage each group's activation codes (in the
//    128B-swizzled K-major layout the MMA reads) and scales, promote, and run
//    the split-K reduction, SwiGLU, hidden quantization and stores;
//  * warp 8 (producer): one elected lane streams 32 KB TMA boxes (128 rows x
//    2 k-blocks) of the CTA's units into the ring, evict-first in L2 (each
//    tile is read once).  A CTA without units instead prefetches its share
//    of the next kernel's weights (l2_next) into L2, evict-last;
//  * warp 9 (MMA): allocates 128 TMEM columns, issues the MMAs and commits.
// Units are (128-row tile, K split) pairs, a contiguous range per CTA; the
// split-K publication and the last-CTA reduction are those of pw_gemv_mma.cu
// (so results do not depend on the split).  Every wait is bounded (1 s); a
// timeout raises PW_FLAG_WAIT_TIMEOUT and the roles unwind.
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

#include "pw_device.cuh"
#include "pw_internal.h"
#include "pw_tc.cuh"

namespace pw {
namespace gtc {

using namespace tc;

constexpr int kEpiWarps = 8;
constexpr int kProducerWarp = 8;
constexpr int kMmaWarp = 9;
constexpr int kThreads = 10 * 32;
constexpr uint32_t kEpiThreads = kEpiWarps * 32;
constexpr uint32_t kTileRows = 128;
constexpr uint32_t kStageBytes = 32u * 1024u;  // one 3-D box: 128 rows x 2 k-blocks x 128 B
constexpr uint32_t kMaxK = 4096;
constexpr uint32_t kMaxStages = 6;
constexpr uint32_t kNacc = 8;       // rotating accumulator slots
constexpr uint32_t kSlotCols = 16;  // N = 16 columns per slot
constexpr uint32_t kTmemCols = 128;
constexpr uint32_t kLeaves = 8;
constexpr uint32_t kBarStage = 1;   // named barrier: x staged (epilogue warps + MMA warp)
constexpr uint32_t kBarEpi = 2;     // named barrier: epilogue warps only

struct Layout {
  uint32_t x, xs, amax, bars, misc, total;
};

// ring [nst][32 KB] | x codes [K/128][8 rows][128 B] | x scales [8][32] (the
// 1 KB the N = 16 descriptor's second 8-row group reads past the last block:
// columns 8-15, never used) | amax [4][8] | mbarriers | tmem base, abort, last
__host__ __device__ inline Layout make_layout(uint32_t K, uint32_t nst) {
  Layout l;
  l.x = nst * kStageBytes;
  l.xs = l.x + (K / 128u) * 1024u;
  l.amax = l.xs + 8u * 32u * 4u;
  l.bars = l.amax + 4u * 8u * 4u;
  l.misc = l.bars + (2u * nst + 2u * kNacc) * 8u;
  l.total = l.misc + 16u;
  return l;
}

struct Shared {
  uint8_t *ring, *x;
  float *xs, *amax;
  uint64_t *full, *empty, *tfull, *tempty;
  uint32_t *tmem_base;
  volatile int *abort;
  volatile int *last;
};

__device__ __forceinline__ bool swait(const Shared &sh, uint64_t *bar, uint32_t parity, uint32_t *flags) {
  if (*sh.abort) return false;
  if (mbar_wait(bar, parity)) return true;
  *sh.abort = 1;
  raise_flag(flags, PW_FLAG_WAIT_TIMEOUT);
  return false;
}

// 32 lanes x 4 consecutive f32 columns of the warp's lane quarter.
__device__ __forceinline__ void tmem_ld4(uint32_t taddr, float (&v)[4]) {
  uint32_t r0, r1, r2, r3;
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" : "+r"(r0), "+r"(r1), "+r"(r2), "+r"(r3)::"memory");
  v[0] = __uint_as_float(r0);
  v[1] = __uint_as_float(r1);
  v[2] = __uint_as_float(r2);
  v[3] = __uint_as_float(r3);
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Unit geometry: stages run kc-major, then matrix (gate, up); a stage is one
// kc = 2 k-blocks.  The K tree has 8 leaves when the kc count divides by 8.
struct Geo {
  uint32_t kcs, splits, leaves, leaf_kc;
};

__device__ __forceinline__ Geo make_geo(const GemvArgs &a) {
  Geo g;
  g.kcs = (a.K / 128u + 1u) / 2u;
  const bool tree = g.kcs % kLeaves == 0u;
  g.splits = tree && a.splits > 1u ? a.splits : 1u;
  g.leaves = tree ? kLeaves / g.splits : 1u;
  g.leaf_kc = tree ? g.kcs / kLeaves : g.kcs;
  return g;
}

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

// KIND 0: one projection (w0); 2: fused gate (w0) / up (w1) + staged SwiGLU +
// the hidden's dynamic FP8 quantization; 3: one projection of w1 (up).
template <int KIND>
__global__ void __launch_bounds__(kThreads, 1) k_gemv_tc(const GemvArgs a, const uint32_t nst) {
  constexpr bool FUSED = KIND == 2;
  constexpr int MATS = FUSED ? 2 : 1;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const Layout L = make_layout(a.K, nst);
  Shared sh;
  sh.ring = smem;
  sh.x = smem + L.x;
  sh.xs = reinterpret_cast<float *>(smem + L.xs);
  sh.amax = reinterpret_cast<float *>(smem + L.amax);
  sh.full = reinterpret_cast<uint64_t *>(smem + L.bars);
  sh.empty = sh.full + nst;
  sh.tfull = sh.empty + nst;
  sh.tempty = sh.tfull + kNacc;
  sh.tmem_base = reinterpret_cast<uint32_t *>(smem + L.misc);
  sh.abort = reinterpret_cast<volatile int *>(smem + L.misc + 4);
  sh.last = reinterpret_cast<volatile int *>(smem + L.misc + 8);

  const uint32_t warp = threadIdx.x / 32u, lane = threadIdx.x % 32u;
  if (threadIdx.x == 0) {
    for (uint32_t i = 0; i < nst; ++i) {
      mbar_init(&sh.full[i], 1);
      mbar_init(&sh.empty[i], 1);  // tcgen05.commit after the stage's MMAs
    }
    for (uint32_t i = 0; i < kNacc; ++i) {
      mbar_init(&sh.tfull[i], 1);           // tcgen05.commit after a k-block's MMAs
      mbar_init(&sh.tempty[i], kEpiWarps);  // one arrive per epilogue warp
    }
    *sh.abort = 0;
    mbar_fence_init();
  }
  if (warp == (uint32_t)kMmaWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(sh.tmem_base)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  // Under programmatic dependent launch the previous kernel may still run.
  // With early_weights the groups and weights are final (they come from two
  // launches back), so only the activations must wait: the producer streams
  // weights at once and the epilogue warps wait before staging x.
  if (!a.early_weights) pdl_wait();
  pdl_launch_dependents();

  const uint32_t tmem = *sh.tmem_base;
  const uint32_t n_groups = a.n_groups_dev ? min(*a.n_groups_dev, a.n_groups) : a.n_groups;
  const uint32_t tpg = a.rows / kTileRows;
  const Geo geo = make_geo(a);
  const uint64_t total = (uint64_t)n_groups * tpg * geo.splits;  // units: (tile, split)
  const uint32_t u_begin = (uint32_t)(total * blockIdx.x / gridDim.x);
  const uint32_t u_end = (uint32_t)(total * (blockIdx.x + 1) / gridDim.x);
  const uint32_t kblocks = a.K / 128u;
  const uint32_t per_unit = geo.leaves * geo.leaf_kc * (uint32_t)MATS;  // stages per unit

  if (warp == (uint32_t)kProducerWarp) {
    // ------------------------------------------------------------ producer
    // Weights are read once: evict-first, so the stream does not displace
    // what a CTA without units prefetches for the next kernel (evict-last):
    // that CTA's share of the next groups' weights, in 32 KB pieces.
    const uint64_t pol_stream = policy_evict_first();
    if (a.l2_next && u_begin == u_end && total < gridDim.x) {
      const uint64_t pol_keep = policy_evict_last();
      const uint32_t idle_rank = blockIdx.x - u_begin, n_idle = gridDim.x - (uint32_t)total;
      const uint64_t per = (uint64_t)a.l2_rows * a.l2_cols, pieces_per = (per + 32767u) / 32768u;
      for (uint64_t c = (uint64_t)idle_rank * 32u + lane; c < pieces_per * n_groups; c += (uint64_t)n_idle * 32u) {
        const uint64_t off = (c % pieces_per) * 32768u;
        prefetch_l2_hint(a.l2_next[c / pieces_per].w0 + off, (uint32_t)min((uint64_t)32768u, per - off), pol_keep);
      }
    }
    uint32_t slot = 0, phase = 0, issued = 0, parity = 0;
    for (uint32_t u = u_begin; u < u_end; ++u) {
      const uint32_t tile = u / geo.splits;
      const uint32_t kc0 = (u % geo.splits) * geo.leaves * geo.leaf_kc;
      const GemvGroup &g = a.groups[tile / tpg];
      const CUtensorMap *m0 = KIND == 3 ? g.tm1 : g.tm0;
      const CUtensorMap *m1 = g.tm1;
      // the maps were written through the generic proxy (host copy or bank
      // build); make those writes visible to the TMA unit before first use
      tensormap_acquire(m0);
      if (MATS == 2) tensormap_acquire(m1);
      const int row0 = (int)((tile % tpg) * kTileRows);
      for (uint32_t st = 0; st < per_unit; ++st) {
        const uint32_t m = st % (uint32_t)MATS, kc = kc0 + st / (uint32_t)MATS;
        if (swait(sh, &sh.empty[slot], phase ^ 1u, a.flags)) {
          if (elect_one()) {
            mbar_arrive_expect_tx(&sh.full[slot], kStageBytes);
            tma_load_3d_hint(sh.ring + slot * kStageBytes, m == 0u ? m0 : m1, 0, row0, (int)(kc * 2u), &sh.full[slot],
                             pol_stream);
          }
          __syncwarp();
          issued |= 1u << slot;
          parity = (parity & ~(1u << slot)) | (phase << slot);
        }
        if (++slot == nst) {
          slot = 0;
          phase ^= 1u;
        }
      }
    }
    // every copy in flight lands before the CTA can exit
    for (uint32_t i = 0; i < nst; ++i)
      if (issued & (1u << i))
        if (!mbar_wait(&sh.full[i], (parity >> i) & 1u)) raise_flag(a.flags, PW_FLAG_WAIT_TIMEOUT);
  } else if (warp == (uint32_t)kMmaWarp) {
    // ----------------------------------------------------------------- MMA
    const uint32_t idesc = instr_desc(kSlotCols, kTileRows);  // M = 128 rows, N = 16 token columns
    const uint64_t ring_desc = smem_desc_sw128(smem_addr(sh.ring));
    const uint64_t x_desc = smem_desc_sw128(smem_addr(sh.x));
    uint32_t slot = 0, phase = 0, acc = 0, aphase = 0;
    uint32_t pending = 0, pend_parity = 0;  // accumulator slots with a commit in flight
    uint32_t cur_group = 0xffffffffu;
    for (uint32_t u = u_begin; u < u_end; ++u) {
      const uint32_t tile = u / geo.splits;
      const uint32_t gi = tile / tpg;
      const uint32_t kc0 = (u % geo.splits) * geo.leaves * geo.leaf_kc;
      if (gi != cur_group) {
        named_bar_sync(kBarStage, kEpiThreads + 32u);  // this group's x is staged
        cur_group = gi;
      }
      for (uint32_t st = 0; st < per_unit; ++st) {
        const uint32_t kc = kc0 + st / (uint32_t)MATS;
        const bool ok_full = swait(sh, &sh.full[slot], phase, a.flags);
        tc_fence_after();
#pragma unroll
        for (uint32_t j = 0; j < 2; ++j) {
          const uint32_t kb = kc * 2u + j;
          if (kb >= kblocks) break;
          const bool ok_acc = swait(sh, &sh.tempty[acc], aphase ^ 1u, a.flags);
          tc_fence_after();
          if (ok_full && ok_acc) {
            const uint32_t d = tmem + acc * kSlotCols;
            const uint64_t ad = ring_desc + ((slot * kStageBytes + j * (kTileRows * 128u)) >> 4);
            const uint64_t bd = x_desc + ((kb * 1024u) >> 4);
#pragma unroll
            for (uint32_t s = 0; s < 4; ++s) mma_f8_elect(d, ad + 2u * s, bd + 2u * s, idesc, s > 0 ? 1u : 0u);
          }
          mma_commit_elect(&sh.tfull[acc]);  // this k-block's sums ready for the epilogue
          pending |= 1u << acc;
          pend_parity = (pend_parity & ~(1u << acc)) | (aphase << acc);
          if (++acc == kNacc) {
            acc = 0;
            aphase ^= 1u;
          }
        }
        mma_commit_elect(&sh.empty[slot]);  // stage reusable once these MMAs are done
        if (++slot == nst) {
          slot = 0;
          phase ^= 1u;
        }
      }
    }
    // every MMA is complete before the columns are freed
    for (uint32_t i = 0; i < kNacc; ++i)
      if (pending & (1u << i))
        if (!mbar_wait(&sh.tfull[i], (pend_parity >> i) & 1u)) raise_flag(a.flags, PW_FLAG_WAIT_TIMEOUT);
  } else {
    // ------------------------------------------------------------ epilogue
    if (a.early_weights) pdl_wait();
    const uint32_t quarter = warp % 4u, th = warp / 4u;
    const uint32_t r_loc = quarter * 32u + lane;  // this thread's row of the tile
    const uint32_t t0 = th * 4u;                  // its token slots t0 .. t0 + 3
    const uint32_t tcol = tmem + ((quarter * 32u) << 16) + t0;
    uint32_t acc_slot = 0, aphase = 0;
    uint32_t cur_group = 0xffffffffu;
    for (uint32_t u = u_begin; u < u_end; ++u) {
      const uint32_t tile = u / geo.splits, split = u % geo.splits;
      const uint32_t gi = tile / tpg;
      const GemvGroup grp = a.groups[gi];
      const uint32_t row0 = (tile % tpg) * kTileRows;
      const uint32_t kc0 = split * geo.leaves * geo.leaf_kc;
      if (gi != cur_group) {
        // Stage the group's activation codes in the 128B-swizzled K-major
        // layout (block kb: 8 rows of 128 B at x + 1024 kb, 16-byte chunk c of
        // row t at position c ^ t) and its scales.  The previous group's MMAs
        // are complete: every one of its k-blocks was waited on (tfull).
        if (cur_group != 0xffffffffu) named_bar_sync(kBarEpi, kEpiThreads);
        // all of a thread's loads (at most 8: 8 rows x K / 16 vectors over
        // 256 threads) are in flight before its first store
        const uint32_t vec_per_row = a.K / 16u;
        constexpr uint32_t kXVec = 8u * (kMaxK / 16u) / kEpiThreads;
        uint4 q[kXVec];
#pragma unroll
        for (uint32_t k = 0; k < kXVec; ++k) {
          const uint32_t i = threadIdx.x + k * kEpiThreads, t = i / vec_per_row, v = i % vec_per_row;
          q[k] = make_uint4(0u, 0u, 0u, 0u);
          if (i < 8u * vec_per_row && t < grp.count) {
            const uint32_t xrow = a.tok_list ? __ldg(a.tok_list + grp.tok_begin + t) : grp.tok_begin + t;
            q[k] = __ldg(reinterpret_cast<const uint4 *>(a.x_codes + (size_t)xrow * a.K) + v);
          }
        }
#pragma unroll
        for (uint32_t k = 0; k < kXVec; ++k) {
          const uint32_t i = threadIdx.x + k * kEpiThreads, t = i / vec_per_row, v = i % vec_per_row;
          const uint32_t kb = v / 8u, c = v % 8u;
          if (i < 8u * vec_per_row) *reinterpret_cast<uint4 *>(sh.x + kb * 1024u + t * 128u + ((c ^ t) << 4)) = q[k];
        }
        for (uint32_t i = threadIdx.x; i < 8u * 32u; i += kEpiThreads) {
          const uint32_t t = i / 32u, kbi = i % 32u;
          float v = 0.0f;
          if (t < grp.count && kbi < kblocks) {
            const uint32_t xrow = a.tok_list ? __ldg(a.tok_list + grp.tok_begin + t) : grp.tok_begin + t;
            v = __ldg(a.x_scales + (size_t)xrow * kblocks + kbi);
          }
          sh.xs[t * 32u + kbi] = v;
        }
        fence_proxy_async_smem();  // generic writes of x -> the MMA's async-proxy reads
        named_bar_sync(kBarStage, kEpiThreads + 32u);
        cur_group = gi;
      }
      // the tile's weight-scale row: lane l holds column l of each matrix
      const uint32_t srow = row0 / 128u;
      float w0 = 0.0f, w1 = 0.0f;
      if (lane < kblocks) {
        w0 = __ldg((KIND == 3 ? grp.s1 : grp.s0) + (size_t)srow * a.scale_cols + lane);
        if (MATS == 2) w1 = __ldg(grp.s1 + (size_t)srow * a.scale_cols + lane);
      }

      float acc[MATS][4];
      float s0[MATS][4], s1[MATS][4], s2[MATS][4];  // pending left subtrees (1, 2, 4 leaves)
      const uint32_t st_leaf = geo.leaf_kc * (uint32_t)MATS;
#pragma unroll 1
      for (uint32_t leaf = 0; leaf < geo.leaves; ++leaf) {
#pragma unroll
        for (int m = 0; m < MATS; ++m)
#pragma unroll
          for (int i = 0; i < 4; ++i) acc[m][i] = 0.0f;
#pragma unroll 1
        for (uint32_t sl = 0; sl < st_leaf; ++sl) {
          const uint32_t st = leaf * st_leaf + sl;
          const uint32_t m = st % (uint32_t)MATS, kc = kc0 + st / (uint32_t)MATS;
#pragma unroll
          for (uint32_t j = 0; j < 2; ++j) {
            const uint32_t kb = kc * 2u + j;
            if (kb >= kblocks) break;
            const float ws = __shfl_sync(0xffffffffu, m == 0u ? w0 : w1, kb);
            const bool ok = swait(sh, &sh.tfull[acc_slot], aphase, a.flags);
            tc_fence_after();
            float v[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            if (ok) tmem_ld4(tcol + acc_slot * kSlotCols, v);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&sh.tempty[acc_slot]);
            if (++acc_slot == kNacc) {
              acc_slot = 0;
              aphase ^= 1u;
            }
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const float c = __fmul_rn(ws, sh.xs[(t0 + (uint32_t)i) * 32u + kb]);
              if (m == 0u)
                acc[0][i] = __fmaf_rn(v[i], c, acc[0][i]);
              else
                acc[MATS - 1][i] = __fmaf_rn(v[i], c, acc[MATS - 1][i]);
            }
          }
        }
        // fold the leaf into the pairwise tree (left subtree + right, fixed
        // order); after the unit's last leaf acc holds its whole subtree
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
        // split-K: publish this subtree ([matrix][row][token slot]); the last
        // CTA of the tile adds all subtrees in the same pairwise tree
        float *mine = a.split_ws + ((size_t)(tile * geo.splits + split) * MATS) * 1024u;
#pragma unroll
        for (int m = 0; m < MATS; ++m)
#pragma unroll
          for (int i = 0; i < 4; ++i) mine[m * 1024 + r_loc * 8u + t0 + (uint32_t)i] = acc[m][i];
        __threadfence();
        named_bar_sync(kBarEpi, kEpiThreads);
        if (threadIdx.x == 0) *sh.last = atomicAdd(a.split_cnt + tile, 1u) == geo.splits - 1u;
        named_bar_sync(kBarEpi, kEpiThreads);
        if (!*sh.last) continue;
        __threadfence();
        float part[8][MATS][4];
#pragma unroll
        for (uint32_t sp = 0; sp < 8u; ++sp) {
          const float *src = a.split_ws + ((size_t)(tile * geo.splits + sp) * MATS) * 1024u;
#pragma unroll
          for (int m = 0; m < MATS; ++m)
#pragma unroll
            for (int i = 0; i < 4; ++i)
              part[sp][m][i] = sp == split         ? acc[m][i]
                               : sp < geo.splits ? __ldcg(src + m * 1024 + r_loc * 8u + t0 + (uint32_t)i)
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

      // epilogue: thread holds row r_loc x token slots t0 .. t0 + 3
      float outv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint32_t t = t0 + (uint32_t)i;
        float out = 0.0f;
        if (t < grp.count) {
          if (FUSED) {
            out = staged_swiglu(acc[0][i], acc[MATS - 1][i]);
            if (!finite(out)) raise_flag(a.flags, PW_FLAG_NONFINITE_FUSED);
          } else {
            out = a.round_bf16 ? round_bf16(acc[0][i]) : acc[0][i];
            if (!finite(out)) raise_flag(a.flags, PW_FLAG_NONFINITE_ROUND);
          }
          if (a.out) a.out[(size_t)(grp.tok_begin + t) * a.out_stride + row0 + r_loc] = out;
        }
        outv[i] = out;
      }
      if (FUSED && a.q_codes) {
        // The tile's 128 rows are exactly one 128-column group of the down
        // projection's input, so its dynamic FP8 quantization
        // (src/text_endpoint.rs:3008) is finished here: per-token absmax over
        // the 128 rows, scale = max(absmax, 1e-10) / 448, RNE e4m3 codes --
        // the same IEEE steps as the stand-alone quantizer, so the bytes
        // match it.
        float mx[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          mx[i] = fabsf(outv[i]);
#pragma unroll
          for (int o = 1; o <= 16; o <<= 1) mx[i] = fmaxf(mx[i], __shfl_xor_sync(0xffffffffu, mx[i], o));
        }
        if (lane == 0)
#pragma unroll
          for (int i = 0; i < 4; ++i) sh.amax[quarter * 8u + t0 + (uint32_t)i] = mx[i];
        named_bar_sync(kBarEpi, kEpiThreads);
        const uint32_t I = a.rows;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const uint32_t t = t0 + (uint32_t)i;
          const float M = fmaxf(fmaxf(sh.amax[t], sh.amax[8u + t]), fmaxf(sh.amax[16u + t], sh.amax[24u + t]));
          const Fp8GroupScale g = Fp8GroupScale::of(M);
          if (t < grp.count) {
            const float q = g.quotient(outv[i]);
            a.q_codes[(size_t)(grp.tok_begin + t) * I + row0 + r_loc] = (uint8_t)(encode2(q, 0.0f) & 0xffu);
            if (quarter == 0u && lane == 0u) a.q_scales[(size_t)(grp.tok_begin + t) * (I / 128u) + row0 / 128u] = g.scale;
          }
        }
        named_bar_sync(kBarEpi, kEpiThreads);  // amax is rewritten by the next tile
      }
    }
  }

  // free the accumulator columns once every role is done with them
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == (uint32_t)kMmaWarp)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
}

constexpr uint32_t kSmemLimit = 227u * 1024u;

template <int KIND>
static cudaError_t launch_one(const GemvArgs &a, int grid, cudaStream_t stream) {
  // deepest ring that fits next to this K's activation tile
  uint32_t nst = kMaxStages;
  while (nst > 2 && make_layout(a.K, nst).total + 1024u > kSmemLimit) --nst;
  const uint32_t smem = make_layout(a.K, nst).total + 1024u;
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(k_gemv_tc<KIND>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemLimit);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  return launch_kernel(k_gemv_tc<KIND>, dim3(grid), dim3(kThreads), smem, stream, a, nst);
}

}  // namespace gtc

cudaError_t launch_gemv_tc(int kind, const GemvArgs &a, int grid, cudaStream_t stream) {
  if (a.K == 0 || a.K % 128u || a.K > gtc::kMaxK || a.rows % gtc::kTileRows || grid <= 0 ||
      a.layout != PW_LAYOUT_PLAIN)
    return cudaErrorInvalidValue;
  switch (kind) {
    case 0: return gtc::launch_one<0>(a, grid, stream);
    case 2: return gtc::launch_one<2>(a, grid, stream);
    case 3: return gtc::launch_one<3>(a, grid, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace pw
