// pw_gemm_tc.cu -- grouped block-scaled FP8 GEMM on tcgen05 / TMEM (wide widths).
//
// For prefill-width groups (tens to hundreds of tokens per weight matrix) the
// same equation as the GEMV (src/wide_metal_moe.rs:404-423)
//   y[t, r] = sum_kb ( sum_{c in kb} dec(W[r, c]) * dec(code[t, c]) ) * S[r/128, kb] * xs[t, kb]
// runs on the 5th-generation tensor cores:
//  * A = 128 token rows x 32 columns, B = 128 weight rows x 32 columns, both
//    K-major e4m3 in shared memory (128B swizzle, written by TMA); D[t, r]
//    puts tokens on TMEM lanes and weight rows on columns.  Only the group's
//    tokens rounded up to 32 are loaded; the lanes past them hold whatever
//    the slot held before and are never read back;
//  * one elected thread issues tcgen05.mma.kind::f8f6f4 into a TMEM
//    accumulator; every 128-column block gets a fresh accumulator (the
//    checkpoint's f32 block scales are not power-of-two UE8M0 scales, so the
//    hardware block-scaled MMA cannot apply them);
//  * eight epilogue warps (two per TMEM lane quarter, each owning 64 of the
//    128 weight rows) tcgen05.ld each block's result and promote it into f32
//    registers, acc += v * (S * xs) with packed f32x2 FMAs.  A thread holds
//    one token, so its scale S * xs is one value per block (with weight rows
//    on the lanes every thread needed all 32 token scales of its chunk per
//    block, broadcast reads that took half of the shared-memory bandwidth),
//    and its outputs are one contiguous run of the output row, written with
//    16-byte stores.  Meanwhile the MMA fills the next of the rotating
//    128-column TMEM accumulator slots;
//  * a producer warp streams stages of {128 rows x 2 blocks} weights (one
//    32 KB 3-D TMA box) and {n tokens x 2 blocks} activation codes, n the
//    group's tokens rounded up to 32.  The fused kind runs all gate stages of
//    a tile, parks the finished gate sums in a spare TMEM slot (tcgen05.st),
//    runs the up stages in the same registers and stores bf16(gate) and
//    bf16(up) -- the first two roundings of the staged SwiGLU.  The rest of
//    the SwiGLU and the hidden's dynamic FP8 quantization run in
//    k_swiglu_quant at full occupancy: inside this kernel only eight warps
//    per SM would execute them, on the pipeline's critical path (measured
//    ~15k cycles per 128 x 64 tile, a third of the tile's HBM time).
// Work: persistent CTAs over (group, 128-row tile); a group is <= 128 tokens
// of one weight matrix (an expert's placements, or a chunk of a projection).
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

#include "pw_device.cuh"
#include "pw_internal.h"
#include "pw_tc.cuh"

namespace pw {
namespace tc {

// Warp roles: producer (warp 0), MMA issuer and TMEM owner (warp 1), epilogue
// (warps 2-9, two per TMEM lane quarter).
constexpr int kProducerWarp = 0;
constexpr int kMmaWarp = 1;
constexpr int kEpiWarp0 = 2;
constexpr int kEpiWarps = 8;
constexpr int kThreads = (2 + kEpiWarps) * 32;
constexpr int kTileRows = 128;
constexpr int kTN = 128;           // tokens per group
constexpr int kWBox = 32 * 1024;   // weights: 128 rows x 2 k-blocks x 128 B
constexpr int kXBox = kTN * 256;   // activations: 128 tokens x 2 k-blocks x 128 B
constexpr int kStage = kWBox + kXBox;
constexpr int kNst = 3;
constexpr int kTmemCols = 512;                 // four 128-column slots

template <int KIND>
struct Cfg {
  static constexpr bool FUSED = KIND == 2;
  static constexpr int MATS = FUSED ? 2 : 1;
  static constexpr int RING = kNst * kStage;
  static constexpr int XS = RING;                     // token scales [2 bufs][4 quarters][32 kb][32 t] f32
  static constexpr int BARS = XS + 2 * 4 * 32 * 32 * 4;  // mbarriers
  static constexpr int NACC = FUSED ? 3 : 4;          // rotating accumulator slots (fused: + gate stash)
  static constexpr int NBARS = 2 * kNst + 2 * NACC;   // full, empty, tfull[NACC], tempty[NACC]
  static constexpr int MISC = BARS + NBARS * 8;       // tmem base, abort
  static constexpr int SMEM = MISC + 16 + 1024;       // + alignment slack
  static_assert((NACC + (FUSED ? 1 : 0)) * kTN <= kTmemCols, "TMEM holds 512 columns");
  static_assert(SMEM <= 227 * 1024, "shared memory");
};

struct Shared {
  uint8_t *ring;
  float *xs;
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

// MMA columns of a group: its token count rounded up to whole 32-token chunks.
__device__ __forceinline__ uint32_t mma_cols(uint32_t count) {
  const uint32_t n = (min(count, (uint32_t)kTN) + 31u) & ~31u;
  return n ? n : 32u;
}

template <int KIND>
__global__ void __launch_bounds__(kThreads, 1) k_gemm_tc(const __grid_constant__ GemmArgs A) {
  using C = Cfg<KIND>;
  constexpr int MATS = C::MATS;
  constexpr uint32_t NACC = (uint32_t)C::NACC;
  const GemvArgs &a = A.g;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Shared sh;
  sh.ring = smem;
  sh.xs = reinterpret_cast<float *>(smem + C::XS);
  sh.full = reinterpret_cast<uint64_t *>(smem + C::BARS);
  sh.empty = sh.full + kNst;
  sh.tfull = sh.empty + kNst;
  sh.tempty = sh.tfull + NACC;
  sh.tmem_base = reinterpret_cast<uint32_t *>(smem + C::MISC);
  sh.abort = reinterpret_cast<volatile int *>(smem + C::MISC + 4);

  const uint32_t warp = threadIdx.x / 32u, lane = threadIdx.x % 32u;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kNst; ++i) {
      mbar_init(&sh.full[i], 1);
      mbar_init(&sh.empty[i], 1);  // arrived by the MMA warp's tcgen05.commit
    }
    for (uint32_t i = 0; i < NACC; ++i) {
      mbar_init(&sh.tfull[i], 1);           // tcgen05.commit after a k-block's MMAs
      mbar_init(&sh.tempty[i], kEpiWarps);  // one arrive per epilogue warp
    }
    *sh.abort = 0;
    mbar_fence_init();
  }
  if (warp == kMmaWarp) {
    // allocate the accumulator columns (whole warp), then let other CTAs allocate
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(sh.tmem_base)),
                 "r"((uint32_t)kTmemCols)
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
  // tiles are dealt round-robin: at any moment the CTAs work on neighbouring
  // tiles, i.e. a few groups, whose activation rows stay in L2 across the
  // group's row tiles (contiguous ranges per CTA spread the working set over
  // ~150 groups and the weight stream evicted it: ~30% more HBM traffic)
  const uint32_t u_begin = blockIdx.x;
  const uint32_t u_end = (uint32_t)total;
  const uint32_t u_step = gridDim.x;
  const uint32_t kblocks = a.K / 128u;
  const uint32_t kcs = (kblocks + 1u) / 2u;          // stages per matrix per tile
  const uint32_t per_tile = kcs * (uint32_t)MATS;   // stages per tile; fused: all gate, then all up
  const bool qkv = KIND == 0 && a.layout != PW_LAYOUT_PLAIN;

  if (warp == kProducerWarp) {
    // converged like the MMA warp: every lane waits, one elected lane issues
    {
      uint32_t slot = 0, phase = 0, issued = 0, parity = 0;
      for (uint32_t u = u_begin; u < u_end; u += u_step) {
        const GemvGroup &g = a.groups[u / tpg];
        const CUtensorMap *m0 = KIND == 3 ? g.tm1 : g.tm0;
        tensormap_acquire(m0);
        if (MATS == 2) tensormap_acquire(g.tm1);
        const uint32_t row0 = (u % tpg) * kTileRows;
        // QKV layouts: the tile's two 64-row halves are each one run of
        // consecutive checkpoint rows (map_row); load them as {128, 64, 1} boxes
        uint32_t src0 = 0, src1 = 0, sr_unused = 0;
        if (qkv) {
          map_row(a.layout, row0, src0, sr_unused);
          map_row(a.layout, row0 + 64u, src1, sr_unused);
        }
        const uint32_t n = mma_cols(g.count);  // token rows loaded: whole 32-token chunks
        const CUtensorMap *xm = &A.xmap[n / 32u - 1u];
        const uint32_t bytes = (uint32_t)kWBox + n * 256u;
        for (uint32_t st = 0; st < per_tile; ++st) {
          const uint32_t m = st / kcs, kc = st % kcs;
          if (bwait(sh, &sh.empty[slot], phase ^ 1u, a.flags)) {
            uint8_t *dst = sh.ring + slot * kStage;
            if (elect_one()) {
              mbar_arrive_expect_tx(&sh.full[slot], bytes);
              if (!qkv) {
                tma_load_3d(dst, m == 0 ? m0 : g.tm1, 0, (int)row0, (int)(kc * 2u), &sh.full[slot]);
              } else {
#pragma unroll
                for (uint32_t j = 0; j < 2; ++j) {
                  tma_load_3d(dst + j * (kTileRows * 128u), m0, 0, (int)src0, (int)(kc * 2u + j), &sh.full[slot]);
                  tma_load_3d(dst + j * (kTileRows * 128u) + 64u * 128u, m0, 0, (int)src1, (int)(kc * 2u + j),
                              &sh.full[slot]);
                }
              }
              tma_load_3d(dst + kWBox, xm, 0, (int)g.tok_begin, (int)(kc * 2u), &sh.full[slot]);
            }
            __syncwarp();
            issued |= 1u << slot;
            parity = (parity & ~(1u << slot)) | (phase << slot);
          }
          if (++slot == (uint32_t)kNst) {
            slot = 0;
            phase ^= 1u;
          }
        }
      }
      for (int i = 0; i < kNst; ++i)
        if (issued & (1u << i))
          if (!mbar_wait(&sh.full[i], (parity >> i) & 1u)) raise_flag(a.flags, PW_FLAG_WAIT_TIMEOUT);
    }
  } else if (warp == kMmaWarp) {
    // The whole warp walks the pipeline (every lane waits); one elected lane
    // issues each MMA and commit.  Descriptors are the ring's base descriptor
    // plus constant offsets (the start-address field counts 16-byte units).
    {
      const uint32_t ring = smem_addr(sh.ring);
      const uint64_t ring_desc = smem_desc_sw128(ring);
      uint32_t slot = 0, phase = 0, acc = 0, aphase = 0;
      uint32_t pending = 0, pend_parity = 0;  // accumulator slots with a commit in flight
      uint32_t n_next = u_begin < u_end ? mma_cols(a.groups[u_begin / tpg].count) : 32u;
      for (uint32_t u = u_begin; u < u_end; u += u_step) {
        const uint32_t n = n_next;  // token rows loaded
        if (u + u_step < u_end) n_next = mma_cols(a.groups[(u + u_step) / tpg].count);
        const uint32_t idesc = instr_desc((uint32_t)kTileRows, 128u);
        for (uint32_t st = 0; st < per_tile; ++st) {
          const uint32_t kc = st % kcs;
          const bool ok_full = bwait(sh, &sh.full[slot], phase, a.flags);
          tc_fence_after();
#pragma unroll
          for (uint32_t j = 0; j < 2; ++j) {
            if (kc * 2u + j >= kblocks) break;
            const bool ok_acc = bwait(sh, &sh.tempty[acc], aphase ^ 1u, a.flags);
            tc_fence_after();
            if (ok_full && ok_acc) {
              const uint32_t d = tmem + acc * (uint32_t)kTN;
              const uint64_t ad = ring_desc + ((slot * (uint32_t)kStage + (uint32_t)kWBox + j * (n * 128u)) >> 4);
              const uint64_t bd = ring_desc + ((slot * (uint32_t)kStage + j * (kTileRows * 128u)) >> 4);
#pragma unroll
              for (uint32_t s = 0; s < 4; ++s) mma_f8_elect(d, ad + 2u * s, bd + 2u * s, idesc, s > 0 ? 1u : 0u);
            }
            mma_commit_elect(&sh.tfull[acc]);  // this k-block's sums ready for the epilogue
            pending |= 1u << acc;
            pend_parity = (pend_parity & ~(1u << acc)) | (aphase << acc);
            if (++acc == NACC) {
              acc = 0;
              aphase ^= 1u;
            }
          }
          mma_commit_elect(&sh.empty[slot]);  // stage reusable once these MMAs are done
          if (++slot == (uint32_t)kNst) {
            slot = 0;
            phase ^= 1u;
          }
        }
      }
      // every MMA must be complete before the columns are freed
      for (uint32_t i = 0; i < NACC; ++i)
        if (pending & (1u << i))
          if (!mbar_wait(&sh.tfull[i], (pend_parity >> i) & 1u)) raise_flag(a.flags, PW_FLAG_WAIT_TIMEOUT);
    }
  } else {
    // ---------------------------------------------------------- epilogue
    const uint32_t ew = warp - kEpiWarp0;          // 0..7
    const uint32_t quarter = warp % 4u;            // TMEM lane quarter this warp may access
    const uint32_t half = ew / 4u;                 // owns weight rows 64 * half .. + 63 of the tile
    const uint32_t t_local = quarter * 32u + lane;  // token of the group owned by this thread
    const uint32_t lane_base = (quarter * 32u) << 16;
    const uint32_t col0 = half * 64u;
    const uint32_t stash = tmem + lane_base + NACC * (uint32_t)kTN + col0;  // fused: gate sums
    uint32_t acc_slot = 0, aphase = 0;
    // Token scales: the two warps of a lane quarter copy their 32 tokens'
    // scales ([kb][t], conflict-free reads by lane) for the NEXT tile with
    // cp.async while this tile runs, double-buffered; a 64-thread barrier
    // per quarter at the tile start is the only synchronisation.
    auto xs_fetch = [&](uint32_t uu, uint32_t buf) {
      const GemvGroup &gg = a.groups[uu / tpg];
      const uint32_t c = min(gg.count, (uint32_t)kTN);
      float *dst = sh.xs + (buf * 4u + quarter) * 1024u;
      for (uint32_t e = half * 32u + lane; e < 32u * kblocks; e += 64u) {
        const uint32_t kb = e / 32u, t = e % 32u, tok = quarter * 32u + t;
        if (tok < c) cp_async4(dst + kb * 32u + t, a.x_scales + (size_t)(gg.tok_begin + tok) * kblocks + kb);
      }
      cp_async_commit();
    };
    // Weight scales live in registers: lane l of every epilogue warp holds
    // the tile's two scale rows at k-block l (row 0: the first matrix, or
    // QKV rows 0-63; row 1: the up matrix, or QKV rows 64-127) and each
    // k-block's value is a shuffle.  The next tile's are fetched while this
    // one runs, so a tile boundary needs neither a load round trip nor a
    // barrier; only a group change (new token scales in shared memory) does.
    auto ws_load = [&](uint32_t uu, float &w0, float &w1) {
      const GemvGroup &gg = a.groups[uu / tpg];
      const uint32_t trow0 = (uu % tpg) * kTileRows;
      uint32_t srow = trow0 / 128u, srow1 = srow;
      if (qkv) {
        uint32_t src_unused = 0;
        map_row(a.layout, trow0, src_unused, srow);
        map_row(a.layout, trow0 + 64u, src_unused, srow1);
      }
      w0 = 0.0f;
      w1 = 0.0f;
      if (lane < kblocks) {
        w0 = __ldg((KIND == 3 ? gg.s1 : gg.s0) + (size_t)srow * a.scale_cols + lane);
        if (MATS == 2) w1 = __ldg(gg.s1 + (size_t)srow * a.scale_cols + lane);
        if (qkv) w1 = __ldg(gg.s0 + (size_t)srow1 * a.scale_cols + lane);
      }
    };
    float wn0 = 0.0f, wn1 = 0.0f;
    if (u_begin < u_end) {
      ws_load(u_begin, wn0, wn1);
      xs_fetch(u_begin, 0u);
    }
    uint32_t ti = 0;  // tile ordinal: token-scale buffer ti & 1
    for (uint32_t u = u_begin; u < u_end; u += u_step, ++ti) {
      const uint32_t gi = u / tpg;
      const GemvGroup grp = a.groups[gi];
      const uint32_t row0 = (u % tpg) * kTileRows;
      const uint32_t cnt = min(grp.count, (uint32_t)kTN);
      const bool active = quarter * 32u < cnt;  // this warp's lane quarter holds tokens
      // this tile's token scales have landed (both warps), the other buffer is free
      cp_async_wait_all();
      named_bar_sync(2u + quarter, 64u);
      const float *xsb = sh.xs + ((ti & 1u) * 4u + quarter) * 1024u;
      if (u + u_step < u_end) xs_fetch(u + u_step, (ti & 1u) ^ 1u);
      const float wc0 = wn0, wc1 = wn1;
      if (u + u_step < u_end) ws_load(u + u_step, wn0, wn1);

      float2 acc[32];  // weight rows col0 + 2i, col0 + 2i + 1
#pragma unroll 1
      for (int m = 0; m < MATS; ++m) {
        if (m == 1 && active) {
          // gate finished: park its sums in the stash slot, start the up sums
          tmem_st32(stash, *reinterpret_cast<const float2(*)[16]>(&acc[0]));
          tmem_st32(stash + 32u, *reinterpret_cast<const float2(*)[16]>(&acc[16]));
          tmem_wait_st();
        }
#pragma unroll
        for (int i = 0; i < 32; ++i) acc[i] = make_float2(0.0f, 0.0f);
        const uint32_t sel = qkv ? half : (uint32_t)m;
        const uint32_t cols = tmem + lane_base + col0;
        // Two-deep software pipeline over the k-blocks: the second 32 columns
        // of a block load while the first 32 are promoted, and the first 32
        // of the next block load while the second 32 are.  The slot goes
        // back to the MMA as soon as both halves sit in registers.  Every
        // value still gets the same single FMA per k-block, in k order.
        if (active) {
          float v0[32], v1[32];
          bool ok = bwait(sh, &sh.tfull[acc_slot], aphase, a.flags);
          tc_fence_after();
          tmem_ld32(cols + acc_slot * (uint32_t)kTN, v0);
          tmem_wait_ld(v0);
          for (uint32_t kb = 0; kb < kblocks; ++kb) {
            const float ws = __shfl_sync(0xffffffffu, sel == 0u ? wc0 : wc1, kb);
            const float c = ok ? __fmul_rn(ws, xsb[kb * 32u + lane]) : 0.0f;
            const float2 c2 = make_float2(c, c);
            tmem_ld32(cols + acc_slot * (uint32_t)kTN + 32u, v1);
#pragma unroll
            for (int i = 0; i < 16; ++i) acc[i] = __ffma2_rn(make_float2(v0[2 * i], v0[2 * i + 1]), c2, acc[i]);
            tmem_wait_ld(v1);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&sh.tempty[acc_slot]);
            if (++acc_slot == NACC) {
              acc_slot = 0;
              aphase ^= 1u;
            }
            const bool more = kb + 1u < kblocks;
            if (more) {
              ok = bwait(sh, &sh.tfull[acc_slot], aphase, a.flags);
              tc_fence_after();
              tmem_ld32(cols + acc_slot * (uint32_t)kTN, v0);
            }
#pragma unroll
            for (int i = 0; i < 16; ++i)
              acc[16 + i] = __ffma2_rn(make_float2(v1[2 * i], v1[2 * i + 1]), c2, acc[16 + i]);
            if (more) tmem_wait_ld(v0);
          }
        } else {
          // no tokens in this lane quarter: keep the slot handshake only
          for (uint32_t kb = 0; kb < kblocks; ++kb) {
            bwait(sh, &sh.tfull[acc_slot], aphase, a.flags);
            tc_fence_after();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&sh.tempty[acc_slot]);
            if (++acc_slot == NACC) {
              acc_slot = 0;
              aphase ^= 1u;
            }
          }
        }
      }

      if (!active) continue;

      // outputs: this warp's tokens, weight rows row0 + col0 .. + 63 (one
      // contiguous run of each output row).  They leave through staging rows
      // in this tile's token-scale buffer, which the quarter no longer needs
      // once both of its warps are past the last k-block (the next tile's
      // scales are in the other buffer; this one is refilled only after the
      // next tile's barrier): each thread writes a 64-byte piece of its row
      // (16-byte chunk i at position i ^ ((row >> 1) & 3), so neither the
      // row-wise writes nor the column-wise reads conflict), and each store
      // instruction then covers 8 rows x 64 B instead of 32 rows x 16 B.
      named_bar_sync(2u + quarter, 64u);
      uint8_t *stg = reinterpret_cast<uint8_t *>(sh.xs + ((ti & 1u) * 4u + quarter) * 1024u) + half * 2048u;
      const uint32_t rows_here = min(cnt - quarter * 32u, 32u);
      const size_t p0 = grp.tok_begin + quarter * 32u;  // the warp's first token row
      // dst(r): byte address of row r's piece (r < rows_here)
      auto put_rows = [&](const uint4 (&w)[4], auto &&dst) {
#pragma unroll
        for (uint32_t i = 0; i < 4; ++i)
          *reinterpret_cast<uint4 *>(stg + lane * 64u + ((i ^ ((lane >> 1) & 3u)) << 4)) = w[i];
        __syncwarp();
#pragma unroll
        for (uint32_t j = 0; j < 4; ++j) {
          const uint32_t r = 8u * j + lane / 4u, c = lane % 4u;
          const uint4 v = *reinterpret_cast<const uint4 *>(stg + r * 64u + ((c ^ ((r >> 1) & 3u)) << 4));
          if (r < rows_here) *reinterpret_cast<uint4 *>(dst(r) + c * 16u) = v;
        }
        __syncwarp();  // the staging rows are rewritten by the next piece
      };
      if (KIND != 2) {
        // bf16 rounding by the conversion instruction; an output is non-finite
        // when its f32 sum is, or when rounding carries it past the largest bf16
        const bool rb = a.round_bf16 != 0u;
        uint32_t mx = 0u;
#pragma unroll
        for (int i = 0; i < 32; ++i)
          mx = max(mx, max(__float_as_uint(acc[i].x) & 0x7fffffffu, __float_as_uint(acc[i].y) & 0x7fffffffu));
        if (mx >= (rb ? kBf16OverflowBits : 0x7f800000u) && t_local < cnt) raise_flag(a.flags, PW_FLAG_NONFINITE_ROUND);
        uint32_t pk[32];  // bf16 pairs of weight rows col0 + 2i, col0 + 2i + 1
#pragma unroll
        for (int i = 0; i < 32; ++i) pk[i] = pack_bf16x2_rn(acc[i].x, acc[i].y);
        if (a.out_bf16 || a.peer_base) {  // exact: the values are bf16-rounded
          const size_t seg = (size_t)(row0 + col0) * 2u;
#pragma unroll
          for (uint32_t h = 0; h < 2; ++h) {
            uint4 w[4];
#pragma unroll
            for (int i = 0; i < 4; ++i)
              w[i] = make_uint4(pk[16 * h + 4 * i], pk[16 * h + 4 * i + 1], pk[16 * h + 4 * i + 2],
                                pk[16 * h + 4 * i + 3]);
            if (a.peer_base) {
              put_rows(w, [&](uint32_t r) {
                const size_t p = p0 + r;
                return a.peer_base[a.row_rank[p]] + a.peer_off + (size_t)a.row_place[p] * a.out_stride * 2u + seg +
                       h * 64u;
              });
            } else {
              uint8_t *base = reinterpret_cast<uint8_t *>(a.out_bf16) + p0 * a.out_stride * 2u + seg + h * 64u;
              put_rows(w, [&](uint32_t r) { return base + (size_t)r * a.out_stride * 2u; });
            }
          }
        } else {
          float o[64];
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            o[2 * i] = rb ? __uint_as_float(pk[i] << 16) : acc[i].x;
            o[2 * i + 1] = rb ? __uint_as_float(pk[i] & 0xffff0000u) : acc[i].y;
          }
          if ((a.out_stride & 3u) == 0u && (reinterpret_cast<uintptr_t>(a.out) & 15u) == 0u) {
            uint8_t *base = reinterpret_cast<uint8_t *>(a.out + p0 * a.out_stride + row0 + col0);
#pragma unroll
            for (uint32_t h = 0; h < 4; ++h) {
              uint4 w[4];
#pragma unroll
              for (int i = 0; i < 4; ++i)
                w[i] = make_uint4(__float_as_uint(o[16 * h + 4 * i]), __float_as_uint(o[16 * h + 4 * i + 1]),
                                  __float_as_uint(o[16 * h + 4 * i + 2]), __float_as_uint(o[16 * h + 4 * i + 3]));
              put_rows(w, [&](uint32_t r) { return base + (size_t)r * a.out_stride * 4u + h * 64u; });
            }
          } else if (t_local < cnt) {
            float *dst = a.out + (size_t)(grp.tok_begin + t_local) * a.out_stride + row0 + col0;
#pragma unroll
            for (int i = 0; i < 64; ++i) dst[i] = o[i];
          }
        }
      } else {
        // bf16(gate) (from the stash) and bf16(up) (registers): the staged
        // SwiGLU's first roundings; k_swiglu_quant finishes the hidden
        const uint32_t I = a.rows;
        const size_t seg = (size_t)(row0 + col0) * 2u;
        uint8_t *gbase = reinterpret_cast<uint8_t *>(a.gate_bf16) + p0 * I * 2u + seg;
        uint8_t *ubase = reinterpret_cast<uint8_t *>(a.up_bf16) + p0 * I * 2u + seg;
#pragma unroll
        for (uint32_t h = 0; h < 2; ++h) {
          float g[32];
          tmem_ld32(stash + h * 32u, g);
          tmem_wait_ld();
          uint4 w[4];
#pragma unroll
          for (int i = 0; i < 4; ++i)
            w[i] = make_uint4(pack_bf16x2_rn(g[8 * i], g[8 * i + 1]), pack_bf16x2_rn(g[8 * i + 2], g[8 * i + 3]),
                              pack_bf16x2_rn(g[8 * i + 4], g[8 * i + 5]),
                              pack_bf16x2_rn(g[8 * i + 6], g[8 * i + 7]));
          put_rows(w, [&](uint32_t r) { return gbase + (size_t)r * I * 2u + h * 64u; });
        }
#pragma unroll
        for (uint32_t h = 0; h < 2; ++h) {
          uint4 w[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float2 *us = acc + 16 * h + 4 * i;
            w[i] = make_uint4(pack_bf16x2_rn(us[0].x, us[0].y), pack_bf16x2_rn(us[1].x, us[1].y),
                              pack_bf16x2_rn(us[2].x, us[2].y), pack_bf16x2_rn(us[3].x, us[3].y));
          }
          put_rows(w, [&](uint32_t r) { return ubase + (size_t)r * I * 2u + h * 64u; });
        }
      }
    }
  }

  // rows stored into other GPUs' memory are made visible before the release
  // kernel that follows this one publishes them
  if (KIND == 0 && a.peer_base) __threadfence_system();
  // free the accumulator columns once every role is done with them
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == kMmaWarp)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)kTmemCols)
                 : "memory");
}

template <int KIND>
static cudaError_t launch_one(const GemmArgs &a, int grid, cudaStream_t stream) {
  using C = Cfg<KIND>;
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(k_gemm_tc<KIND>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  return launch_kernel(k_gemm_tc<KIND>, dim3(grid), dim3(kThreads), C::SMEM, stream, a);
}

}  // namespace tc

int gemm_tc_tokens(int) { return tc::kTN; }

cudaError_t launch_gemm_tc(int kind, const GemmArgs &a, int grid, cudaStream_t stream) {
  const GemvArgs &g = a.g;
  if (g.K == 0 || g.K % 128u || g.K > 4096u || g.rows % tc::kTileRows || grid <= 0 ||
      (g.layout != PW_LAYOUT_PLAIN && kind != 0))
    return cudaErrorInvalidValue;
  switch (kind) {
    case 0: return tc::launch_one<0>(a, grid, stream);
    case 2: return tc::launch_one<2>(a, grid, stream);
    case 3: return tc::launch_one<3>(a, grid, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace pw
