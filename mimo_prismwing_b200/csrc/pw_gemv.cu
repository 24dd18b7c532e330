// pw_gemv.cu -- width-specialised block-FP8 GEMV for sm_100a (widths 1..8).
//
// Computes, for every group g of <= 8 tokens sharing one e4m3 weight matrix,
//   y[t, r] = sum_kb ( sum_{c in kb} dec(W[src(r), c]) * x_t[c] ) * S[srow(r), kb] * xs_t[kb]
// (the block-scaled equation of src/wide_metal_moe.rs:404-423 and
// kernels/block_fp8_gemv.metal:935-1046), or with x unquantized and xs = 1
// (the readable projection, src/lib.rs:1272), or gate and up together with
// the staged bf16 SwiGLU in the epilogue (kernels/block_fp8_gemv.metal:1048).
//
// B200 design (HBM-bound at these widths):
//  * persistent CTAs, one per SM, 8 warps;
//  * lane 0 of warp 0 streams weight rows into a 128 KB shared-memory ring
//    with 1-D bulk copies (cp.async.bulk, mbarrier complete_tx), staying
//    NST-1 stages ahead of the consumers, so each SM keeps 96-112 KB of HBM
//    reads in flight (a separate producer warp would put 3 warps on one SM
//    sub-partition and cap every thread at 168 registers);
//  * consumer warp w owns a fixed 512-column K slice (lane = 16 columns, one
//    128-bit shared load per row); its slice of every token's decoded
//    activation lives in registers for the whole group, so each weight byte
//    is decoded once and used `count` times;
//  * per-lane partial dots are scaled per 128-block and kept per (row, token);
//    at the end of a row tile a 32-slot transposing butterfly (31 shuffles)
//    and an 8-way shared-memory sum give the outputs.
// Work is split in units of 64 output rows; CTA b takes a contiguous range of
// units so activations are reloaded only when the group changes.
#include <cstdint>
#include <cuda_runtime.h>

#include "pw_device.cuh"
#include "pw_internal.h"

namespace pw {

constexpr int kConsumerWarps = 8;
constexpr int kGemvThreads = kConsumerWarps * 32;
constexpr int kRingBytes = 128 * 1024;
constexpr uint32_t kUnitRows = 64;

template <int NSL, int KIND>
struct Cfg {
  static constexpr int RG = 8 / NSL;            // row groups of warps
  static constexpr bool FUSED = KIND == 2;
  static constexpr int MATS = FUSED ? 2 : 1;
  static constexpr int SMAX = 32 / NSL;         // stage rows at the padded K
  static constexpr int MAT_BYTES = SMAX * NSL * 512;
  static constexpr int SLOT_BYTES = MAT_BYTES * MATS;
  static constexpr int NST = kRingBytes / SLOT_BYTES;
  static constexpr int SMEM = kRingBytes + 2 * NST * 8 + 256 * 4 + 16;
};

// Item rows R (bounded so that rows-per-warp x tokens x matrices <= 32
// accumulator slots) and stage rows S for a width bucket.
__host__ __device__ constexpr int tile_rows(int nsl, bool fused, int cmax) {
  return ((fused ? 16 : 32) * (8 / nsl) / cmax) < 64 ? ((fused ? 16 : 32) * (8 / nsl) / cmax) : 64;
}
__host__ __device__ constexpr int stage_rows(int nsl, bool fused, int cmax) {
  return (32 / nsl) < tile_rows(nsl, fused, cmax) ? (32 / nsl) : tile_rows(nsl, fused, cmax);
}

template <int NSL, int KIND, int CMAX>
struct Tile {
  using C = Cfg<NSL, KIND>;
  static constexpr int R = tile_rows(NSL, C::FUSED, CMAX);   // item rows
  static constexpr int S = stage_rows(NSL, C::FUSED, CMAX);  // stage rows
  static constexpr int STAGES = R / S;
  static constexpr int RS = R / C::RG;             // rows per warp per item
  static constexpr int NSLOT = RS * CMAX * C::MATS;  // <= 32
  static_assert(R % S == 0 && S % C::RG == 0 && NSLOT <= 32, "tile shape");
};

struct Ring {
  uint32_t slot = 0;
  uint32_t phase = 0;
  uint32_t issued = 0;   // producer: slots that ever received a copy
  uint32_t parity = 0;   // producer: phase parity of each slot's last copy
  __device__ __forceinline__ void advance(int nst) {
    if (++slot == (uint32_t)nst) {
      slot = 0;
      phase ^= 1u;
    }
  }
};

struct Shared {
  uint8_t *ring;
  uint64_t *full;
  uint64_t *empty;
  float *red;
  volatile int *abort;
};

__device__ __forceinline__ bool ring_wait(const Shared &sh, uint64_t *bar, uint32_t parity, uint32_t *flags) {
  if (*sh.abort) return false;
  if (mbar_wait(bar, parity)) return true;
  *sh.abort = 1;
  raise_flag(flags, PW_FLAG_WAIT_TIMEOUT);
  return false;
}

__device__ __forceinline__ int bucket_of(uint32_t count) { return count <= 1 ? 0 : count <= 2 ? 1 : count <= 4 ? 2 : 3; }

// ------------------------------------------------------------------ producer
__device__ __forceinline__ int bucket_cmax(int b) { return 1 << b; }

// Walks the same (unit, item, stage) sequence as the consumers and issues one
// stage of bulk copies per call.  Lives in lane 0 of warp 0.
template <int NSL, int KIND>
struct Producer {
  using C = Cfg<NSL, KIND>;
  uint32_t u, u_end, upg;
  uint32_t it, st, items, stages, R, S;
  uint32_t unit_row0;
  const uint8_t *w0;
  const uint8_t *w1;
  Ring ring;

  __device__ __forceinline__ void enter_unit(const GemvArgs &a) {
    if (u >= u_end) return;
    const GemvGroup &grp = a.groups[u / upg];
    w0 = KIND == 3 ? grp.w1 : grp.w0;
    w1 = grp.w1;
    const int cmax = bucket_cmax(bucket_of(grp.count));
    R = tile_rows(NSL, C::FUSED, cmax);
    S = stage_rows(NSL, C::FUSED, cmax);
    items = kUnitRows / R;
    stages = R / S;
    unit_row0 = (u % upg) * kUnitRows;
    it = 0;
    st = 0;
  }

  __device__ __forceinline__ void init(const GemvArgs &a, uint32_t ub, uint32_t ue, uint32_t upg_) {
    u = ub;
    u_end = ue;
    upg = upg_;
    enter_unit(a);
  }

  __device__ __forceinline__ void issue_next(const GemvArgs &a, const Shared &sh) {
    if (u >= u_end) return;
    uint32_t src0, srow;
    map_row(a.layout, unit_row0 + it * R, src0, srow);
    if (ring_wait(sh, &sh.empty[ring.slot], ring.phase ^ 1u, a.flags)) {
      const uint32_t mat_bytes = S * a.K;
      uint8_t *dst = sh.ring + ring.slot * C::SLOT_BYTES;
      const size_t off = (size_t)(src0 + st * S) * a.K;
      mbar_arrive_expect_tx(&sh.full[ring.slot], mat_bytes * C::MATS);
      bulk_g2s(dst, w0 + off, mat_bytes, &sh.full[ring.slot]);
      if (C::FUSED) bulk_g2s(dst + C::MAT_BYTES, w1 + off, mat_bytes, &sh.full[ring.slot]);
      ring.issued |= 1u << ring.slot;
      ring.parity = (ring.parity & ~(1u << ring.slot)) | (ring.phase << ring.slot);
    }
    ring.advance(C::NST);
    if (++st == stages) {
      st = 0;
      if (++it == items) {
        ++u;
        enter_unit(a);
      }
    }
  }

  // Every bulk copy issued must land before the CTA exits.  Normally the
  // consumers already waited on each; after an abort they did not.
  __device__ __forceinline__ void drain(const GemvArgs &a, const Shared &sh) {
    for (int i = 0; i < C::NST; ++i) {
      if (ring.issued & (1u << i)) {
        if (!mbar_wait(&sh.full[i], (ring.parity >> i) & 1u)) raise_flag(a.flags, PW_FLAG_WAIT_TIMEOUT);
      }
    }
  }
};

// ------------------------------------------------------------------ consumer
template <int CMAX>
struct Acts {
  float xv[CMAX][16];
  float xs[CMAX];
};

template <int NSL, int KIND, int CMAX>
__device__ __forceinline__ void load_acts(const GemvArgs &a, const GemvGroup &grp, uint32_t col0, bool col_ok,
                                          Acts<CMAX> &acts) {
  const uint32_t kb = col0 / 128u;
#pragma unroll
  for (int t = 0; t < CMAX; ++t) {
    acts.xs[t] = 0.0f;
#pragma unroll
    for (int i = 0; i < 16; ++i) acts.xv[t][i] = 0.0f;
    if (t < (int)grp.count && col_ok) {
      const uint32_t slot = grp.tok_begin + t;
      const uint32_t xrow = a.tok_list ? __ldg(a.tok_list + slot) : slot;
      if (KIND == 1) {
        const float4 *p = reinterpret_cast<const float4 *>(a.x_f32 + (size_t)xrow * a.K + col0);
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          const float4 f = __ldg(p + v);
          acts.xv[t][4 * v + 0] = f.x;
          acts.xv[t][4 * v + 1] = f.y;
          acts.xv[t][4 * v + 2] = f.z;
          acts.xv[t][4 * v + 3] = f.w;
        }
        acts.xs[t] = 1.0f;
      } else {
        const uint4 q = __ldg(reinterpret_cast<const uint4 *>(a.x_codes + (size_t)xrow * a.K + col0));
        decode16(q, acts.xv[t]);
        acts.xs[t] = __ldg(a.x_scales + (size_t)xrow * (a.K / 128u) + kb);
      }
    }
  }
}

// Transposing butterfly: lane l ends with the warp sum of slot l.
__device__ __forceinline__ float butterfly32(float (&v)[32], uint32_t lane) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
    const bool upper = (lane & o) != 0;
#pragma unroll
    for (int j = 0; j < o; ++j) {
      const float send = upper ? v[j] : v[j + o];
      const float keep = upper ? v[j + o] : v[j];
      v[j] = keep + __shfl_xor_sync(0xffffffffu, send, o);
    }
  }
  return v[0];
}

template <int NSL, int KIND, int CMAX>
__device__ __forceinline__ void consume_unit(const GemvArgs &a, const Shared &sh, Ring &ring,
                                             Producer<NSL, KIND> &prod, const GemvGroup &grp,
                                             uint32_t unit_row0, const Acts<CMAX> &acts, uint32_t warp,
                                             uint32_t lane, uint32_t col0, bool col_ok) {
  using C = Cfg<NSL, KIND>;
  using T = Tile<NSL, KIND, CMAX>;
  const uint32_t g = warp / NSL;   // row group
  const uint32_t kb = col0 / 128u;
  const uint32_t count = grp.count;
#pragma unroll 1
  for (uint32_t it = 0; it < kUnitRows / T::R; ++it) {
    const uint32_t row0 = unit_row0 + it * T::R;
    uint32_t src0, srow;
    map_row(a.layout, row0, src0, srow);
    float sc[C::MATS][CMAX];
    {
      const float *s0 = KIND == 3 ? grp.s1 : grp.s0;
      const float w0s = col_ok ? __ldg(s0 + (size_t)srow * a.scale_cols + kb) : 0.0f;
      const float w1s = (C::FUSED && col_ok) ? __ldg(grp.s1 + (size_t)srow * a.scale_cols + kb) : 0.0f;
#pragma unroll
      for (int t = 0; t < CMAX; ++t) {
        sc[0][t] = w0s * acts.xs[t];
        if (C::FUSED) sc[C::MATS - 1][t] = w1s * acts.xs[t];
      }
    }
    float acc[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) acc[i] = 0.0f;

#pragma unroll
    for (int st = 0; st < T::STAGES; ++st) {
      if (warp == 0 && lane == 0) prod.issue_next(a, sh);  // keep NST-1 stages in flight
      __syncwarp();
      const bool ok = ring_wait(sh, &sh.full[ring.slot], ring.phase, a.flags);
      if (ok && col_ok) {
        const uint8_t *base = sh.ring + ring.slot * C::SLOT_BYTES;
#pragma unroll
        for (int j = 0; j < T::S / C::RG; ++j) {
          const int srow_in_stage = (int)g + C::RG * j;
          const int rs = st * (T::S / C::RG) + j;  // row slot within the item
#pragma unroll
          for (int m = 0; m < C::MATS; ++m) {
            const uint4 q = *reinterpret_cast<const uint4 *>(base + m * C::MAT_BYTES + srow_in_stage * a.K + col0);
            float wf[16];
            decode16(q, wf);
#pragma unroll
            for (int t = 0; t < CMAX; ++t) {
              if (t < (int)count) {
                float d0 = 0.0f, d1 = 0.0f;
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                  d0 = fmaf(wf[2 * i], acts.xv[t][2 * i], d0);
                  d1 = fmaf(wf[2 * i + 1], acts.xv[t][2 * i + 1], d1);
                }
                const int s = m * (T::RS * CMAX) + rs * CMAX + t;
                acc[s] = fmaf(d0 + d1, sc[m][t], acc[s]);
              }
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&sh.empty[ring.slot]);
      ring.advance(C::NST);
    }

    // reduce: lanes, then the NSL warps of this row group
    const float mine = butterfly32(acc, lane);
    sh.red[warp * 32 + lane] = mine;
    named_bar_sync(1, kConsumerWarps * 32);
    const uint32_t tid = warp * 32 + lane;
    if (!C::FUSED) {
      const uint32_t gg = tid / 32u, slot = tid % 32u;
      if (gg < (uint32_t)C::RG && slot < (uint32_t)(T::RS * CMAX)) {
        float v = 0.0f;
#pragma unroll
        for (int k = 0; k < NSL; ++k) v += sh.red[(gg * NSL + k) * 32 + slot];
        const uint32_t rsl = slot / CMAX, t = slot % CMAX;
        if (t < count) {
          const uint32_t r = row0 + rsl * C::RG + gg;
          float out = a.round_bf16 ? round_bf16(v) : v;
          if (!finite(out)) raise_flag(a.flags, PW_FLAG_NONFINITE_ROUND);
          a.out[(size_t)(grp.tok_begin + t) * a.out_stride + r] = out;
        }
      }
    } else {
      const uint32_t gg = tid / 32u, p = tid % 32u;
      if (gg < (uint32_t)C::RG && p < (uint32_t)(T::RS * CMAX)) {
        float gv = 0.0f, uv = 0.0f;
#pragma unroll
        for (int k = 0; k < NSL; ++k) {
          gv += sh.red[(gg * NSL + k) * 32 + p];
          uv += sh.red[(gg * NSL + k) * 32 + T::RS * CMAX + p];
        }
        const uint32_t rsl = p / CMAX, t = p % CMAX;
        if (t < count) {
          const uint32_t r = row0 + rsl * C::RG + gg;
          const float h = staged_swiglu(gv, uv);
          if (!finite(h)) raise_flag(a.flags, PW_FLAG_NONFINITE_FUSED);
          a.out[(size_t)(grp.tok_begin + t) * a.out_stride + r] = h;
        }
      }
    }
    named_bar_sync(1, kConsumerWarps * 32);
  }
}

template <int NSL, int KIND>
__global__ void __launch_bounds__(kGemvThreads, 1) k_gemv(const GemvArgs a) {
  using C = Cfg<NSL, KIND>;
  extern __shared__ __align__(1024) uint8_t smem[];
  Shared sh;
  sh.ring = smem;
  sh.full = reinterpret_cast<uint64_t *>(smem + kRingBytes);
  sh.empty = sh.full + C::NST;
  sh.red = reinterpret_cast<float *>(sh.empty + C::NST);
  sh.abort = reinterpret_cast<volatile int *>(sh.red + 256);

  const uint32_t warp = threadIdx.x / 32u, lane = threadIdx.x % 32u;
  if (threadIdx.x == 0) {
    for (int i = 0; i < C::NST; ++i) {
      mbar_init(&sh.full[i], 1);
      mbar_init(&sh.empty[i], kConsumerWarps);
    }
    *sh.abort = 0;
    mbar_fence_init();
  }
  __syncthreads();

  const uint32_t n_groups = a.n_groups_dev ? min(*a.n_groups_dev, a.n_groups) : a.n_groups;
  const uint32_t upg = a.rows / kUnitRows;
  const uint64_t total = (uint64_t)n_groups * upg;
  const uint32_t u_begin = (uint32_t)(total * blockIdx.x / gridDim.x);
  const uint32_t u_end = (uint32_t)(total * (blockIdx.x + 1) / gridDim.x);

  Producer<NSL, KIND> prod;
  if (warp == 0 && lane == 0) {
    prod.init(a, u_begin, u_end, upg);
    for (int i = 0; i < C::NST - 1; ++i) prod.issue_next(a, sh);
  }
  __syncwarp();

  Ring ring;
  const uint32_t col0 = (warp % NSL) * 512u + lane * 16u;
  const bool col_ok = col0 < a.K;
  // Activations are reloaded per 64-row unit: a few hundred bytes of L2
  // reads against 256-512 KB of weight rows.
  for (uint32_t u = u_begin; u < u_end; ++u) {
    const GemvGroup grp = a.groups[u / upg];
    const uint32_t row0 = (u % upg) * kUnitRows;
    switch (bucket_of(grp.count)) {
      case 0: {
        Acts<1> acts;
        load_acts<NSL, KIND, 1>(a, grp, col0, col_ok, acts);
        consume_unit<NSL, KIND, 1>(a, sh, ring, prod, grp, row0, acts, warp, lane, col0, col_ok);
        break;
      }
      case 1: {
        Acts<2> acts;
        load_acts<NSL, KIND, 2>(a, grp, col0, col_ok, acts);
        consume_unit<NSL, KIND, 2>(a, sh, ring, prod, grp, row0, acts, warp, lane, col0, col_ok);
        break;
      }
      case 2: {
        Acts<4> acts;
        load_acts<NSL, KIND, 4>(a, grp, col0, col_ok, acts);
        consume_unit<NSL, KIND, 4>(a, sh, ring, prod, grp, row0, acts, warp, lane, col0, col_ok);
        break;
      }
      default: {
        Acts<8> acts;
        load_acts<NSL, KIND, 8>(a, grp, col0, col_ok, acts);
        consume_unit<NSL, KIND, 8>(a, sh, ring, prod, grp, row0, acts, warp, lane, col0, col_ok);
        break;
      }
    }
  }
  if (warp == 0 && lane == 0) prod.drain(a, sh);
}

template <int NSL, int KIND>
static cudaError_t launch_one(const GemvArgs &a, int grid, cudaStream_t stream) {
  using C = Cfg<NSL, KIND>;
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(k_gemv<NSL, KIND>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  k_gemv<NSL, KIND><<<grid, kGemvThreads, C::SMEM, stream>>>(a);
  return cudaGetLastError();
}

template <int KIND>
static cudaError_t launch_kind(const GemvArgs &a, int grid, cudaStream_t stream) {
  const uint32_t slices = (a.K + 511u) / 512u;
  if (slices <= 1) return launch_one<1, KIND>(a, grid, stream);
  if (slices <= 2) return launch_one<2, KIND>(a, grid, stream);
  if (slices <= 4) return launch_one<4, KIND>(a, grid, stream);
  return launch_one<8, KIND>(a, grid, stream);
}

// The block-scaled kinds (0, 2, 3) run on the FP8 tensor-core GEMV
// (pw_gemv_mma.cu); this CUDA-core kernel keeps the readable projection,
// whose activation is an unquantized f32 vector.
cudaError_t launch_gemv(int kind, const GemvArgs &a, int grid, cudaStream_t stream) {
  if (a.K == 0 || a.K % 128u || a.K > 4096u || a.rows % kUnitRows || grid <= 0) return cudaErrorInvalidValue;
  switch (kind) {
    case 1: return launch_kind<1>(a, grid, stream);
    case 0:
    case 2:
    case 3: return launch_gemv_mma(kind, a, grid, stream);
    default: return cudaErrorInvalidValue;
  }
}

int gemv_max_ctas(int num_sms) { return num_sms; }

}  // namespace pw
