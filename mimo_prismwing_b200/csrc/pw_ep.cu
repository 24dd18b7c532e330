// pw_ep.cu -- expert-parallel dispatch and combine over peer memory.
//
// Every rank owns a window (one cudaMalloc, mapped into every other rank's
// process through CUDA IPC; layout in EpWindow).  Per layer, with an epoch
// number that all ranks advance together:
//   k_ep_dispatch  first publishes flag_ready[r] = epoch in every window and
//                  waits (bounded) until every peer's flag_ready has reached
//                  this epoch in its own window: a peer that has left never
//                  publishes it, so no row is ever stored into a departed
//                  rank's window, and the wait times out instead; then it
//                  stores this rank's per-expert counts and its FP8 rows
//                  (codes + per-128 scales, in its expert-major placement
//                  order) straight into each expert owner's window -- source
//                  slot r, so no rank needs the others' counts to know where
//                  to write -- then, once every CTA's stores are visible
//                  system-wide, releases flag_data[r] = epoch in each window;
//   k_ep_plan      (owner) waits for every source's flag, then builds on the
//                  device what the host planner builds for the NCCL path:
//                  the rows in expert order, each row's source rank and
//                  placement, and the GEMV/GEMM groups;
//   k_ep_gather    lays the received rows out in expert order for the GEMM;
//   k_ep_return    stores each bf16-rounded down row as bf16 straight into
//                  its source's window at the source's placement index, then
//                  releases flag_ret[owner] = epoch in every source's window;
//   k_ep_wait      waits for every owner's return flag before the combine.
// Stores are plain 16-byte peer stores over NVLink; flags use release /
// acquire at system scope.  Every wait is bounded by the caller's deadline
// and raises PW_FLAG_WAIT_TIMEOUT when it runs out.  One window per rank is
// enough: a rank starts layer l + 1 only after every owner returned its rows
// of layer l, and an owner returns rows only after it has read that layer's
// input.
#include <cstdint>
#include <cuda_runtime.h>

#include "pw_device.cuh"
#include "pw_internal.h"

namespace pw {

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(uint32_t *p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

template <class T>
__device__ __forceinline__ T *win_at(const EpArgs &e, uint32_t rank, uint64_t off) {
  return reinterpret_cast<T *>(e.peers[rank] + off);
}

// Bounded wait until flags[0..n) all equal epoch; false on timeout.
__device__ bool wait_flags(const uint32_t *flags, uint32_t n, uint32_t epoch, uint64_t deadline_ns) {
  const uint64_t t0 = global_timer_ns();
  for (uint32_t i = 0; i < n; ++i) {
    while (ld_acquire_sys(flags + i) != epoch) {
      if (global_timer_ns() - t0 > deadline_ns) return false;
      __nanosleep(200);
    }
  }
  return true;
}

// ------------------------------------------------------------------ dispatch
__global__ void __launch_bounds__(256) k_ep_dispatch(const EpArgs e, const uint32_t *__restrict__ offsets,
                                                     const uint8_t *__restrict__ codes, const float *__restrict__ scales,
                                                     uint32_t P, uint32_t *ctr) {
  pdl_wait();
  const EpWindow &w = e.w;
  const uint32_t G = w.G, L = w.L, r = e.rank;
  __shared__ uint32_t gbeg[9];
  __shared__ int last, ready;
  // readiness: this rank has finished the previous layer (its receive slots
  // are free); every peer must say the same before any row goes to it.
  // Every CTA publishes (the same value), so no CTA's wait depends on another
  // CTA of this grid being resident.
  if (threadIdx.x < G) st_release_sys(win_at<uint32_t>(e, threadIdx.x, w.flag_ready) + r, e.epoch);
  __syncthreads();
  if (threadIdx.x == 0) {
    ready = wait_flags(win_at<uint32_t>(e, r, w.flag_ready), G, e.epoch, e.deadline_ns) ? 1 : 0;
    if (!ready) raise_flag(e.flags, PW_FLAG_WAIT_TIMEOUT);
  }
  if (threadIdx.x <= G) gbeg[threadIdx.x] = offsets[threadIdx.x * L];
  __syncthreads();
  const bool go = ready != 0;
  // the mailbox: this rank's counts for each owner's experts and the
  // placement index of its first row for that owner
  if (blockIdx.x == 0 && go) {
    for (uint32_t i = threadIdx.x; i < G * L + G; i += blockDim.x) {
      if (i < G * L) {
        const uint32_t g = i / L, le = i % L, ex = g * L + le;
        win_at<uint32_t>(e, g, w.mail_cnt)[r * L + le] = offsets[ex + 1] - offsets[ex];
      } else {
        const uint32_t g = i - G * L;
        win_at<uint32_t>(e, g, w.mail_base)[r] = gbeg[g];
      }
    }
  }
  // the rows: warp per row, 16-byte stores into the owner's slot r
  const uint32_t warp = (blockIdx.x * blockDim.x + threadIdx.x) / 32u, lane = threadIdx.x % 32u;
  const uint32_t nwarps = gridDim.x * blockDim.x / 32u;
  const uint32_t vc = w.H / 16u, vs = w.H / 128u / 4u;  // uint4 per row: codes, scales
  for (uint32_t i = warp; go && i < P; i += nwarps) {
    uint32_t g = 0;
    while (g + 1u < G && gbeg[g + 1] <= i) ++g;
    const uint64_t dst_row = (uint64_t)r * w.slot_rows + (i - gbeg[g]);
    const uint4 *src = reinterpret_cast<const uint4 *>(codes + (size_t)i * w.H);
    uint4 *dst = win_at<uint4>(e, g, w.recv_codes + dst_row * w.H);
    for (uint32_t v = lane; v < vc; v += 32u) dst[v] = __ldg(src + v);
    const uint4 *ss = reinterpret_cast<const uint4 *>(scales + (size_t)i * (w.H / 128u));
    uint4 *ds = win_at<uint4>(e, g, w.recv_scales + dst_row * (w.H / 128u) * 4u);
    for (uint32_t v = lane; v < vs; v += 32u) ds[v] = __ldg(ss + v);
  }
  // release: the last CTA to finish raises flag_data[r] in every window
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) last = atomicAdd(ctr, 1u) == gridDim.x - 1u;
  __syncthreads();
  if (last) {
    __threadfence_system();
    if (go && threadIdx.x < G) st_release_sys(win_at<uint32_t>(e, threadIdx.x, w.flag_data) + r, e.epoch);
    if (threadIdx.x == 0) *ctr = 0u;
  }
  pdl_launch_dependents();
}

// ---------------------------------------------------------------------- plan
// One CTA (the plan is a few hundred words; what takes time is the wait for
// the slowest source's rows).  Outputs (expert order j): perm[j] = received row (slot s, row),
// src_rank[j], src_place[j]; groups over each local expert's rows in chunks
// of `chunk`; *n_groups; *p_recv = rows received and p_recv[1] = local
// experts with at least one row.  Rows beyond `cap` are an error.
__global__ void __launch_bounds__(1024) k_ep_plan(const EpArgs e, BankTable bank, uint32_t chunk, uint32_t cap,
                                                  uint32_t *__restrict__ perm, uint32_t *__restrict__ src_rank,
                                                  uint32_t *__restrict__ src_place, GemvGroup *__restrict__ gu,
                                                  GemvGroup *__restrict__ dn, uint32_t *n_groups, uint32_t *p_recv) {
  pdl_wait();
  const EpWindow &w = e.w;
  const uint32_t G = w.G, L = w.L, r = e.rank;
  extern __shared__ uint32_t sm[];
  uint32_t *cnt = sm;                  // [G][L]
  uint32_t *pre = cnt + G * L;         // [G][L]: a source's rows before expert le
  uint32_t *base = pre + G * L;        // [G]
  uint32_t *beg = base + G;            // [L + 1] expert-order begin
  uint32_t *gbeg = beg + L + 1;        // [L + 1] group begin
  __shared__ int ok;
  if (threadIdx.x == 0) ok = 1;
  __syncthreads();
  if (threadIdx.x == 0)
    if (!wait_flags(win_at<uint32_t>(e, r, w.flag_data), G, e.epoch, e.deadline_ns)) {
      ok = 0;
      raise_flag(e.flags, PW_FLAG_WAIT_TIMEOUT);
    }
  __syncthreads();
  if (!ok) {
    if (threadIdx.x == 0) {
      *n_groups = 0u;
      *p_recv = 0u;
      p_recv[1] = 0u;
    }
    return;
  }
  const uint32_t *mc = win_at<uint32_t>(e, r, w.mail_cnt), *mb = win_at<uint32_t>(e, r, w.mail_base);
  for (uint32_t i = threadIdx.x; i < G * L; i += blockDim.x) cnt[i] = __ldcv(mc + i);
  for (uint32_t i = threadIdx.x; i < G; i += blockDim.x) base[i] = __ldcv(mb + i);
  __syncthreads();
  for (uint32_t s = threadIdx.x; s < G; s += blockDim.x) {
    uint32_t run = 0;
    for (uint32_t le = 0; le < L; ++le) {
      pre[s * L + le] = run;
      run += cnt[s * L + le];
    }
  }
  if (threadIdx.x == 0) {
    uint32_t run = 0, grun = 0;
    for (uint32_t le = 0; le < L; ++le) {
      beg[le] = run;
      gbeg[le] = grun;
      uint32_t t = 0;
      for (uint32_t s = 0; s < G; ++s) t += cnt[s * L + le];
      run += t;
      grun += (t + chunk - 1u) / chunk;
    }
    beg[L] = run;
    gbeg[L] = grun;
    uint32_t used = 0;
    for (uint32_t le = 0; le < L; ++le) used += beg[le + 1] > beg[le] ? 1u : 0u;
    p_recv[1] = used;
    if (run > cap) {
      ok = 0;
      raise_flag(e.flags, PW_FLAG_BAD_EXPERT_COUNT);
    }
  }
  __syncthreads();
  if (!ok) {
    if (threadIdx.x == 0) {
      *n_groups = 0u;
      *p_recv = 0u;
      p_recv[1] = 0u;
    }
    return;
  }
  // a warp per local expert: its rows (source rank, then the source's
  // order) and its groups, lanes striding over them
  const uint32_t lane = threadIdx.x % 32u, nwarps = blockDim.x / 32u;
  for (uint32_t le = threadIdx.x / 32u; le < L; le += nwarps) {
    uint32_t j0 = beg[le];
    for (uint32_t s = 0; s < G; ++s) {
      const uint32_t c = cnt[s * L + le], p0 = pre[s * L + le];
      for (uint32_t k = lane; k < c; k += 32u) {
        perm[j0 + k] = s * w.slot_rows + p0 + k;
        src_rank[j0 + k] = s;
        src_place[j0 + k] = base[s] + p0 + k;
      }
      j0 += c;
    }
    const uint32_t t = beg[le + 1] - beg[le];
    for (uint32_t c = lane; c * chunk < t; c += 32u) {
      GemvGroup g;
      g.tok_begin = beg[le] + c * chunk;
      g.count = min(chunk, t - c * chunk);
      g.expert = r * L + le;
      g.pad = 0;
      g.w0 = bank.gate_w[le];
      g.s0 = bank.gate_s[le];
      g.w1 = bank.up_w[le];
      g.s1 = bank.up_s[le];
      g.tm0 = bank.gate_tm + le;
      g.tm1 = bank.up_tm + le;
      gu[gbeg[le] + c] = g;
      GemvGroup d = g;
      d.w0 = bank.down_w[le];
      d.s0 = bank.down_s[le];
      d.w1 = nullptr;
      d.s1 = nullptr;
      d.tm0 = bank.down_tm + le;
      d.tm1 = nullptr;
      dn[gbeg[le] + c] = d;
    }
  }
  if (threadIdx.x == 0) {
    *n_groups = gbeg[L];
    *p_recv = beg[L];
  }
  __syncthreads();
  pdl_launch_dependents();
}

// ---------------------------------------------------------------- gather
// out row j = received row perm[j] (codes and scales), j < p_recv.
__global__ void __launch_bounds__(256) k_ep_gather(const EpArgs e, const uint32_t *__restrict__ perm,
                                                   const uint32_t *p_recv, uint8_t *__restrict__ out_codes,
                                                   float *__restrict__ out_scales) {
  pdl_wait();
  const EpWindow &w = e.w;
  const uint32_t n = *p_recv;
  const uint8_t *codes = win_at<uint8_t>(e, e.rank, w.recv_codes);
  const float *scales = win_at<float>(e, e.rank, w.recv_scales);
  const uint32_t warp = (blockIdx.x * blockDim.x + threadIdx.x) / 32u, lane = threadIdx.x % 32u;
  const uint32_t nwarps = gridDim.x * blockDim.x / 32u;
  const uint32_t vc = w.H / 16u, vs = w.H / 128u / 4u;
  for (uint32_t j = warp; j < n; j += nwarps) {
    const uint32_t src = perm[j];
    const uint4 *sc = reinterpret_cast<const uint4 *>(codes + (size_t)src * w.H);
    uint4 *dc = reinterpret_cast<uint4 *>(out_codes + (size_t)j * w.H);
    for (uint32_t v = lane; v < vc; v += 32u) dc[v] = __ldcv(sc + v);
    const uint4 *ss = reinterpret_cast<const uint4 *>(scales + (size_t)src * (w.H / 128u));
    uint4 *ds = reinterpret_cast<uint4 *>(out_scales + (size_t)j * (w.H / 128u));
    for (uint32_t v = lane; v < vs; v += 32u) ds[v] = __ldcv(ss + v);
  }
  pdl_launch_dependents();
}

// ---------------------------------------------------------------- return
__global__ void __launch_bounds__(256) k_ep_return(const EpArgs e, const float *__restrict__ down,
                                                   const uint32_t *__restrict__ src_rank,
                                                   const uint32_t *__restrict__ src_place, const uint32_t *p_recv,
                                                   uint32_t *ctr) {
  pdl_wait();
  const EpWindow &w = e.w;
  const uint32_t n = *p_recv;
  const uint32_t warp = (blockIdx.x * blockDim.x + threadIdx.x) / 32u, lane = threadIdx.x % 32u;
  const uint32_t nwarps = gridDim.x * blockDim.x / 32u;
  __shared__ int last;
  for (uint32_t j = warp; j < n; j += nwarps) {
    const float4 *src = reinterpret_cast<const float4 *>(down + (size_t)j * w.H);
    uint4 *dst = win_at<uint4>(e, src_rank[j], w.ret_rows + (uint64_t)src_place[j] * w.H * 2u);
    // 8 bf16-rounded floats -> one 16-byte store of their bf16 bits
    for (uint32_t v = lane; v < w.H / 8u; v += 32u) {
      const float4 a = __ldg(src + 2u * v), b = __ldg(src + 2u * v + 1u);
      dst[v] = make_uint4((__float_as_uint(a.x) >> 16) | (__float_as_uint(a.y) & 0xffff0000u),
                          (__float_as_uint(a.z) >> 16) | (__float_as_uint(a.w) & 0xffff0000u),
                          (__float_as_uint(b.x) >> 16) | (__float_as_uint(b.y) & 0xffff0000u),
                          (__float_as_uint(b.z) >> 16) | (__float_as_uint(b.w) & 0xffff0000u));
    }
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) last = atomicAdd(ctr, 1u) == gridDim.x - 1u;
  __syncthreads();
  if (last) {
    __threadfence_system();
    if (threadIdx.x < w.G) st_release_sys(win_at<uint32_t>(e, threadIdx.x, w.flag_ret) + e.rank, e.epoch);
    if (threadIdx.x == 0) *ctr = 0u;
  }
  pdl_launch_dependents();
}

// ------------------------------------------------------------- release
// The down GEMM stored the rows into the sources' windows itself (fused
// return); publish them: a system-scope fence, then flag_ret[rank] = epoch in
// every window.
__global__ void k_ep_release(const EpArgs e) {
  pdl_wait();
  __threadfence_system();
  if (threadIdx.x < e.w.G) st_release_sys(win_at<uint32_t>(e, threadIdx.x, e.w.flag_ret) + e.rank, e.epoch);
  pdl_launch_dependents();
}

// ------------------------------------------------------------------ wait
__global__ void k_ep_wait_returns(const EpArgs e) {
  pdl_wait();
  if (threadIdx.x == 0 &&
      !wait_flags(win_at<uint32_t>(e, e.rank, e.w.flag_ret), e.w.G, e.epoch, e.deadline_ns))
    raise_flag(e.flags, PW_FLAG_WAIT_TIMEOUT);
  pdl_launch_dependents();
}

// ------------------------------------------------------------------ launchers
cudaError_t launch_ep_dispatch(const EpArgs &e, const uint32_t *offsets, const uint8_t *codes, const float *scales,
                               uint32_t P, uint32_t *ctr, int grid, cudaStream_t stream) {
  if (e.w.G > 8u || e.w.H % 512u) return cudaErrorInvalidValue;
  return launch_kernel(k_ep_dispatch, dim3(grid), dim3(256), 0, stream, e, offsets, codes, scales, P, ctr);
}

cudaError_t launch_ep_plan(const EpArgs &e, const BankTable &bank, uint32_t chunk, uint32_t cap, uint32_t *perm,
                           uint32_t *src_rank, uint32_t *src_place, GemvGroup *gu, GemvGroup *dn, uint32_t *n_groups,
                           uint32_t *p_recv, cudaStream_t stream) {
  const size_t smem = (size_t)(2u * e.w.G * e.w.L + e.w.G + 2u * (e.w.L + 1u)) * sizeof(uint32_t);
  if (smem > 48u * 1024u) return cudaErrorInvalidValue;
  return launch_kernel(k_ep_plan, dim3(1), dim3(1024), smem, stream, e, bank, chunk, cap, perm, src_rank, src_place,
                       gu, dn, n_groups, p_recv);
}

cudaError_t launch_ep_gather(const EpArgs &e, const uint32_t *perm, const uint32_t *p_recv, uint8_t *codes,
                             float *scales, int grid, cudaStream_t stream) {
  return launch_kernel(k_ep_gather, dim3(grid), dim3(256), 0, stream, e, perm, p_recv, codes, scales);
}

cudaError_t launch_ep_return(const EpArgs &e, const float *down, const uint32_t *src_rank, const uint32_t *src_place,
                             const uint32_t *p_recv, uint32_t *ctr, int grid, cudaStream_t stream) {
  return launch_kernel(k_ep_return, dim3(grid), dim3(256), 0, stream, e, down, src_rank, src_place, p_recv, ctr);
}

cudaError_t launch_ep_release(const EpArgs &e, cudaStream_t stream) {
  return launch_kernel(k_ep_release, dim3(1), dim3(32), 0, stream, e);
}

cudaError_t launch_ep_wait_returns(const EpArgs &e, cudaStream_t stream) {
  return launch_kernel(k_ep_wait_returns, dim3(1), dim3(32), 0, stream, e);
}

}  // namespace pw
