// pw_static.cu -- an expert forward pass that allocates nothing.
//
// pw_expert_forward_static() runs the same kernels as pw_expert_forward()
// (dynamic FP8 quantization, fused gate/up + staged SwiGLU + hidden
// quantization, down projection with bf16 rounding), but its scratch --
// activation codes and scales, the hidden's codes and scales, the GEMV group
// records, the TMA descriptors and the error-flag word -- lives in one
// file-scope __device__ array instead of a runtime's cudaMalloc'd arena.  It
// needs no pw_runtime either.  It is meant for callers that must not allocate
// device memory at call time: code running under a fixed memory budget that
// was reserved up front, plug-in hosts whose allocator is not CUDA's, or
// serving loops that have to stay free of cudaMalloc/cudaFree because those
// calls synchronise the device.
//
// Host code must not pass `g_static_scratch` itself to a kernel: in host code
// that name is a host-side stand-in, not a device address.  The device address
// comes from cudaGetSymbolAddress, taken once per device (see scratch_base).
#include <cstdint>
#include <cstring>
#include <mutex>

#include <cuda.h>
#include <cuda_runtime.h>

#include "pw_cuda.h"
#include "pw_internal.h"

namespace {

using namespace pw;

constexpr uint32_t kMaxWidth = 8;
constexpr uint32_t kMaxDim = 4096;
constexpr size_t kAlign = 256;

constexpr size_t align_up(size_t v) { return (v + kAlign - 1) / kAlign * kAlign; }

// Fixed layout of the static scratch (offsets in bytes).
constexpr size_t kOffXCodes = 0;                                                   // [8][4096] u8
constexpr size_t kOffXScales = align_up(kOffXCodes + kMaxWidth * kMaxDim);          // [8][32] f32
constexpr size_t kOffHCodes = align_up(kOffXScales + kMaxWidth * (kMaxDim / 128) * 4);  // [8][4096] u8
constexpr size_t kOffHScales = align_up(kOffHCodes + kMaxWidth * kMaxDim);          // [8][32] f32
constexpr size_t kOffMaps = align_up(kOffHScales + kMaxWidth * (kMaxDim / 128) * 4);  // 3 x CUtensorMap
constexpr size_t kOffGroups = align_up(kOffMaps + 3 * sizeof(CUtensorMap));         // 2 x GemvGroup
constexpr size_t kOffFlags = align_up(kOffGroups + 2 * sizeof(GemvGroup));          // u32
constexpr size_t kScratchBytes = align_up(kOffFlags + sizeof(uint32_t));

}  // namespace

// Every device that loads this library holds this array until the process
// exits.  All calls share it and it keeps the last call's contents.
static __device__ __align__(256) unsigned char g_static_scratch[kScratchBytes];

namespace {

constexpr int kMaxDevices = 64;
std::mutex g_setup_mutex;
void *g_scratch_ptr[kMaxDevices] = {};

// Device address of g_static_scratch on the current device, looked up once
// per device (with that device current) and cached for the life of the
// process.  cudaDeviceReset destroys the context that address belongs to, so
// the entry point must not be called after a reset.
cudaError_t scratch_base(int device, unsigned char **out) {
  if (device < 0 || device >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (!g_scratch_ptr[device]) {
    void *p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_static_scratch);
    if (e != cudaSuccess) return e;
    g_scratch_ptr[device] = p;
  }
  *out = static_cast<unsigned char *>(g_scratch_ptr[device]);
  return cudaSuccess;
}

bool plain_tensor_ok(const pw_fp8_tensor &t) {
  return t.weight && t.scale && t.rows && t.cols && t.rows % 128u == 0 && t.cols % 128u == 0 &&
         t.scale_rows == t.rows / 128u && t.scale_cols == t.cols / 128u;
}

}  // namespace

extern "C" int pw_expert_forward_static(const pw_expert_weights *w, const float *x, uint32_t width, float *y,
                                        void *cuda_stream) {
  if (!w || !x || !y) return PW_ERR_ARGUMENT;
  if (!plain_tensor_ok(w->gate) || !plain_tensor_ok(w->up) || !plain_tensor_ok(w->down)) return PW_ERR_SHAPE;
  const uint32_t H = w->gate.cols, I = w->gate.rows;
  if (w->up.rows != I || w->up.cols != H || w->down.rows != H || w->down.cols != I) return PW_ERR_SHAPE;
  // the fixed scratch holds at most 8 tokens of 4096 columns each
  if (width == 0 || width > kMaxWidth || H > kMaxDim || I > kMaxDim) return PW_ERR_UNSUPPORTED;
  cudaStream_t stream = static_cast<cudaStream_t>(cuda_stream);

  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess) return PW_ERR_CUDA;
  // the scratch used is the current device's, so the stream must belong to it
  int stream_device = device;
  if (cudaStreamGetDevice(stream, &stream_device) != cudaSuccess) return PW_ERR_CUDA;
  if (stream_device != device) return PW_ERR_ARGUMENT;
  unsigned char *base = nullptr;
  if (scratch_base(device, &base) != cudaSuccess) return PW_ERR_CUDA;
  uint8_t *xc = base + kOffXCodes;
  float *xs = reinterpret_cast<float *>(base + kOffXScales);
  uint8_t *hc = base + kOffHCodes;
  float *hs = reinterpret_cast<float *>(base + kOffHScales);
  CUtensorMap *maps = reinterpret_cast<CUtensorMap *>(base + kOffMaps);
  GemvGroup *groups = reinterpret_cast<GemvGroup *>(base + kOffGroups);
  uint32_t *flags = reinterpret_cast<uint32_t *>(base + kOffFlags);

  // host-side descriptors, copied into the static scratch (no allocation)
  CUtensorMap hmaps[3];
  if (!encode_weight_map(&hmaps[0], w->gate.weight, I, H, 128u) ||
      !encode_weight_map(&hmaps[1], w->up.weight, I, H, 128u) ||
      !encode_weight_map(&hmaps[2], w->down.weight, H, I, 128u))
    return PW_ERR_CUDA;
  GemvGroup hgroups[2];
  memset(hgroups, 0, sizeof hgroups);
  hgroups[0].w0 = w->gate.weight;
  hgroups[0].s0 = w->gate.scale;
  hgroups[0].w1 = w->up.weight;
  hgroups[0].s1 = w->up.scale;
  hgroups[0].tm0 = &maps[0];
  hgroups[0].tm1 = &maps[1];
  hgroups[0].count = width;
  hgroups[1].w0 = w->down.weight;
  hgroups[1].s0 = w->down.scale;
  hgroups[1].tm0 = &maps[2];
  hgroups[1].count = width;

  if (cudaMemcpyAsync(maps, hmaps, sizeof hmaps, cudaMemcpyHostToDevice, stream) != cudaSuccess) return PW_ERR_CUDA;
  if (cudaMemcpyAsync(groups, hgroups, sizeof hgroups, cudaMemcpyHostToDevice, stream) != cudaSuccess)
    return PW_ERR_CUDA;
  // the flag word must start at zero; everything else is fully written
  // before it is read by the kernels below
  if (cudaMemsetAsync(flags, 0, sizeof(uint32_t), stream) != cudaSuccess) return PW_ERR_CUDA;

  if (launch_quantize(x, width, H, xc, xs, flags, stream) != cudaSuccess) return PW_ERR_CUDA;
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  GemvArgs gu{};
  gu.groups = &groups[0];
  gu.n_groups = 1;
  gu.rows = I;
  gu.K = H;
  gu.scale_cols = H / 128u;
  gu.layout = PW_LAYOUT_PLAIN;
  gu.x_codes = xc;
  gu.x_scales = xs;
  gu.out = nullptr;
  gu.out_stride = I;
  gu.q_codes = hc;
  gu.q_scales = hs;
  gu.flags = flags;
  const int grid_gu = (int)((I / 128u) < (uint32_t)sms ? (I / 128u) : (uint32_t)sms);
  if (launch_gemv(2, gu, grid_gu, stream) != cudaSuccess) return PW_ERR_CUDA;
  GemvArgs dn{};
  dn.groups = &groups[1];
  dn.n_groups = 1;
  dn.rows = H;
  dn.K = I;
  dn.scale_cols = I / 128u;
  dn.layout = PW_LAYOUT_PLAIN;
  dn.x_codes = hc;
  dn.x_scales = hs;
  dn.out = y;
  dn.out_stride = H;
  dn.round_bf16 = 1;
  dn.flags = flags;
  const int grid_dn = (int)((H / 128u) < (uint32_t)sms ? (H / 128u) : (uint32_t)sms);
  if (launch_gemv(0, dn, grid_dn, stream) != cudaSuccess) return PW_ERR_CUDA;

  uint32_t hflags = 0;
  if (cudaMemcpyAsync(&hflags, flags, sizeof hflags, cudaMemcpyDeviceToHost, stream) != cudaSuccess)
    return PW_ERR_CUDA;
  if (cudaStreamSynchronize(stream) != cudaSuccess) return PW_ERR_CUDA;
  if (hflags & PW_FLAG_WAIT_TIMEOUT) return PW_ERR_TIMEOUT;
  if (hflags & (PW_FLAG_NONFINITE_INPUT | PW_FLAG_NONFINITE_FUSED | PW_FLAG_NONFINITE_ROUND)) return PW_ERR_NONFINITE;
  if (hflags) return PW_ERR_DEVICE_FLAGS;
  return PW_OK;
}
