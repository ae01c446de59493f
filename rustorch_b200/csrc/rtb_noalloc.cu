// rtb_conv2d_fwd_noalloc: the Conv2d(+bias, +residual, +ReLU) forward of
// rtb_conv2d_fwd for callers that cannot allocate device memory.
//
// Some callers cannot call cudaMalloc (or any allocator) on the path that
// runs a conv: a host framework that owns the GPU's memory through its own
// allocator and counts every other allocation against a fixed budget, or a
// latency-critical loop where an allocation call may block on device-wide
// synchronisation.  rtb_conv2d_fwd needs scratch memory for the channel-padded
// NHWC copy of the input and the repacked weight, which it takes from the
// stream-ordered pool.  This variant takes that scratch from a fixed array
// compiled into the library instead, so the call itself allocates nothing.
//
// The scratch is a file-scope __device__ array of kNoAllocScratchBytes
// (16 MiB).  Every GPU that loads this library holds those 16 MiB until the
// process exits.  All calls on a device share the one array:
//   - calls that overlap on the GPU (different streams, or different host
//     threads without ordering) race on it and corrupt each other's results;
//     callers must order them (same stream, or events);
//   - the array keeps the previous call's contents; every byte a call reads is
//     first written by that call (the padding channels and padding taps are
//     written as zeros by the packing kernels), so nothing needs clearing.
// The first call on each device looks up the array's device address with
// cudaGetSymbolAddress while that device is current (once per device); that
// first call should come before any stream capture.  The address is kept per
// device together with the CUDA context it belongs to: after the context is
// torn down and recreated (cudaDeviceReset), the next call looks it up again.
//
// The stem-shaped case (stride 2 over <= 4 input channels) runs here as the
// 4-channel cp.async im2col gather, not through the space-to-depth rewrite
// rtb_conv2d_fwd uses (that rewrite needs a second copy of the input); the
// results agree to the same tolerance, the gather is the slower producer for
// that shape (measured on the ResNet stem at 256 images: about 1.2 against
// 0.95 ms through rtb_conv2d_fwd, a size beyond this scratch anyway).
#include <cstdint>
#include <mutex>

#include "rtb_internal.h"

constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;  // 16 MiB

// Host code never touches this array directly: its name in host code is only
// a handle for cudaGetSymbolAddress, not a device address.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

namespace {

constexpr int kMaxDevices = 64;

std::mutex g_mu;
void* g_addr[kMaxDevices] = {nullptr};
CUcontext g_addr_ctx[kMaxDevices] = {nullptr};  // the context each address belongs to

typedef CUresult (*CtxGetCurrentFn)(CUcontext*);

CtxGetCurrentFn ctx_get_current() {
  static CtxGetCurrentFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<CtxGetCurrentFn>(p);
  });
  return fn;
}

// Device address of the scratch array on `device` (which must be current).
int scratch_address(int device, void** out) {
  if (device < 0 || device >= kMaxDevices)
    return rtb::set_error(RTB_E_UNSUPPORTED, "conv2d_fwd_noalloc: device index too large");
  CtxGetCurrentFn get = ctx_get_current();
  if (!get) return rtb::set_error(RTB_E_CUDA, "conv2d_fwd_noalloc: cuCtxGetCurrent unavailable");
  CUcontext cur = nullptr;
  if (get(&cur) != CUDA_SUCCESS) cur = nullptr;
  std::lock_guard<std::mutex> lk(g_mu);
  if (cur && g_addr[device] && g_addr_ctx[device] == cur) {
    *out = g_addr[device];
    return RTB_OK;
  }
  // first call on this device (or its context was recreated): look the
  // address up, which also makes the device's primary context current
  void* p = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
  if (e != cudaSuccess) return rtb::cuda_status(e, "conv2d_fwd_noalloc: cudaGetSymbolAddress");
  if (get(&cur) != CUDA_SUCCESS) cur = nullptr;
  g_addr[device] = p;
  g_addr_ctx[device] = cur;
  *out = p;
  return RTB_OK;
}

inline int64_t round_up64(int64_t v, int64_t m) { return (v + m - 1) / m * m; }

}  // namespace

extern "C" {

int rtb_conv2d_fwd_noalloc(rtb_ctx* ctx, int64_t N, int64_t Ci, int64_t H, int64_t W, int64_t Co,
                           int64_t kh, int64_t kw, int64_t sh, int64_t sw, int64_t ph, int64_t pw,
                           const float* x, int x_layout, const float* w, const float* bias,
                           const float* residual, int act, float* y, int y_layout, int precision,
                           void* stream) {
  if (!ctx) return rtb::set_error(RTB_E_INVALID, "null rtb_ctx");
  if (N < 0 || Ci <= 0 || H <= 0 || W <= 0 || Co <= 0 || kh <= 0 || kw <= 0 || sh <= 0 ||
      sw <= 0 || ph < 0 || pw < 0 || H + 2 * ph < kh || W + 2 * pw < kw)
    return rtb::set_error(RTB_E_INVALID, "conv2d_fwd_noalloc: bad shape, stride or padding");
  if (x_layout != RTB_LAYOUT_NCHW && x_layout != RTB_LAYOUT_NHWC)
    return rtb::set_error(RTB_E_INVALID, "conv2d_fwd_noalloc: bad x_layout");
  // Every argument is checked before the first launch, so a rejected call
  // leaves the shared scratch as it was.
  if (y_layout != RTB_LAYOUT_NCHW && y_layout != RTB_LAYOUT_NHWC)
    return rtb::set_error(RTB_E_INVALID, "conv2d_fwd_noalloc: bad y_layout");
  if (act < RTB_ACT_NONE || act > RTB_ACT_TANH)
    return rtb::set_error(RTB_E_INVALID, "conv2d_fwd_noalloc: unknown activation");
  if (precision != RTB_PREC_3XTF32 && precision != RTB_PREC_TF32 && precision != RTB_PREC_DEFAULT)
    return rtb::set_error(RTB_E_INVALID,
                          "conv2d_fwd_noalloc: precision must be RTB_PREC_3XTF32, RTB_PREC_TF32 or "
                          "DEFAULT");
  if (N == 0) return RTB_OK;
  if (!x || !w || !y) return rtb::set_error(RTB_E_INVALID, "conv2d_fwd_noalloc: null pointer");

  const int64_t Cp = round_up64(Ci, 4);
  const bool x_direct = x_layout == RTB_LAYOUT_NHWC && Cp == Ci &&
                        (reinterpret_cast<uintptr_t>(x) & 15u) == 0;
  const int64_t x_bytes = x_direct ? 0 : round_up64(N * H * W * Cp * 4, 256);
  const int64_t w_bytes = Co * kh * kw * Cp * 4;
  if (x_bytes + w_bytes > (int64_t)kNoAllocScratchBytes)
    return rtb::set_error(
        RTB_E_INVALID,
        "conv2d_fwd_noalloc: padded input + packed weight need more than the 16 MiB scratch "
        "(use rtb_conv2d_fwd)");

  rtb::DeviceGuard g(ctx->device);
  void* base = nullptr;
  int st = scratch_address(ctx->device, &base);
  if (st) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  float* xs = x_direct ? nullptr : static_cast<float*>(base);
  float* wp = reinterpret_cast<float*>(static_cast<unsigned char*>(base) + x_bytes);

  if (!x_direct) {
    st = x_layout == RTB_LAYOUT_NCHW ? rtb::launch_nchw_to_nhwc_padded(x, N, Ci, H, W, Cp, xs, s)
                                     : rtb::launch_pack_kmajor(x, N * H * W, Ci, Ci, 1, xs, Cp, s);
    if (st) return st;
  }
  st = rtb::launch_prepack_weight(w, Co, Ci, kh, kw, Cp, wp, nullptr, s);
  if (st) return st;
  return rtb::conv2d_fwd_packed_noalloc(ctx, N, Ci, H, W, Co, kh, kw, sh, sw, ph, pw,
                                        x_direct ? x : xs, wp, bias, residual, act, y, y_layout,
                                        precision, stream);
}

}  // extern "C"
