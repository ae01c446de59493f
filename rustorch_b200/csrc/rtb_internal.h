// Internal declarations shared by the C-ABI implementation files.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>
#include <string>
#include <unordered_map>

#include "../../include/rustorch_b200.h"

struct rtb_ctx {
  int device = 0;
  int sm_count = 0;
  int cc_major = 0, cc_minor = 0;
  size_t total_mem = 0;
  cudaStream_t stream = nullptr;  // the context's own non-blocking stream (rtb_context_stream)
  int* d_err = nullptr;           // device error word (bounded-wait timeouts)
  uint64_t timeout_ns = 2000000000ull;
  int default_precision = RTB_PREC_3XTF32;
  unsigned long long* trace = nullptr;  // kernel timeline trace buffer (diagnostics)
  int64_t trace_capacity = 0;           // in 64-bit stamps
  // Split-tile arrival counters, one block per stream this context launches
  // on (launches on one stream run in order, so they can share it).  A word
  // holds (launch generation << 8 | arrivals): a launch counts only arrivals
  // tagged with its own generation, so the block never needs re-zeroing.
  struct SplitCounters {
    unsigned long long* d = nullptr;
    unsigned long long gen = 0;
  };
  std::mutex cnt_mu;
  std::unordered_map<cudaStream_t, SplitCounters> split_cnt;
};

namespace rtb {

// Clears the calling thread's CUDA "last error" (a non-sticky error left by an
// earlier, already reported call, possibly another library's) so the check
// after our own kernel launch sees only that launch's outcome.
inline void clear_stale_cuda_error() { (void)cudaGetLastError(); }

// Records `msg` as this thread's last error and returns `status`.
int set_error(int status, const std::string& msg);
int cuda_status(cudaError_t e, const char* what);

// NULL is the legacy default stream, as everywhere in the CUDA runtime (and
// what torch's default stream handle is), so work on it orders with other
// libraries' work on that stream.
inline cudaStream_t pick_stream(rtb_ctx* ctx, void* stream) {
  (void)ctx;
  return static_cast<cudaStream_t>(stream);
}

// RAII guard making ctx->device current for the calling thread.  The device
// is set even when it already is the thread's current device: cudaSetDevice
// also binds the device's primary context to the thread, which the driver-API
// calls made here (tensor-map encoding) need in a thread that has not used
// the runtime yet (e.g. a worker thread of the caller's pool).
struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    cudaGetDevice(&prev);
    cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

// 2-D fp32 tensor map (innermost dim0 contiguous, row stride in elements),
// 128-byte swizzle with 16-byte atoms, or 32-byte atoms when atom32 is set.
int make_tmap_2d(CUtensorMap* map, const void* base, uint64_t dim0, uint64_t dim1,
                 uint64_t row_stride_elems, uint32_t box0, uint32_t box1, bool atom32);
// Same with the shared-memory layout chosen explicitly (no swizzle allows an
// inner box wider than 128 bytes).
constexpr int kTmapSwizzleNone = 0, kTmapSwizzle128 = 1, kTmapSwizzle128Atom32 = 2;
int make_tmap_2d_swz(CUtensorMap* map, const void* base, uint64_t dim0, uint64_t dim1,
                     uint64_t row_stride_elems, uint32_t box0, uint32_t box1, int swizzle);

// 4-D im2col map over an NHWC tensor [N, H, W, Cp] for a forward conv with
// filter R x S, stride (sh, sw), padding (ph, pw): channels_per_pixel x
// pixels_per_column boxes, rows swizzled in 16-byte units over swizzle_bytes
// (128, 64 or 32; 0 = dense rows).
int make_tmap_im2col(CUtensorMap* map, const void* x, int N, int H, int W, int Cp, int R, int S,
                     int sh, int sw, int ph, int pw, uint32_t channels_per_pixel,
                     uint32_t pixels_per_column, int swizzle_bytes);

// What the GEMM engine computes; see rtb_gemm.cuh (GemmParams) for the epilogue.
struct GemmDesc {
  int64_t M = 0, N = 0, K = 0;
  // A: K-major [M, K] with row stride lda (GATHER: unused; see conv fields)
  const float* A = nullptr;
  int64_t lda = 0;
  // B: b_mn_major=0 -> [N, K] row stride ldb; 1 -> [K, N] row stride ldb
  const float* B = nullptr;
  int64_t ldb = 0;
  int b_mn_major = 0;
  // epilogue
  float* C = nullptr;
  int64_t ldc = 0;
  const float* bias = nullptr;
  const float* residual = nullptr;
  int64_t ldr = 0;
  int act = 0;  // RTB_ACT_* applied after bias and residual
  int out_mode = 0;  // 0 row-major, 1 NCHW scatter, 2 every rank's C (N-split)
  int hw = 0;
  float* const* peer_c = nullptr;  // out_mode 2: device array of npeers C bases
  int npeers = 0;
  int64_t col_off = 0;
  // conv A producer: 0 = none (A is a matrix), 1 = cp.async gather, 2 = TMA im2col
  // (one tap x 32 channels per k-block), 3 = multi-tap TMA im2col (32 / Cp taps
  // of Cp channels per k-block, Cp in {4, 8, 16}; 3xTF32 only; selected for 8, 16)
  int gather = 0;
  const float* x = nullptr;
  int Nimg = 0;
  int H = 0, W = 0, Cp = 0, Ho = 0, Wo = 0, R = 0, S = 0, sh = 1, sw = 1, ph = 0, pw = 0;
  // optional: B's 3xTF32 low part (B - trunc_tf32(B)) in B's layout and ldb,
  // computed by the caller (e.g. with a weight pack); null = gemm_run decides
  const float* B_lo = nullptr;
  int split3 = 1;     // 3xTF32 (1) or TF32 (0)
  int bn = 0;         // 0 = heuristic
  int allow_workspace = 1;  // 0: never allocate (tail balancing off)
  // A given MN-major: [K, M] row-major with row stride lda (3xTF32, no conv
  // producer; the converters read the tile transposed).  Used by the skinny
  // GEMM's transposed form, whose A is the caller's [K,N] B.
  int a_mn_major = 0;
  // bias per row of C (out_mode 1 only): the transposed skinny GEMM's bias,
  // which indexes the caller's columns
  const float* row_bias = nullptr;
};

// Validated launch of the tcgen05 engine (A/B already TMA-compatible).
int gemm_run(rtb_ctx* ctx, const GemmDesc& d, cudaStream_t stream);

// Small-M path (M <= kSmallMMax, no conv producer): packed fp32 FMAs on the
// CUDA cores with B streamed once from HBM (rtb_smallm.cu).  Measured on B200
// for M x 8192 x 8192 (B row-major): 52.9 / 54.2 / 68.6 / 123.2 us at M = 1 /
// 8 / 16 / 32 against 106.9-109.3 us for the 128-row tensor-core tile (M = 48,
// 64) and 73-79 us for the tensor cores' transposed form (C^T = B^T . A^T,
// which takes 72.5-78 us at M = 16), so rows beyond 16 go to the tensor cores.
constexpr int64_t kSmallMMax = 16;
int smallm_run(rtb_ctx* ctx, const GemmDesc& d, cudaStream_t stream);

// Aux kernels (rtb_aux.cu).
int launch_pack_kmajor(const float* src, int64_t rows, int64_t k, int64_t rs, int64_t cs,
                       float* dst, int64_t kp, cudaStream_t s);
int launch_fill_rows(float* C, int64_t M, int64_t N, int64_t ldc, const float* bias, int act,
                     cudaStream_t s);
int launch_nchw_to_nhwc_padded(const float* x, int64_t N, int64_t C, int64_t H, int64_t W,
                               int64_t Cp, float* y, cudaStream_t s);
// w [Co, Ci, kh, kw] -> wp [Co, kh*kw*Cp] (channels padded to Cp); wlo
// (nullable) receives wp's 3xTF32 low part in the same layout.
int launch_prepack_weight(const float* w, int64_t Co, int64_t Ci, int64_t kh, int64_t kw,
                          int64_t Cp, float* wp, float* wlo, cudaStream_t s);
// NCHW -> NHWC (channels padded to Cp) of x and the weight prepack of
// launch_prepack_weight in one launch (two launches when Cp == 4).
// out[r][c] = B[r][c] - trunc_tf32(B[r][c]) over rows x cols (row stride ldb),
// padding columns [cols, ldo) zeroed; ldo % 4 == 0, out 16-byte aligned.
int launch_tf32_lo(const float* b, int64_t rows, int64_t cols, int64_t ldb, float* out,
                   int64_t ldo, cudaStream_t s);
int launch_conv_prologue(const float* x, int64_t N, int64_t C, int64_t H, int64_t W, int64_t Cp,
                         float* y, const float* w, int64_t Co, int64_t kh, int64_t kw, float* wp,
                         float* wlo, cudaStream_t s);
// Stride-2 conv over <= 4 input channels as a stride-1 conv of its space-to-
// depth form: NCHW x -> NHWC [N, Hs, Ws, 16] (padding applied) and w [Co, C,
// kh, kw] -> [Co, ceil(kh/2)*ceil(kw/2), 16], in one launch.
int launch_conv_prologue_s2d(const float* x, int64_t N, int64_t C, int64_t H, int64_t W,
                             int64_t ph, int64_t pw, int64_t Hs, int64_t Ws, float* y,
                             const float* w, int64_t Co, int64_t kh, int64_t kw, float* w2,
                             float* w2lo, cudaStream_t s);
int launch_max_pool2d(const float* x, float* y, int64_t N, int64_t C, int64_t H, int64_t W,
                      int64_t kh, int64_t kw, int64_t sh, int64_t sw, int64_t ph, int64_t pw,
                      int layout, cudaStream_t s);
int launch_global_avg_pool(const float* x, float* y, int64_t N, int64_t C, int64_t HW, int layout,
                           cudaStream_t s);
int launch_add(const float* a, const float* b, float* y, int64_t n, cudaStream_t s);
int launch_relu(const float* x, float* y, int64_t n, cudaStream_t s);
int launch_broadcast(int op, int ndim, const int64_t* shape, const float* a,
                     const int64_t* sa, const float* b, const int64_t* sb, float* y,
                     cudaStream_t s);
int launch_wait_probe(int* err, uint64_t timeout_ns, cudaStream_t s);
int launch_unsplit_cols(const float* parts, float* C, int64_t P, int64_t M, int64_t Nl,
                        cudaStream_t s);
int launch_nhwc_to_nchw(const float* x, float* y, int64_t N, int64_t C, int64_t HW,
                        cudaStream_t s);

// rtb_conv2d_fwd_packed without any device allocation (rtb_noalloc.cu).
int conv2d_fwd_packed_noalloc(rtb_ctx* ctx, int64_t N, int64_t Ci, int64_t H, int64_t W,
                              int64_t Co, int64_t kh, int64_t kw, int64_t sh, int64_t sw,
                              int64_t ph, int64_t pw, const float* x_nhwc_padded,
                              const float* w_packed, const float* bias, const float* residual,
                              int act, float* y, int y_layout, int precision, void* stream);

// Backward-pass layout kernels (rtb_backward.cu).
int launch_dilate_nchw_to_nhwc(const float* dy, int64_t N, int64_t Co, int64_t Ho, int64_t Wo,
                               int64_t sh, int64_t sw, int64_t Hd, int64_t Wd, int64_t Cop,
                               float* out, cudaStream_t s);
int launch_prepack_flip(const float* w, int64_t Co, int64_t Ci, int64_t R, int64_t S, int64_t Cop,
                        float* wt, cudaStream_t s);
int launch_im2col_nhwc(const float* x, int64_t N, int64_t H, int64_t W, int64_t Cp, int64_t Ho,
                       int64_t Wo, int64_t R, int64_t S, int64_t sh, int64_t sw, int64_t ph,
                       int64_t pw, float* col, cudaStream_t s);
int launch_nchw_to_cmajor(const float* dy, int64_t N, int64_t Co, int64_t HW, int64_t ldp,
                          float* dyt, cudaStream_t s);
int launch_unpack_weight_grad(const float* dwp, int64_t Co, int64_t Ci, int64_t R, int64_t S,
                              int64_t Cp, int accumulate, float* dw, cudaStream_t s);

// Row-wise LayerNorm (last dimension, two-pass variance) + activation:
// Y = act((X - mean) / sqrt(var + eps) * g + b) over row-major [M, N]
// matrices (X == Y allowed); g / b optional.
int launch_layernorm_act(rtb_ctx* ctx, const float* X, int64_t ldx, float* Y, int64_t ldy,
                         int64_t M, int64_t N, const float* g, const float* b, float eps, int act,
                         cudaStream_t s);

// Stream-ordered workspace.
int ws_alloc(rtb_ctx* ctx, void** p, size_t bytes, cudaStream_t s);
void ws_free(void* p, cudaStream_t s);
// Launch with programmatic stream serialization (programmatic dependent
// launch): the kernel may be scheduled while the previous kernel on the
// stream finishes, so it must call griddep_wait() before its first access
// to global memory.  Used for the kernels of the contraction chains.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t s, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, args...);
}
// Capacity (words) of a stream's split-counter block: >= the tail tiles of
// one wave split (at most half the SMs).
constexpr int kSplitCounters = 256;
// The split-counter block for `s` and the next launch generation on it;
// RTB_E_UNSUPPORTED (no error recorded) while `s` is capturing a graph or is
// cudaStreamPerThread (a different stream in every host thread), when the
// caller allocates and zeroes counters for the launch itself (gen 1).
int split_counters(rtb_ctx* ctx, cudaStream_t s, unsigned long long** d, unsigned long long* gen);

}  // namespace rtb
