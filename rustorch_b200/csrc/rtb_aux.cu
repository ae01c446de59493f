// Small device kernels around the contraction engine: operand packing,
// layout conversion, max/avg pooling, elementwise ops, N-split repacking.
// These are HBM-bound byte movers; grids are sized in multiples of the SM
// count by the CUDA occupancy rules (256-thread blocks, grid-stride loops).
#include <cfloat>

#include "rtb_act.cuh"
#include "rtb_internal.h"
#include "rtb_ptx.cuh"

namespace rtb {

namespace {

constexpr int kThreads = 256;

inline int grid_for(int64_t n, int per_thread = 1) {
  int64_t blocks = (n / per_thread + kThreads - 1) / kThreads;
  if (blocks < 1) blocks = 1;
  if (blocks > 148 * 32) blocks = 148 * 32;
  return (int)blocks;
}

inline int launch_check(const char* what) {
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? RTB_OK : cuda_status(e, what);
}

// dst[r, k] = src[r*rs + k*cs] for k < K, 0 for K <= k < Kp.  32x32 tiles
// through shared memory so both the strided read and the row write coalesce.
__global__ void pack_kmajor_kernel(const float* __restrict__ src, int64_t rows, int64_t K,
                                   int64_t rs, int64_t cs, float* __restrict__ dst, int64_t Kp) {
  __shared__ float tile[32][33];
  const int64_t r0 = (int64_t)blockIdx.y * 32, k0 = (int64_t)blockIdx.x * 32;
  const int tx = threadIdx.x, ty = threadIdx.y;  // 32 x 8
  const bool k_fast = (cs == 1);
  for (int i = ty; i < 32; i += 8) {
    int64_t r, k;
    if (k_fast) { r = r0 + i; k = k0 + tx; }
    else        { r = r0 + tx; k = k0 + i; }
    float v = 0.0f;
    if (r < rows && k < K) v = src[r * rs + k * cs];
    if (k_fast) tile[i][tx] = v; else tile[tx][i] = v;
  }
  __syncthreads();
  for (int i = ty; i < 32; i += 8) {
    const int64_t r = r0 + i, k = k0 + tx;
    if (r < rows && k < Kp) dst[r * Kp + k] = tile[i][tx];
  }
}

__global__ void fill_rows_kernel(float* C, int64_t M, int64_t N, int64_t ldc,
                                 const float* bias, int act) {
  const int64_t total = M * N;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t m = i / N, n = i - m * N;
    C[m * ldc + n] = activate(bias ? bias[n] : 0.0f, act);
  }
}

// NCHW -> NHWC with channel stride Cp (zero pad).  Tiled transpose per image:
// tile of 32 pixels x 32 channels.
// NCHW [N, C, HW] -> NHWC [N, HW, Cp] (channels >= C zero-filled).  A block
// moves a 32-channel x 128-pixel tile (16 KB): each warp reads 512 contiguous
// bytes of one channel plane (16-byte loads when HW % 4 == 0), the tile is
// transposed through shared memory (row pitch 129: conflict-free), and each
// warp writes 4 pixels x 32 channels as 16-byte stores.  32-bit index math
// within an image.
constexpr int kT2Pix = 128;
// One 32-channel x 128-pixel tile (tile index p_t, channel block c_t, image n);
// `tile` is 32 x (kT2Pix + 1) floats of shared memory.
__device__ __forceinline__ void nchw_to_nhwc_tile(const float* __restrict__ x, int C, int HW,
                                                  int Cp, int vec, int vec_out,
                                                  float* __restrict__ y, int p_t, int c_t,
                                                  int64_t n, float (*tile)[kT2Pix + 1]) {
  const int p0 = p_t * kT2Pix, c0 = c_t * 32;
  const float* xi = x + n * C * HW;
  float* yi = y + n * HW * Cp;
  const int t = threadIdx.x;
  // load: 32 channels x 32 four-pixel groups, 4 per thread
#pragma unroll
  for (int it = 0; it < 4; ++it) {
    const int idx = t + 256 * it;
    const int cl = idx >> 5, g = idx & 31;
    const int c = c0 + cl, p = p0 + 4 * g;
    float v[4] = {0.f, 0.f, 0.f, 0.f};
    if (c < C) {
      const float* src = xi + (int64_t)c * HW + p;
      if (vec && p + 3 < HW) {
        const float4 q = __ldg(reinterpret_cast<const float4*>(src));
        v[0] = q.x; v[1] = q.y; v[2] = q.z; v[3] = q.w;
      } else {
#pragma unroll
        for (int e = 0; e < 4; ++e)
          if (p + e < HW) v[e] = __ldg(src + e);
      }
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) tile[cl][4 * g + e] = v[e];
  }
  __syncthreads();
  // store: 128 pixels x 8 four-channel groups, 4 per thread
#pragma unroll
  for (int it = 0; it < 4; ++it) {
    const int idx = t + 256 * it;
    const int pl = idx >> 3, cg = idx & 7;
    const int p = p0 + pl, c = c0 + 4 * cg;
    if (p >= HW || c >= Cp) continue;
    float* dst = yi + (int64_t)p * Cp + c;
    const float4 o = make_float4(tile[4 * cg][pl], tile[4 * cg + 1][pl], tile[4 * cg + 2][pl],
                                 tile[4 * cg + 3][pl]);
    if (vec_out && c + 3 < Cp) {
      *reinterpret_cast<float4*>(dst) = o;  // y 16-byte aligned, Cp % 4 == 0
    } else {
      const float ov[4] = {o.x, o.y, o.z, o.w};
      for (int e = 0; e < 4 && c + e < Cp; ++e) dst[e] = ov[e];
    }
  }
}

__global__ void __launch_bounds__(256) nchw_to_nhwc_kernel(const float* __restrict__ x, int C,
                                                            int HW, int Cp, int vec,
                                                            int vec_out, float* __restrict__ y) {
  __shared__ float tile[32][kT2Pix + 1];
  nchw_to_nhwc_tile(x, C, HW, Cp, vec, vec_out, y, blockIdx.x, blockIdx.y, blockIdx.z, tile);
}

// Small-channel variant (C <= 4, Cp == 4): one thread per pixel reads its C
// channel values (coalesced across threads within each plane) and writes one
// 16-byte NHWC pixel.
__global__ void nchw_to_nhwc_c4_kernel(const float* __restrict__ x, int C, int HW, int64_t npix,
                                       float4* __restrict__ y) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < npix;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t img = i / HW;
    const int p = (int)(i - img * HW);
    const float* xi = x + img * C * HW + p;
    float v[4] = {0.f, 0.f, 0.f, 0.f};
    for (int c = 0; c < C; ++c) v[c] = __ldg(xi + (int64_t)c * HW);
    y[i] = make_float4(v[0], v[1], v[2], v[3]);
  }
}

// NHWC [N, HW, C] -> NCHW [N, C, HW].
__global__ void nhwc_to_nchw_kernel(const float* __restrict__ x, int64_t C, int64_t HW,
                                    float* __restrict__ y) {
  __shared__ float tile[32][33];
  const int64_t img = blockIdx.z;
  const int64_t p0 = (int64_t)blockIdx.x * 32, c0 = (int64_t)blockIdx.y * 32;
  const int tx = threadIdx.x, ty = threadIdx.y;
  const float* xi = x + img * HW * C;
  for (int i = ty; i < 32; i += 8) {
    const int64_t p = p0 + i, c = c0 + tx;
    tile[i][tx] = (c < C && p < HW) ? xi[p * C + c] : 0.0f;
  }
  __syncthreads();
  float* yi = y + img * C * HW;
  for (int i = ty; i < 32; i += 8) {
    const int64_t c = c0 + i, p = p0 + tx;
    if (c < C && p < HW) yi[c * HW + p] = tile[tx][i];
  }
}

// w [Co, Ci, kh, kw] -> wp [Co, kh*kw*Cp] with k = (r*kw + s)*Cp + ci.
// One block per output channel: its Ci*kh*kw weights are read contiguously
// into shared memory (when they fit), then written in (tap, ci) order.
constexpr int kPrepackSmemFloats = 12288;  // 48 KB
// Output channel co's weights; `sw` is kPrepackSmemFloats floats of shared memory.
// The 3xTF32 low part of a weight value: x - trunc_tf32(x) (the tensor core
// reads the raw value as its truncated TF32 hi part).
__device__ __forceinline__ float tf32_lo(float x) {
  return x - __uint_as_float(__float_as_uint(x) & 0xFFFFE000u);
}

// Co row `co` of the packed weight; wlo (nullable) receives its 3xTF32 low part
// in the same layout.
__device__ __forceinline__ void prepack_weight_block(const float* __restrict__ w, int Ci, int taps,
                                                     int Cp, float* __restrict__ wp, int co,
                                                     float* sw, int sw_floats,
                                                     float* __restrict__ wlo) {
  const int n_in = Ci * taps;
  const float* src = w + (int64_t)co * n_in;
  float* dst = wp + (int64_t)co * taps * Cp;
  float* dlo = wlo ? wlo + (int64_t)co * taps * Cp : nullptr;
  const int Kw = taps * Cp;
  if (n_in <= sw_floats) {
    for (int i = threadIdx.x; i < n_in; i += blockDim.x) sw[i] = __ldg(src + i);
    __syncthreads();
    for (int k = threadIdx.x; k < Kw; k += blockDim.x) {
      const int tap = k / Cp, ci = k - tap * Cp;
      const float v = ci < Ci ? sw[ci * taps + tap] : 0.0f;
      dst[k] = v;
      if (dlo) dlo[k] = tf32_lo(v);
    }
  } else {
    for (int k = threadIdx.x; k < Kw; k += blockDim.x) {
      const int tap = k / Cp, ci = k - tap * Cp;
      const float v = ci < Ci ? __ldg(src + ci * taps + tap) : 0.0f;
      dst[k] = v;
      if (dlo) dlo[k] = tf32_lo(v);
    }
  }
}

__global__ void __launch_bounds__(256) prepack_weight_kernel(const float* __restrict__ w, int Ci,
                                                              int taps, int Cp,
                                                              float* __restrict__ wp,
                                                              float* __restrict__ wlo) {
  __shared__ float sw[kPrepackSmemFloats];
  prepack_weight_block(w, Ci, taps, Cp, wp, blockIdx.x, sw, kPrepackSmemFloats, wlo);
}

// A conv call's two input repacks in one launch: blocks [0, n_tiles) move
// NCHW -> NHWC tiles (tiles_p x tiles_c per image), the next Co blocks repack
// the weight (one output channel each).  Shared memory is the transpose
// tile (16.5 KB), which the weight role reuses when one output channel's
// weights fit (Ci*kh*kw <= 4128, else it reads them from global), so 8 CTAs
// fit on an SM.
constexpr int kPrologueSmemFloats = 32 * (kT2Pix + 1);
__global__ void __launch_bounds__(256) conv_prologue_kernel(
    const float* __restrict__ x, int C, int HW, int Cp, int vec, int vec_out,
    float* __restrict__ y, int tiles_p, int tiles_c, int64_t n_tiles,
    const float* __restrict__ w, int taps, float* __restrict__ wp, float* __restrict__ wlo) {
  __shared__ __align__(16) float buf[kPrologueSmemFloats];
  griddep_wait();  // launched with programmatic stream serialization
  griddep_launch_dependents();
  const int64_t b = blockIdx.x;
  if (b < n_tiles) {
    const int64_t per_img = (int64_t)tiles_p * tiles_c;
    const int64_t n = b / per_img;
    const int r = (int)(b - n * per_img);
    const int c_t = r / tiles_p, p_t = r - c_t * tiles_p;
    nchw_to_nhwc_tile(x, C, HW, Cp, vec, vec_out, y, p_t, c_t, n,
                      reinterpret_cast<float (*)[kT2Pix + 1]>(buf));
  } else {
    prepack_weight_block(w, C, taps, Cp, wp, (int)(b - n_tiles), buf, kPrologueSmemFloats, wlo);
  }
}

// B's 3xTF32 low part, out[r][c] = x - trunc_tf32(x) (x = B[r][c]; the
// tensor core reads the raw fp32 B as its truncated TF32 hi part), with the
// padding columns [cols, ldo) zeroed.  One float4 of the output per thread.
__global__ void __launch_bounds__(256) tf32_lo_kernel(const float* __restrict__ b, int64_t rows,
                                                      int64_t cols, int64_t ldb, int vec,
                                                      float* __restrict__ out, int64_t ldo) {
  griddep_wait();  // launched with programmatic stream serialization
  griddep_launch_dependents();
  const int64_t q4 = ldo / 4;
  const int64_t n = rows * q4;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / q4;
    const int64_t c = (i - r * q4) * 4;
    const float* src = b + r * ldb + c;
    float v[4];
    if (vec && c + 4 <= cols) {
      const float4 x = __ldg(reinterpret_cast<const float4*>(src));
      v[0] = x.x; v[1] = x.y; v[2] = x.z; v[3] = x.w;
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) v[j] = c + j < cols ? __ldg(src + j) : 0.0f;
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) v[j] -= __uint_as_float(__float_as_uint(v[j]) & 0xFFFFE000u);
    reinterpret_cast<float4*>(out + r * ldo)[c / 4] = make_float4(v[0], v[1], v[2], v[3]);
  }
}

// ops::max_pool2d semantics (-inf init, padding skipped, strict >).
__global__ void max_pool_nchw_kernel(const float* __restrict__ x, float* __restrict__ y, int64_t N,
                                     int64_t C, int64_t H, int64_t W, int64_t Ho, int64_t Wo,
                                     int kh, int kw, int sh, int sw, int ph, int pw) {
  const int64_t total = N * C * Ho * Wo;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t ow = i % Wo, oh = (i / Wo) % Ho, nc = i / (Wo * Ho);
    const float* xp = x + nc * H * W;
    float m = -INFINITY;
    for (int r = 0; r < kh; ++r) {
      const int64_t hh = oh * sh - ph + r;
      if (hh < 0 || hh >= H) continue;
      for (int s = 0; s < kw; ++s) {
        const int64_t ww = ow * sw - pw + s;
        if (ww < 0 || ww >= W) continue;
        const float v = xp[hh * W + ww];
        if (v > m) m = v;
      }
    }
    y[i] = m;
  }
}

// NHWC variant: one thread per output pixel and 4 consecutive channels
// (16-byte loads/stores, C % 4 == 0), 32-bit index math.
__global__ void max_pool_nhwc4_kernel(const float4* __restrict__ x, float4* __restrict__ y,
                                      int N, int C4, int H, int W, int Ho, int Wo, int kh, int kw,
                                      int sh, int sw, int ph, int pw) {
  griddep_wait();  // launched with programmatic stream serialization
  griddep_launch_dependents();
  const int total = N * Ho * Wo * C4;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const int c = i % C4;
    const int pix = i / C4;
    const int ow = pix % Wo;
    const int oh = (pix / Wo) % Ho;
    const int n = pix / (Wo * Ho);
    float4 m = make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
    for (int r = 0; r < kh; ++r) {
      const int hh = oh * sh - ph + r;
      if (hh < 0 || hh >= H) continue;
      for (int s = 0; s < kw; ++s) {
        const int ww = ow * sw - pw + s;
        if (ww < 0 || ww >= W) continue;
        const float4 v = __ldg(x + ((size_t)(n * H + hh) * W + ww) * C4 + c);
        if (v.x > m.x) m.x = v.x;
        if (v.y > m.y) m.y = v.y;
        if (v.z > m.z) m.z = v.z;
        if (v.w > m.w) m.w = v.w;
      }
    }
    y[i] = m;
  }
}

// 3x3 stride-2 NHWC max pool (ResNet's), C % 4 == 0: a thread owns one 4-channel
// group of one output column and walks a strip of `rows` output rows.  Output
// row oh reads input rows 2oh-ph .. 2oh-ph+2 and the next one starts at the
// last of them, so each row's horizontal maximum over its three columns is
// carried over: 6 float4 loads per output instead of 9.  Taking the maxima
// of each row first, then over the rows in order, with the strict > and the
// -inf start of ops::max_pool2d keeps its result bit for bit (the first
// occurrence of the maximum in row-major window order; NaN never wins).
__device__ __forceinline__ void max4_into(float4& m, const float4 v) {
  if (v.x > m.x) m.x = v.x;
  if (v.y > m.y) m.y = v.y;
  if (v.z > m.z) m.z = v.z;
  if (v.w > m.w) m.w = v.w;
}

__global__ void max_pool3s2_nhwc4_kernel(const float4* __restrict__ x, float4* __restrict__ y,
                                         int N, int C4, int H, int W, int Ho, int Wo, int ph,
                                         int pw, int rows) {
  griddep_wait();  // launched with programmatic stream serialization
  griddep_launch_dependents();
  const int strips = (Ho + rows - 1) / rows;
  const int64_t total = (int64_t)N * strips * Wo * C4;
  const float4 ninf = make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int c = (int)(i % C4);
    int64_t t = i / C4;
    const int ow = (int)(t % Wo);
    t /= Wo;
    const int strip = (int)(t % strips);
    const int n = (int)(t / strips);
    const int iw0 = 2 * ow - pw;
    const bool v0 = iw0 >= 0 && iw0 < W, v1 = iw0 + 1 >= 0 && iw0 + 1 < W,
               v2 = iw0 + 2 >= 0 && iw0 + 2 < W;
    const float4* xn = x + (int64_t)n * H * W * C4 + c;
    // the horizontal maximum of input row hh over the window's columns
    auto hrow = [&](int hh) -> float4 {
      float4 m = ninf;
      if (hh < 0 || hh >= H) return m;
      const float4* xr = xn + (int64_t)hh * W * C4;
      float4 a = ninf, b = ninf, d = ninf;
      if (v0) a = __ldg(xr + (int64_t)iw0 * C4);
      if (v1) b = __ldg(xr + (int64_t)(iw0 + 1) * C4);
      if (v2) d = __ldg(xr + (int64_t)(iw0 + 2) * C4);
      if (v0) max4_into(m, a);
      if (v1) max4_into(m, b);
      if (v2) max4_into(m, d);
      return m;
    };
    const int oh0 = strip * rows;
    const int oh1 = oh0 + rows < Ho ? oh0 + rows : Ho;
    float4 carry = hrow(2 * oh0 - ph);
    float4* yo = y + ((int64_t)n * Ho * Wo + ow) * C4 + c;
    for (int oh = oh0; oh < oh1; ++oh) {
      const int r0 = 2 * oh - ph;
      const float4 a = hrow(r0 + 1);
      const float4 b = hrow(r0 + 2);
      float4 m = ninf;
      max4_into(m, carry);
      max4_into(m, a);
      max4_into(m, b);
      yo[(int64_t)oh * Wo * C4] = m;
      carry = b;
    }
  }
}

// Generic NHWC fallback (any C), one thread per output element.
__global__ void max_pool_nhwc_kernel(const float* __restrict__ x, float* __restrict__ y, int64_t N,
                                     int64_t C, int64_t H, int64_t W, int64_t Ho, int64_t Wo,
                                     int kh, int kw, int sh, int sw, int ph, int pw) {
  const int64_t total = N * Ho * Wo * C;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t c = i % C, ow = (i / C) % Wo, oh = (i / (C * Wo)) % Ho, n = i / (C * Wo * Ho);
    float m = -INFINITY;
    for (int r = 0; r < kh; ++r) {
      const int64_t hh = oh * sh - ph + r;
      if (hh < 0 || hh >= H) continue;
      for (int s = 0; s < kw; ++s) {
        const int64_t ww = ow * sw - pw + s;
        if (ww < 0 || ww >= W) continue;
        const float v = x[((n * H + hh) * W + ww) * C + c];
        if (v > m) m = v;
      }
    }
    y[i] = m;
  }
}

// Global average pool: one warp per (n, c) for NCHW (contiguous HW run);
// NHWC: one thread per (n, c) striding over pixels (coalesced across c).
__global__ void avg_pool_nchw_kernel(const float* __restrict__ x, float* __restrict__ y,
                                     int64_t NC, int64_t HW) {
  const int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= NC) return;
  const float* xp = x + warp * HW;
  double s = 0.0;
  for (int64_t j = lane; j < HW; j += 32) s += (double)xp[j];
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (lane == 0) y[warp] = (float)(s / (double)HW);
}

__global__ void avg_pool_nhwc_kernel(const float* __restrict__ x, float* __restrict__ y, int64_t N,
                                     int64_t C, int64_t HW) {
  griddep_wait();  // launched with programmatic stream serialization
  griddep_launch_dependents();
  const int64_t total = N * C;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t n = i / C, c = i - n * C;
    const float* xp = x + n * HW * C + c;
    double s = 0.0;
    for (int64_t j = 0; j < HW; ++j) s += (double)xp[j * C];
    y[i] = (float)(s / (double)HW);
  }
}

__global__ void add_kernel(const float* __restrict__ a, const float* __restrict__ b,
                           float* __restrict__ y, int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    y[i] = a[i] + b[i];
}

// Rust f32::max(x, 0.0): NaN -> 0.
__global__ void relu_kernel(const float* __restrict__ x, float* __restrict__ y, int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float v = x[i];
    y[i] = (v > 0.0f) ? v : 0.0f;
  }
}

// y[i] = a[.] op b[.] over an n-d output shape with per-operand element
// strides (0 for a broadcast dimension), as ops::add / ops::mul do through
// Tensor::expand (rustorch-core/src/broadcast.rs:23-136).
struct BcastDesc {
  int ndim;
  int64_t shape[8];
  int64_t sa[8];
  int64_t sb[8];
};

__global__ void bcast_kernel(const float* __restrict__ a, const float* __restrict__ b,
                             float* __restrict__ y, int64_t n, BcastDesc d, int op) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    int64_t rem = i, oa = 0, ob = 0;
    for (int k = d.ndim - 1; k >= 0; --k) {
      const int64_t c = rem % d.shape[k];
      rem /= d.shape[k];
      oa += c * d.sa[k];
      ob += c * d.sb[k];
    }
    const float x = a[oa], z = b[ob];
    y[i] = op == 0 ? x + z : x * z;
  }
}

// Failure-detection probe: one thread waits, with the library's bounded wait,
// on an mbarrier that nothing ever arrives on; the wait expires after
// timeout_ns, records DEV_TIMEOUT_PROBE in the error word and the kernel
// returns normally (no trap, no hang).
__global__ void wait_probe_kernel(int* err, unsigned long long timeout_ns) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0)
    mbar_wait_bounded(&bar, 0, reinterpret_cast<volatile int*>(&abort_flag), err,
                      DEV_TIMEOUT_PROBE, timeout_ns);
  __syncthreads();
}

// parts [P, M, Nl] -> C [M, P*Nl].
__global__ void unsplit_cols_kernel(const float* __restrict__ parts, float* __restrict__ C,
                                    int64_t P, int64_t M, int64_t Nl) {
  const int64_t N = P * Nl, total = M * N;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t m = i / N, n = i - m * N;
    const int64_t pr = n / Nl, j = n - pr * Nl;
    C[i] = parts[(pr * M + m) * Nl + j];
  }
}

}  // namespace

int launch_pack_kmajor(const float* src, int64_t rows, int64_t k, int64_t rs, int64_t cs,
                       float* dst, int64_t kp, cudaStream_t s) {
  dim3 grid((unsigned)((kp + 31) / 32), (unsigned)((rows + 31) / 32));
  if (grid.y > 65535) return set_error(RTB_E_UNSUPPORTED, "pack: too many rows");
  clear_stale_cuda_error();
  pack_kmajor_kernel<<<grid, dim3(32, 8), 0, s>>>(src, rows, k, rs, cs, dst, kp);
  return launch_check("pack_kmajor");
}

int launch_fill_rows(float* C, int64_t M, int64_t N, int64_t ldc, const float* bias, int act,
                     cudaStream_t s) {
  clear_stale_cuda_error();
  fill_rows_kernel<<<grid_for(M * N), kThreads, 0, s>>>(C, M, N, ldc, bias, act);
  return launch_check("fill_rows");
}

int launch_nchw_to_nhwc_padded(const float* x, int64_t N, int64_t C, int64_t H, int64_t W,
                               int64_t Cp, float* y, cudaStream_t s) {
  const int64_t HW = H * W;
  if (Cp == 4 && HW < INT32_MAX && (reinterpret_cast<uintptr_t>(y) & 15u) == 0) {
    clear_stale_cuda_error();
    nchw_to_nhwc_c4_kernel<<<grid_for(N * HW), kThreads, 0, s>>>(x, (int)C, (int)HW, N * HW,
                                                                 reinterpret_cast<float4*>(y));
    return launch_check("nchw_to_nhwc (C<=4)");
  }
  if (HW > INT32_MAX || C > INT32_MAX || Cp > INT32_MAX || N > 65535)
    return set_error(RTB_E_UNSUPPORTED, "nchw_to_nhwc: too large");
  dim3 grid((unsigned)((HW + kT2Pix - 1) / kT2Pix), (unsigned)((Cp + 31) / 32), (unsigned)N);
  if (grid.y > 65535) return set_error(RTB_E_UNSUPPORTED, "nchw_to_nhwc: too many channels");
  const int vec = (HW % 4 == 0) && (reinterpret_cast<uintptr_t>(x) & 15u) == 0;
  const int vec_out = (Cp % 4 == 0) && (reinterpret_cast<uintptr_t>(y) & 15u) == 0;
  clear_stale_cuda_error();
  nchw_to_nhwc_kernel<<<grid, 256, 0, s>>>(x, (int)C, (int)HW, (int)Cp, vec, vec_out, y);
  return launch_check("nchw_to_nhwc");
}

int launch_tf32_lo(const float* b, int64_t rows, int64_t cols, int64_t ldb, float* out,
                   int64_t ldo, cudaStream_t s) {
  if (rows <= 0 || cols <= 0 || ldo < cols || ldo % 4 != 0 ||
      (reinterpret_cast<uintptr_t>(out) & 15u) != 0)
    return set_error(RTB_E_INVALID, "tf32_lo: bad arguments");
  const int vec = (ldb % 4 == 0) && (reinterpret_cast<uintptr_t>(b) & 15u) == 0;
  const int64_t n = rows * (ldo / 4);
  const int64_t blocks64 = (n + 255) / 256;
  const unsigned blocks = (unsigned)(blocks64 < 148 * 16 ? blocks64 : 148 * 16);
  clear_stale_cuda_error();
  cudaError_t e = launch_pdl(tf32_lo_kernel, dim3(blocks), dim3(256), 0, s, b, rows, cols, ldb,
                             vec, out, ldo);
  if (e != cudaSuccess) return cuda_status(e, "tf32_lo launch");
  return launch_check("tf32_lo");
}

int launch_conv_prologue(const float* x, int64_t N, int64_t C, int64_t H, int64_t W, int64_t Cp,
                         float* y, const float* w, int64_t Co, int64_t kh, int64_t kw, float* wp,
                         float* wlo, cudaStream_t s) {
  const int64_t HW = H * W, taps = kh * kw;
  if (Cp == 4 || HW > INT32_MAX || C > INT32_MAX || Cp > INT32_MAX || Co > INT32_MAX ||
      C * taps > INT32_MAX || taps * Cp > INT32_MAX) {
    // small-channel inputs keep their own transform kernel
    int st = launch_nchw_to_nhwc_padded(x, N, C, H, W, Cp, y, s);
    return st ? st : launch_prepack_weight(w, Co, C, kh, kw, Cp, wp, wlo, s);
  }
  const int tiles_p = (int)((HW + kT2Pix - 1) / kT2Pix);
  const int tiles_c = (int)((Cp + 31) / 32);
  const int64_t n_tiles = N * tiles_p * tiles_c;
  const int64_t blocks = n_tiles + Co;
  if (blocks > INT32_MAX) return set_error(RTB_E_UNSUPPORTED, "conv prologue: too large");
  const int vec = (HW % 4 == 0) && (reinterpret_cast<uintptr_t>(x) & 15u) == 0;
  const int vec_out = (Cp % 4 == 0) && (reinterpret_cast<uintptr_t>(y) & 15u) == 0;
  clear_stale_cuda_error();
  cudaError_t e = launch_pdl(conv_prologue_kernel, dim3((unsigned)blocks), dim3(256), 0, s, x,
                             (int)C, (int)HW, (int)Cp, vec, vec_out, y, tiles_p, tiles_c, n_tiles,
                             w, (int)taps, wp, wlo);
  if (e != cudaSuccess) return cuda_status(e, "conv prologue launch");
  return launch_check("conv prologue");
}

// Space-to-depth form of a stride-2 conv over an input of at most 4 channels:
//   y[n][hs][ws][(pr*2 + pc)*4 + c] = x[n][c][2*hs + pr - ph][2*ws + pc - pw]
// (zero outside the image, c >= C zero), an NHWC tensor of 16 channels whose
// stride-1, unpadded conv with the kernel
//   w2[co][(R*kw2 + S)][(pr*2 + pc)*4 + c] = w[co][c][2R + pr][2S + pc]
// (zero where 2R + pr >= kh or 2S + pc >= kw), kh2 = ceil(kh/2), equals the
// original conv.  Blocks [0, pix_blocks) write one s2d pixel (64 bytes) per
// thread; the next Co blocks write one output channel's repacked weights.
__global__ void __launch_bounds__(256) conv_prologue_s2d_kernel(
    const float* __restrict__ x, int C, int H, int W, int ph, int pw, int Hs, int Ws,
    int64_t npix, int64_t pix_blocks, float4* __restrict__ y, const float* __restrict__ w,
    int kh, int kw, int kh2, int kw2, float* __restrict__ w2, float* __restrict__ w2lo) {
  griddep_wait();  // launched with programmatic stream serialization
  griddep_launch_dependents();
  const int64_t b = blockIdx.x;
  if (b < pix_blocks) {
    const int64_t i = b * 256 + threadIdx.x;
    if (i >= npix) return;
    const int64_t n = i / ((int64_t)Hs * Ws);
    const int rem = (int)(i - n * Hs * Ws);
    const int hs = rem / Ws, ws = rem - hs * Ws;
    const float* xn = x + n * C * H * W;
    float v[16];
#pragma unroll
    for (int ph2 = 0; ph2 < 4; ++ph2) {
      const int ih = 2 * hs + (ph2 >> 1) - ph, iw = 2 * ws + (ph2 & 1) - pw;
      const bool in = ih >= 0 && ih < H && iw >= 0 && iw < W;
#pragma unroll
      for (int c = 0; c < 4; ++c)
        v[ph2 * 4 + c] = (in && c < C) ? __ldg(xn + ((int64_t)c * H + ih) * W + iw) : 0.0f;
    }
    float4* dst = y + i * 4;
#pragma unroll
    for (int q = 0; q < 4; ++q) dst[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
  } else {
    const int co = (int)(b - pix_blocks);
    const int n_out = kh2 * kw2 * 16;
    for (int k = threadIdx.x; k < n_out; k += 256) {
      const int tap = k >> 4, j = k & 15;
      const int R = tap / kw2, S = tap - R * kw2;
      const int r = 2 * R + (j >> 3), sc = 2 * S + ((j >> 2) & 1), c = j & 3;
      const float v =
          (r < kh && sc < kw && c < C) ? __ldg(w + (((int64_t)co * C + c) * kh + r) * kw + sc) : 0.0f;
      w2[(int64_t)co * n_out + k] = v;
      if (w2lo) w2lo[(int64_t)co * n_out + k] = tf32_lo(v);
    }
  }
}

int launch_conv_prologue_s2d(const float* x, int64_t N, int64_t C, int64_t H, int64_t W,
                             int64_t ph, int64_t pw, int64_t Hs, int64_t Ws, float* y,
                             const float* w, int64_t Co, int64_t kh, int64_t kw, float* w2,
                             float* w2lo, cudaStream_t s) {
  const int64_t npix = N * Hs * Ws;
  const int64_t pix_blocks = (npix + 255) / 256;
  if (C > 4 || H * W > INT32_MAX || Hs * Ws > INT32_MAX || pix_blocks + Co > INT32_MAX ||
      (reinterpret_cast<uintptr_t>(y) & 15u) != 0)
    return set_error(RTB_E_UNSUPPORTED, "conv s2d prologue: unsupported shape");
  clear_stale_cuda_error();
  cudaError_t e = launch_pdl(conv_prologue_s2d_kernel, dim3((unsigned)(pix_blocks + Co)), dim3(256),
                             0, s, x, (int)C, (int)H, (int)W, (int)ph, (int)pw, (int)Hs, (int)Ws,
                             npix, pix_blocks, reinterpret_cast<float4*>(y), w, (int)kh, (int)kw,
                             (int)((kh + 1) / 2), (int)((kw + 1) / 2), w2, w2lo);
  if (e != cudaSuccess) return cuda_status(e, "conv s2d prologue launch");
  return launch_check("conv s2d prologue");
}

int launch_nhwc_to_nchw(const float* x, float* y, int64_t N, int64_t C, int64_t HW,
                        cudaStream_t s) {
  dim3 grid((unsigned)((HW + 31) / 32), (unsigned)((C + 31) / 32), (unsigned)N);
  if (N > 65535 || grid.y > 65535) return set_error(RTB_E_UNSUPPORTED, "nhwc_to_nchw: too large");
  clear_stale_cuda_error();
  nhwc_to_nchw_kernel<<<grid, dim3(32, 8), 0, s>>>(x, C, HW, y);
  return launch_check("nhwc_to_nchw");
}

int launch_prepack_weight(const float* w, int64_t Co, int64_t Ci, int64_t kh, int64_t kw,
                          int64_t Cp, float* wp, float* wlo, cudaStream_t s) {
  const int64_t taps = kh * kw;
  if (Co > INT32_MAX || Ci * taps > INT32_MAX || taps * Cp > INT32_MAX)
    return set_error(RTB_E_UNSUPPORTED, "prepack_weight: too large");
  clear_stale_cuda_error();
  prepack_weight_kernel<<<(unsigned)Co, 256, 0, s>>>(w, (int)Ci, (int)taps, (int)Cp, wp, wlo);
  return launch_check("prepack_weight");
}

int launch_max_pool2d(const float* x, float* y, int64_t N, int64_t C, int64_t H, int64_t W,
                      int64_t kh, int64_t kw, int64_t sh, int64_t sw, int64_t ph, int64_t pw,
                      int layout, cudaStream_t s) {
  const int64_t Ho = (H + 2 * ph - kh) / sh + 1, Wo = (W + 2 * pw - kw) / sw + 1;
  const int64_t total = N * C * Ho * Wo;
  clear_stale_cuda_error();
  if (layout == RTB_LAYOUT_NCHW)
    max_pool_nchw_kernel<<<grid_for(total), kThreads, 0, s>>>(x, y, N, C, H, W, Ho, Wo, (int)kh,
                                                             (int)kw, (int)sh, (int)sw, (int)ph,
                                                             (int)pw);
  else if (C % 4 == 0 && kh == 3 && kw == 3 && sh == 2 && sw == 2 && N < INT32_MAX &&
           H < INT32_MAX && W < INT32_MAX && C / 4 < INT32_MAX &&
           (reinterpret_cast<uintptr_t>(x) & 15u) == 0 && (reinterpret_cast<uintptr_t>(y) & 15u) == 0)
  {
    // strips of 8 output rows: ResNet-18's [256, 112, 112, 64] input gives
    // 1.6M threads, several waves of the SMs
    const int rows = 8;
    const int64_t strips = (Ho + rows - 1) / rows;
    cudaError_t e = launch_pdl(max_pool3s2_nhwc4_kernel,
                               dim3(grid_for(N * strips * Wo * (C / 4))), dim3(kThreads), 0, s,
                               reinterpret_cast<const float4*>(x), reinterpret_cast<float4*>(y),
                               (int)N, (int)(C / 4), (int)H, (int)W, (int)Ho, (int)Wo, (int)ph,
                               (int)pw, rows);
    if (e != cudaSuccess) return cuda_status(e, "max_pool2d launch");
  }
  else if (C % 4 == 0 && total / 4 < INT32_MAX && N * H * W * C < INT32_MAX * 4LL &&
           (reinterpret_cast<uintptr_t>(x) & 15u) == 0 && (reinterpret_cast<uintptr_t>(y) & 15u) == 0)
  {
    cudaError_t e = launch_pdl(max_pool_nhwc4_kernel, dim3(grid_for(total / 4)), dim3(kThreads), 0,
                               s, reinterpret_cast<const float4*>(x), reinterpret_cast<float4*>(y),
                               (int)N, (int)(C / 4), (int)H, (int)W, (int)Ho, (int)Wo, (int)kh,
                               (int)kw, (int)sh, (int)sw, (int)ph, (int)pw);
    if (e != cudaSuccess) return cuda_status(e, "max_pool2d launch");
  }
  else
    max_pool_nhwc_kernel<<<grid_for(total), kThreads, 0, s>>>(x, y, N, C, H, W, Ho, Wo, (int)kh,
                                                             (int)kw, (int)sh, (int)sw, (int)ph,
                                                             (int)pw);
  return launch_check("max_pool2d");
}

int launch_global_avg_pool(const float* x, float* y, int64_t N, int64_t C, int64_t HW, int layout,
                           cudaStream_t s) {
  if (layout == RTB_LAYOUT_NCHW) {
    const int64_t threads = N * C * 32;
    clear_stale_cuda_error();
    avg_pool_nchw_kernel<<<(unsigned)((threads + kThreads - 1) / kThreads), kThreads, 0, s>>>(
        x, y, N * C, HW);
  } else {
    clear_stale_cuda_error();
    cudaError_t e = launch_pdl(avg_pool_nhwc_kernel, dim3(grid_for(N * C)), dim3(kThreads), 0, s,
                               x, y, N, C, HW);
    if (e != cudaSuccess) return cuda_status(e, "global_avg_pool launch");
  }
  return launch_check("global_avg_pool");
}

int launch_add(const float* a, const float* b, float* y, int64_t n, cudaStream_t s) {
  clear_stale_cuda_error();
  add_kernel<<<grid_for(n), kThreads, 0, s>>>(a, b, y, n);
  return launch_check("add");
}

int launch_relu(const float* x, float* y, int64_t n, cudaStream_t s) {
  clear_stale_cuda_error();
  relu_kernel<<<grid_for(n), kThreads, 0, s>>>(x, y, n);
  return launch_check("relu");
}

int launch_broadcast(int op, int ndim, const int64_t* shape, const float* a,
                     const int64_t* sa, const float* b, const int64_t* sb, float* y,
                     cudaStream_t s) {
  if (ndim < 1 || ndim > 8) return set_error(RTB_E_UNSUPPORTED, "broadcast: 1..8 dimensions");
  BcastDesc d;
  d.ndim = ndim;
  int64_t n = 1;
  for (int k = 0; k < ndim; ++k) {
    d.shape[k] = shape[k];
    d.sa[k] = sa[k];
    d.sb[k] = sb[k];
    n *= shape[k];
  }
  if (n == 0) return RTB_OK;
  clear_stale_cuda_error();
  bcast_kernel<<<grid_for(n), kThreads, 0, s>>>(a, b, y, n, d, op);
  return launch_check("broadcast elementwise");
}

int launch_wait_probe(int* err, uint64_t timeout_ns, cudaStream_t s) {
  clear_stale_cuda_error();
  wait_probe_kernel<<<1, 32, 0, s>>>(err, (unsigned long long)timeout_ns);
  return launch_check("wait probe");
}

int launch_unsplit_cols(const float* parts, float* C, int64_t P, int64_t M, int64_t Nl,
                        cudaStream_t s) {
  clear_stale_cuda_error();
  unsplit_cols_kernel<<<grid_for(P * M * Nl), kThreads, 0, s>>>(parts, C, P, M, Nl);
  return launch_check("unsplit_cols");
}

}  // namespace rtb
