// Layout kernels for the backward contractions (MatmulBackward,
// Conv2dBackward: rustorch-core/src/ops.rs:529-570, ops/conv.rs:336-736).
// The contractions themselves run on the tcgen05 engine:
//   grad_input  = a forward conv of the zero-dilated gradient with the
//                 transposed, flipped filter (stride 1, padding k-1-p);
//   grad_weight = dY^T [Co, P] . im2col(x) [P, R*S*Cp], P = N*Ho*Wo.
// These kernels only move bytes (HBM-bound); 32-bit index math inside an
// image, 64-bit across images.
#include "rtb_internal.h"
#include "rtb_ptx.cuh"

namespace rtb {

namespace {

constexpr int kT = 256;

inline int grid_for(int64_t n) {
  int64_t blocks = (n + kT - 1) / kT;
  if (blocks < 1) blocks = 1;
  if (blocks > 148 * 32) blocks = 148 * 32;
  return (int)blocks;
}

inline int launch_check(const char* what) {
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? RTB_OK : cuda_status(e, what);
}

// dy NCHW [N, Co, Ho, Wo] -> zero-dilated NHWC [N, Hd, Wd, Cop]: element
// (ho, wo, co) lands at (ho*sh, wo*sw, co); the buffer is cleared beforehand,
// so the inserted rows/columns and channels >= Co stay zero.  32 pixels x 32
// channels per tile through shared memory (coalesced read and write).
__global__ void dilate_nchw_to_nhwc_kernel(const float* __restrict__ dy, int Co, int Ho, int Wo,
                                           int sh, int sw, int Hd, int Wd, int Cop,
                                           float* __restrict__ out) {
  griddep_wait();  // launched with programmatic stream serialization
  griddep_launch_dependents();
  __shared__ float tile[32][33];
  const int HoWo = Ho * Wo;
  const int p0 = blockIdx.x * 32, c0 = blockIdx.y * 32;
  const int64_t n = blockIdx.z;
  const float* src = dy + n * Co * (int64_t)HoWo;
  float* dst = out + n * (int64_t)Hd * Wd * Cop;
  const int tx = threadIdx.x, ty = threadIdx.y;  // 32 x 8
  for (int i = ty; i < 32; i += 8) {
    const int c = c0 + i, p = p0 + tx;
    tile[i][tx] = (c < Co && p < HoWo) ? src[(int64_t)c * HoWo + p] : 0.0f;
  }
  __syncthreads();
  for (int i = ty; i < 32; i += 8) {
    const int p = p0 + i, c = c0 + tx;
    if (p < HoWo && c < Co) {
      const int ho = p / Wo, wo = p - ho * Wo;
      dst[((int64_t)ho * sh * Wd + (int64_t)wo * sw) * Cop + c] = tile[tx][i];
    }
  }
}

// w [Co, Ci, R, S] -> wt [Ci, R*S*Cop] with wt[ci][(r*S + s)*Cop + co] =
// w[co][ci][R-1-r][S-1-s]: grad_input's filter as a forward conv (input
// channels = Co, output channels = Ci); co >= Co zero.
__global__ void prepack_flip_kernel(const float* __restrict__ w, int Co, int Ci, int R, int S,
                                    int Cop, float* __restrict__ wt) {
  griddep_wait();  // launched with programmatic stream serialization
  griddep_launch_dependents();
  const int64_t total = (int64_t)Ci * R * S * Cop;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int co = (int)(i % Cop);
    const int64_t t = i / Cop;
    const int tap = (int)(t % (R * S));
    const int ci = (int)(t / (R * S));
    const int r = tap / S, s = tap - r * S;
    wt[i] = co < Co ? w[(((int64_t)co * Ci + ci) * R + (R - 1 - r)) * S + (S - 1 - s)] : 0.0f;
  }
}

// x NHWC [N, H, W, Cp] -> col [P, R*S*Cp], col[p][(r*S + s)*Cp + c] =
// x[n][oh*sh - ph + r][ow*sw - pw + s][c] (zero outside the image), the same
// (tap, channel) order as the forward conv's packed weight.  One block row per
// output pixel p (grid.x strides over P), threads over the row's 16-byte
// groups: both the read (a tap's Cp channels) and the write are contiguous.
__global__ void im2col_nhwc_kernel(const float4* __restrict__ x, int H, int W, int Cp4, int Ho,
                                   int Wo, int R, int S, int sh, int sw, int ph, int pw,
                                   int64_t P, float4* __restrict__ col) {
  griddep_wait();  // launched with programmatic stream serialization
  griddep_launch_dependents();
  const int Kp4 = R * S * Cp4;
  const int HoWo = Ho * Wo;
  for (int64_t p = blockIdx.x; p < P; p += gridDim.x) {
    const int64_t n = p / HoWo;
    const int pix = (int)(p - n * HoWo);
    const int oh = pix / Wo, ow = pix - oh * Wo;
    const float4* xn = x + n * H * W * Cp4;
    float4* dst = col + p * Kp4;
    for (int k4 = threadIdx.x; k4 < Kp4; k4 += blockDim.x) {
      const int tap = k4 / Cp4, c4 = k4 - tap * Cp4;
      const int r = tap / S, s = tap - r * S;
      const int ih = oh * sh - ph + r, iw = ow * sw - pw + s;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (ih >= 0 && ih < H && iw >= 0 && iw < W) v = xn[((int64_t)ih * W + iw) * Cp4 + c4];
      dst[k4] = v;
    }
  }
}

// dy NCHW [N, Co, HW] -> dyt [Co, ldp], dyt[co][n*HW + pix] = dy[n][co][pix]
// (the K-major left operand of grad_weight): one block row per (n, co) plane,
// a contiguous copy.
__global__ void nchw_to_cmajor_kernel(const float* __restrict__ dy, int64_t N, int Co, int HW,
                                      int64_t ldp, float* __restrict__ dyt) {
  griddep_wait();  // launched with programmatic stream serialization
  griddep_launch_dependents();
  const int64_t planes = N * Co;
  for (int64_t pl = blockIdx.x; pl < planes; pl += gridDim.x) {
    const int64_t n = pl / Co;
    const int co = (int)(pl - n * Co);
    const float* src = dy + pl * HW;
    float* dst = dyt + (int64_t)co * ldp + n * HW;
    for (int i = threadIdx.x; i < HW; i += blockDim.x) dst[i] = src[i];
  }
}

// dwp [Co, R*S*Cp] -> dw [Co, Ci, R, S] (added to dw when accumulate).
__global__ void unpack_weight_grad_kernel(const float* __restrict__ dwp, int Co, int Ci, int R,
                                          int S, int Cp, int accumulate, float* __restrict__ dw) {
  griddep_wait();  // launched with programmatic stream serialization
  griddep_launch_dependents();
  const int64_t total = (int64_t)Co * Ci * R * S;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int s = (int)(i % S);
    const int r = (int)((i / S) % R);
    const int ci = (int)((i / ((int64_t)R * S)) % Ci);
    const int64_t co = i / ((int64_t)Ci * R * S);
    const float v = dwp[co * R * S * Cp + (int64_t)(r * S + s) * Cp + ci];
    dw[i] = accumulate ? dw[i] + v : v;
  }
}

}  // namespace

int launch_dilate_nchw_to_nhwc(const float* dy, int64_t N, int64_t Co, int64_t Ho, int64_t Wo,
                               int64_t sh, int64_t sw, int64_t Hd, int64_t Wd, int64_t Cop,
                               float* out, cudaStream_t s) {
  if (N > 65535 || Co > INT32_MAX || Ho * Wo > INT32_MAX || Hd * Wd > INT32_MAX)
    return set_error(RTB_E_UNSUPPORTED, "dilate: too large");
  dim3 grid((unsigned)((Ho * Wo + 31) / 32), (unsigned)((Co + 31) / 32), (unsigned)N);
  if (grid.y > 65535) return set_error(RTB_E_UNSUPPORTED, "dilate: too many channels");
  clear_stale_cuda_error();
  cudaError_t e = launch_pdl(dilate_nchw_to_nhwc_kernel, grid, dim3(32, 8), 0, s, dy, (int)Co,
                             (int)Ho, (int)Wo, (int)sh, (int)sw, (int)Hd, (int)Wd, (int)Cop, out);
  if (e != cudaSuccess) return cuda_status(e, "dilate_nchw_to_nhwc launch");
  return launch_check("dilate_nchw_to_nhwc");
}

int launch_prepack_flip(const float* w, int64_t Co, int64_t Ci, int64_t R, int64_t S, int64_t Cop,
                        float* wt, cudaStream_t s) {
  clear_stale_cuda_error();
  cudaError_t e = launch_pdl(prepack_flip_kernel, dim3(grid_for(Ci * R * S * Cop)), dim3(kT), 0, s,
                             w, (int)Co, (int)Ci, (int)R, (int)S, (int)Cop, wt);
  if (e != cudaSuccess) return cuda_status(e, "prepack_flip launch");
  return launch_check("prepack_flip");
}

int launch_im2col_nhwc(const float* x, int64_t N, int64_t H, int64_t W, int64_t Cp, int64_t Ho,
                       int64_t Wo, int64_t R, int64_t S, int64_t sh, int64_t sw, int64_t ph,
                       int64_t pw, float* col, cudaStream_t s) {
  const int64_t P = N * Ho * Wo;
  if (R * S * (Cp / 4) > INT32_MAX || H * W > INT32_MAX || Ho * Wo > INT32_MAX)
    return set_error(RTB_E_UNSUPPORTED, "im2col: too large");
  const int64_t blocks = P < 148 * 64 ? P : 148 * 64;
  clear_stale_cuda_error();
  cudaError_t e = launch_pdl(im2col_nhwc_kernel, dim3((unsigned)blocks), dim3(128), 0, s,
                             reinterpret_cast<const float4*>(x), (int)H, (int)W, (int)(Cp / 4),
                             (int)Ho, (int)Wo, (int)R, (int)S, (int)sh, (int)sw, (int)ph, (int)pw, P,
                             reinterpret_cast<float4*>(col));
  if (e != cudaSuccess) return cuda_status(e, "im2col_nhwc launch");
  return launch_check("im2col_nhwc");
}

int launch_nchw_to_cmajor(const float* dy, int64_t N, int64_t Co, int64_t HW, int64_t ldp,
                          float* dyt, cudaStream_t s) {
  if (HW > INT32_MAX || Co > INT32_MAX) return set_error(RTB_E_UNSUPPORTED, "nchw_to_cmajor: too large");
  const int64_t planes = N * Co;
  const int64_t blocks = planes < 148 * 64 ? planes : 148 * 64;
  clear_stale_cuda_error();
  cudaError_t e = launch_pdl(nchw_to_cmajor_kernel, dim3((unsigned)blocks), dim3(256), 0, s, dy, N,
                             (int)Co, (int)HW, ldp, dyt);
  if (e != cudaSuccess) return cuda_status(e, "nchw_to_cmajor launch");
  return launch_check("nchw_to_cmajor");
}

int launch_unpack_weight_grad(const float* dwp, int64_t Co, int64_t Ci, int64_t R, int64_t S,
                              int64_t Cp, int accumulate, float* dw, cudaStream_t s) {
  clear_stale_cuda_error();
  cudaError_t e = launch_pdl(unpack_weight_grad_kernel, dim3(grid_for(Co * Ci * R * S)), dim3(kT),
                             0, s, dwp, (int)Co, (int)Ci, (int)R, (int)S, (int)Cp, accumulate, dw);
  if (e != cudaSuccess) return cuda_status(e, "unpack_weight_grad launch");
  return launch_check("unpack_weight_grad");
}

}  // namespace rtb
