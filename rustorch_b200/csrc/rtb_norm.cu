// Row-wise LayerNorm + activation over a row-major [M, N] matrix, in place:
// the second half of matmul_bias_norm_activation (rustorch-core/src/ops.rs:
// 1815-1886, layer_norm at ops/norm.rs:613-700, activations at
// ops/activations.rs).  One 256-thread CTA per row (grid = resident CTAs, rows
// strided): the row is read from HBM once into shared memory (or re-read
// through L2 when it does not fit), the mean and the variance are two passes
// over that copy (sum, then sum of squared deviations, accumulated in double),
// and the normalised, scaled, shifted and activated row is written back with
// streaming stores.  HBM-bound: 8 bytes per element.
#include <cmath>

#include "rtb_internal.h"

namespace rtb {

namespace {

constexpr int kLnThreads = 256;
constexpr int kLnMaxOnChip = 16384;  // rows up to 16384 columns are kept in shared memory (64 KB)

__device__ __forceinline__ double block_sum(double v, double* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();  // red[] free from the previous reduction
  if (l == 0) red[w] = v;
  __syncthreads();
  double t = 0.0;
  if (threadIdx.x < kLnThreads / 32) t = red[threadIdx.x];
  if (w == 0) {
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (l == 0) red[0] = t;
  }
  __syncthreads();
  return red[0];
}

__device__ __forceinline__ float activate(float y, int act) {
  if (act == RTB_ACT_RELU) return fmaxf(y, 0.0f);  // NaN -> 0, as f32::max
  if (act == RTB_ACT_SIGMOID) return 1.0f / (1.0f + expf(-y));
  if (act == RTB_ACT_TANH) return tanhf(y);
  return y;
}

// VEC: the row is read and written as float4 (N % 4 == 0, 16-byte aligned rows).
// ON_CHIP: the row is staged in dynamic shared memory (N <= kLnMaxOnChip);
// otherwise the second and third passes re-read it (from L2).
// X and Y may be the same matrix (in place): every element is read before its
// row's first write.
template <bool VEC, bool ON_CHIP>
__global__ void __launch_bounds__(kLnThreads) layernorm_act_kernel(const float* X, int64_t ldx,
                                                                   float* Y, int64_t ldy,
                                                                   int64_t M, int N,
                                                                   const float* __restrict__ g,
                                                                   const float* __restrict__ b,
                                                                   float eps, int act) {
  extern __shared__ float4 srow4[];
  float* srow = reinterpret_cast<float*>(srow4);
  __shared__ double red[kLnThreads / 32];
  const int n4 = N >> 2;
  for (int64_t m = blockIdx.x; m < M; m += gridDim.x) {
    const float* row = X + m * ldx;
    const float4* row4 = reinterpret_cast<const float4*>(row);
    float* out = Y + m * ldy;
    float4* out4 = reinterpret_cast<float4*>(out);
    double s = 0.0;
    if (VEC) {
      for (int j = threadIdx.x; j < n4; j += kLnThreads) {
        const float4 v = row4[j];
        if (ON_CHIP) srow4[j] = v;
        s += ((double)v.x + (double)v.y) + ((double)v.z + (double)v.w);
      }
    } else {
      for (int j = threadIdx.x; j < N; j += kLnThreads) {
        const float v = row[j];
        if (ON_CHIP) srow[j] = v;
        s += (double)v;
      }
    }
    const double mean = block_sum(s, red) / N;
    double q = 0.0;
    if (VEC) {
      for (int j = threadIdx.x; j < n4; j += kLnThreads) {
        const float4 v = ON_CHIP ? srow4[j] : row4[j];
        const double dx = v.x - mean, dy = v.y - mean, dz = v.z - mean, dw = v.w - mean;
        q += (dx * dx + dy * dy) + (dz * dz + dw * dw);
      }
    } else {
      for (int j = threadIdx.x; j < N; j += kLnThreads) {
        const double d = (double)(ON_CHIP ? srow[j] : row[j]) - mean;
        q += d * d;
      }
    }
    const double var = block_sum(q, red) / N;
    const float inv_std = (float)(1.0 / sqrt(var + (double)eps));
    const float meanf = (float)mean;
    if (VEC) {
      const float4* g4 = reinterpret_cast<const float4*>(g);
      const float4* b4 = reinterpret_cast<const float4*>(b);
      for (int j = threadIdx.x; j < n4; j += kLnThreads) {
        float4 v = ON_CHIP ? srow4[j] : row4[j];
        v.x = (v.x - meanf) * inv_std;
        v.y = (v.y - meanf) * inv_std;
        v.z = (v.z - meanf) * inv_std;
        v.w = (v.w - meanf) * inv_std;
        if (g) {
          const float4 gv = g4[j];
          v.x *= gv.x; v.y *= gv.y; v.z *= gv.z; v.w *= gv.w;
        }
        if (b) {
          const float4 bv = b4[j];
          v.x += bv.x; v.y += bv.y; v.z += bv.z; v.w += bv.w;
        }
        v.x = activate(v.x, act);
        v.y = activate(v.y, act);
        v.z = activate(v.z, act);
        v.w = activate(v.w, act);
        __stcs(out4 + j, v);
      }
    } else {
      for (int j = threadIdx.x; j < N; j += kLnThreads) {
        float y = ((ON_CHIP ? srow[j] : row[j]) - meanf) * inv_std;
        if (g) y *= g[j];
        if (b) y += b[j];
        out[j] = activate(y, act);
      }
    }
    if (ON_CHIP) __syncthreads();  // srow is reused by the next row
  }
}

template <bool VEC, bool ON_CHIP>
int launch_ln(const float* X, int64_t ldx, float* Y, int64_t ldy, int64_t M, int N,
              const float* g, const float* b, float eps, int act, cudaStream_t s) {
  auto* k = layernorm_act_kernel<VEC, ON_CHIP>;
  const size_t smem = ON_CHIP ? (size_t)((N + 3) & ~3) * sizeof(float) : 0;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return cuda_status(e, "layernorm smem attribute");
  }
  int per_sm = 1;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, kLnThreads, smem);
  if (per_sm < 1) per_sm = 1;
  const int64_t cap = (int64_t)sms * per_sm;
  const int64_t blocks = M < cap ? M : cap;
  clear_stale_cuda_error();
  k<<<(unsigned)blocks, kLnThreads, smem, s>>>(X, ldx, Y, ldy, M, N, g, b, eps, act);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? RTB_OK : cuda_status(e, "layernorm kernel launch");
}

}  // namespace

int launch_layernorm_act(const float* X, int64_t ldx, float* Y, int64_t ldy, int64_t M, int64_t N,
                         const float* g, const float* b, float eps, int act, cudaStream_t s) {
  if (M <= 0 || N <= 0) return RTB_OK;
  if (N > INT32_MAX) return set_error(RTB_E_UNSUPPORTED, "layernorm: N too large");
  auto al16 = [](const void* p) { return ((uintptr_t)p & 15) == 0; };
  const bool vec = N % 4 == 0 && ldx % 4 == 0 && ldy % 4 == 0 && al16(X) && al16(Y) &&
                   (!g || al16(g)) && (!b || al16(b));
  const bool on_chip = N <= kLnMaxOnChip;
  if (vec) return on_chip ? launch_ln<true, true>(X, ldx, Y, ldy, M, (int)N, g, b, eps, act, s)
                          : launch_ln<true, false>(X, ldx, Y, ldy, M, (int)N, g, b, eps, act, s);
  return on_chip ? launch_ln<false, true>(X, ldx, Y, ldy, M, (int)N, g, b, eps, act, s)
                 : launch_ln<false, false>(X, ldx, Y, ldy, M, (int)N, g, b, eps, act, s);
}

}  // namespace rtb
