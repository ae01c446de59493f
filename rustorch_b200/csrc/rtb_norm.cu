// Row-wise LayerNorm + activation, Y = act(LN(X)) over row-major [M, N]
// matrices (Y may be X):
// the second half of matmul_bias_norm_activation (rustorch-core/src/ops.rs:
// 1815-1886, layer_norm at ops/norm.rs:613-700, activations at
// ops/activations.rs).  HBM-bound: 8 bytes per element (read once, written
// once); the mean and the variance are two passes over an on-chip copy of the
// row (sum, then sum of squared deviations).
//   float4-aligned rows of up to 16384 columns (scalar rows up to 512): the
//     row in registers of a group of 32..256 threads (up to 64 values per
//     thread), reductions by shuffles and the group's named barrier; all of a
//     row's loads are issued before its first reduction, so many rows are in
//     flight per SM;
//   other rows: one 256-thread CTA per row, block reductions in double, the
//     row staged in shared memory (or re-read through L2 beyond 16384).
// Both grids are the resident CTAs with rows strided over them; the output is
// written with streaming stores.
#include <cmath>

#include "rtb_act.cuh"
#include "rtb_internal.h"
#include "rtb_ptx.cuh"

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

__device__ __forceinline__ double warp_sum(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// A group of T threads (32..256, whole warps) per row, the row in registers:
// E (4..64) elements per thread, thread t of the group holding columns
// t + T*i (scalar) or float4 groups t + T*i (VEC).  A 256-thread CTA works on
// 256/T rows at once.  Per-thread partial sums in fp32 (at most 64 terms),
// combined in double by shuffles and, across the group's warps, through
// shared memory and the group's named barrier (ids 1..8).
template <int T, int E, bool VEC>
__global__ void __launch_bounds__(256) layernorm_act_rows_kernel(const float* X, int64_t ldx,
                                                                 float* Y, int64_t ldy,
                                                                 int64_t M, int N,
                                                                 const float* __restrict__ g,
                                                                 const float* __restrict__ b,
                                                                 float eps, int act) {
  constexpr int G = VEC ? E / 4 : E;  // loads per thread
  constexpr int R = 256 / T;          // rows per CTA
  constexpr int W = T / 32;           // warps per row
  __shared__ double red_s[R][W], red_q[R][W];
  griddep_wait();  // launched with programmatic stream serialization
  griddep_launch_dependents();
  const int t = threadIdx.x % T, grp = threadIdx.x / T, w = t >> 5;
  const int64_t groups = (int64_t)gridDim.x * R;
  const int units = VEC ? (N >> 2) : N;
  auto group_sum = [&](double v, double (*red)[W]) -> double {
    v = warp_sum(v);
    if (W == 1) return v;
    if ((t & 31) == 0) red[grp][w] = v;
    asm volatile("bar.sync %0, %1;" ::"r"(1 + grp), "r"(T) : "memory");
    double tot = 0.0;
#pragma unroll
    for (int k = 0; k < W; ++k) tot += red[grp][k];
    return tot;
  };
  for (int64_t m = (int64_t)blockIdx.x * R + grp; m < M; m += groups) {
    float v[E];
    const float* row = X + m * ldx;
#pragma unroll
    for (int i = 0; i < G; ++i) {
      const int u = t + T * i;
      if (VEC) {
        float4 x4 = make_float4(0.f, 0.f, 0.f, 0.f);
        if (u < units) x4 = reinterpret_cast<const float4*>(row)[u];
        v[4 * i] = x4.x; v[4 * i + 1] = x4.y; v[4 * i + 2] = x4.z; v[4 * i + 3] = x4.w;
      } else {
        v[i] = u < units ? row[u] : 0.0f;
      }
    }
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < E; ++i) s += v[i];
    const float meanf = (float)(group_sum((double)s, red_s) / N);
    float q = 0.0f;
#pragma unroll
    for (int i = 0; i < G; ++i) {
      const int u = t + T * i;
      if (u < units) {
#pragma unroll
        for (int c = 0; c < E / G; ++c) {
          const float d = v[i * (E / G) + c] - meanf;
          q = fmaf(d, d, q);
        }
      }
    }
    const double var = group_sum((double)q, red_q) / N;
    const float inv_std = (float)(1.0 / sqrt(var + (double)eps));
    float* out = Y + m * ldy;
#pragma unroll
    for (int i = 0; i < G; ++i) {
      const int u = t + T * i;
      if (u >= units) continue;
      if (VEC) {
        float4 o;
        float* ov = &o.x;
        const float4 gv = g ? reinterpret_cast<const float4*>(g)[u] : make_float4(1.f, 1.f, 1.f, 1.f);
        const float4 bv = b ? reinterpret_cast<const float4*>(b)[u] : make_float4(0.f, 0.f, 0.f, 0.f);
        const float* gp = &gv.x;
        const float* bp = &bv.x;
#pragma unroll
        for (int c = 0; c < 4; ++c)
          ov[c] = activate((v[4 * i + c] - meanf) * inv_std * gp[c] + bp[c], act);
        __stcs(reinterpret_cast<float4*>(out) + u, o);
      } else {
        float y = (v[i] - meanf) * inv_std;
        if (g) y *= g[u];
        if (b) y += b[u];
        out[u] = activate(y, act);
      }
    }
  }
}

// One 256-thread CTA per row.  X and Y may be the same matrix (in place):
// every element is read before its row's first write.
// VEC: the row is read and written as float4 (N % 4 == 0, 16-byte aligned rows).
// ON_CHIP: the row is staged in dynamic shared memory (N <= kLnMaxOnChip);
// otherwise the second and third passes re-read it (from L2).
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
  griddep_wait();  // launched with programmatic stream serialization
  griddep_launch_dependents();
  const int n4 = N >> 2;
  for (int64_t m = blockIdx.x; m < M; m += gridDim.x) {
    const float* row = X + m * ldx;
    const float4* row4 = reinterpret_cast<const float4*>(row);
    float* out = Y + m * ldy;
    float4* out4 = reinterpret_cast<float4*>(out);
    double s = 0.0;
    if (VEC) {
      #pragma unroll 4
      for (int j = threadIdx.x; j < n4; j += kLnThreads) {
        const float4 v = row4[j];
        if (ON_CHIP) srow4[j] = v;
        s += ((double)v.x + (double)v.y) + ((double)v.z + (double)v.w);
      }
    } else {
      #pragma unroll 4
      for (int j = threadIdx.x; j < N; j += kLnThreads) {
        const float v = row[j];
        if (ON_CHIP) srow[j] = v;
        s += (double)v;
      }
    }
    const double mean = block_sum(s, red) / N;
    double q = 0.0;
    if (VEC) {
      #pragma unroll 4
      for (int j = threadIdx.x; j < n4; j += kLnThreads) {
        const float4 v = ON_CHIP ? srow4[j] : row4[j];
        const double dx = v.x - mean, dy = v.y - mean, dz = v.z - mean, dw = v.w - mean;
        q += (dx * dx + dy * dy) + (dz * dz + dw * dw);
      }
    } else {
      #pragma unroll 4
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
      #pragma unroll 4
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
      #pragma unroll 4
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
  cudaError_t e = launch_pdl(k, dim3((unsigned)blocks), dim3(kLnThreads), smem, s, X, ldx, Y, ldy,
                             M, N, g, b, eps, act);
  if (e == cudaSuccess) e = cudaGetLastError();
  return e == cudaSuccess ? RTB_OK : cuda_status(e, "layernorm kernel launch");
}

template <int T, int E, bool VEC>
int launch_ln_rows(rtb_ctx* ctx, const float* X, int64_t ldx, float* Y, int64_t ldy, int64_t M,
                   int N, const float* g, const float* b, float eps, int act, cudaStream_t s) {
  auto* k = layernorm_act_rows_kernel<T, E, VEC>;
  int per_sm = 1;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, 256, 0);
  if (per_sm < 1) per_sm = 1;
  const int64_t need = (M + 256 / T - 1) / (256 / T);
  const int64_t cap = (int64_t)ctx->sm_count * per_sm;
  const int64_t blocks = need < cap ? need : cap;
  clear_stale_cuda_error();
  cudaError_t e = launch_pdl(k, dim3((unsigned)blocks), dim3(256), 0, s, X, ldx, Y, ldy, M, N, g, b,
                             eps, act);
  if (e == cudaSuccess) e = cudaGetLastError();
  return e == cudaSuccess ? RTB_OK : cuda_status(e, "layernorm (rows) kernel launch");
}

}  // namespace

int launch_layernorm_act(rtb_ctx* ctx, const float* X, int64_t ldx, float* Y, int64_t ldy,
                         int64_t M, int64_t N, const float* g, const float* b, float eps, int act,
                         cudaStream_t s) {
  if (M <= 0 || N <= 0) return RTB_OK;
  if (N > INT32_MAX) return set_error(RTB_E_UNSUPPORTED, "layernorm: N too large");
  auto al16 = [](const void* p) { return ((uintptr_t)p & 15) == 0; };
  const bool vec = N % 4 == 0 && ldx % 4 == 0 && ldy % 4 == 0 && al16(X) && al16(Y) &&
                   (!g || al16(g)) && (!b || al16(b));
  const int n = (int)N;
  if (vec && N <= 16384) {  // T threads per row, up to 16 float4 per thread, in registers
    const int per = (int)((N / 4 + 31) / 32);  // float4 per lane of one warp
    if (per <= 1) return launch_ln_rows<32, 4, true>(ctx, X, ldx, Y, ldy, M, n, g, b, eps, act, s);
    if (per <= 2) return launch_ln_rows<32, 8, true>(ctx, X, ldx, Y, ldy, M, n, g, b, eps, act, s);
    if (per <= 4) return launch_ln_rows<32, 16, true>(ctx, X, ldx, Y, ldy, M, n, g, b, eps, act, s);
    if (per <= 8) return launch_ln_rows<32, 32, true>(ctx, X, ldx, Y, ldy, M, n, g, b, eps, act, s);
    if (per <= 16) return launch_ln_rows<64, 32, true>(ctx, X, ldx, Y, ldy, M, n, g, b, eps, act, s);
    if (per <= 32) return launch_ln_rows<128, 32, true>(ctx, X, ldx, Y, ldy, M, n, g, b, eps, act, s);
    if (per <= 64) return launch_ln_rows<256, 32, true>(ctx, X, ldx, Y, ldy, M, n, g, b, eps, act, s);
    return launch_ln_rows<256, 64, true>(ctx, X, ldx, Y, ldy, M, n, g, b, eps, act, s);
  }
  if (!vec && N <= 512) {  // one warp per row, scalar
    const int per = (int)((N + 31) / 32);
    if (per <= 4) return launch_ln_rows<32, 4, false>(ctx, X, ldx, Y, ldy, M, n, g, b, eps, act, s);
    if (per <= 8) return launch_ln_rows<32, 8, false>(ctx, X, ldx, Y, ldy, M, n, g, b, eps, act, s);
    return launch_ln_rows<32, 16, false>(ctx, X, ldx, Y, ldy, M, n, g, b, eps, act, s);
  }
  // a CTA per row: float4-aligned rows beyond 16384 columns (re-read through
  // L2), other rows staged in shared memory up to 16384 columns
  if (vec) return launch_ln<true, false>(X, ldx, Y, ldy, M, n, g, b, eps, act, s);
  return N <= kLnMaxOnChip ? launch_ln<false, true>(X, ldx, Y, ldy, M, n, g, b, eps, act, s)
                           : launch_ln<false, false>(X, ldx, Y, ldy, M, n, g, b, eps, act, s);
}

}  // namespace rtb
