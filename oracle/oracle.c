/*
 * ORACLE — test infrastructure only.
 *
 * A plain-C restatement of RusTorch's CPU dense-contraction path, used as the
 * parity checker for the B200 kernels and as the timed CPU baseline.  Nothing
 * in the product (rustorch_b200/) links or calls this file; only tests/,
 * __graft_entry__.smoke() and bench.py's cpu_baseline / reference arm do.
 *
 * Every function cites the reference file:line it restates (paths relative to
 * the RusTorch project root).  The reference is Rust and no Rust toolchain is
 * available, so the reference itself cannot be built; this restatement is
 * pinned against the reference's own known-answer tests (tests/golden/).
 *
 * Numerics notes
 *  - matmul_cpu_parallel_core (rustorch-core/src/ops.rs:1204-1236) is restated
 *    bit-exactly: sequential f32 sum, unrolled x8, no FMA contraction (Rust does
 *    not contract a*b+c).  This file is compiled with -ffp-contract=off.
 *  - matrixmultiply 0.3.10 sgemm (called at rustorch-core/src/ops.rs:1099-1114)
 *    is a third-party crate not vendored in the reference.  Its published
 *    algorithm is a BLIS-style blocked GEMM: the k dimension is split into
 *    KC=256 blocks, each block's contribution is an f32 FMA chain over k
 *    (fused multiply-add microkernel on FMA-capable x86), and blocks are
 *    accumulated into C left to right (beta=0 for the first block, then C+=).
 *    orc_sgemm_mm restates that per-element summation order; bit-exactness with
 *    the crate is unpinned (the crate is absent).
 *  - The direct conv (rustorch-core/src/ops/conv.rs:156-205) accumulates in f64,
 *    restated exactly.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define ORC_API __attribute__((visibility("default")))

/* ------------------------------------------------------------------------ */
/* PRNG                                                                      */
/* ------------------------------------------------------------------------ */

/* SplitMix64 finaliser, as in the reference's deterministic_unit
 * (demo_visual/src/bin/bench_alignment_ci.rs:12-20). */
static inline uint64_t orc_splitmix_fin(uint64_t x) {
  x ^= x >> 30;
  x *= 0xBF58476D1CE4E5B9ULL;
  x ^= x >> 27;
  x *= 0x94D049BB133111EBULL;
  x ^= x >> 31;
  return x;
}

/* Stream key for (seed, tensor id): one SplitMix64 step of seed, offset by id. */
ORC_API uint64_t orc_stream_key(uint64_t seed, uint64_t tensor_id) {
  return orc_splitmix_fin(seed * 0x9E3779B97F4A7C15ULL + tensor_id * 0xD1B54A32D192ED03ULL + 1ULL);
}

/* 64-bit draw number idx of stream key. */
static inline uint64_t orc_draw(uint64_t key, uint64_t idx) {
  return orc_splitmix_fin(idx + key * 0x9E3779B97F4A7C15ULL);
}

/* The reference's deterministic_unit(idx, seed) verbatim in meaning:
 * (u32)(splitmix(idx + seed*golden)) / u32::MAX, computed in f32. */
ORC_API float orc_unit(uint64_t idx, uint64_t seed) {
  uint64_t x = orc_splitmix_fin(idx + seed * 0x9E3779B97F4A7C15ULL);
  return (float)(uint32_t)x / (float)UINT32_MAX;
}

/* U(lo, hi): lo + (hi - lo) * u, u = (top 24 bits of draw i + 0.5) / 2^24. */
ORC_API void orc_fill_uniform(float* out, int64_t n, uint64_t seed, uint64_t tensor_id, float lo,
                              float hi) {
  const uint64_t key = orc_stream_key(seed, tensor_id);
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) {
    const uint64_t d = orc_draw(key, (uint64_t)i);
    const double u = ((double)(d >> 40) + 0.5) * (1.0 / 16777216.0);
    out[i] = (float)((double)lo + ((double)hi - (double)lo) * u);
  }
}

/* N(mean, std) by Box-Muller on pairs: element 2j uses cos, 2j+1 uses sin of
 * draws (2j, 2j+1) of the stream; u1 = (top 53 bits + 0.5) / 2^53. */
ORC_API void orc_fill_normal(float* out, int64_t n, uint64_t seed, uint64_t tensor_id, float mean,
                             float stdv) {
  const uint64_t key = orc_stream_key(seed, tensor_id);
  const int64_t npairs = (n + 1) / 2;
#pragma omp parallel for schedule(static)
  for (int64_t j = 0; j < npairs; ++j) {
    const uint64_t d1 = orc_draw(key, (uint64_t)(2 * j));
    const uint64_t d2 = orc_draw(key, (uint64_t)(2 * j + 1));
    const double u1 = ((double)(d1 >> 11) + 0.5) * (1.0 / 9007199254740992.0);
    const double u2 = ((double)(d2 >> 11) + 0.5) * (1.0 / 9007199254740992.0);
    const double r = sqrt(-2.0 * log(u1));
    const double t = 6.283185307179586476925286766559 * u2;
    out[2 * j] = (float)((double)mean + (double)stdv * r * cos(t));
    if (2 * j + 1 < n) out[2 * j + 1] = (float)((double)mean + (double)stdv * r * sin(t));
  }
}

/* ------------------------------------------------------------------------ */
/* Helpers                                                                   */
/* ------------------------------------------------------------------------ */

static void orc_set_threads(int nthreads) {
#ifdef _OPENMP
  if (nthreads > 0) omp_set_num_threads(nthreads);
#else
  (void)nthreads;
#endif
}

ORC_API int orc_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

/* Tensor::contiguous of a 2-D strided view (rustorch-core/src/ops/view.rs:113-178). */
static float* orc_contig2d(const float* src, int64_t rows, int64_t cols, int64_t rs, int64_t cs) {
  float* dst = (float*)malloc((size_t)(rows * cols) * sizeof(float));
  if (!dst) return NULL;
  for (int64_t i = 0; i < rows; ++i)
    for (int64_t j = 0; j < cols; ++j) dst[i * cols + j] = src[i * rs + j * cs];
  return dst;
}

/* ------------------------------------------------------------------------ */
/* GEMM                                                                      */
/* ------------------------------------------------------------------------ */

#define ORC_KC 256
#define ORC_MR 8
#define ORC_NR 8

/* matrixmultiply::sgemm restatement (call site rustorch-core/src/ops.rs:1099-1114,
 * alpha=1, beta=0, C row-major with ldc=n).  C[i,j] = sum over KC=256 k-blocks,
 * left to right, of fma-chains over the block.  Packed MRxNR = 8x8 register
 * blocking with an AVX2/FMA microkernel (one 8-wide accumulator per row, an FMA
 * per k step), as the crate's x86 FMA kernel does; the per-element summation
 * order is independent of the tiling.  Rows [r0, r1) only, so the all-cores
 * variant can split rows without changing numerics. */
#if defined(__AVX2__) && defined(__FMA__)
#include <immintrin.h>
#endif
#define ORC_MC 64
#define ORC_NC 512
static void orc_sgemm_rows(int64_t r0, int64_t r1, int64_t k, int64_t n, const float* A, int64_t rsa,
                           int64_t csa, const float* B, int64_t rsb, int64_t csb, float* C) {
  float* bpack = (float*)aligned_alloc(64, (size_t)ORC_KC * ORC_NC * sizeof(float));
  float* apack = (float*)aligned_alloc(64, (size_t)ORC_KC * ORC_MC * sizeof(float));
  for (int64_t j1 = 0; j1 < n; j1 += ORC_NC) {
    const int64_t nc = (n - j1) < ORC_NC ? (n - j1) : ORC_NC;
    const int64_t npan = (nc + ORC_NR - 1) / ORC_NR;
    for (int64_t k0 = 0; k0 < k; k0 += ORC_KC) {
      const int64_t kb = (k - k0) < ORC_KC ? (k - k0) : ORC_KC;
      /* B[k0:k0+kb, j1:j1+nc] -> panels of NR columns, p-major inside a panel */
      for (int64_t jp = 0; jp < npan; ++jp)
        for (int64_t p = 0; p < kb; ++p)
          for (int64_t jj = 0; jj < ORC_NR; ++jj) {
            const int64_t j = j1 + jp * ORC_NR + jj;
            bpack[(jp * kb + p) * ORC_NR + jj] = j < j1 + nc ? B[(k0 + p) * rsb + j * csb] : 0.0f;
          }
      for (int64_t i1 = r0; i1 < r1; i1 += ORC_MC) {
        const int64_t mc = (r1 - i1) < ORC_MC ? (r1 - i1) : ORC_MC;
        const int64_t mpan = (mc + ORC_MR - 1) / ORC_MR;
        for (int64_t ip = 0; ip < mpan; ++ip)
          for (int64_t p = 0; p < kb; ++p)
            for (int64_t ii = 0; ii < ORC_MR; ++ii) {
              const int64_t i = i1 + ip * ORC_MR + ii;
              apack[(ip * kb + p) * ORC_MR + ii] = i < i1 + mc ? A[i * rsa + (k0 + p) * csa] : 0.0f;
            }
        for (int64_t jp = 0; jp < npan; ++jp) {
          const float* bp0 = bpack + jp * kb * ORC_NR;
          const int64_t j0 = j1 + jp * ORC_NR;
          const int64_t nj = (j1 + nc - j0) < ORC_NR ? (j1 + nc - j0) : ORC_NR;
          for (int64_t ip = 0; ip < mpan; ++ip) {
            const float* ap0 = apack + ip * kb * ORC_MR;
            const int64_t i0 = i1 + ip * ORC_MR;
            const int64_t mi = (i1 + mc - i0) < ORC_MR ? (i1 + mc - i0) : ORC_MR;
            float acc[ORC_MR][ORC_NR] __attribute__((aligned(32)));
#if defined(__AVX2__) && defined(__FMA__)
            __m256 c0 = _mm256_setzero_ps(), c1 = c0, c2 = c0, c3 = c0, c4 = c0, c5 = c0,
                   c6 = c0, c7 = c0;
            for (int64_t p = 0; p < kb; ++p) {
              const __m256 bv = _mm256_load_ps(bp0 + p * ORC_NR);
              const float* ap = ap0 + p * ORC_MR;
              c0 = _mm256_fmadd_ps(_mm256_broadcast_ss(ap + 0), bv, c0);
              c1 = _mm256_fmadd_ps(_mm256_broadcast_ss(ap + 1), bv, c1);
              c2 = _mm256_fmadd_ps(_mm256_broadcast_ss(ap + 2), bv, c2);
              c3 = _mm256_fmadd_ps(_mm256_broadcast_ss(ap + 3), bv, c3);
              c4 = _mm256_fmadd_ps(_mm256_broadcast_ss(ap + 4), bv, c4);
              c5 = _mm256_fmadd_ps(_mm256_broadcast_ss(ap + 5), bv, c5);
              c6 = _mm256_fmadd_ps(_mm256_broadcast_ss(ap + 6), bv, c6);
              c7 = _mm256_fmadd_ps(_mm256_broadcast_ss(ap + 7), bv, c7);
            }
            _mm256_store_ps(acc[0], c0); _mm256_store_ps(acc[1], c1);
            _mm256_store_ps(acc[2], c2); _mm256_store_ps(acc[3], c3);
            _mm256_store_ps(acc[4], c4); _mm256_store_ps(acc[5], c5);
            _mm256_store_ps(acc[6], c6); _mm256_store_ps(acc[7], c7);
#else
            memset(acc, 0, sizeof(acc));
            for (int64_t p = 0; p < kb; ++p)
              for (int64_t ii = 0; ii < ORC_MR; ++ii)
                for (int64_t jj = 0; jj < ORC_NR; ++jj)
                  acc[ii][jj] = fmaf(ap0[p * ORC_MR + ii], bp0[p * ORC_NR + jj], acc[ii][jj]);
#endif
            for (int64_t ii = 0; ii < mi; ++ii)
              for (int64_t jj = 0; jj < nj; ++jj) {
                float* c = &C[(i0 + ii) * n + (j0 + jj)];
                *c = (k0 == 0) ? acc[ii][jj] : (*c + acc[ii][jj]);
              }
          }
        }
      }
    }
  }
  free(apack);
  free(bpack);
}

/* Single-threaded, as the reference's matrixmultiply build has no threading
 * feature (Cargo.lock:1258-1265).  nthreads > 1 gives the all-cores variant
 * used only as an extra, stronger CPU baseline (same numerics). */
ORC_API void orc_sgemm_mm(int64_t m, int64_t k, int64_t n, const float* A, int64_t rsa, int64_t csa,
                          const float* B, int64_t rsb, int64_t csb, float* C, int nthreads) {
  if (k == 0) {
    memset(C, 0, (size_t)(m * n) * sizeof(float));
    return;
  }
  if (nthreads <= 1) {
    orc_sgemm_rows(0, m, k, n, A, rsa, csa, B, rsb, csb, C);
    return;
  }
  orc_set_threads(nthreads);
  const int64_t chunk = 64;
#pragma omp parallel for schedule(dynamic, 1)
  for (int64_t r0 = 0; r0 < m; r0 += chunk) {
    const int64_t r1 = (r0 + chunk) < m ? (r0 + chunk) : m;
    orc_sgemm_rows(r0, r1, k, n, A, rsa, csa, B, rsb, csb, C);
  }
}

/* matmul_cpu_parallel_core (rustorch-core/src/ops.rs:1204-1236), bit-exact:
 * per output sum starts at bias[j] (or 0), then sequential f32 mul+add over k
 * unrolled by 8 (same order), contiguous A[m,k], B[k,n]. */
ORC_API void orc_matmul_parallel_core(int64_t m, int64_t k, int64_t n, const float* A,
                                      const float* B, const float* bias, float* C, int nthreads) {
  orc_set_threads(nthreads);
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < m; ++i) {
    const float* a = A + i * k;
    for (int64_t j = 0; j < n; ++j) {
      float sum = bias ? bias[j] : 0.0f;
      int64_t p = 0;
      while (p + 8 <= k) {
        sum += a[p] * B[p * n + j];
        sum += a[p + 1] * B[(p + 1) * n + j];
        sum += a[p + 2] * B[(p + 2) * n + j];
        sum += a[p + 3] * B[(p + 3) * n + j];
        sum += a[p + 4] * B[(p + 4) * n + j];
        sum += a[p + 5] * B[(p + 5) * n + j];
        sum += a[p + 6] * B[(p + 6) * n + j];
        sum += a[p + 7] * B[(p + 7) * n + j];
        p += 8;
      }
      while (p < k) {
        sum += a[p] * B[p * n + j];
        p += 1;
      }
      C[i * n + j] = sum;
    }
  }
}

/* should_use_parallel_auto (rustorch-core/src/ops.rs:1075-1078) with the
 * default thresholds of cpu_matmul_config (ops.rs:1050-1073). */
ORC_API int orc_matmul_auto_parallel(int64_t m, int64_t k, int64_t n) {
  return (m >= 128 && k >= 256 && n <= 128) ? 1 : 0;
}

/* ops::matmul CPU branch (rustorch-core/src/ops.rs:1888-2066): make inputs
 * contiguous, choose kernel by the auto rule, run it.  Returns the choice
 * (0 = sgemm, 1 = parallel core), or -1 on allocation failure. */
ORC_API int orc_matmul(int64_t m, int64_t k, int64_t n, const float* A, int64_t rsa, int64_t csa,
                       const float* B, int64_t rsb, int64_t csb, const float* bias, float* C,
                       int nthreads) {
  const int contig_a = (csa == 1 && rsa == k);
  const int contig_b = (csb == 1 && rsb == n);
  float* a = contig_a ? (float*)A : orc_contig2d(A, m, k, rsa, csa);
  float* b = contig_b ? (float*)B : orc_contig2d(B, k, n, rsb, csb);
  if (!a || !b) return -1;
  const int par = orc_matmul_auto_parallel(m, k, n);
  if (par) {
    orc_matmul_parallel_core(m, k, n, a, b, bias, C, nthreads);
  } else {
    orc_sgemm_mm(m, k, n, a, k, 1, b, n, 1, C, 1);
    if (bias) /* matmul_cpu_sgemm_core bias: per row v += b[j] (ops.rs:1116-1122) */
      for (int64_t i = 0; i < m; ++i)
        for (int64_t j = 0; j < n; ++j) C[i * n + j] += bias[j];
  }
  if (!contig_a) free(a);
  if (!contig_b) free(b);
  return par;
}

/* f64-accumulated truth GEMM for error metrics (not a reference kernel). */
ORC_API void orc_matmul_f64(int64_t m, int64_t k, int64_t n, const float* A, int64_t rsa,
                            int64_t csa, const float* B, int64_t rsb, int64_t csb, double* C,
                            int nthreads) {
  orc_set_threads(nthreads);
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < m; ++i) {
    double* c = C + i * n;
    for (int64_t j = 0; j < n; ++j) c[j] = 0.0;
    for (int64_t p = 0; p < k; ++p) {
      const double a = (double)A[i * rsa + p * csa];
      const float* b = B + p * rsb;
      if (csb == 1)
        for (int64_t j = 0; j < n; ++j) c[j] += a * (double)b[j];
      else
        for (int64_t j = 0; j < n; ++j) c[j] += a * (double)b[j * csb];
    }
  }
}

/* f64 truth for a sampled subset of output entries: C[rows[t], cols[t]]. */
ORC_API void orc_matmul_f64_sampled(int64_t k, const float* A, int64_t rsa, int64_t csa,
                                    const float* B, int64_t rsb, int64_t csb, const int64_t* rows,
                                    const int64_t* cols, int64_t count, double* out, int nthreads) {
  orc_set_threads(nthreads);
#pragma omp parallel for schedule(static)
  for (int64_t t = 0; t < count; ++t) {
    double s = 0.0;
    for (int64_t p = 0; p < k; ++p)
      s += (double)A[rows[t] * rsa + p * csa] * (double)B[p * rsb + cols[t] * csb];
    out[t] = s;
  }
}

/* ------------------------------------------------------------------------ */
/* Elementwise                                                               */
/* ------------------------------------------------------------------------ */

/* ops::relu (rustorch-core/src/ops.rs:449-491): x.max(0.0). Rust's f32::max
 * returns the non-NaN operand, so NaN -> 0. */
ORC_API void orc_relu(float* x, int64_t n) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) {
    const float v = x[i];
    x[i] = (v != v) ? 0.0f : (v > 0.0f ? v : 0.0f);
  }
}

/* Broadcast add of bias [1,C,1,1] onto NCHW output (rustorch-nn/src/conv.rs:52-63
 * via ops::add broadcast, rustorch-core/src/ops.rs:223-291): y += b[c]. */
ORC_API void orc_add_bias_nchw(float* y, const float* bias, int64_t n, int64_t c, int64_t hw) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n * c; ++i) {
    const float b = bias[i % c];
    float* p = y + i * hw;
    for (int64_t j = 0; j < hw; ++j) p[j] = p[j] + b;
  }
}

/* Row-broadcast add of bias [n] onto a [m,n] matrix (Linear::forward,
 * rustorch-nn/src/linear.rs:75-95). */
ORC_API void orc_add_bias_rows(float* y, const float* bias, int64_t m, int64_t n) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < m; ++i)
    for (int64_t j = 0; j < n; ++j) y[i * n + j] = y[i * n + j] + bias[j];
}

/* Same-shape add (rustorch-core/src/ops.rs:223-291). */
ORC_API void orc_add(const float* a, const float* b, float* out, int64_t n) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) out[i] = a[i] + b[i];
}

/* ------------------------------------------------------------------------ */
/* Conv2d                                                                    */
/* ------------------------------------------------------------------------ */

/* conv2d_direct_core (rustorch-core/src/ops/conv.rs:156-205): f64 accumulate in
 * (ci, kh, kw) order, zero padding by bounds check, cast to f32. */
ORC_API void orc_conv2d_direct(int64_t n, int64_t ci, int64_t h, int64_t w, int64_t co, int64_t kh,
                               int64_t kw, int64_t sh, int64_t sw, int64_t ph, int64_t pw,
                               const float* x, const float* wt, float* y, int nthreads) {
  const int64_t ho = (h + 2 * ph - kh) / sh + 1;
  const int64_t wo = (w + 2 * pw - kw) / sw + 1;
  const int64_t total = n * co * ho * wo;
  orc_set_threads(nthreads);
#pragma omp parallel for schedule(static)
  for (int64_t idx = 0; idx < total; ++idx) {
    const int64_t o_w = idx % wo;
    const int64_t o_h = (idx / wo) % ho;
    const int64_t c_o = (idx / (wo * ho)) % co;
    const int64_t b = idx / (wo * ho * co);
    double sum = 0.0;
    for (int64_t c = 0; c < ci; ++c)
      for (int64_t r = 0; r < kh; ++r)
        for (int64_t s = 0; s < kw; ++s) {
          const int64_t hi = o_h * sh + r, wi = o_w * sw + s;
          if (hi >= ph && wi >= pw) {
            const int64_t hh = hi - ph, ww = wi - pw;
            if (hh < h && ww < w)
              sum += (double)x[((b * ci + c) * h + hh) * w + ww] *
                     (double)wt[((c_o * ci + c) * kh + r) * kw + s];
          }
        }
    y[idx] = (float)sum;
  }
}

/* conv2d_im2col_core (rustorch-core/src/ops/conv.rs:207-274): build
 * col[N*Ho*Wo, Ci*kh*kw] with column order (ci, kh, kw), out2d = col . W^T via
 * ops::matmul (W^T made contiguous first), scatter to NCHW.  Returns the
 * matmul kernel choice, or -1 on allocation failure. */
ORC_API int orc_conv2d_im2col(int64_t n, int64_t ci, int64_t h, int64_t w, int64_t co, int64_t kh,
                              int64_t kw, int64_t sh, int64_t sw, int64_t ph, int64_t pw,
                              const float* x, const float* wt, float* y, int nthreads) {
  const int64_t ho = (h + 2 * ph - kh) / sh + 1;
  const int64_t wo = (w + 2 * pw - kw) / sw + 1;
  const int64_t ksz = ci * kh * kw, patches = n * ho * wo;
  float* col = (float*)malloc((size_t)(patches * ksz) * sizeof(float));
  float* out2d = (float*)malloc((size_t)(patches * co) * sizeof(float));
  if (!col || !out2d) {
    free(col);
    free(out2d);
    return -1;
  }
  orc_set_threads(nthreads);
#pragma omp parallel for schedule(static)
  for (int64_t row = 0; row < patches; ++row) {
    const int64_t o_w = row % wo, o_h = (row / wo) % ho, b = row / (wo * ho);
    int64_t cidx = 0;
    for (int64_t c = 0; c < ci; ++c)
      for (int64_t r = 0; r < kh; ++r)
        for (int64_t s = 0; s < kw; ++s) {
          const int64_t hi = o_h * sh + r, wi = o_w * sw + s;
          float v = 0.0f;
          if (hi >= ph && wi >= pw) {
            const int64_t hh = hi - ph, ww = wi - pw;
            if (hh < h && ww < w) v = x[((b * ci + c) * h + hh) * w + ww];
          }
          col[row * ksz + cidx++] = v;
        }
  }
  /* weight_t = Tensor::new(weight, [co, ksz]).t(): strides (1, ksz). */
  const int choice = orc_matmul(patches, ksz, co, col, ksz, 1, wt, 1, ksz, NULL, out2d, nthreads);
#pragma omp parallel for schedule(static)
  for (int64_t row = 0; row < patches; ++row) {
    const int64_t o_w = row % wo, o_h = (row / wo) % ho, b = row / (wo * ho);
    for (int64_t c = 0; c < co; ++c) y[((b * co + c) * ho + o_h) * wo + o_w] = out2d[row * co + c];
  }
  free(col);
  free(out2d);
  return choice;
}

/* ops::conv2d auto dispatch (rustorch-core/src/ops/conv.rs:738-919, choice at
 * 794-862 with min_work default 65536, conv.rs:90-109).  Returns
 * 0 = direct, 1 = im2col+sgemm, 2 = im2col+parallel core, -1 = failure. */
ORC_API int orc_conv2d(int64_t n, int64_t ci, int64_t h, int64_t w, int64_t co, int64_t kh,
                       int64_t kw, int64_t sh, int64_t sw, int64_t ph, int64_t pw, const float* x,
                       const float* wt, float* y, int nthreads) {
  const int64_t ho = (h + 2 * ph - kh) / sh + 1;
  const int64_t wo = (w + 2 * pw - kw) / sw + 1;
  const int64_t work = n * co * ho * wo * ci * kh * kw;
  if (work < 65536) {
    orc_conv2d_direct(n, ci, h, w, co, kh, kw, sh, sw, ph, pw, x, wt, y, nthreads);
    return 0;
  }
  const int r = orc_conv2d_im2col(n, ci, h, w, co, kh, kw, sh, sw, ph, pw, x, wt, y, nthreads);
  return r < 0 ? -1 : 1 + r;
}

/* f64 truth conv for error metrics, output in double (NCHW). */
ORC_API void orc_conv2d_f64(int64_t n, int64_t ci, int64_t h, int64_t w, int64_t co, int64_t kh,
                            int64_t kw, int64_t sh, int64_t sw, int64_t ph, int64_t pw,
                            const float* x, const float* wt, double* y, int nthreads) {
  const int64_t ho = (h + 2 * ph - kh) / sh + 1;
  const int64_t wo = (w + 2 * pw - kw) / sw + 1;
  orc_set_threads(nthreads);
#pragma omp parallel for collapse(2) schedule(static)
  for (int64_t b = 0; b < n; ++b)
    for (int64_t c_o = 0; c_o < co; ++c_o) {
      double* out = y + (b * co + c_o) * ho * wo;
      for (int64_t i = 0; i < ho * wo; ++i) out[i] = 0.0;
      for (int64_t c = 0; c < ci; ++c)
        for (int64_t r = 0; r < kh; ++r)
          for (int64_t s = 0; s < kw; ++s) {
            const double wv = (double)wt[((c_o * ci + c) * kh + r) * kw + s];
            for (int64_t oh = 0; oh < ho; ++oh) {
              const int64_t hh = oh * sh + r - ph;
              if (hh < 0 || hh >= h) continue;
              const float* xr = x + ((b * ci + c) * h + hh) * w;
              double* orow = out + oh * wo;
              for (int64_t ow = 0; ow < wo; ++ow) {
                const int64_t ww = ow * sw + s - pw;
                if (ww >= 0 && ww < w) orow[ow] += wv * (double)xr[ww];
              }
            }
          }
    }
}

/* ------------------------------------------------------------------------ */
/* Conv2dBackward (rustorch-core/src/ops/conv.rs:336-736)                     */
/* ------------------------------------------------------------------------ */

/* grad_input, restating conv2d_grad_input_direct_core (conv.rs:336-389): for
 * every input element (b, ci, h, w), the f64 sum over the output positions
 * whose window covers it, ho in [ceil((h+ph-kh+1)/sh), min(ho_n, (h+ph)/sh+1))
 * with kh_idx = h + ph - ho*sh (same for w), and over co, of g * w.  Output in
 * double (the reference casts this sum to f32). */
ORC_API void orc_conv2d_grad_input_f64(int64_t n, int64_t ci, int64_t h, int64_t w, int64_t co,
                                       int64_t kh, int64_t kw, int64_t sh, int64_t sw,
                                       int64_t ph, int64_t pw, const float* gy, const float* wt,
                                       double* gx, int nthreads) {
  const int64_t ho_n = (h + 2 * ph - kh) / sh + 1;
  const int64_t wo_n = (w + 2 * pw - kw) / sw + 1;
  orc_set_threads(nthreads);
#pragma omp parallel for collapse(2) schedule(static)
  for (int64_t b = 0; b < n; ++b)
    for (int64_t c = 0; c < ci; ++c)
      for (int64_t hh = 0; hh < h; ++hh)
        for (int64_t ww = 0; ww < w; ++ww) {
          double sum = 0.0;
          const int64_t ho0 = hh + ph >= kh ? (hh + ph - kh + 1 + sh - 1) / sh : 0;
          int64_t ho1 = (hh + ph) / sh + 1;
          if (ho1 > ho_n) ho1 = ho_n;
          for (int64_t oh = ho0; oh < ho1; ++oh) {
            const int64_t r = hh + ph - oh * sh;
            const int64_t wo0 = ww + pw >= kw ? (ww + pw - kw + 1 + sw - 1) / sw : 0;
            int64_t wo1 = (ww + pw) / sw + 1;
            if (wo1 > wo_n) wo1 = wo_n;
            for (int64_t ow = wo0; ow < wo1; ++ow) {
              const int64_t s = ww + pw - ow * sw;
              for (int64_t c_o = 0; c_o < co; ++c_o)
                sum += (double)gy[((b * co + c_o) * ho_n + oh) * wo_n + ow] *
                       (double)wt[((c_o * ci + c) * kh + r) * kw + s];
            }
          }
          gx[((b * ci + c) * h + hh) * w + ww] = sum;
        }
}

/* grad_weight, restating conv2d_grad_weight_direct_core (conv.rs:455-502): for
 * every weight (co, ci, r, s) the f64 sum over (b, ho, wo) of x * g, padding
 * positions skipped.  Output in double. */
ORC_API void orc_conv2d_grad_weight_f64(int64_t n, int64_t ci, int64_t h, int64_t w, int64_t co,
                                        int64_t kh, int64_t kw, int64_t sh, int64_t sw,
                                        int64_t ph, int64_t pw, const float* x, const float* gy,
                                        double* gw, int nthreads) {
  const int64_t ho_n = (h + 2 * ph - kh) / sh + 1;
  const int64_t wo_n = (w + 2 * pw - kw) / sw + 1;
  orc_set_threads(nthreads);
#pragma omp parallel for collapse(2) schedule(static)
  for (int64_t c_o = 0; c_o < co; ++c_o)
    for (int64_t c = 0; c < ci; ++c)
      for (int64_t r = 0; r < kh; ++r)
        for (int64_t s = 0; s < kw; ++s) {
          double sum = 0.0;
          for (int64_t b = 0; b < n; ++b)
            for (int64_t oh = 0; oh < ho_n; ++oh) {
              const int64_t hh = oh * sh + r - ph;
              if (hh < 0 || hh >= h) continue;
              const float* xr = x + ((b * ci + c) * h + hh) * w;
              const float* gr = gy + ((b * co + c_o) * ho_n + oh) * wo_n;
              for (int64_t ow = 0; ow < wo_n; ++ow) {
                const int64_t ww = ow * sw + s - pw;
                if (ww >= 0 && ww < w) sum += (double)xr[ww] * (double)gr[ow];
              }
            }
          gw[((c_o * ci + c) * kh + r) * kw + s] = sum;
        }
}

/* ------------------------------------------------------------------------ */
/* Pooling                                                                   */
/* ------------------------------------------------------------------------ */

/* ops::max_pool2d (rustorch-core/src/ops/pool.rs:115-191): -inf init, padding
 * positions skipped, strict '>' comparison. NCHW. */
ORC_API void orc_max_pool2d(int64_t n, int64_t c, int64_t h, int64_t w, int64_t kh, int64_t kw,
                            int64_t sh, int64_t sw, int64_t ph, int64_t pw, const float* x,
                            float* y) {
  const int64_t ho = (h + 2 * ph - kh) / sh + 1;
  const int64_t wo = (w + 2 * pw - kw) / sw + 1;
  const int64_t total = n * c * ho * wo;
#pragma omp parallel for schedule(static)
  for (int64_t idx = 0; idx < total; ++idx) {
    const int64_t o_w = idx % wo, o_h = (idx / wo) % ho, cc = (idx / (wo * ho)) % c,
                  b = idx / (wo * ho * c);
    const int64_t h0 = o_h * sh - ph, w0 = o_w * sw - pw;
    float m = -INFINITY;
    for (int64_t r = 0; r < kh; ++r)
      for (int64_t s = 0; s < kw; ++s) {
        const int64_t hh = h0 + r, ww = w0 + s;
        if (hh >= 0 && hh < h && ww >= 0 && ww < w) {
          const float v = x[((b * c + cc) * h + hh) * w + ww];
          if (v > m) m = v;
        }
      }
    y[idx] = m;
  }
}

/* Global average pool NCHW -> [N, C]: absent from the reference (a grep for
 * avg pooling finds nothing); restated as sum in f64 over H*W, / (H*W). */
ORC_API void orc_global_avg_pool(int64_t n, int64_t c, int64_t hw, const float* x, float* y) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n * c; ++i) {
    double s = 0.0;
    for (int64_t j = 0; j < hw; ++j) s += (double)x[i * hw + j];
    y[i] = (float)(s / (double)hw);
  }
}

/* ------------------------------------------------------------------------ */
/* LayerNorm + activation (matmul_bias_norm_activation's second half)        */
/* ------------------------------------------------------------------------ */

/* layer_norm over the last dimension, in place, f32, the reference's own
 * formula (rustorch-core/src/ops/norm.rs:613-700 with the scalar row kernel
 * norm.rs:536-544): s += v; q += v*v sequentially in f32, m = s/D,
 * var = q/D - m*m, inv_s = 1/sqrt(var + eps), out = (v - m)*inv_s*g + b
 * (g = 1, b = 0 when absent). */
ORC_API void orc_layer_norm_ref(float* x, int64_t rows, int64_t d, const float* g, const float* b,
                                float eps) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < rows; ++i) {
    float* row = x + i * d;
    float s = 0.0f, q = 0.0f;
    for (int64_t j = 0; j < d; ++j) {
      s += row[j];
      q += row[j] * row[j];
    }
    const float m = s / (float)d;
    const float v = q / (float)d - m * m;
    const float inv_s = 1.0f / sqrtf(v + eps);
    for (int64_t j = 0; j < d; ++j) {
      const float xh = (row[j] - m) * inv_s;
      row[j] = xh * (g ? g[j] : 1.0f) + (b ? b[j] : 0.0f);
    }
  }
}

/* The same normalisation in f64 with a two-pass variance (mean first, then the
 * mean of squared deviations): the exact value the reference's f32 formula
 * approximates.  x is f64 [rows, d], in place. */
ORC_API void orc_layer_norm_f64(double* x, int64_t rows, int64_t d, const float* g, const float* b,
                                double eps) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < rows; ++i) {
    double* row = x + i * d;
    double s = 0.0;
    for (int64_t j = 0; j < d; ++j) s += row[j];
    const double m = s / (double)d;
    double q = 0.0;
    for (int64_t j = 0; j < d; ++j) q += (row[j] - m) * (row[j] - m);
    const double inv_s = 1.0 / sqrt(q / (double)d + eps);
    for (int64_t j = 0; j < d; ++j)
      row[j] = (row[j] - m) * inv_s * (g ? (double)g[j] : 1.0) + (b ? (double)b[j] : 0.0);
  }
}

/* apply_activation (rustorch-core/src/ops.rs:1773-1780): 1 ReLU, 2 sigmoid
 * 1/(1+exp(-x)) (ops/activations.rs:47-50), 3 tanh (activations.rs:213),
 * 0 none.  In place, f32. */
ORC_API void orc_activation(float* x, int64_t n, int act) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) {
    const float v = x[i];
    if (act == 1) x[i] = v > 0.0f ? v : 0.0f;
    else if (act == 2) x[i] = 1.0f / (1.0f + expf(-v));
    else if (act == 3) x[i] = tanhf(v);
  }
}

/* The same activations in f64. */
ORC_API void orc_activation_f64(double* x, int64_t n, int act) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) {
    const double v = x[i];
    if (act == 1) x[i] = v > 0.0 ? v : 0.0;
    else if (act == 2) x[i] = 1.0 / (1.0 + exp(-v));
    else if (act == 3) x[i] = tanh(v);
  }
}

/* ------------------------------------------------------------------------ */
/* Error metrics                                                             */
/* ------------------------------------------------------------------------ */

/* ||x - ref||_F / ||ref||_F in f64. */
ORC_API double orc_rel_frob(const float* x, const double* ref, int64_t n) {
  double num = 0.0, den = 0.0;
#pragma omp parallel for reduction(+ : num, den) schedule(static)
  for (int64_t i = 0; i < n; ++i) {
    const double d = (double)x[i] - ref[i];
    num += d * d;
    den += ref[i] * ref[i];
  }
  return den > 0.0 ? sqrt(num / den) : sqrt(num);
}
