// Small-M GEMM path (M <= kSmallMMax): C[M,N] = act(A[M,K] . B[K,N] + bias[N]).
//
// With so few rows the problem is a stream over B (K x N x 4 bytes, read once
// from HBM), not a tensor-core problem: a 128-row UMMA tile would be at least
// three quarters padding, and the 3xTF32 split would triple the work.  Here B
// is cut into 256-column blocks and 32-k chunks; the chunk sequence (block-
// major) is shared out to the resident CTAs as equal contiguous ranges
// ("stream-K"), so every SM streams the same number of B bytes whatever N is.
// A CTA's range covers the tail of one block and the head of the next; a block
// touched by several CTAs gets its partial sums from each, and the last CTA to
// arrive (per-block arrival word) adds them in CTA order, so the result does
// not depend on arrival order.
//
// Per CTA: one producer warp issues TMA loads of the A chunk (all M rows) and
// the B chunk into an mbarrier ring; eight consumer warps do the products as
// packed fp32 FMAs (fma.rn.f32x2: two round-to-nearest fp32 FMAs per
// instruction, the same arithmetic as two fmaf) and release each stage with
// one arrival per warp, so the warps drift freely between stages.
//   B [K,N] row-major (Tensor::matmul's rhs): a thread owns 8 rows x 8 columns
//     (4q..4q+3 and 128+4q..), pairs of adjacent columns packed; A values are
//     duplicated into both halves of a pair.
//   B [N,K] row-major (Linear's weight, transposed view): a thread owns 8 rows
//     x 4 columns (q + 64j), each accumulator a pair of even-k and odd-k sums
//     (A's and B's 4-k vectors already hold the pairs).
// The k range of a chunk is split over KG thread groups; at the end of a
// block segment the groups are added in group order through shared memory.
// Accumulation is exact fp32 FMA (more accurate than either tensor-core mode,
// so both precision settings use this path).
#include <cstdint>
#include <cstring>

#include "rtb_act.cuh"
#include "rtb_internal.h"
#include "rtb_ptx.cuh"

namespace rtb {

namespace {

constexpr int kSmCols = 256;  // columns of C per block
constexpr int kSmKC = 32;     // k per chunk (one 128-byte row of A)
constexpr int kSmConsumers = 256;
constexpr int kSmThreads = kSmConsumers + 32;  // + the producer warp
static_assert(kSmConsumers == kSmCols, "the fix-up gives every consumer thread one column");

struct SmallMParams {
  int M, N, K;
  int nch;       // chunks per block: ceil(K / 32)
  int nblk;      // column blocks
  int64_t T;     // nblk * nch: the chunk sequence shared out to the CTAs
  int G;         // CTAs (gridDim.x)
  int whole;     // 1: CTA b owns block b alone (no partials)
  float* C;
  int64_t ldc;
  const float* bias;
  int act;       // RTB_ACT_*
  float* ws;     // [G][2][M][256] partial sums of blocks shared with other CTAs
  unsigned long long* cnt;  // [nblk] arrival words (generation << 8 | count)
  unsigned long long cnt_gen;
  int* err;
  unsigned long long timeout_ns;
};

__device__ __forceinline__ int64_t sm_lo(const SmallMParams& p, int c) {
  return (int64_t)c * p.T / p.G;
}

// The CTA whose chunk range holds chunk x.
__device__ __forceinline__ int sm_owner(const SmallMParams& p, int64_t x) {
  int c = (int)((x * p.G) / p.T);
  while (c + 1 < p.G && sm_lo(p, c + 1) <= x) ++c;
  while (c > 0 && sm_lo(p, c) > x) --c;
  return c;
}

template <int MP, int B_MN>
struct SmCfg {
  // MP: rows padded to 8 or 16 (rows >= M are the TMA's zero fill)
  static constexpr int RGN = MP / 8;                        // row groups of 8 rows
  static constexpr int CGN = B_MN ? 32 : 64;                // column groups
  static constexpr int KG = kSmConsumers / (RGN * CGN);     // k groups
  static constexpr int TPG = kSmConsumers / KG;             // threads per k group
  static constexpr int NV = B_MN ? 64 : 32;                 // finished values per thread
  static constexpr int kABytes = MP * kSmKC * 4;
  static constexpr int kBBytes = kSmKC * kSmCols * 4;       // 32 KB
  static constexpr int kStage = kABytes + kBBytes;
  static constexpr int kRedBytes = (KG - 1) * TPG * NV * 4;
  static constexpr int kStagesRaw = (224 * 1024 - kRedBytes) / kStage;
  static constexpr int kStages = kStagesRaw > 8 ? 8 : kStagesRaw;
  static constexpr int kSmem = kStages * kStage + kRedBytes + 1024 /*align*/ + 256 /*bars*/;
  static_assert(KG >= 1 && RGN * CGN * KG == kSmConsumers, "thread layout");
  static_assert(kStages >= 3, "ring depth");
};

__device__ __forceinline__ void fma2(unsigned long long& d, unsigned long long a,
                                     unsigned long long b) {
  asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(d) : "l"(a), "l"(b));
}
__device__ __forceinline__ unsigned long long dup2(float a) {
  unsigned long long r;
  asm("mov.b64 %0, {%1, %1};" : "=l"(r) : "f"(a));
  return r;
}
__device__ __forceinline__ void lds2x64(uint32_t addr, unsigned long long& lo,
                                        unsigned long long& hi) {
  asm volatile("ld.shared.v2.u64 {%0, %1}, [%2];" : "=l"(lo), "=l"(hi) : "r"(addr));
}
__device__ __forceinline__ float lo_f(unsigned long long v) {
  return __uint_as_float((uint32_t)(v & 0xFFFFFFFFull));
}
__device__ __forceinline__ float hi_f(unsigned long long v) {
  return __uint_as_float((uint32_t)(v >> 32));
}

// Column (within the block) and row of value e of a consumer thread.
template <int B_MN>
__device__ __forceinline__ int sm_col(int e, int q) {
  if (B_MN) {
    const int j = (e & 7) >> 1;
    return (j >= 2 ? 128 : 0) + 4 * q + 2 * (j & 1) + (e & 1);
  }
  return q + 64 * (e & 3);
}
template <int B_MN>
__device__ __forceinline__ int sm_row(int e, int rg) {
  return 8 * rg + (B_MN ? (e >> 3) : (e >> 2));
}

// Bias, activation and the store of a thread's finished values.
template <int B_MN, int NV>
__device__ __forceinline__ void sm_finish(const SmallMParams& p, const float (&w)[NV], int rg,
                                          int q, int n0) {
#pragma unroll
  for (int e = 0; e < NV; ++e) {
    const int m = sm_row<B_MN>(e, rg), n = n0 + sm_col<B_MN>(e, q);
    if (m < p.M && n < p.N) {
      float x = w[e];
      if (p.bias) x += __ldg(p.bias + n);
      p.C[(int64_t)m * p.ldc + n] = activate(x, p.act);
    }
  }
}

template <int MP, int B_MN>
__global__ void __launch_bounds__(kSmThreads, 1)
    smallm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                  const SmallMParams p) {
  using Cfg = SmCfg<MP, B_MN>;
  constexpr int S_ = Cfg::kStages;
  constexpr int KG = Cfg::KG;
  constexpr int TPG = Cfg::TPG;
  constexpr int NV = Cfg::NV;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  float* red = reinterpret_cast<float*>(base + S_ * Cfg::kStage);  // [KG-1][NV][TPG]
  uint64_t* full = reinterpret_cast<uint64_t*>(base + S_ * Cfg::kStage + Cfg::kRedBytes);
  uint64_t* empty = full + S_;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + S_);
  volatile int* last_flag = abort_flag + 1;

  const int tid = threadIdx.x;
  const int c = blockIdx.x;
  // chunk range of this CTA: whole blocks (block c) or its share of the sequence
  const int64_t lo = p.whole ? (int64_t)c * p.nch : sm_lo(p, c);
  const int64_t hi = p.whole ? lo + p.nch : sm_lo(p, c + 1);

  if (tid == 0) {
    for (int s = 0; s < S_; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kSmConsumers / 32);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  // global memory only after the previous kernel on the stream has completed
  // (launched with programmatic stream serialization)
  griddep_wait();
  griddep_launch_dependents();

  if (tid < 32) {
    // ------------------------------------------------------------ producer
    if (tid == 0) {
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmB);
      int s = 0;
      uint32_t ph = 0;
      for (int64_t u = lo; u < hi; ++u) {
        if (!mbar_wait_bounded(&empty[s], ph ^ 1, abort_flag, p.err, DEV_TIMEOUT_EMPTY,
                               p.timeout_ns))
          break;
        const int blk = (int)(u / p.nch);
        const int ch = (int)(u - (int64_t)blk * p.nch);
        uint8_t* sa = base + s * Cfg::kStage;
        mbar_arrive_expect_tx(&full[s], Cfg::kStage);
        tma_load_2d(sa, &tmA, &full[s], ch * kSmKC, 0);
        if (B_MN)
          tma_load_2d(sa + Cfg::kABytes, &tmB, &full[s], blk * kSmCols, ch * kSmKC);
        else
          tma_load_2d(sa + Cfg::kABytes, &tmB, &full[s], ch * kSmKC, blk * kSmCols);
        if (++s == S_) { s = 0; ph ^= 1; }
      }
    }
  } else {
    // ------------------------------------------------------------ consumers
    const int ct = tid - 32;
    const int lane = ct & 31;
    const int kg = ct / TPG;      // k group
    const int tig = ct % TPG;     // thread in its k group
    const int rg = B_MN ? tig / 32 : tig / 64;  // row group (rows 8rg .. 8rg+7)
    const int q = B_MN ? tig % 32 : tig % 64;   // column group
    int s = 0;
    uint32_t ph = 0;
    bool ok = true;
    for (int64_t u0 = lo; u0 < hi;) {
      const int blk = (int)(u0 / p.nch);
      const int64_t seg_end = ((int64_t)blk + 1) * p.nch < hi ? ((int64_t)blk + 1) * p.nch : hi;
      unsigned long long acc[8][4];
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = 0ull;
      for (int64_t u = u0; u < seg_end; ++u) {
        // a failed wait raises the abort flag, after which every wait returns
        // at once: the loop structure (and the barriers below) stay uniform
        const bool got = mbar_wait_bounded(&full[s], ph, abort_flag, p.err, DEV_TIMEOUT_FULL,
                                           p.timeout_ns);
        ok = ok && got;
        if (got) {
          const uint32_t sa = smem_u32(base + s * Cfg::kStage);
          const uint32_t sb = sa + Cfg::kABytes;
#pragma unroll 1
          for (int k4 = kg; k4 < kSmKC / 4; k4 += KG) {
            if (B_MN) {
              // B: 4 k rows x this thread's 8 columns as 4 column pairs each
              unsigned long long b[4][4];
#pragma unroll
              for (int kk = 0; kk < 4; ++kk) {
                const uint32_t bk = sb + ((4 * k4 + kk) * kSmCols + 4 * q) * 4;
                lds2x64(bk, b[kk][0], b[kk][1]);
                lds2x64(bk + 512, b[kk][2], b[kk][3]);
              }
              float4 a[8];
#pragma unroll
              for (int i = 0; i < 8; ++i) {
                const int r = 8 * rg + i;
                a[i] = lds128(sa + r * 128 + ((k4 ^ (r & 7)) << 4));
              }
              // k outermost: successive FMAs on one accumulator are 32
              // instructions apart (the FMA pipe's latency is hidden)
#pragma unroll
              for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                  const float av =
                      kk == 0 ? a[i].x : kk == 1 ? a[i].y : kk == 2 ? a[i].z : a[i].w;
                  const unsigned long long ad = dup2(av);
#pragma unroll
                  for (int j = 0; j < 4; ++j) fma2(acc[i][j], ad, b[kk][j]);
                }
              }
            } else {
              // B: this thread's 4 columns, 4 k each as two (k, k+1) pairs
              unsigned long long b0[4], b1[4];
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                const int col = q + 64 * j;
                lds2x64(sb + col * 128 + ((k4 ^ (col & 7)) << 4), b0[j], b1[j]);
              }
              unsigned long long a0[8], a1[8];
#pragma unroll
              for (int i = 0; i < 8; ++i) {
                const int r = 8 * rg + i;
                lds2x64(sa + r * 128 + ((k4 ^ (r & 7)) << 4), a0[i], a1[i]);
              }
              // (k, k+1) products for every accumulator, then (k+2, k+3): the
              // two FMAs on one accumulator are 32 instructions apart
#pragma unroll
              for (int i = 0; i < 8; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) fma2(acc[i][j], a0[i], b0[j]);
#pragma unroll
              for (int i = 0; i < 8; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) fma2(acc[i][j], a1[i], b1[j]);
            }
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
        if (++s == S_) { s = 0; ph ^= 1; }
      }
      // ---- end of a block segment: fold the k groups, then finish the block
      // (alone), or publish this CTA's partial and let the last CTA finish it
      float v[NV];
      if (B_MN) {
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            v[i * 8 + 2 * j] = lo_f(acc[i][j]);
            v[i * 8 + 2 * j + 1] = hi_f(acc[i][j]);
          }
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) v[i * 4 + j] = lo_f(acc[i][j]) + hi_f(acc[i][j]);
      }
      if (KG > 1) {
        const uint32_t rb = smem_u32(red);
        named_bar_sync(1, kSmConsumers);  // the previous segment's readers are done
        if (kg > 0) {
#pragma unroll
          for (int e = 0; e < NV; ++e) sts32(rb + (((kg - 1) * NV + e) * TPG + tig) * 4, v[e]);
        }
        named_bar_sync(1, kSmConsumers);
        if (kg == 0) {
#pragma unroll 1
          for (int g = 1; g < KG; ++g)
#pragma unroll
            for (int e = 0; e < NV; ++e) v[e] += lds32(rb + (((g - 1) * NV + e) * TPG + tig) * 4);
        }
      }
      const int n0 = blk * kSmCols;
      const int c_first = p.whole ? c : sm_owner(p, (int64_t)blk * p.nch);
      const int c_last = p.whole ? c : sm_owner(p, ((int64_t)blk + 1) * p.nch - 1);
      if (c_first == c_last) {
        if (kg == 0 && ok) sm_finish<B_MN, NV>(p, v, rg, q, n0);
      } else {
        // slot of (CTA x, this block): x's ranges span at most two blocks
        auto slot_of = [&](int x) {
          return 2 * x + (blk - (int)(sm_lo(p, x) / p.nch));
        };
        if (kg == 0 && ok) {
          float* part = p.ws + (size_t)slot_of(c) * p.M * kSmCols;
#pragma unroll
          for (int e = 0; e < NV; ++e) {
            const int m = sm_row<B_MN>(e, rg);
            if (m < p.M) __stcg(part + (size_t)m * kSmCols + sm_col<B_MN>(e, q), v[e]);
          }
        }
        __threadfence();
        named_bar_sync(1, kSmConsumers);
        if (ct == 0) {
          int last = 0;
          if (!*abort_flag) {
            const int arrived = tagged_arrive(p.cnt + blk, p.cnt_gen);
            if (arrived < 0) {
              atomicCAS(p.err, 0, (int)DEV_BAD_CONFIG);
              *abort_flag = 1;
            }
            last = arrived == c_last - c_first;
          }
          *last_flag = last;
        }
        named_bar_sync(1, kSmConsumers);
        if (*last_flag && ok) {
          // The last CTA to arrive sums the block's partials in CTA order (its
          // own read back too, so the order is the same whoever is last).
          // All consumer threads take part: thread t owns column t of the
          // block for every row, so each warp reads whole 128-byte rows and
          // the next partial's loads are in flight while one is added.
          __threadfence();
          const int col = ct;  // kSmConsumers == kSmCols
          const int n = n0 + col;
          float a[MP], t0[MP], t1[MP];
          auto load = [&](int x, float (&t)[MP]) {
            const float* part = p.ws + (size_t)slot_of(x) * p.M * kSmCols + col;
#pragma unroll
            for (int r = 0; r < MP; ++r) t[r] = r < p.M ? __ldcg(part + (size_t)r * kSmCols) : 0.0f;
          };
          load(c_first, t0);
#pragma unroll
          for (int r = 0; r < MP; ++r) a[r] = 0.0f;
#pragma unroll 1
          for (int x = c_first; x <= c_last; x += 2) {
            if (x + 1 <= c_last) load(x + 1, t1);
#pragma unroll
            for (int r = 0; r < MP; ++r) a[r] = x == c_first ? t0[r] : a[r] + t0[r];
            if (x + 1 > c_last) break;
            if (x + 2 <= c_last) load(x + 2, t0);
#pragma unroll
            for (int r = 0; r < MP; ++r) a[r] += t1[r];
          }
          if (n < p.N) {
            const float bv = p.bias ? __ldg(p.bias + n) : 0.0f;
#pragma unroll
            for (int r = 0; r < MP; ++r)
              if (r < p.M) p.C[(int64_t)r * p.ldc + n] = activate(a[r] + bv, p.act);
          }
        }
      }
      u0 = seg_end;
    }
  }
  __syncthreads();
  if (*abort_flag) {
    // copies already issued may still land in shared memory: give them time
    const uint64_t t0 = globaltimer_ns();
    while (globaltimer_ns() - t0 < 1000000ull) __nanosleep(1000);
  }
}

}  // namespace

}  // namespace rtb

namespace rtb {

namespace {

template <int MP, int B_MN>
int launch_smallm(const CUtensorMap& tmA, const CUtensorMap& tmB, const SmallMParams& p,
                  cudaStream_t s) {
  using Cfg = SmCfg<MP, B_MN>;
  auto kern = smallm_kernel<MP, B_MN>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmem);
  if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute(smallm smem)");
  clear_stale_cuda_error();
  e = launch_pdl(kern, dim3((unsigned)p.G), dim3(kSmThreads), Cfg::kSmem, s, tmA, tmB, p);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_status(e, "smallm kernel launch");
  return RTB_OK;
}

template <int MP>
int launch_mp(const CUtensorMap& tmA, const CUtensorMap& tmB, const SmallMParams& p, int b_mn,
              cudaStream_t s) {
  return b_mn ? launch_smallm<MP, 1>(tmA, tmB, p, s) : launch_smallm<MP, 0>(tmA, tmB, p, s);
}

}  // namespace

int smallm_run(rtb_ctx* ctx, const GemmDesc& d, cudaStream_t stream) {
  if (d.M <= 0 || d.M > kSmallMMax || d.N <= 0 || d.K <= 0 || d.gather)
    return set_error(RTB_E_INVALID, "smallm_run: bad problem");
  if (d.N > INT32_MAX || d.K > INT32_MAX)
    return set_error(RTB_E_UNSUPPORTED, "smallm_run: dimension exceeds 2^31-1");
  const int MP = d.M <= 8 ? 8 : 16;

  CUtensorMap tmA, tmB;
  // A: K-major [M, K]; box 32 k x MP rows (rows >= M read as zero)
  int st = make_tmap_2d_swz(&tmA, d.A, (uint64_t)d.K, (uint64_t)d.M, (uint64_t)d.lda, kSmKC,
                            (uint32_t)MP, kTmapSwizzle128);
  if (st != RTB_OK) return st;
  if (d.b_mn_major)  // [K, N]: box 256 n x 32 k, dense
    st = make_tmap_2d_swz(&tmB, d.B, (uint64_t)d.N, (uint64_t)d.K, (uint64_t)d.ldb, kSmCols, kSmKC,
                          kTmapSwizzleNone);
  else               // [N, K]: box 32 k x 256 n, 128B-swizzled
    st = make_tmap_2d_swz(&tmB, d.B, (uint64_t)d.K, (uint64_t)d.N, (uint64_t)d.ldb, kSmKC, kSmCols,
                          kTmapSwizzle128);
  if (st != RTB_OK) return st;

  SmallMParams p{};
  p.M = (int)d.M;
  p.N = (int)d.N;
  p.K = (int)d.K;
  p.nch = (int)((d.K + kSmKC - 1) / kSmKC);
  p.nblk = (int)((d.N + kSmCols - 1) / kSmCols);
  p.T = (int64_t)p.nblk * p.nch;
  p.C = d.C;
  p.ldc = d.ldc;
  p.bias = d.bias;
  p.act = d.act;
  p.err = ctx->d_err;
  p.timeout_ns = ctx->timeout_ns;
  // Stream-K over the chunk sequence when every CTA gets >= 4 chunks and at
  // most two blocks (CTAs >= blocks), a counter word exists for every block
  // and the caller allows a workspace; otherwise one CTA per block.
  const int64_t G = (int64_t)ctx->sm_count < p.T / 4 ? (int64_t)ctx->sm_count : p.T / 4;
  p.whole = !(d.allow_workspace && p.nch >= 4 && p.nblk < ctx->sm_count &&
              p.nblk <= kSplitCounters && G >= p.nblk && G >= 2);
  p.G = p.whole ? p.nblk : (int)G;
  void* ws = nullptr;
  if (!p.whole) {
    const size_t part_bytes = (size_t)p.G * 2 * d.M * kSmCols * sizeof(float);
    const size_t cnt_off = (part_bytes + 255) & ~size_t(255);
    st = split_counters(ctx, stream, &p.cnt, &p.cnt_gen);
    const bool own = (st == RTB_E_UNSUPPORTED);  // capture / per-thread stream: own counters
    if (st != RTB_OK && !own) return st;
    st = ws_alloc(ctx, &ws, own ? cnt_off + (size_t)p.nblk * 8 : part_bytes, stream);
    if (st != RTB_OK) return st;
    if (own) {
      p.cnt = reinterpret_cast<unsigned long long*>(static_cast<char*>(ws) + cnt_off);
      p.cnt_gen = 1;
      cudaError_t e = cudaMemsetAsync(p.cnt, 0, (size_t)p.nblk * 8, stream);
      if (e != cudaSuccess) {
        ws_free(ws, stream);
        return cuda_status(e, "smallm counters memset");
      }
    }
    p.ws = static_cast<float*>(ws);
  }
  st = MP == 8 ? launch_mp<8>(tmA, tmB, p, d.b_mn_major, stream)
               : launch_mp<16>(tmA, tmB, p, d.b_mn_major, stream);
  ws_free(ws, stream);
  return st;
}

}  // namespace rtb
