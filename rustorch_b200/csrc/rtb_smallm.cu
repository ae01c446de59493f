// Small-M GEMM path (M <= kSmallMMax): C[M,N] = act(A[M,K] . B[K,N] + bias[N]).
//
// With so few rows the problem is a stream over B (K x N x 4 bytes, read once
// from HBM), not a tensor-core problem: a 128-row UMMA tile would be at least
// half padding, and the 3xTF32 split would triple the work.  Here every CTA
// owns a 256-column block of C for one K slice, all M rows at once, so each B
// element is fetched exactly once; B and A chunks of 32 k arrive by TMA in a
// small mbarrier ring and the products are plain fp32 FMAs (exact fp32
// accumulation in k order, more accurate than either tensor-core mode).
//
// Thread layout (256 threads, one CTA per SM): row group rg owns rows
// 16*rg .. 16*rg+15 (RG = 1, 2 or 4 groups for M <= 16, 32, 64); the other
// 4/RG-fold of threads split each chunk's k range and are summed through
// shared memory in a fixed order at the end; column group cg = tid % 64 owns
// 4 columns:
//   B [K,N] row-major (Tensor::matmul's rhs): columns n0 + 4cg .. 4cg+3
//   B [N,K] row-major (Linear's weight, transposed view): columns n0 + cg + 64j
// so that each warp's shared-memory reads are conflict-free.
// K is split into S slices when N alone gives too few CTAs; every slice
// writes its fp32 partial block to a workspace and the last slice of a column
// block to arrive (per-block counter) sums the slices in slice order, adds
// the bias and applies the activation, so the result does not depend on arrival order.
#include <cstdint>
#include <cstring>

#include "rtb_act.cuh"
#include "rtb_internal.h"
#include "rtb_ptx.cuh"

namespace rtb {

namespace {

constexpr int kSmCols = 256;  // columns of C per CTA
constexpr int kSmKC = 32;     // k per chunk (one 128-byte row of A)

struct SmallMParams {
  int M, N, K;
  int nchunks;   // ceil(K / 32)
  int nblk;      // column blocks
  int S;         // K slices
  float* C;
  int64_t ldc;
  const float* bias;
  int act;       // RTB_ACT_*
  float* ws;     // [S][M][ws_ld] partial sums (S > 1)
  int64_t ws_ld;
  unsigned long long* cnt;  // [nblk] arrival words (generation << 8 | count), S > 1
  unsigned long long cnt_gen;
  int* err;
  unsigned long long timeout_ns;
};

template <int RG>
struct SmCfg {
  // 256 threads: RG row groups of 16 rows x KG k groups, 64 column groups each
  static constexpr int kThreads = 256;
  static constexpr int KG = 4 / RG;
  static constexpr int kABytes = 16 * RG * 128;            // 16*RG rows x 32 fp32
  static constexpr int kBBytes = kSmKC * kSmCols * 4;      // 32 KB
  static constexpr int kStage = kABytes + kBBytes;
  // one CTA per SM with a deep ring: the HBM latency is covered by several
  // 32 KB chunks in flight per CTA
  static constexpr int kStagesRaw = (220 * 1024) / kStage;
  static constexpr int kStages = kStagesRaw > 8 ? 8 : kStagesRaw;
  static constexpr int kSmem = kStages * kStage + 1024 /*align*/ + 256 /*barriers*/;
  static_assert(kStages * kStage >= 256 * 64 * 4, "reduction buffer must fit in the ring");
};

template <int RG, int B_MN>
__global__ void __launch_bounds__(256, 1)
    smallm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                  const SmallMParams p) {
  using Cfg = SmCfg<RG>;
  constexpr int S_ = Cfg::kStages;
  constexpr int KG = Cfg::KG;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(base + S_ * Cfg::kStage);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(full + S_);
  volatile int* last_flag = abort_flag + 1;

  const int tid = threadIdx.x;
  const int cg = tid & 63;
  const int rg = (tid >> 6) % RG;   // row group
  const int kg = (tid >> 6) / RG;   // k group: k4 = kg, kg + KG, ... of each chunk
  const int blk = blockIdx.x % p.nblk;
  const int slice = blockIdx.x / p.nblk;
  const int n0 = blk * kSmCols;
  const int c0 = (int)((int64_t)slice * p.nchunks / p.S);
  const int c1 = (int)((int64_t)(slice + 1) * p.nchunks / p.S);
  const int nch = c1 - c0;

  if (tid == 0) {
    for (int s = 0; s < S_; ++s) mbar_init(&full[s], 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  // global memory only after the previous kernel on the stream has completed
  // (launched with programmatic stream serialization)
  griddep_wait();
  griddep_launch_dependents();
  auto issue = [&](int s, int chunk) {
    uint8_t* sa = base + s * Cfg::kStage;
    mbar_arrive_expect_tx(&full[s], Cfg::kStage);
    tma_load_2d(sa, &tmA, &full[s], chunk * kSmKC, 0);
    if (B_MN)
      tma_load_2d(sa + Cfg::kABytes, &tmB, &full[s], n0, chunk * kSmKC);
    else
      tma_load_2d(sa + Cfg::kABytes, &tmB, &full[s], chunk * kSmKC, n0);
  };
  if (tid == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    for (int s = 0; s < S_ && s < nch; ++s) issue(s, c0 + s);
  }

  float acc[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;

  bool ok = true;
  for (int c = 0; c < nch; ++c) {
    const int s = c % S_;
    const bool got = mbar_wait_bounded(&full[s], (uint32_t)((c / S_) & 1), abort_flag, p.err,
                                       DEV_TIMEOUT_FULL, p.timeout_ns);
    if (__syncthreads_or(!got)) {
      ok = false;
      break;
    }
    const uint32_t sa = smem_u32(base + s * Cfg::kStage);
    const uint32_t sb = sa + Cfg::kABytes;
#pragma unroll 1
    for (int k4 = kg; k4 < kSmKC / 4; k4 += KG) {
      float4 bv[4];
      if (B_MN) {
        // bv[j] = B[k = 4*k4 + j][4 columns]   (dense [32 k][256 n] tile)
#pragma unroll
        for (int j = 0; j < 4; ++j) bv[j] = lds128(sb + ((4 * k4 + j) * kSmCols + 4 * cg) * 4);
      } else {
        // bv[j] = B[column cg + 64j][4 k]   ([256 n][32 k] tile, 128B-swizzled rows)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int r = cg + 64 * j;
          bv[j] = lds128(sb + r * 128 + ((k4 ^ (r & 7)) << 4));
        }
      }
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int r = 16 * rg + i;  // A row, 128B-swizzled like B's K-major tile
        const float4 a = lds128(sa + r * 128 + ((k4 ^ (r & 7)) << 4));
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          if (B_MN) {
            const float b0 = j == 0 ? bv[0].x : j == 1 ? bv[0].y : j == 2 ? bv[0].z : bv[0].w;
            const float b1 = j == 0 ? bv[1].x : j == 1 ? bv[1].y : j == 2 ? bv[1].z : bv[1].w;
            const float b2 = j == 0 ? bv[2].x : j == 1 ? bv[2].y : j == 2 ? bv[2].z : bv[2].w;
            const float b3 = j == 0 ? bv[3].x : j == 1 ? bv[3].y : j == 2 ? bv[3].z : bv[3].w;
            acc[i][j] = fmaf(a.x, b0, acc[i][j]);
            acc[i][j] = fmaf(a.y, b1, acc[i][j]);
            acc[i][j] = fmaf(a.z, b2, acc[i][j]);
            acc[i][j] = fmaf(a.w, b3, acc[i][j]);
          } else {
            acc[i][j] = fmaf(a.x, bv[j].x, acc[i][j]);
            acc[i][j] = fmaf(a.y, bv[j].y, acc[i][j]);
            acc[i][j] = fmaf(a.z, bv[j].z, acc[i][j]);
            acc[i][j] = fmaf(a.w, bv[j].w, acc[i][j]);
          }
        }
      }
    }
    __syncthreads();  // stage s fully read by every thread
    if (tid == 0 && c + S_ < nch) issue(s, c0 + c + S_);
  }
  if (!ok) {
    // copies already issued may still land in shared memory: give them time
    const uint64_t t0 = globaltimer_ns();
    while (globaltimer_ns() - t0 < 1000000ull) __nanosleep(1000);
    return;  // uniform: decided by __syncthreads_or
  }

  if (KG > 1) {
    // sum the k groups in order kg = 0, 1, ... through the (now idle) ring
    float* red = reinterpret_cast<float*>(base);  // [KG][RG*64 threads][64]
    const int slot = tid - kg * 64 * RG;          // thread within its k group
    if (kg > 0) {
#pragma unroll
      for (int i = 0; i < 16; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) red[((kg * 64 * RG + slot) * 16 + i) * 4 + j] = acc[i][j];
    }
    __syncthreads();
    if (kg == 0) {
      for (int g = 1; g < KG; ++g)
#pragma unroll
        for (int i = 0; i < 16; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) acc[i][j] += red[((g * 64 * RG + slot) * 16 + i) * 4 + j];
    }
  }
  const bool owner = kg == 0;  // this thread holds finished sums for its rows/columns

  auto col = [&](int j) { return B_MN ? n0 + 4 * cg + j : n0 + cg + 64 * j; };
  auto finish = [&](int m, int n, float v) {
    if (p.bias) v += __ldg(p.bias + n);
    v = activate(v, p.act);
    p.C[(int64_t)m * p.ldc + n] = v;
  };
  if (p.S == 1) {
    if (!owner) return;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int m = 16 * rg + i;
      if (m >= p.M) break;
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (col(j) < p.N) finish(m, col(j), acc[i][j]);
    }
    return;
  }
  // split K: publish this slice, the last slice of the block sums all of them
  if (owner) {
    float* part = p.ws + (size_t)slice * p.M * p.ws_ld;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int m = 16 * rg + i;
      if (m >= p.M) break;
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (col(j) < p.N) __stcg(part + (size_t)m * p.ws_ld + col(j), acc[i][j]);
    }
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const int arrived = tagged_arrive(p.cnt + blk, p.cnt_gen);
    if (arrived < 0) atomicCAS(p.err, 0, (int)DEV_BAD_CONFIG);
    *last_flag = (arrived == p.S - 1);
  }
  __syncthreads();
  if (!*last_flag || !owner) return;
  __threadfence();
#pragma unroll 1
  for (int i = 0; i < 16; ++i) {
    const int m = 16 * rg + i;
    if (m >= p.M) break;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int n = col(j);
      if (n >= p.N) continue;
      float v = 0.0f;
      for (int sl = 0; sl < p.S; ++sl) v += __ldcg(p.ws + ((size_t)sl * p.M + m) * p.ws_ld + n);
      finish(m, n, v);
    }
  }
}

template <int RG, int B_MN>
int launch_smallm(rtb_ctx* ctx, const CUtensorMap& tmA, const CUtensorMap& tmB,
                  const SmallMParams& p, cudaStream_t s) {
  using Cfg = SmCfg<RG>;
  auto kern = smallm_kernel<RG, B_MN>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmem);
  if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute(smallm smem)");
  // all of the unified L1/shared storage as shared memory (deep ring)
  e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout,
                           cudaSharedmemCarveoutMaxShared);
  if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute(smallm carveout)");
  clear_stale_cuda_error();
  e = launch_pdl(kern, dim3((unsigned)(p.nblk * p.S)), dim3(Cfg::kThreads), Cfg::kSmem, s, tmA, tmB,
                 p);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_status(e, "smallm kernel launch");
  (void)ctx;
  return RTB_OK;
}

}  // namespace

int smallm_run(rtb_ctx* ctx, const GemmDesc& d, cudaStream_t stream) {
  if (d.M <= 0 || d.M > kSmallMMax || d.N <= 0 || d.K <= 0 || d.gather)
    return set_error(RTB_E_INVALID, "smallm_run: bad problem");
  if (d.N > INT32_MAX || d.K > INT32_MAX)
    return set_error(RTB_E_UNSUPPORTED, "smallm_run: dimension exceeds 2^31-1");
  const int RG = d.M <= 16 ? 1 : (d.M <= 32 ? 2 : 4);  // 4: M up to 64 if the threshold moves

  CUtensorMap tmA, tmB;
  // A: K-major [M, K]; box 32 k x 16*RG rows (rows >= M read as zero)
  int st = make_tmap_2d_swz(&tmA, d.A, (uint64_t)d.K, (uint64_t)d.M, (uint64_t)d.lda, kSmKC,
                            (uint32_t)(16 * RG), kTmapSwizzle128);
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
  p.nchunks = (int)((d.K + kSmKC - 1) / kSmKC);
  p.nblk = (int)((d.N + kSmCols - 1) / kSmCols);
  p.C = d.C;
  p.ldc = d.ldc;
  p.bias = d.bias;
  p.act = d.act;
  p.err = ctx->d_err;
  p.timeout_ns = ctx->timeout_ns;
  // K slices: one wave of CTAs (one per SM), at least 4 chunks per slice.
  int S = ctx->sm_count / p.nblk;
  if (S > p.nchunks / 4) S = p.nchunks / 4;
  if (S < 1 || !d.allow_workspace) S = 1;
  p.S = S;
  void* ws = nullptr;
  if (S > 1 && p.nblk > kSplitCounters) S = p.S = 1;  // no counter word for every column block
  if (S > 1) {
    p.ws_ld = (d.N + 3) / 4 * 4;
    const size_t part_bytes = (size_t)S * d.M * p.ws_ld * sizeof(float);
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
  if (RG == 1)
    st = d.b_mn_major ? launch_smallm<1, 1>(ctx, tmA, tmB, p, stream)
                      : launch_smallm<1, 0>(ctx, tmA, tmB, p, stream);
  else if (RG == 2)
    st = d.b_mn_major ? launch_smallm<2, 1>(ctx, tmA, tmB, p, stream)
                      : launch_smallm<2, 0>(ctx, tmA, tmB, p, stream);
  else
    st = d.b_mn_major ? launch_smallm<4, 1>(ctx, tmA, tmB, p, stream)
                      : launch_smallm<4, 0>(ctx, tmA, tmB, p, stream);
  ws_free(ws, stream);
  return st;
}

}  // namespace rtb
