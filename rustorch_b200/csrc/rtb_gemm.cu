// Instantiation and launch of the tcgen05 GEMM engine (rtb_gemm.cuh).
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "rtb_gemm.cuh"
#include "rtb_internal.h"

namespace rtb {

namespace {

template <int BN, bool SPLIT, int A_MODE, int B_MN>
int launch_variant(rtb_ctx* ctx, const CUtensorMap& tmA, const CUtensorMap& tmB,
                   const CUtensorMap& tmC, const GemmParams& p, cudaStream_t stream) {
  using Cfg = GemmCfg<BN, SPLIT>;
  using Roles = GemmRoles<SPLIT, A_MODE == 1>;
  auto kern = rtb_gemm_kernel<BN, SPLIT, A_MODE, B_MN>;
  // The attribute is per function and per device; setting it is idempotent
  // and cheap, so it is set on every launch (covers multi-device processes).
  cudaError_t e =
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes);
  if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute(gemm smem)");
  const int grid = p.num_units < ctx->sm_count ? p.num_units : ctx->sm_count;
  // programmatic dependent launch: the kernel's setup (barriers, TMEM)
  // overlaps the end of the previous kernel; it waits for that kernel before
  // its first global-memory access (griddep_wait in the kernel)
  clear_stale_cuda_error();
  e = launch_pdl(kern, dim3((unsigned)grid), dim3(Roles::kThreads), Cfg::kSmemBytes, stream, tmA,
                 tmB, tmC, p);
  if (e != cudaSuccess) return cuda_status(e, "gemm kernel launch");
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_status(e, "gemm kernel launch");
  return RTB_OK;
}

template <int BN, bool SPLIT>
int launch_prec(rtb_ctx* ctx, const CUtensorMap& tmA, const CUtensorMap& tmB,
                const CUtensorMap& tmC, const GemmParams& p, const GemmDesc& d, cudaStream_t s) {
  if (d.gather == 1) return launch_variant<BN, SPLIT, 1, 0>(ctx, tmA, tmB, tmC, p, s);
  if (d.gather == 2) return launch_variant<BN, SPLIT, 2, 0>(ctx, tmA, tmB, tmC, p, s);
  if (d.gather == 3) {
    if constexpr (SPLIT) return launch_variant<BN, SPLIT, 3, 0>(ctx, tmA, tmB, tmC, p, s);
    else return set_error(RTB_E_INVALID, "multi-tap im2col needs the 3xTF32 converters");
  }
  if (d.b_mn_major) return launch_variant<BN, SPLIT, 0, 1>(ctx, tmA, tmB, tmC, p, s);
  return launch_variant<BN, SPLIT, 0, 0>(ctx, tmA, tmB, tmC, p, s);
}

template <int BN>
int launch_bn(rtb_ctx* ctx, const CUtensorMap& tmA, const CUtensorMap& tmB,
              const CUtensorMap& tmC, const GemmParams& p, const GemmDesc& d, cudaStream_t s) {
  if (!d.split3) return launch_prec<BN, false>(ctx, tmA, tmB, tmC, p, d, s);
  if constexpr (BN <= 128) {
    return launch_prec<BN, true>(ctx, tmA, tmB, tmC, p, d, s);
  } else {
    return set_error(RTB_E_INVALID, "3xTF32 tiles are at most 128 columns wide");
  }
}

int env_int(const char* name, int dflt) {
  const char* v = std::getenv(name);
  return v ? std::atoi(v) : dflt;
}

// Column-tile width: the widest tile that still fills every SM once; narrower
// tiles for small problems (more CTAs), 3xTF32 caps at 128 so the smem ring
// keeps three stages.
int pick_bn(rtb_ctx* ctx, const GemmDesc& d) {
  static const int forced = env_int("RTB_GEMM_BN", 0);
  if (forced == 64 || forced == 128 || (forced == 256 && !d.split3)) return forced;
  const int64_t tm = (d.M + kBM - 1) / kBM;
  const int cands_split[2] = {128, 64};
  const int cands_fast[3] = {256, 128, 64};
  const int* c = d.split3 ? cands_split : cands_fast;
  const int nc = d.split3 ? 2 : 3;
  const int64_t num_kb = (d.K + kBK - 1) / kBK;
  for (int i = 0; i < nc; ++i) {
    if (c[i] > 64 && d.N <= c[i] / 2) continue;  // half the tile (or more) would be padding
    const int64_t tiles = tm * ((d.N + c[i] - 1) / c[i]);
    if (tiles >= ctx->sm_count) return c[i];
    // few tiles but a long K: the K split of the work units fills the SMs,
    // and a wider tile halves the per-k-block overhead per flop
    if (c[i] == 128 && d.allow_workspace && tiles * 2 <= ctx->sm_count &&
        num_kb >= 4 * ((ctx->sm_count + tiles - 1) / tiles))
      return 128;
  }
  return 64;
}

}  // namespace

int gemm_run(rtb_ctx* ctx, const GemmDesc& d, cudaStream_t stream) {
  if (d.M <= 0 || d.N <= 0 || d.K <= 0) return set_error(RTB_E_INVALID, "gemm_run: empty problem");
  if (d.M > INT32_MAX || d.N > INT32_MAX || d.K > INT32_MAX)
    return set_error(RTB_E_UNSUPPORTED, "gemm_run: dimension exceeds 2^31-1");
  const int bn = d.bn ? d.bn : pick_bn(ctx, d);

  CUtensorMap tmA, tmB;
  int st;
  if (d.gather == 1) {
    // A is gathered by the kernel; give the unused map a valid encoding.
    st = make_tmap_2d(&tmA, d.B, (uint64_t)d.K, (uint64_t)d.N, (uint64_t)d.ldb, kBK, 64, false);
  } else if (d.gather == 2) {
    st = make_tmap_im2col(&tmA, d.x, d.Nimg, d.H, d.W, d.Cp, d.R, d.S, d.sh, d.sw, d.ph, d.pw,
                          kBK, kBM, true);
  } else if (d.gather == 3) {  // one dense [128 pixels][Cp] box per filter tap
    st = make_tmap_im2col(&tmA, d.x, d.Nimg, d.H, d.W, d.Cp, d.R, d.S, d.sh, d.sw, d.ph, d.pw,
                          (uint32_t)d.Cp, kBM, false);
  } else {
    st = make_tmap_2d(&tmA, d.A, (uint64_t)d.K, (uint64_t)d.M, (uint64_t)d.lda, kBK, kBM, false);
  }
  if (st != RTB_OK) return st;
  if (d.b_mn_major)  // MN-major TF32 tiles use the 32-byte-atom 128B swizzle
    st = make_tmap_2d(&tmB, d.B, (uint64_t)d.N, (uint64_t)d.K, (uint64_t)d.ldb, 32, kBK, true);
  else
    st = make_tmap_2d(&tmB, d.B, (uint64_t)d.K, (uint64_t)d.N, (uint64_t)d.ldb, kBK, (uint32_t)bn,
                      false);
  if (st != RTB_OK) return st;

  GemmParams p{};
  p.M = (int)d.M;
  p.N = (int)d.N;
  p.K = (int)d.K;
  p.num_kb = (int)((d.K + kBK - 1) / kBK);
  // 3xTF32 promotion interval: the tensor core's accumulation error grows with
  // the length of one accumulation unit, not with K.  Measured relative
  // Frobenius errors for 8 k-blocks (256 K) per unit: 2.2e-6 on N(0,1) data,
  // 5.1e-6 on all-positive data (4 k-blocks: 1.2e-6 / 2.6e-6; 16: 4.0e-6 /
  // 1.0e-5), against the 1e-5 bound.
  static const int kb_acc_env = env_int("RTB_KB_PER_ACC", 0);
  p.kb_per_acc = d.split3 ? (kb_acc_env > 0 ? kb_acc_env : 8) : p.num_kb;
  // L2 prefetch measured no gain on B200 (the ring already hides the latency):
  // off unless RTB_PREFETCH_KB asks for it.
  static const int pf_env = env_int("RTB_PREFETCH_KB", 0);
  p.prefetch_kb = pf_env > 0 ? pf_env : 0;
  // The tensor core truncates fp32 operands to TF32 (pinned by a GPU test), so
  // the raw tile already is the "hi" part; RTB_SPLIT_TRUNC=0 selects the
  // round-to-nearest hi written back in place instead.
  static const int trunc_env = env_int("RTB_SPLIT_TRUNC", 1);
  p.split_trunc = trunc_env != 0;
  p.tiles_m = (int)((d.M + kBM - 1) / kBM);
  p.tiles_n = (int)((d.N + bn - 1) / bn);
  p.group_m = p.tiles_m < 16 ? p.tiles_m : 16;
  p.C = d.C;
  p.ldc = d.ldc;
  p.bias = d.bias;
  p.residual = d.residual;
  p.ldr = d.ldr;
  p.relu = d.relu;
  p.out_mode = d.out_mode;
  p.hw = d.hw;
  p.peer_c = d.peer_c;
  p.npeers = d.npeers;
  p.col_off = d.col_off;
  if (d.out_mode == 2 && (!d.peer_c || d.npeers <= 0 || d.residual))
    return set_error(RTB_E_INVALID, "gemm_run: peer output needs peer pointers and no residual");
  auto al16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; };
  p.vec_ok = (d.out_mode == 0) && al16(d.C) && (d.ldc % 4 == 0) && (!d.bias || al16(d.bias)) &&
             (!d.residual || (al16(d.residual) && d.ldr % 4 == 0));
  p.vec4_nchw = (d.out_mode == 1) && al16(d.C) && (!d.residual || al16(d.residual));
  // Row-major C leaves through TMA stores when the tensor map can describe it.
  CUtensorMap tmC;
  std::memset(&tmC, 0, sizeof tmC);
  p.c_tma = 0;
  if (d.out_mode == 0 && al16(d.C) && d.ldc % 4 == 0) {
    if (make_tmap_2d(&tmC, d.C, (uint64_t)d.N, (uint64_t)d.M, (uint64_t)d.ldc, 32, kBM, false) ==
        RTB_OK)
      p.c_tma = 1;
  }
  p.x = d.x;
  p.H = d.H;
  p.W = d.W;
  p.Cp = d.Cp;
  p.Ho = d.Ho;
  p.Wo = d.Wo;
  p.R = d.R;
  p.S = d.S;
  p.sh = d.sh;
  p.sw = d.sw;
  p.ph = d.ph;
  p.pw = d.pw;
  p.err = ctx->d_err;
  p.timeout_ns = ctx->timeout_ns;

  // Tail balancing: when the last wave of tiles would leave at least half of
  // the SMs idle, its tiles are cut along K into split_k pieces that run on
  // the otherwise idle SMs (e.g. 196 tiles on 148 SMs: 148 whole tiles, then
  // 48 tiles x 3 pieces).  The pieces' partial tiles go through a stream-
  // ordered workspace; RTB_TAIL_SPLIT=0 turns this off.
  const int64_t tiles = (int64_t)p.tiles_m * p.tiles_n;
  if (tiles > INT32_MAX / 8) return set_error(RTB_E_UNSUPPORTED, "gemm_run: too many tiles");
  p.full_units = (int)tiles;
  p.split_k = 1;
  p.num_units = (int)tiles;
  p.ws = nullptr;
  p.ws_cnt = nullptr;
  p.cnt_gen = 0;
  void* split_ws = nullptr;
  static const int tail_env = env_int("RTB_TAIL_SPLIT", 1);
  if (tail_env && d.allow_workspace) {
    const int64_t G = ctx->sm_count;
    const int64_t rem = tiles % G;
    if (rem > 0 && rem * 2 <= G) {
      // up to 16 pieces (a few tiles with a very long K, e.g. a conv's weight
      // gradient: 9 tiles x 784 k-blocks), each piece >= 4 k-blocks once the
      // split passes 8 (the last piece's fix-up reads every piece)
      int sk = (int)(G / rem);
      if (sk > 16) sk = 16;
      if (sk > 8 && sk > p.num_kb / 4) sk = p.num_kb / 4 > 8 ? p.num_kb / 4 : 8;
      if (sk > p.num_kb / 2) sk = p.num_kb / 2;  // every piece keeps >= 2 k-blocks
      if (sk >= 2 && rem <= kSplitCounters) {
        const size_t part_bytes = (size_t)rem * sk * bn * kBM * sizeof(float);
        const size_t cnt_off = (part_bytes + 255) & ~size_t(255);
        st = split_counters(ctx, stream, &p.ws_cnt, &p.cnt_gen);
        const bool own = (st == RTB_E_UNSUPPORTED);  // capturing: counters of this launch
        if (st != RTB_OK && !own) return st;
        st = ws_alloc(ctx, &split_ws, own ? cnt_off + (size_t)rem * 8 : part_bytes, stream);
        if (st != RTB_OK) return st;
        if (own) {
          p.ws_cnt = reinterpret_cast<unsigned long long*>(static_cast<char*>(split_ws) + cnt_off);
          p.cnt_gen = 1;
          cudaError_t e = cudaMemsetAsync(p.ws_cnt, 0, (size_t)rem * 8, stream);
          if (e != cudaSuccess) {
            ws_free(split_ws, stream);
            return cuda_status(e, "split counters memset");
          }
        }
        p.full_units = (int)(tiles - rem);
        p.split_k = sk;
        p.num_units = (int)(tiles - rem + rem * sk);
        p.ws = static_cast<float*>(split_ws);
      }
    }
  }
  {
    const int64_t grid = p.num_units < ctx->sm_count ? p.num_units : ctx->sm_count;
    p.trace = (ctx->trace && ctx->trace_capacity >= grid * kTraceSlots) ? ctx->trace : nullptr;
  }

  switch (bn) {
    case 64: st = launch_bn<64>(ctx, tmA, tmB, tmC, p, d, stream); break;
    case 128: st = launch_bn<128>(ctx, tmA, tmB, tmC, p, d, stream); break;
    case 256: st = launch_bn<256>(ctx, tmA, tmB, tmC, p, d, stream); break;
    default: st = set_error(RTB_E_INVALID, "gemm_run: bad tile width");
  }
  ws_free(split_ws, stream);
  return st;
}

}  // namespace rtb
