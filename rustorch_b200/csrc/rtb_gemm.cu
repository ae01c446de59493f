// Tile selection, tensor maps, work units and launch of the tcgen05 GEMM
// engine (rtb_gemm.cuh).
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "rtb_gemm.cuh"
#include "rtb_internal.h"

namespace rtb {

// One instantiation per tile width, each in its own translation unit
// (rtb_gemm_bn64.cu, rtb_gemm_bn128.cu, rtb_gemm_bn256.cu) so they compile in
// parallel.
template <int BN>
int launch_bn(rtb_ctx* ctx, const CUtensorMap& tmA, const CUtensorMap& tmB,
              const CUtensorMap& tmBlo, const CUtensorMap& tmC, const GemmParams& p,
              const GemmDesc& d, cudaStream_t s);
extern template int launch_bn<64>(rtb_ctx*, const CUtensorMap&, const CUtensorMap&,
                                  const CUtensorMap&, const CUtensorMap&, const GemmParams&,
                                  const GemmDesc&, cudaStream_t);
extern template int launch_bn<128>(rtb_ctx*, const CUtensorMap&, const CUtensorMap&,
                                   const CUtensorMap&, const CUtensorMap&, const GemmParams&,
                                   const GemmDesc&, cudaStream_t);
extern template int launch_bn<256>(rtb_ctx*, const CUtensorMap&, const CUtensorMap&,
                                   const CUtensorMap&, const CUtensorMap&, const GemmParams&,
                                   const GemmDesc&, cudaStream_t);

namespace {

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

// Work-unit schedule of one launch: the first `full` tiles run whole, the
// other tiles - full are cut along K into `sk` pieces (consecutive k-block
// ranges) whose partial tiles are summed in piece order by the last to arrive.
struct SplitPlan {
  int64_t full = 0;
  int sk = 1;
  double cost = 0.0;  // estimated span in k-block times
};

// Cost model in k-block times: units are dealt round-robin to the G resident
// CTAs (CTA c runs units c, c + G, ...), a whole tile costs its k-blocks plus
// one for the pipeline fill and the epilogue tail, a piece its k-blocks plus
// 8 (the partial tile's round trip through the workspace and the arrival
// count: fitted to B200 timings of 1024^3, 2048^3 and ResNet convs with 2 to
// 5 pieces per tile, where a piece cost 7.6 to 13 k-block times more than its
// share of the mainloop) plus the share of its tile's fix-up (every partial
// read back: 1 per piece when the partials are staged through the idle load
// ring, which holds two chunks of up to 5 pieces; 2 per piece read straight
// from L2 beyond that; a trace of R50 stage 4 with 5 pieces per tile showed
// the queued fix-ups running 6.5-12.5 us past the CTAs' last units).
double plan_cost(int64_t tiles, int64_t split, int sk, int num_kb, int64_t G) {
  const int64_t full = tiles - split;
  const int64_t units = full + split * sk;
  const int64_t grid = units < G ? units : G;
  const double c_tile = num_kb + 1.0;
  const double c_piece = (double)((num_kb + sk - 1) / sk) + 8.0 + (sk <= 5 ? 1.0 : 2.0) * sk;
  double worst = 0.0;
  for (int64_t c = 0; c < grid; ++c) {
    const int64_t n_full = full > c ? (full - c + grid - 1) / grid : 0;
    // first unit index >= full that CTA c runs
    int64_t first = c + n_full * grid;
    const int64_t n_piece = first < units ? (units - 1 - first) / grid + 1 : 0;
    const double t = n_full * c_tile + n_piece * c_piece;
    worst = t > worst ? t : worst;
  }
  return worst;
}

// The cheapest schedule for `tiles` tiles of num_kb k-blocks on G CTAs: no
// split, or the last `split` tiles (the partial last wave, plus whole waves
// before it) cut into 2..16 pieces of >= 2 k-blocks (>= 4 beyond 8 pieces),
// within the split-counter block and a 256 MiB partial-tile workspace.
SplitPlan plan_split(int64_t tiles, int num_kb, int64_t G, int bn) {
  SplitPlan best;
  best.full = tiles;
  best.cost = plan_cost(tiles, 0, 1, num_kb, G);
  const double base = best.cost;
  const int64_t rem = tiles % G;
  if (rem == 0) return best;
  // RTB_SPLIT_K: the last wave's tiles cut into exactly that many pieces
  // (measurements)
  static const int forced_sk = env_int("RTB_SPLIT_K", 0);
  if (forced_sk >= 2 && forced_sk <= 16 && num_kb / forced_sk >= 2 && rem <= kSplitCounters) {
    best.full = tiles - rem;
    best.sk = forced_sk;
    best.cost = plan_cost(tiles, rem, forced_sk, num_kb, G);
    return best;
  }
  for (int64_t split = rem; split <= tiles && split <= kSplitCounters; split += G) {
    for (int sk = 2; sk <= 16; ++sk) {
      const int kbp = num_kb / sk;
      if (kbp < 2 || (sk > 8 && kbp < 4)) break;
      if ((double)split * sk * bn * kBM * 4.0 > 256.0 * (1 << 20)) break;
      const double c = plan_cost(tiles, split, sk, num_kb, G);
      if (c < best.cost && c < base - 0.5) {  // a split must beat no split by half a k-block
        best.full = tiles - split;
        best.sk = sk;
        best.cost = c;
      }
    }
  }
  return best;
}

}  // namespace

// The tensor core truncates fp32 operands to TF32 (pinned by a GPU test), so
// the raw tile already is the 3xTF32 "hi" part; RTB_SPLIT_TRUNC=0 selects the
// round-to-nearest hi written back in place instead.
static bool trunc_split_enabled() {
  static const int trunc_env = env_int("RTB_SPLIT_TRUNC", 1);
  return trunc_env != 0;
}

int gemm_run(rtb_ctx* ctx, const GemmDesc& d, cudaStream_t stream) {
  if (d.M <= 0 || d.N <= 0 || d.K <= 0) return set_error(RTB_E_INVALID, "gemm_run: empty problem");
  if (d.M > INT32_MAX || d.N > INT32_MAX || d.K > INT32_MAX)
    return set_error(RTB_E_UNSUPPORTED, "gemm_run: dimension exceeds 2^31-1");
  if (d.gather == 3 && d.Cp != 8 && d.Cp != 16)
    return set_error(RTB_E_INVALID, "gemm_run: multi-tap im2col takes 8 or 16 channels");
  if (d.a_mn_major && (!d.split3 || d.gather != 0))
    return set_error(RTB_E_INVALID, "gemm_run: an MN-major A needs 3xTF32 and no conv producer");
  if (d.row_bias && (d.out_mode != 1 || d.bias))
    return set_error(RTB_E_INVALID, "gemm_run: a row bias needs the transposed output, no column bias");
  static const int tail_env = env_int("RTB_TAIL_SPLIT", 1);
  const bool can_split = tail_env && d.allow_workspace;
  const int64_t num_kb64 = (d.K + kBK - 1) / kBK;
  const int64_t tiles_m64 = (d.M + kBM - 1) / kBM;
  int bn = d.bn ? d.bn : pick_bn(ctx, d);
  SplitPlan plan;
  plan.full = tiles_m64 * ((d.N + bn - 1) / bn);
  if (can_split && num_kb64 <= INT32_MAX) {
    plan = plan_split(plan.full, (int)num_kb64, ctx->sm_count, bn);
    // 3xTF32 with the tile width left open: 128 and 64 columns compared under
    // their schedules, at the measured k-block times of the two modes (B200,
    // 4096^3 forced to each width: 0.70 us per 128-column k-block, 0.47 us per
    // 64-column one in the wide mode, which does half the work; 1024^3 then
    // runs as one wave of 64-column tiles, 92 TFLOP/s, instead of 128-column
    // tiles cut in two K pieces, 77)
    if (d.split3 && !d.bn && std::getenv("RTB_GEMM_BN") == nullptr && d.N > 64) {
      const int alt = bn == 128 ? 64 : 128;
      const int64_t tiles_alt = tiles_m64 * ((d.N + alt - 1) / alt);
      const SplitPlan pa = plan_split(tiles_alt, (int)num_kb64, ctx->sm_count, alt);
      const double t_cur = plan.cost * (bn == 128 ? 0.70 : 0.47);
      const double t_alt = pa.cost * (alt == 128 ? 0.70 : 0.47);
      if (t_alt < t_cur * 0.97) {
        bn = alt;
        plan = pa;
      }
    }
  }

  CUtensorMap tmA, tmB;
  int st;
  if (d.gather == 1) {
    // A is gathered by the kernel; give the unused map a valid encoding.
    st = make_tmap_2d(&tmA, d.B, (uint64_t)d.K, (uint64_t)d.N, (uint64_t)d.ldb, kBK, 64, false);
  } else if (d.gather == 2) {
    st = make_tmap_im2col(&tmA, d.x, d.Nimg, d.H, d.W, d.Cp, d.R, d.S, d.sh, d.sw, d.ph, d.pw,
                          kBK, kBM, 128);
  } else if (d.gather == 3) {
    // one [128 pixels][Cp] box per filter tap, its Cp*4-byte rows swizzled
    // over their own width (the converters' reads of one 16-byte chunk of
    // 32 consecutive rows then spread over all banks; dense 64-byte rows
    // collide 16 ways)
    const int swz = (d.Cp * 4 == 32 || d.Cp * 4 == 64) ? d.Cp * 4 : 0;
    st = make_tmap_im2col(&tmA, d.x, d.Nimg, d.H, d.W, d.Cp, d.R, d.S, d.sh, d.sw, d.ph, d.pw,
                          (uint32_t)d.Cp, kBM, swz);
  } else if (d.a_mn_major) {
    // [K, M] row-major: unswizzled [32 k][128 m] boxes (512-byte rows), read
    // by the converters only
    st = make_tmap_2d_swz(&tmA, d.A, (uint64_t)d.M, (uint64_t)d.K, (uint64_t)d.lda, kBM, kBK,
                          kTmapSwizzleNone);
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
  // L2 prefetch measured no gain on B200 (the ring already hides the latency,
  // also for the transposed skinny GEMM that streams B from DRAM: 2-16
  // k-blocks ahead within 1%): off unless RTB_PREFETCH_KB asks for it.
  static const int pf_env = env_int("RTB_PREFETCH_KB", 0);
  p.prefetch_kb = pf_env > 0 ? pf_env : 0;
  p.split_trunc = trunc_split_enabled();
  p.tiles_m = (int)((d.M + kBM - 1) / kBM);
  p.tiles_n = (int)((d.N + bn - 1) / bn);
  // Raster: consecutive tiles walk down group_m M-tiles, then across N
  // (RTB_GROUP_M overrides the band height for measurements).
  // Bands of 12 M-tiles make a wave of 148 tiles about square (12 x 12.3),
  // the fewest A and B panels per wave: 8192^3 reads 3.34 GB from DRAM per
  // launch (8: 3.40, 16: 3.59, 4: 5.08), at the same speed within run-to-run
  // noise (196-209 TFLOP/s for every band from 4 to 16, interleaved
  // processes on one B200; the kernel is bound by its mainloop, not DRAM).
  static const int gm_env = env_int("RTB_GROUP_M", 12);
  const int gm = gm_env > 0 ? gm_env : 12;
  p.group_m = p.tiles_m < gm ? p.tiles_m : gm;
  p.C = d.C;
  p.ldc = d.ldc;
  p.bias = d.bias;
  p.residual = d.residual;
  p.ldr = d.ldr;
  p.act = d.act;
  p.out_mode = d.out_mode;
  p.hw = d.hw;
  p.row_bias = d.row_bias;
  p.peer_c = d.peer_c;
  p.npeers = d.npeers;
  p.col_off = d.col_off;
  if (d.out_mode == 2 && (!d.peer_c || d.npeers <= 0 || d.residual))
    return set_error(RTB_E_INVALID, "gemm_run: peer output needs peer pointers and no residual");
  auto al16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; };
  p.vec_ok = (d.out_mode == 0) && al16(d.C) && (d.ldc % 4 == 0) && (!d.bias || al16(d.bias)) &&
             (!d.residual || (al16(d.residual) && d.ldr % 4 == 0));
  p.vec4_nchw = (d.out_mode == 1) && al16(d.C) && (!d.residual || al16(d.residual)) &&
                (!d.row_bias || al16(d.row_bias));
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

  // K-split schedule (plan_split above): the last `rem` tiles (the partial
  // last wave, or whole waves more when that balances better) are cut along K
  // into split_k pieces, e.g. R50 stage-3 3x3 (98 tiles of 72 k-blocks on
  // 148 SMs): 98 x 3 pieces instead of 98 whole tiles on 98 SMs.  The pieces'
  // partial tiles go through a stream-ordered workspace; RTB_TAIL_SPLIT=0
  // turns splitting off.
  const int64_t tiles = (int64_t)p.tiles_m * p.tiles_n;
  if (tiles > INT32_MAX / 8) return set_error(RTB_E_UNSUPPORTED, "gemm_run: too many tiles");
  p.full_units = (int)tiles;
  p.split_k = 1;
  p.num_units = (int)tiles;
  p.ws = nullptr;
  p.ws_cnt = nullptr;
  p.cnt_gen = 0;
  void* split_ws = nullptr;
  if (plan.sk > 1 && plan.full < tiles) {
    const int64_t rem = tiles - plan.full;
    const int sk = plan.sk;
    const size_t part_bytes = (size_t)rem * sk * bn * kBM * sizeof(float);
    const size_t cnt_off = (part_bytes + 255) & ~size_t(255);
    st = split_counters(ctx, stream, &p.ws_cnt, &p.cnt_gen);
    const bool own = (st == RTB_E_UNSUPPORTED);  // capture / per-thread stream: own counters
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
  {
    const int64_t grid = p.num_units < ctx->sm_count ? p.num_units : ctx->sm_count;
    p.trace = (ctx->trace && ctx->trace_capacity >= grid * kTraceSlots) ? ctx->trace : nullptr;
  }

  // 3xTF32 tiles with a B_lo slot in the ring stage: B's low part
  // (B - trunc_tf32(B), a property of B alone) computed once per call by a
  // prepass and brought in by TMA beside B, instead of by the converter warps
  // of every CTA that reads the B tile (once per M-tile).  Measured on B200
  // (4096^3): converters 714 -> 341 clocks per k-block, mainloop 1219 -> 970.
  // The prepass is one more launch the GEMM waits for, so it is left to the
  // converters below 16 M-tiles (1024^3: 85 -> 70 TFLOP/s with it), and when
  // no workspace may be allocated.
  static const int blo_env = env_int("RTB_BLO_PREPASS", -1);
  const bool blo_slot = d.split3 && (bn == 64 || (bn == 128 && d.gather != 3));
  const bool want_blo = blo_env >= 0 ? blo_env != 0 : tiles_m64 >= 16;
  CUtensorMap tmBlo = tmB;
  void* blo_ws = nullptr;
  bool blo_given = false;
  if (blo_slot && d.B_lo && trunc_split_enabled() && blo_env != 0) {
    // computed by the caller (a weight pack): B's layout and row stride
    if (d.b_mn_major)
      st = make_tmap_2d(&tmBlo, d.B_lo, (uint64_t)d.N, (uint64_t)d.K, (uint64_t)d.ldb, 32, kBK, true);
    else
      st = make_tmap_2d(&tmBlo, d.B_lo, (uint64_t)d.K, (uint64_t)d.N, (uint64_t)d.ldb, kBK,
                        (uint32_t)bn, false);
    if (st != RTB_OK) {
      ws_free(split_ws, stream);
      return st;
    }
    blo_given = true;
  } else if (blo_slot && want_blo && d.allow_workspace && trunc_split_enabled()) {
    const int64_t rows = d.b_mn_major ? d.K : d.N;
    const int64_t cols = d.b_mn_major ? d.N : d.K;
    const int64_t ldo = (cols + 3) & ~int64_t(3);
    st = ws_alloc(ctx, &blo_ws, (size_t)(rows * ldo) * sizeof(float), stream);
    if (st != RTB_OK) {
      ws_free(split_ws, stream);
      return st;
    }
    float* blo = static_cast<float*>(blo_ws);
    st = launch_tf32_lo(d.B, rows, cols, d.ldb, blo, ldo, stream);
    if (st == RTB_OK) {
      if (d.b_mn_major)
        st = make_tmap_2d(&tmBlo, blo, (uint64_t)d.N, (uint64_t)d.K, (uint64_t)ldo, 32, kBK, true);
      else
        st = make_tmap_2d(&tmBlo, blo, (uint64_t)d.K, (uint64_t)d.N, (uint64_t)ldo, kBK,
                          (uint32_t)bn, false);
    }
    if (st != RTB_OK) {
      ws_free(blo_ws, stream);
      ws_free(split_ws, stream);
      return st;
    }
  }
  p.blo_tma = blo_given || blo_ws != nullptr;


  switch (bn) {
    case 64: st = launch_bn<64>(ctx, tmA, tmB, tmBlo, tmC, p, d, stream); break;
    case 128: st = launch_bn<128>(ctx, tmA, tmB, tmBlo, tmC, p, d, stream); break;
    case 256: st = launch_bn<256>(ctx, tmA, tmB, tmBlo, tmC, p, d, stream); break;
    default: st = set_error(RTB_E_INVALID, "gemm_run: bad tile width");
  }
  ws_free(split_ws, stream);
  ws_free(blo_ws, stream);
  return st;
}

}  // namespace rtb
