// Persistent, warp-specialised tcgen05 GEMM / implicit-GEMM conv for sm_100a.
//
//   C[M,N] = act( A[M,K] . B[K,N] + bias[N] + residual[M,N] )
//
// Tiles: BM=128 rows x BN (64/128/256) columns, k-blocks of BK=32 fp32 (one
// 128-byte swizzle atom).  Roles (warp index):
//   0        TMA producer: A (unless gathered) and B tiles -> smem ring
//   1        TMEM allocator + single-thread UMMA issuer (kind::tf32, M=128)
//   2..5     epilogue: TMEM -> registers -> bias/residual/activation -> global
//   6..9     (3xTF32 only) converters: split each fp32 tile in smem into a
//            TF32 "hi" part (in place, round-to-nearest) and the exact fp32
//            remainder "lo" (separate plane); UMMA then accumulates
//            hi*hi + hi*lo + lo*hi (split-precision TF32, Ootomo & Yokota 2022)
//   next 4   (conv, A_MODE 1) im2col gather: 16-byte cp.async of NHWC input
//            rows into the swizzled A tile, zero-filling padding taps
// A operand modes: 0 = tiled TMA of a K-major matrix; 1 = cp.async im2col
// gather (any Cp % 4 == 0); 2 = TMA im2col (Cp % 32 == 0: every k-block is one
// filter tap x 32 channels, fetched by one bulk tensor copy per k-block);
// 3 = multi-tap TMA im2col; 4 = tiled TMA of an MN-major matrix ([K, M]
// row-major, 3xTF32 only: the converters read the unswizzled [32 k][128 m]
// tile column-wise, so the MMAs never see its layout).
// The accumulator is double-buffered in TMEM (2 x BN columns) so the epilogue
// of tile i overlaps the mainloop of tile i+1.
//
// Accumulator promotion (3xTF32): the tensor core's internal accumulation does
// not round every addition to nearest fp32, so its error grows linearly with
// the length of the accumulation chain.  The MMA issuer therefore restarts the
// TMEM accumulator every `kb_per_acc` k-blocks (one "accumulation unit"), and
// the epilogue warps add each unit's partial sum into an fp32 running sum kept
// in a third TMEM buffer (round-to-nearest adds on the CUDA cores), emitting
// the tile after its last unit.  TF32 mode uses one unit per tile.
//
// Layouts in shared memory (all 128B-swizzled, 1024-byte aligned):
//   A tile, K-major:  row r (M) at r*128 B, 32 fp32 of K per row.
//   B tile, K-major:  same with BN rows (B given as [N,K], e.g. Linear.weight).
//   B tile, MN-major: BN/32 boxes of 32 K-rows x 128 B (32 N values), 4 KB each
//                     (B given as [K,N] row-major, e.g. Tensor::matmul's rhs).
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

#include "rtb_act.cuh"
#include "rtb_ptx.cuh"

namespace rtb {

constexpr int kBM = 128;
constexpr uint32_t kConvSleepNs = 64;  // converters' back-off between barrier tests
constexpr int kBK = 32;                      // fp32 elements per k-block (128 B)
constexpr int kABytes = kBM * kBK * 4;       // 16 KB
constexpr int kSmemLimit = 232448;           // 227 KB dynamic shared memory per CTA
constexpr int kSmemReserve = 3072;           // bias staging (1 KB) + barriers + alignment slack
constexpr int kOutChunkBytes = kBM * 32 * 4;  // one 128 x 32 fp32 output chunk (16 KB)

struct GemmParams {
  int M, N, K;
  int num_kb;            // ceil(K / 32)
  int kb_per_acc;        // k-blocks accumulated on the tensor core before promotion
  int prefetch_kb;       // L2 prefetch distance in k-blocks (0 = off)
  int split_trunc;       // 3xTF32 hi part: 1 = the tensor core's own truncation of the
                         // raw fp32 (lo = x - trunc(x)); 0 = round-to-nearest hi
                         // written back in place
  int tiles_m, tiles_n;
  int group_m;           // raster: tiles grouped by this many M-tiles
  // output / epilogue
  float* C;
  int64_t ldc;
  const float* bias;     // [N] or null
  const float* residual; // same indexing as C, or null
  int64_t ldr;
  int act;               // RTB_ACT_*: none, ReLU, sigmoid, tanh (after bias and residual)
  int out_mode;          // 0: C[m*ldc+n]; 1: NCHW scatter, m=(img,pix), C[(img*N+n)*hw+pix];
                         // 2: every rank's C, peer_c[r][m*ldc + col_off + n] (N-split)
  int hw;                // Ho*Wo for out_mode 1
  const float* row_bias; // out_mode 1: [M] bias per row (C^T of a skinny GEMM), or null
  int vec_ok;            // 16-byte aligned C/residual/bias with ldc, ldr % 4 == 0
  int c_tma;             // out_mode 0 with a TMA-storable C (tmC valid)
  int vec4_nchw;         // out_mode 1: C and residual 16-byte aligned
  // implicit-GEMM conv (A gathered from NHWC input with Cp channels, Cp % 4 == 0)
  const float* x;
  int H, W, Cp, Ho, Wo, R, S, sh, sw, ph, pw;
  // out_mode 2: base pointers of the npeers ranks' C (this rank's own included),
  // written over NVLink by the epilogue; col_off = this rank's first column
  float* const* peer_c;
  int npeers;
  int64_t col_off;
  // failure reporting
  int* err;
  unsigned long long timeout_ns;
  // optional timeline trace: per CTA kTraceSlots globaltimer stamps (null = off)
  unsigned long long* trace;
  // Work units (tail balancing).  Units [0, full_units) are whole tiles
  // 0..full_units-1; the remaining tiles_m*tiles_n - full_units "tail" tiles
  // are each cut into split_k pieces along K (consecutive k-block ranges),
  // one unit per piece.  A piece leaves its fp32 partial tile in ws; the last
  // piece of a tile to arrive (ws_cnt) sums the pieces in piece order and runs
  // the epilogue, so the result does not depend on arrival order.
  int full_units;
  int split_k;           // 1 = no split
  int num_units;
  float* ws;             // [tail tile][piece][BN/32][8][128] float4
  unsigned long long* ws_cnt;  // [tail tile] arrival words (generation << 8 | count)
  unsigned long long cnt_gen;  // this launch's generation (older tags count as zero)
  // 3xTF32 wide tiles: B's low part arrives by TMA (tmBlo, B's layout) in the
  // ring stage's B_lo slot, and the converters leave B alone
  int blo_tma;
};

struct WorkUnit {
  int tile;
  int kb0, kb1;  // k-block range [kb0, kb1)
  int piece;     // -1 = whole tile
  int slot;      // tail tile index (pieces only)
};

__device__ __forceinline__ WorkUnit work_unit(const GemmParams& p, int w) {
  WorkUnit u;
  if (w < p.full_units) {
    u.tile = w;
    u.kb0 = 0;
    u.kb1 = p.num_kb;
    u.piece = -1;
    u.slot = -1;
  } else {
    const int j = w - p.full_units;
    const int q = j / p.split_k;
    const int piece = j - q * p.split_k;
    u.tile = p.full_units + q;
    u.kb0 = (int)((int64_t)piece * p.num_kb / p.split_k);
    u.kb1 = (int)((int64_t)(piece + 1) * p.num_kb / p.split_k);
    u.piece = piece;
    u.slot = q;
  }
  return u;
}

// Trace slot layout per CTA (first kTraceTiles tiles of the CTA):
//   0 start, 1 end, then per tile j at 2+6j: producer first issue, MMA first
//   k-block ready, MMA last commit, epilogue sees the first accumulation unit,
//   epilogue sees the last unit, epilogue done.
constexpr int kTraceTiles = 3;
constexpr int kTraceSlots = 2 + 6 * kTraceTiles;
__device__ __forceinline__ void trace_stamp(const GemmParams& p, int slot) {
  if (p.trace) p.trace[(size_t)blockIdx.x * kTraceSlots + slot] = globaltimer_ns();
}

// Shared-memory read bandwidth (about 128 B per clock per SM on B200) is
// shared by the tensor core's operand reads and the warps' ld.shared, so the
// 3xTF32 mainloop keeps A's hi and lo parts in TMEM (the MMAs read only B
// and B_lo from shared memory) and the converters read each raw A tile once.
// Per 128-column k-block: 48 KB of operand reads + 16 KB of converter reads
// (+ 16 KB more when the converters also make B's low part), about 500-625
// clocks against the 768 clocks of MMAs.
//
// BLO (3xTF32 with the A tile in the 128B-swizzled K-major layout, i.e. every
// producer but the multi-tap im2col): B's low part has a slot in every ring
// stage, right after the raw B tile, so it can arrive by TMA from a copy
// computed once per call (B - trunc_tf32(B) is a property of B alone) instead
// of being recomputed by the converters of every CTA that reads the B tile.
// (A 128-column tile could then also issue hi . [B | B_lo] as one N=256 MMA,
// but its 256-column partial leaves TMEM room for one partial buffer only,
// and the MMAs idling while the epilogue drains it cost more than the third
// instruction per k-step: three N=128 MMAs, double-buffered partials.)
template <int BN, bool SPLIT, bool BLO = false>
struct GemmCfg {
  static constexpr int kBBytes = BN * kBK * 4;
  // TMEM: the partial-sum buffer(s); with 3xTF32 one fp32 running sum the
  // epilogue warps promote the partials into, then a ring of kAStages
  // converted k-blocks: A's 32-column hi and lo parts.
  // Wide mode: B's low part sits right after the raw B tile in the ring
  // stage, so hi_A . [B | B_lo] is ONE MMA of twice the tile width (partial
  // columns [0,BN) = hi.hi, [BN,2BN) = hi.lo) and lo_A . B one MMA of the
  // tile width: two tensor-core instructions per k-step instead of three; the
  // epilogue adds the two halves.  Otherwise B's low part has its own
  // shared-memory plane of kAStages slots.
  static_assert(!BLO || SPLIT, "BLO is a 3xTF32 layout");
  static constexpr bool kWide = SPLIT && BN == 64;
  static constexpr int kAccW = kWide ? 2 * BN : BN;  // TMEM columns of one partial buffer
  static constexpr int kAccCols = 2 * kAccW + (SPLIT ? BN : 0);
  static constexpr int kAStagesRaw = SPLIT ? (512 - kAccCols) / (2 * kBK) : 0;
  static constexpr int kAStages = kAStagesRaw > 4 ? 4 : kAStagesRaw;
  static constexpr bool kBloInStage = kWide || BLO;
  static constexpr int kBStage = kBloInStage ? 2 * kBBytes : kBBytes;  // B slot of a ring stage
  static constexpr int kBloBytes = (SPLIT && !kBloInStage) ? kAStages * kBBytes : 0;
  // Load ring stage: the raw A and B tiles (TMA) (+ B's low part).
  static constexpr int kStageBytes = kABytes + kBStage;
  // Epilogue staging: two 16 KB chunks alternate, unless dropping one gives
  // the load ring another stage.
  static constexpr int kRingBytes = kSmemLimit - kSmemReserve - kBloBytes;
  static constexpr int kOutBufs =
      (kRingBytes - kOutChunkBytes) / kStageBytes > (kRingBytes - 2 * kOutChunkBytes) / kStageBytes
          ? 1 : 2;
  static constexpr int kOutBytes = kOutBufs * kOutChunkBytes;
  static constexpr int kStagesRaw = (kRingBytes - kOutBytes) / kStageBytes;
  static constexpr int kStages = kStagesRaw > 8 ? 8 : kStagesRaw;
  static constexpr int kSmemBytes =
      kStages * kStageBytes + kBloBytes + kOutBytes + kSmemReserve;
  static constexpr int kTmemNeed = kAccCols + kAStages * 2 * kBK;
  static constexpr int kTmemCols = kTmemNeed <= 128 ? 128 : (kTmemNeed <= 256 ? 256 : 512);
  static_assert(kTmemNeed <= 512, "TMEM holds 512 columns");
  static_assert(!SPLIT || kAStages >= 2, "3xTF32 needs BN <= 128 (two TMEM A stages)");
  static_assert(kStages >= 2, "need at least two pipeline stages");
  static_assert(BN == 64 || BN == 128 || BN == 256, "BN must be 64, 128 or 256");
};

// The configuration a kernel variant uses: B_lo in the ring stage for every
// 3xTF32 producer whose A tile is in the swizzled K-major layout (all but the
// multi-tap im2col, whose tiles the converters read in their own layout).
template <int BN, bool SPLIT, int A_MODE>
using GemmCfgFor = GemmCfg<BN, SPLIT, SPLIT && A_MODE != 3>;

template <bool SPLIT, bool GATHER>
struct GemmRoles {  // GATHER: the cp.async im2col producer warps are present
  static constexpr int kWarpTma = 0;
  static constexpr int kWarpMma = 1;
  static constexpr int kWarpEpi = 2;                        // 4 warps
  static constexpr int kWarpConv = 6;                       // 4 warps if SPLIT
  static constexpr int kWarpGather = 6 + (SPLIT ? 4 : 0);   // 4 warps if GATHER
  // second TMA producer (alternate k-blocks with warp 0)
  static constexpr int kWarpTma2 = 6 + (SPLIT ? 4 : 0) + (GATHER ? 4 : 0);
  static constexpr int kWarps = kWarpTma2 + 1;
  static constexpr int kThreads = kWarps * 32;
};

__device__ __forceinline__ void tile_coords(int t, int tiles_m, int tiles_n, int group_m, int& tm,
                                            int& tn) {
  const int group_size = group_m * tiles_n;
  const int g = t / group_size;
  const int first_m = g * group_m;
  int gm = tiles_m - first_m;
  gm = gm < group_m ? gm : group_m;
  const int r = t - g * group_size;
  tm = first_m + r % gm;
  tn = r / gm;
}

__device__ __forceinline__ float4 tf32_hi4(float4 v) {
  float4 h;
  uint32_t a, b, c, d;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(a) : "f"(v.x));
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(b) : "f"(v.y));
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(c) : "f"(v.z));
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(d) : "f"(v.w));
  h.x = __uint_as_float(a);
  h.y = __uint_as_float(b);
  h.z = __uint_as_float(c);
  h.w = __uint_as_float(d);
  return h;
}

// x - trunc_tf32(x): the exact remainder below the 10 explicit mantissa bits a
// TF32 operand keeps when the low 13 bits of the fp32 pattern are dropped.
__device__ __forceinline__ float4 tf32_trunc_rem4(float4 v) {
  const float hx = __uint_as_float(__float_as_uint(v.x) & 0xFFFFE000u);
  const float hy = __uint_as_float(__float_as_uint(v.y) & 0xFFFFE000u);
  const float hz = __uint_as_float(__float_as_uint(v.z) & 0xFFFFE000u);
  const float hw = __uint_as_float(__float_as_uint(v.w) & 0xFFFFE000u);
  return make_float4(v.x - hx, v.y - hy, v.z - hz, v.w - hw);
}

// The epilogue functions below take `sb`: the shared-window address of the
// chunk's 32 bias values, staged once per tile (zero past N), used when
// p.bias is set; shared memory is addressed through 32-bit shared-window
// addresses (ld/st.shared) throughout.
// Every global load of a chunk is issued before its first store, so loads are
// not serialised behind stores the compiler cannot prove disjoint.

// Row-major epilogue for one thread's row m and 32 consecutive columns n0..n0+31.
__device__ __forceinline__ void epilogue_store32(const GemmParams& p, int m, int n0,
                                                 const uint32_t (&r)[32], uint32_t sb) {
  if (m >= p.M) return;
  float v[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
  if (p.bias) {
#pragma unroll
    for (int j = 0; j < 32; j += 4) {
      const float4 b = lds128(sb + 4 * j);
      v[j] += b.x; v[j + 1] += b.y; v[j + 2] += b.z; v[j + 3] += b.w;
    }
  }
  float* crow = p.C + (int64_t)m * p.ldc;
  const float* rrow = p.residual ? p.residual + (int64_t)m * p.ldr : nullptr;
  if (n0 + 32 <= p.N && p.vec_ok) {
    if (rrow) {
      float4 q[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) q[j] = __ldg(reinterpret_cast<const float4*>(rrow + n0) + j);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        v[4 * j] += q[j].x; v[4 * j + 1] += q[j].y; v[4 * j + 2] += q[j].z; v[4 * j + 3] += q[j].w;
      }
    }
    activate_n<32>(v, p.act);
#pragma unroll
    for (int j = 0; j < 32; j += 4)
      *reinterpret_cast<float4*>(crow + n0 + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
  } else {
    if (rrow) {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (n0 + j < p.N) v[j] += __ldg(rrow + n0 + j);
    }
    activate_n<32>(v, p.act);
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      if (n0 + j < p.N) crow[n0 + j] = v[j];
    }
  }
}

// N-split epilogue, after epilogue_stage_rowmajor has put the 128 x 32 chunk
// (bias/activation applied) into the 128B-swizzled staging buffer: thread et moves
// float4 f = et + 128*i (row f/8, column group f%8), so each warp store covers
// four whole 128-byte rows of C, into every rank's C at column col_off + n0
// (P2P stores over NVLink for the peers; whole-line writes, 16-byte aligned by
// the host's checks).
__device__ __forceinline__ void epilogue_store_peers(const GemmParams& p, uint32_t buf, int et,
                                                     int m0, int n0) {
#pragma unroll 2
  for (int i = 0; i < 8; ++i) {
    const int f = et + 128 * i;
    const int row = f >> 3, c4 = f & 7;
    const int m = m0 + row, n = n0 + 4 * c4;
    if (m >= p.M || n >= p.N) continue;
    const float4 v = lds128(buf + row * 128 + ((c4 ^ (row & 7)) << 4));
    for (int q = 0; q < p.npeers; ++q) {
      float* dst = p.peer_c[q] + (int64_t)m * p.ldc + p.col_off + n;
      if (n + 4 <= p.N) {
        *reinterpret_cast<float4*>(dst) = v;
      } else {
        const float e[4] = {v.x, v.y, v.z, v.w};
        for (int j = 0; j < 4 && n + j < p.N; ++j) dst[j] = e[j];
      }
    }
  }
}

// Row-major epilogue via TMA store: bias, residual and activation in registers, then
// this thread's row (32 fp32) into the 128 x 32 staging chunk, 128-byte
// swizzled (16-byte unit j of row r at position j ^ (r % 8)) to match the
// store map and keep the 8-thread phases of the writes conflict-free.
__device__ __forceinline__ void epilogue_stage_rowmajor(const GemmParams& p, uint32_t buf, int row,
                                                        int n0, int m, const uint32_t (&r)[32],
                                                        uint32_t sb) {
  float v[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
  if (p.bias) {
#pragma unroll
    for (int j = 0; j < 32; j += 4) {
      const float4 b = lds128(sb + 4 * j);
      v[j] += b.x; v[j + 1] += b.y; v[j + 2] += b.z; v[j + 3] += b.w;
    }
  }
  if (p.residual && m < p.M) {
    const float* rrow = p.residual + (int64_t)m * p.ldr;
    if (n0 + 32 <= p.N && p.vec_ok) {
      float4 q[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) q[j] = __ldg(reinterpret_cast<const float4*>(rrow + n0) + j);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        v[4 * j] += q[j].x; v[4 * j + 1] += q[j].y; v[4 * j + 2] += q[j].z; v[4 * j + 3] += q[j].w;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (n0 + j < p.N) v[j] += __ldg(rrow + n0 + j);
    }
  }
  activate_n<32>(v, p.act);
  const uint32_t rowp = buf + row * 128;
#pragma unroll
  for (int j = 0; j < 8; ++j)
    sts128(rowp + ((j ^ (row & 7)) << 4), make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]));
}

// NCHW epilogue: transpose the 128-pixel x 32-channel chunk through shared
// memory ([32 channels][128 pixels]), then each thread writes 4 consecutive
// pixels of 8 channels with 16-byte stores (a warp covers 512 contiguous bytes
// of one channel plane per store), adding bias and the NCHW residual and
// applying the activation there.  A thread keeps the same 4-pixel group (et % 32) for
// all of its channels, so the pixel -> (image, offset) division happens once
// per chunk, and the 8 loads are issued before the 8 stores.
__device__ __forceinline__ void epilogue_nchw_chunk(const GemmParams& p, uint32_t buf, int row,
                                                    int et, int m0, int n0,
                                                    const uint32_t (&r)[32], uint32_t sb) {
#pragma unroll
  for (int j = 0; j < 32; ++j) sts32(buf + (j * kBM + row) * 4, __uint_as_float(r[j]));
  named_bar_sync(1, 128);
  const int q = et & 31;   // 4-pixel group
  const int cw = et >> 5;  // channels cw, cw+4, ..., cw+28 of the chunk
  const int m = m0 + 4 * q;
  // 16-byte stores need every 4-pixel group inside one image and aligned:
  // images of a multiple of 4 pixels and a whole 128-pixel chunk (uniform
  // over the chunk)
  const bool vec = (p.hw % 4 == 0) && p.vec4_nchw && m0 + kBM <= p.M;
  {
    if (vec) {
      // the 4 pixels lie in one image
      const int img = m / p.hw;
      const int pix = m - img * p.hw;
      const float* rbase =
          p.residual ? p.residual + ((int64_t)img * p.N + n0) * p.hw + pix : nullptr;
      float* cbase = p.C + ((int64_t)img * p.N + n0) * p.hw + pix;
      // per-row bias of the 4 rows (16-byte aligned: checked by the host)
      const float4 rb = p.row_bias ? __ldg(reinterpret_cast<const float4*>(p.row_bias + m))
                                   : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int h = 0; h < 2; ++h) {  // two halves of 4 channels: loads, then stores
        float4 o[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int ch = cw + 4 * (4 * h + k);
          o[k] = lds128(buf + (ch * kBM + 4 * q) * 4);
          const float bv = p.bias ? lds32(sb + ch * 4) : 0.0f;
          o[k].x += bv; o[k].y += bv; o[k].z += bv; o[k].w += bv;
          if (p.row_bias) {
            o[k].x += rb.x; o[k].y += rb.y; o[k].z += rb.z; o[k].w += rb.w;
          }
          if (rbase && n0 + ch < p.N) {
            const float4 r4 = __ldg(reinterpret_cast<const float4*>(rbase + (int64_t)ch * p.hw));
            o[k].x += r4.x; o[k].y += r4.y; o[k].z += r4.z; o[k].w += r4.w;
          }
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int ch = cw + 4 * (4 * h + k);
          if (n0 + ch < p.N)
            *reinterpret_cast<float4*>(cbase + (int64_t)ch * p.hw) = activate4(o[k], p.act);
        }
      }
    } else {
      // general case (images of any size, the last chunk): warp cw writes
      // channels cw, cw+4, ..., lane l pixels l, l+32, l+64, l+96, so each
      // store instruction covers 32 consecutive pixels of one channel plane
      const int l = et & 31;
      int64_t pb[4];
      bool pv[4];
      float rbv[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int me = m0 + l + 32 * j;
        pv[j] = me < p.M;
        const int im = pv[j] ? me / p.hw : 0;
        pb[j] = pv[j] ? ((int64_t)im * p.N + n0) * p.hw + (me - im * p.hw) : 0;
        rbv[j] = (pv[j] && p.row_bias) ? __ldg(p.row_bias + me) : 0.0f;
      }
#pragma unroll 1
      for (int k = 0; k < 8; ++k) {
        const int ch = cw + 4 * k;
        if (n0 + ch >= p.N) continue;
        const float bv = p.bias ? lds32(sb + ch * 4) : 0.0f;
        float sv[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) sv[j] = lds32(buf + (ch * kBM + l + 32 * j) * 4) + bv;
        if (p.row_bias) {
#pragma unroll
          for (int j = 0; j < 4; ++j) sv[j] += rbv[j];
        }
        if (p.residual) {
#pragma unroll
          for (int j = 0; j < 4; ++j)
            if (pv[j]) sv[j] += __ldg(p.residual + pb[j] + (int64_t)ch * p.hw);
        }
#pragma unroll
        for (int j = 0; j < 4; ++j)
          if (pv[j]) p.C[pb[j] + (int64_t)ch * p.hw] = activate(sv[j], p.act);
      }
    }
  }
  named_bar_sync(1, 128);
}

// B_MN: 0 = B is K-major ([N,K] in memory), 1 = MN-major ([K,N] row-major).
template <int BN, bool SPLIT, int A_MODE, int B_MN>
__global__ void __launch_bounds__(GemmRoles<SPLIT, A_MODE == 1>::kThreads, 1)
    rtb_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    const __grid_constant__ CUtensorMap tmBlo,
                    const __grid_constant__ CUtensorMap tmC, const GemmParams p) {
  constexpr bool GATHER = (A_MODE == 1);
  constexpr bool IM2COL = (A_MODE == 2 || A_MODE == 3);
  constexpr bool MULTITAP = (A_MODE == 3);
  static_assert(!MULTITAP || SPLIT, "multi-tap im2col tiles are read by the 3xTF32 converters");
  static_assert(A_MODE != 4 || SPLIT, "MN-major A tiles are read by the 3xTF32 converters");
  using Cfg = GemmCfgFor<BN, SPLIT, A_MODE>;
  using Roles = GemmRoles<SPLIT, GATHER>;
  constexpr int S = Cfg::kStages;
  constexpr int kBBytes = Cfg::kBBytes;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  constexpr int kAS = SPLIT ? Cfg::kAStages : 1;
  uint8_t* sA = base;                                  // S x 16 KB
  uint8_t* sB = sA + S * kABytes;                      // S x kBStage (BN*128, + B's low part)
  uint8_t* sBlo = sB + S * Cfg::kBStage;               // SPLIT, B_lo not in the stage: kAS x BN*128
  uint8_t* sOut = sBlo + Cfg::kBloBytes;               // kOutBufs x 16 KB epilogue staging
  uint8_t* tail = sOut + Cfg::kOutBytes;
  float* sBias = reinterpret_cast<float*>(tail);         // epilogue: the tile's BN bias values
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(tail + 1024);
  uint64_t* conv_bar = full_bar + S;                     // SPLIT: [kAS] converted k-block ready
  uint64_t* empty_bar = conv_bar + kAS;
  uint64_t* tfull_bar = empty_bar + S;
  uint64_t* tempty_bar = tfull_bar + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty_bar + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* fix_flag = abort_flag + 1;  // epilogue: this CTA sums a split tile
  volatile int* epi_vote = abort_flag + 2;  // epilogue: per-warp wait outcome (4 ints)
  // epilogue: split tiles this CTA sums after its last unit: [0] = count,
  // then (tile, slot) pairs
  volatile int* pend = abort_flag + 6;
  constexpr int kMaxPending = 8;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full_bar[s], 1 + (GATHER ? 128 : 0));
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull_bar[b], 1);
      mbar_init(&tempty_bar[b], 128);
    }
    for (int j = 0; j < kAS; ++j) mbar_init(&conv_bar[j], 128);
    *abort_flag = 0;
    pend[0] = 0;
    fence_mbar_init();
  }
  if (warp == Roles::kWarpTma && lane == 0) {
    if (!GATHER) tma_prefetch_desc(&tmA);  // tiled or im2col map
    tma_prefetch_desc(&tmB);
    if (p.blo_tma) tma_prefetch_desc(&tmBlo);
    if (p.c_tma) tma_prefetch_desc(&tmC);
  }
  if (warp == Roles::kWarpMma) {
    tmem_alloc(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // Everything above touched only shared memory, TMEM and the kernel
  // parameters; global memory is read and written after the previous kernel
  // on the stream has completed (programmatic dependent launch).
  griddep_wait();
  griddep_launch_dependents();
  if (threadIdx.x == 0) trace_stamp(p, 0);

  if (warp == Roles::kWarpTma || warp == Roles::kWarpTma2) {
    // ------------------------------------------------------------ TMA producers
    // Lane 0 of two warps takes alternate k-blocks of the CTA's sequence: one
    // thread's wait + issue round trip (about 0.2 us on B200, whatever the box
    // size) would cap the ring's fill rate near 10 TB/s over 148 SMs.
    if (lane == 0) {
      const int pidx = warp == Roles::kWarpTma ? 0 : 1;
      int q = 0;  // k-block sequence number of this CTA
      int s = 0;
      uint32_t ph = 0;
      const uint32_t tx = (GATHER ? 0 : kABytes) + kBBytes * (p.blo_tma ? 2 : 1);
      const int HoWo = p.Ho * p.Wo;
      for (int w = blockIdx.x; w < p.num_units && !*abort_flag; w += gridDim.x) {
        const WorkUnit u = work_unit(p, w);
        int tm, tn;
        tile_coords(u.tile, p.tiles_m, p.tiles_n, p.group_m, tm, tn);
        // TMA im2col: input position of the tile's first output pixel.
        int a_w = 0, a_h = 0, a_n = 0;
        if (IM2COL) {
          const int m0 = tm * kBM;
          a_n = m0 / HoWo;
          const int rem = m0 - a_n * HoWo;
          const int oh = rem / p.Wo;
          a_h = oh * p.sh - p.ph;
          a_w = (rem - oh * p.Wo) * p.sw - p.pw;
        }
        const int tj = (w - (int)blockIdx.x) / (int)gridDim.x;
        for (int kb = u.kb0; kb < u.kb1; ++kb, ++q) {
          if ((q & 1) != pidx) {  // the other producer's k-block
            if (++s == S) { s = 0; ph ^= 1; }
            continue;
          }
          if (!mbar_wait_bounded(&empty_bar[s], ph ^ 1, abort_flag, p.err, DEV_TIMEOUT_EMPTY,
                                 p.timeout_ns))
            break;
          if (kb == u.kb0 && tj < kTraceTiles) trace_stamp(p, 2 + 6 * tj);
          // multi-tap: 32 / Cp filter taps per k-block, the last k-block may
          // hold fewer (no copy is issued for taps past R*S)
          const int tpk = MULTITAP ? kBK / p.Cp : 1;
          int ntaps = 0;
          if (MULTITAP) {
            ntaps = p.R * p.S - kb * tpk;
            ntaps = ntaps < tpk ? ntaps : tpk;
          }
          mbar_arrive_expect_tx(&full_bar[s],
                                MULTITAP ? (uint32_t)(ntaps * kBM * p.Cp * 4 + kBBytes *
                                                      (p.blo_tma ? 2 : 1))
                                         : tx);
          // Warm L2 for a k-block `prefetch_kb` ahead (hides DRAM latency beyond
          // what the shared-memory ring can cover).
          const int kp = kb + p.prefetch_kb;
          if (p.prefetch_kb > 0 && kp < u.kb1) {
            if (A_MODE == 0) {
              tma_prefetch_2d(&tmA, kp * kBK, tm * kBM);
              if (B_MN == 0) tma_prefetch_2d(&tmB, kp * kBK, tn * BN);
            } else if (A_MODE == 4) {
              tma_prefetch_2d(&tmA, tm * kBM, kp * kBK);
            } else if (IM2COL && !MULTITAP) {
              const int k0 = kp * kBK, tap = k0 / p.Cp, rr = tap / p.S;
              tma_prefetch_im2col_4d(&tmA, k0 - tap * p.Cp, a_w, a_h, a_n,
                                     (uint16_t)(tap - rr * p.S), (uint16_t)rr);
            }
          }
          if (A_MODE == 0) {
            tma_load_2d(sA + s * kABytes, &tmA, &full_bar[s], kb * kBK, tm * kBM);
          } else if (A_MODE == 4) {
            // [32 k][128 m] box of the [K, M] matrix (m is the inner coordinate)
            tma_load_2d(sA + s * kABytes, &tmA, &full_bar[s], tm * kBM, kb * kBK);
          } else if (MULTITAP) {
            // tap j of the k-block -> dense [128 pixels][Cp] block j of the A tile
            for (int j = 0; j < ntaps; ++j) {
              const int tap = kb * tpk + j;
              const int rr = tap / p.S;
              const int ss = tap - rr * p.S;
              tma_load_im2col_4d(sA + s * kABytes + j * (kBM * p.Cp * 4), &tmA, &full_bar[s], 0,
                                 a_w, a_h, a_n, (uint16_t)ss, (uint16_t)rr);
            }
          } else if (IM2COL) {
            const int k0 = kb * kBK;
            const int tap = k0 / p.Cp;           // one filter tap per k-block (Cp % 32 == 0)
            const int c0 = k0 - tap * p.Cp;
            const int rr = tap / p.S;
            const int ss = tap - rr * p.S;
            tma_load_im2col_4d(sA + s * kABytes, &tmA, &full_bar[s], c0, a_w, a_h, a_n,
                               (uint16_t)ss, (uint16_t)rr);
          }
          // B, then (blo_tma) its low part into the stage's B_lo slot
          for (int part = 0; part < (Cfg::kBloInStage && p.blo_tma ? 2 : 1); ++part) {
            const CUtensorMap* mb = part ? &tmBlo : &tmB;
            uint8_t* dst = sB + s * Cfg::kBStage + part * kBBytes;
            if (B_MN == 0) {
              tma_load_2d(dst, mb, &full_bar[s], kb * kBK, tn * BN);
            } else {
#pragma unroll
              for (int j = 0; j < BN / 32; ++j)
                tma_load_2d(dst + j * 4096, mb, &full_bar[s], tn * BN + j * 32, kb * kBK);
            }
          }
          if (++s == S) { s = 0; ph ^= 1; }
        }
      }
    }
  } else if (warp == Roles::kWarpMma) {
    // ------------------------------------------------------------ UMMA issuer
    // The whole warp walks the schedule (operands stay warp-uniform); lane 0
    // does the barrier waits, one elected lane issues each tcgen05 instruction.
    {
      auto warp_wait = [&](uint64_t* bar, uint32_t parity, int code) -> bool {
        int got = 0;
        if (lane == 0) got = mbar_wait_bounded(bar, parity, abort_flag, p.err, code, p.timeout_ns);
        return __shfl_sync(0xffffffffu, got, 0) != 0;
      };
      constexpr uint32_t idesc = umma_idesc_tf32(kBM, BN, 0, B_MN);
      constexpr uint32_t idesc_w = umma_idesc_tf32(kBM, Cfg::kWide ? 2 * BN : BN, 0, B_MN);
      int s = 0;
      uint32_t ph = 0;
      int g = 0;  // accumulation-unit counter (selects the TMEM partial buffer)
      int ja = 0;  // converted-k-block ring slot (3xTF32)
      uint32_t pa = 0;
      // Lane 0: the next k-block's ready barrier tested complete halfway
      // through this k-block's MMAs.  A wait on a complete barrier still costs
      // the MMA warp ~200 clocks of shared-memory latency in the loaded kernel
      // (B200 trace), which the test hides behind the MMA issue.
      int next_ready = 0;
      bool ok = true;
      for (int w = blockIdx.x; w < p.num_units && ok && !*abort_flag; w += gridDim.x) {
        const WorkUnit u = work_unit(p, w);
        const int tj = (w - (int)blockIdx.x) / (int)gridDim.x;
        for (int kb0 = u.kb0; kb0 < u.kb1 && ok; kb0 += p.kb_per_acc, ++g) {
          const int b = g & 1;
          const uint32_t use = (uint32_t)(g >> 1);
          if (!warp_wait(&tempty_bar[b], (use & 1) ^ 1, DEV_TIMEOUT_TMEM_EMPTY)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d_tmem = tmem_base + (uint32_t)(b * Cfg::kAccW);
          const int kend = (kb0 + p.kb_per_acc) < u.kb1 ? (kb0 + p.kb_per_acc) : u.kb1;
          for (int kb = kb0; kb < kend; ++kb) {
            uint64_t* ready = SPLIT ? &conv_bar[ja] : &full_bar[s];
            // the next k-block's barrier and phase (it follows this one in the
            // ring whatever unit or tile it belongs to; its previous phase was
            // waited for already and the one after needs this k-block's MMAs,
            // so the parity test cannot alias)
            const int jn = (ja + 1 == kAS) ? 0 : ja + 1;
            const int sn = (s + 1 == S) ? 0 : s + 1;
            uint64_t* ready_n = SPLIT ? &conv_bar[jn] : &full_bar[sn];
            const uint32_t par_n =
                SPLIT ? (ja + 1 == kAS ? pa ^ 1u : pa) : (s + 1 == S ? ph ^ 1u : ph);
            if (!__shfl_sync(0xffffffffu, next_ready, 0) &&
                !warp_wait(ready, SPLIT ? pa : ph, SPLIT ? DEV_TIMEOUT_CONV : DEV_TIMEOUT_FULL)) {
              ok = false;
              break;
            }
            next_ready = 0;
            if (lane == 0 && kb == u.kb0 && tj < kTraceTiles) trace_stamp(p, 3 + 6 * tj);
            tc_fence_after();
            // cp.async-gathered A (TF32 mode has no converter pass): make the
            // generic-proxy writes visible to the tensor core's async proxy.
            if (GATHER && !SPLIT) fence_proxy_async_smem();
            const uint32_t a_addr = smem_u32(sA + s * kABytes);
            const uint32_t b_addr = smem_u32(sB + s * Cfg::kBStage);
            const uint32_t blo_addr =
                Cfg::kBloInStage ? b_addr + (uint32_t)kBBytes : smem_u32(sBlo + ja * kBBytes);
            // 3xTF32: A's hi / lo k-block in TMEM columns (lane 0 = tile row 0)
            const uint32_t a_hi = tmem_base + (uint32_t)(Cfg::kAccCols + ja * 2 * kBK);
            const uint32_t a_lo = a_hi + (uint32_t)kBK;
#pragma unroll
            for (int k = 0; k < kBK / 8; ++k) {
              if (k == kBK / 8 - 1 && lane == 0) next_ready = mbar_test_wait(ready_n, par_n);
              // A (K-major, SW128): +32 B per 8-element k step inside the 128 B row.
              // B MN-major (SW128 with 32 B atoms): +1024 B = 8 K-rows per k step;
              // LBO = 4096 B between 32-column boxes, SBO = 512 B per 4 K-rows.
              const uint64_t db =
                  B_MN == 0 ? umma_desc(b_addr + k * 32, 16, 1024, kLayoutSW128)
                            : umma_desc(b_addr + k * 1024, 4096, 512, kLayoutSW128Base32B);
              const uint32_t acc = (kb > kb0 || k > 0) ? 1u : 0u;
              if (Cfg::kWide) {
                // one MMA of twice the tile width over [B | B_lo] (hi.hi and
                // hi.lo side by side), then lo.hi into the hi.hi columns
                umma_tf32_ts_e(d_tmem, a_hi + k * 8, db, idesc_w, acc);
                umma_tf32_ts_e(d_tmem, a_lo + k * 8, db, idesc, 1u);
              } else if (SPLIT) {
                const uint64_t dbl =
                    B_MN == 0 ? umma_desc(blo_addr + k * 32, 16, 1024, kLayoutSW128)
                              : umma_desc(blo_addr + k * 1024, 4096, 512, kLayoutSW128Base32B);
                // small cross terms first, then hi*hi; A from TMEM (8 columns per k step)
                umma_tf32_ts_e(d_tmem, a_hi + k * 8, dbl, idesc, acc);
                umma_tf32_ts_e(d_tmem, a_lo + k * 8, db, idesc, 1u);
                umma_tf32_ts_e(d_tmem, a_hi + k * 8, db, idesc, 1u);
              } else {
                const uint64_t da = umma_desc(a_addr + k * 32, 16, 1024, kLayoutSW128);
                umma_tf32_e(d_tmem, da, db, idesc, acc);
              }
            }
            // one commit frees the ring stage and (3xTF32) the TMEM A stage
            umma_commit_e(&empty_bar[s]);
            if (SPLIT) {
              if (++ja == kAS) { ja = 0; pa ^= 1; }
            }
            if (++s == S) { s = 0; ph ^= 1; }
          }
          if (!ok) break;
          umma_commit_e(&tfull_bar[b]);
          if (lane == 0 && kb0 + p.kb_per_acc >= u.kb1 && tj < kTraceTiles) trace_stamp(p, 4 + 6 * tj);
        }
      }
    }
  } else if (warp >= Roles::kWarpEpi && warp < Roles::kWarpEpi + 4) {
    // ------------------------------------------------------------ epilogue
    const int lane_base = 32 * (warp & 3);
    const int row = lane_base + lane;
    const uint32_t t_lane = tmem_base + ((uint32_t)lane_base << 16);
    const uint32_t t_run = t_lane + (uint32_t)(2 * Cfg::kAccW);  // fp32 running sum (3xTF32)
    const int et = threadIdx.x - Roles::kWarpEpi * 32;  // 0..127 within the epilogue group
    int chunk = 0;  // staging-buffer sequence number
    int g = 0;
    bool ok = true;
    // One finished 128 x 32 chunk (this thread's row, columns n0..n0+31) to C.
    auto emit = [&](int tm, int tn, int c, int m, const uint32_t (&r)[32]) {
      const int n0 = tn * BN + c;
      const uint32_t sb = smem_u32(sBias) + 4 * c;
      if (p.c_tma) {
        uint8_t* stg = sOut + (chunk % Cfg::kOutBufs) * kOutChunkBytes;
        epilogue_stage_rowmajor(p, smem_u32(stg), row, n0, m, r, sb);
        fence_proxy_async_smem();
        named_bar_sync(1, 128);
        if (et == 0) {
          tma_store_2d(&tmC, stg, n0, tm * kBM);
          bulk_commit_group();
          // the buffer used next is free again
          bulk_wait_group_read<Cfg::kOutBufs - 1>();
        }
        named_bar_sync(1, 128);
        ++chunk;
      } else if (p.out_mode == 1) {
        const uint32_t buf = smem_u32(sOut + (chunk % Cfg::kOutBufs) * kOutChunkBytes);
        epilogue_nchw_chunk(p, buf, row, et, tm * kBM, n0, r, sb);
        if (Cfg::kOutBufs == 1) named_bar_sync(1, 128);  // single buffer: readers done first
        ++chunk;
      } else if (p.out_mode == 2) {
        const uint32_t buf = smem_u32(sOut + (chunk % Cfg::kOutBufs) * kOutChunkBytes);
        epilogue_stage_rowmajor(p, buf, row, n0, m, r, sb);
        named_bar_sync(1, 128);
        epilogue_store_peers(p, buf, et, tm * kBM, n0);
        named_bar_sync(1, 128);
        ++chunk;
      } else {
        epilogue_store32(p, m, n0, r, sb);
      }
    };
    // Split-tile fix-up: the sum of the tile's split_k partials (in piece
    // order, so the result does not depend on arrival order) goes through the
    // epilogue like a finished tile.
    constexpr int kFixRoom = S * Cfg::kStageBytes;
    const bool fix_room = 2 * p.split_k * kOutChunkBytes <= kFixRoom;
    // Staged: each thread copies its own row of every piece by cp.async into
    // the idle load ring (one L2 round trip per chunk, the next chunk in
    // flight while this one is summed).  `restage_bias`: the tile is not the
    // one whose bias is in sBias (a queued tile).
    auto fix_staged = [&](int tile, int slot, bool restage_bias) {
      int tm, tn;
      tile_coords(tile, p.tiles_m, p.tiles_n, p.group_m, tm, tn);
      const int m = tm * kBM + row;
      if (restage_bias && p.bias) {
        named_bar_sync(1, 128);
        for (int i = et; i < BN; i += 128) {
          const int n = tn * BN + i;
          sts32(smem_u32(sBias) + 4 * i, n < p.N ? __ldg(p.bias + n) : 0.0f);
        }
        named_bar_sync(1, 128);
      }
      __threadfence();
      const float4* src0 =
          reinterpret_cast<const float4*>(p.ws) + (size_t)slot * p.split_k * (size_t)(BN * kBM / 4);
      const int SK = p.split_k;
      const uint32_t fb = smem_u32(sA);
      auto stage_chunk = [&](int ci) {  // chunk ci of every piece -> buffer ci & 1
        const float4* s0 = src0 + (size_t)ci * 8 * kBM + row;
        const uint32_t d0 = fb + (uint32_t)((ci & 1) * SK * kOutChunkBytes) + row * 16;
#pragma unroll 1
        for (int pc = 0; pc < SK; ++pc) {
#pragma unroll
          for (int j = 0; j < 8; ++j)
            cp_async_16_cg(d0 + (uint32_t)((pc * 8 + j) * kBM * 16),
                           s0 + (size_t)pc * (BN * kBM / 4) + j * kBM);
        }
        cp_async_commit();
      };
      stage_chunk(0);
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        const int ci = c / 32;
        if (c + 32 < BN) {
          stage_chunk(ci + 1);
          cp_async_wait<1>();
        } else {
          cp_async_wait<0>();
        }
        const uint32_t d0 = fb + (uint32_t)((ci & 1) * SK * kOutChunkBytes) + row * 16;
        float v[32];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float4 q = lds128(d0 + (uint32_t)(j * kBM * 16));
          v[4 * j] = q.x; v[4 * j + 1] = q.y; v[4 * j + 2] = q.z; v[4 * j + 3] = q.w;
        }
#pragma unroll 1
        for (int pc = 1; pc < SK; ++pc) {
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float4 q = lds128(d0 + (uint32_t)((pc * 8 + j) * kBM * 16));
            v[4 * j] += q.x; v[4 * j + 1] += q.y; v[4 * j + 2] += q.z; v[4 * j + 3] += q.w;
          }
        }
        uint32_t r[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) r[j] = __float_as_uint(v[j]);
        emit(tm, tn, c, m, r);
      }
    };
    // Straight from L2 (the ring is busy, or too small for every piece): the
    // next piece's loads are issued before the current one is added.
    auto fix_direct = [&](int tile, int slot) {
      int tm, tn;
      tile_coords(tile, p.tiles_m, p.tiles_n, p.group_m, tm, tn);
      const int m = tm * kBM + row;
      __threadfence();
      const float4* src0 =
          reinterpret_cast<const float4*>(p.ws) + (size_t)slot * p.split_k * (size_t)(BN * kBM / 4);
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        const float4* s0 = src0 + (size_t)(c / 32) * 8 * kBM + row;
        float v[32];
        float4 q[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) q[j] = __ldcg(s0 + j * kBM);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          v[4 * j] = q[j].x; v[4 * j + 1] = q[j].y; v[4 * j + 2] = q[j].z; v[4 * j + 3] = q[j].w;
        }
        if (p.split_k > 1) {
#pragma unroll
          for (int j = 0; j < 8; ++j) q[j] = __ldcg(s0 + (size_t)(BN * kBM / 4) + j * kBM);
        }
#pragma unroll 1
        for (int pc = 1; pc < p.split_k; ++pc) {
          float4 nq[8];
          if (pc + 1 < p.split_k) {
            const float4* sp = s0 + (size_t)(pc + 1) * (BN * kBM / 4);
#pragma unroll
            for (int j = 0; j < 8; ++j) nq[j] = __ldcg(sp + j * kBM);
          }
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            v[4 * j] += q[j].x; v[4 * j + 1] += q[j].y; v[4 * j + 2] += q[j].z;
            v[4 * j + 3] += q[j].w;
          }
          if (pc + 1 < p.split_k) {
#pragma unroll
            for (int j = 0; j < 8; ++j) q[j] = nq[j];
          }
        }
        uint32_t r[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) r[j] = __float_as_uint(v[j]);
        emit(tm, tn, c, m, r);
      }
    };
    for (int w = blockIdx.x; w < p.num_units && ok; w += gridDim.x) {
      const WorkUnit u = work_unit(p, w);
      const int tj = (w - (int)blockIdx.x) / (int)gridDim.x;
      int tm, tn;
      tile_coords(u.tile, p.tiles_m, p.tiles_n, p.group_m, tm, tn);
      const int m = tm * kBM + row;
      const bool piece = u.piece >= 0;
      // this piece's partial tile in the workspace, as float4 [BN/32][8][128]
      float4* wsp = piece ? reinterpret_cast<float4*>(p.ws) +
                                ((size_t)u.slot * p.split_k + u.piece) * (size_t)(BN * kBM / 4)
                          : nullptr;
      const int units = (u.kb1 - u.kb0 + p.kb_per_acc - 1) / p.kb_per_acc;
      if (p.bias) {
        // Stage the tile's bias once (the loads overlap the mainloop); the
        // barrier keeps the previous tile's readers ahead of the overwrite,
        // the vote barriers below publish the values.
        named_bar_sync(2, 128);
        for (int i = et; i < BN; i += 128) {
          const int n = tn * BN + i;
          sts32(smem_u32(sBias) + 4 * i, n < p.N ? __ldg(p.bias + n) : 0.0f);
        }
      }
      for (int a = 0; a < units; ++a, ++g) {
        const int b = g & 1;
        const uint32_t use = (uint32_t)(g >> 1);
        // tcgen05.ld is .sync.aligned and the staged stores meet at named
        // barriers: all four warps take the same branch (vote through smem).
        if (lane == 0)
          epi_vote[warp & 3] = mbar_wait_bounded(&tfull_bar[b], use & 1, abort_flag, p.err,
                                                 DEV_TIMEOUT_TMEM_FULL, p.timeout_ns);
        named_bar_sync(2, 128);
        const bool got = epi_vote[0] && epi_vote[1] && epi_vote[2] && epi_vote[3];
        named_bar_sync(2, 128);
        if (!got) {
          ok = false;
          break;
        }
        tc_fence_after();
        const bool last = (a + 1 == units);
        if (warp == Roles::kWarpEpi && lane == 0 && tj < kTraceTiles) {
          if (a == 0) trace_stamp(p, 5 + 6 * tj);
          if (last) trace_stamp(p, 6 + 6 * tj);
        }
        const uint32_t t_part = t_lane + (uint32_t)(b * Cfg::kAccW);
        // the last unit leaves without the running-sum round trip through
        // TMEM when holding the accumulator during the stores costs nothing;
        // otherwise (single-unit tiles too) the partial moves to the running
        // sum and is released before any store: the stem's 8-k-block tiles
        // waited ~2800 clocks per tile for a partial held through a chunk's
        // stores
        const bool emit_now = last && (piece || w + (int)gridDim.x >= p.num_units);
        const bool via_run = SPLIT && !emit_now;
        // One finished chunk: a split piece's partial to the workspace, else to C.
        auto out = [&](int c, const uint32_t (&r)[32]) {
          if (piece) {
            float4* dst = wsp + (size_t)(c / 32) * 8 * kBM + row;
#pragma unroll
            for (int j = 0; j < 8; ++j)
              __stcg(dst + j * kBM, make_float4(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]),
                                                __uint_as_float(r[4 * j + 2]),
                                                __uint_as_float(r[4 * j + 3])));
          } else {
            emit(tm, tn, c, m, r);
          }
        };
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
          // the chunk's partial reads (and its hi.lo half) are issued together
          // and waited for once; the running sum's after the partial is free
          uint32_t r[32], q[32];
          tmem_ld_32x32b_x32(t_part + (uint32_t)c, r);
          if (Cfg::kWide) tmem_ld_32x32b_x32(t_part + (uint32_t)(BN + c), q);
          tmem_ld_wait();
          if (c + 32 == BN) {
            tc_fence_before();
            mbar_arrive(&tempty_bar[b]);  // partial buffer b may be overwritten now
          }
          if (Cfg::kWide) {  // + the hi.lo half
#pragma unroll
            for (int j = 0; j < 32; ++j)
              r[j] = __float_as_uint(__uint_as_float(r[j]) + __uint_as_float(q[j]));
          }
          if (SPLIT && a > 0) {
            tmem_ld_32x32b_x32(t_run + (uint32_t)c, q);
            tmem_ld_wait();
#pragma unroll
            for (int j = 0; j < 32; ++j)
              r[j] = __float_as_uint(__uint_as_float(r[j]) + __uint_as_float(q[j]));
          }
          if (via_run) {
            // running sum; after the last unit the finished tile, which leaves
            // from there so the accumulator is not held during the stores
            tmem_st_32x32b_x32(t_run + (uint32_t)c, r);
          } else {
            // straight from the partial (+ running sum): a tile (or piece) of
            // one unit, a piece (its partial goes to L2 fast), and the CTA's
            // last tile (no later tile waits for the accumulator)
            out(c, r);
          }
        }
        if (via_run) tmem_st_wait();
        if (via_run && last) {
#pragma unroll 1
          for (int c = 0; c < BN; c += 32) {
            uint32_t r[32];
            tmem_ld_32x32b_x32(t_run + (uint32_t)c, r);
            tmem_ld_wait();
            out(c, r);
          }
        }
      }
      if (ok && piece) {
        // Publish this piece, count arrivals; the last piece's CTA sums all of
        // them: at once when this piece is its last work unit (the ring is
        // idle: no more loads are issued and the MMAs that read it have
        // completed) or when there is no room to stage; otherwise the tile is
        // queued and summed after the CTA's last unit, through the idle ring.
        __threadfence();
        named_bar_sync(1, 128);
        if (et == 0) {
          const int arrived = tagged_arrive(p.ws_cnt + u.slot, p.cnt_gen);
          if (arrived < 0) {
            atomicCAS(p.err, 0, (int)DEV_BAD_CONFIG);
            *abort_flag = 1;
          }
          int mode = 0;  // 0 nothing, 1 sum now (staged), 2 queued, 3 sum now (from L2)
          if (arrived == p.split_k - 1) {
            const bool ring_idle = w + (int)gridDim.x >= p.num_units;
            if (!fix_room) mode = 3;
            else if (ring_idle) mode = 1;
            else if (pend[0] < kMaxPending) mode = 2;
            else mode = 3;
            if (mode == 2) {
              const int q = pend[0];
              pend[1 + 2 * q] = u.tile;
              pend[2 + 2 * q] = u.slot;
              pend[0] = q + 1;
            }
          }
          *fix_flag = mode;
        }
        named_bar_sync(1, 128);
        const int mode = *fix_flag;
        if (mode == 1) fix_staged(u.tile, u.slot, false);
        else if (mode == 3) fix_direct(u.tile, u.slot);
      }
      if (ok && warp == Roles::kWarpEpi && lane == 0 && tj < kTraceTiles)
        trace_stamp(p, 7 + 6 * tj);
    }
    if (ok) {  // queued split tiles, now that the ring is idle
      const int np = pend[0];
      for (int i = 0; i < np; ++i) fix_staged(pend[1 + 2 * i], pend[2 + 2 * i], true);
    }
    if (p.c_tma && et == 0) bulk_wait_group<0>();  // all output stores complete
    // peer stores are ordered before anything that follows the kernel on the
    // stream (the cross-rank barrier after an N-split GEMM)
    if (p.out_mode == 2) __threadfence_system();
  } else if (SPLIT && warp >= Roles::kWarpConv && warp < Roles::kWarpConv + 4) {
    // ------------------------------------------------------------ converters
    // Per k-block: thread = tile row (TMEM lane 32*(warp%4)+lane).  The A row
    // (32 fp32, 128B-swizzled in smem) becomes hi = trunc_tf32(x) and
    // lo = x - hi, stored as two 32-column blocks of the TMEM A stage; the B
    // tile's low part goes to its smem plane (its hi part is the raw tile,
    // truncated by the tensor core).
    const int ct = threadIdx.x - Roles::kWarpConv * 32;  // 0..127
    const int lane_base = 32 * (warp & 3);
    const int row = lane_base + lane;
    const uint32_t t_lane = tmem_base + ((uint32_t)lane_base << 16);
    int s = 0;
    uint32_t ph = 0;
    int ja = 0;
    int q = 0;           // k-block sequence number
    int s_rel = 0;       // ring stage and phase parity of k-block q - kAS, whose
    uint32_t ph_rel = 0; // MMAs (one commit) also free TMEM A stage ja
    const bool b_conv = !(Cfg::kBloInStage && p.blo_tma);  // this warp group makes B_lo
    bool ok = true;
    for (int w = blockIdx.x; w < p.num_units && ok && !*abort_flag; w += gridDim.x) {
      const WorkUnit u = work_unit(p, w);
      for (int kb = u.kb0; kb < u.kb1; ++kb, ++q) {
        // every lane waits (acquire for its own smem reads); tcgen05.st is
        // .sync.aligned, so the warp proceeds only if all lanes got through
        bool got = mbar_wait_bounded_sleep(&full_bar[s], ph, abort_flag, p.err,
                                           DEV_TIMEOUT_LOADED, p.timeout_ns, kConvSleepNs);
        if (q >= kAS)
          got = got && mbar_wait_bounded_sleep(&empty_bar[s_rel], ph_rel, abort_flag, p.err,
                                               DEV_TIMEOUT_TMEM_A, p.timeout_ns, kConvSleepNs);
        if (!__all_sync(0xffffffffu, got)) {
          ok = false;
          break;
        }
        tc_fence_after();
        // All shared-memory loads first (A row and this thread's share of B),
        // then the splits, so the converter's latency is one load round trip.
        constexpr int kBPer = kBBytes / 16 / 128;  // float4 of B per thread
        const uint32_t arow = smem_u32(sA + s * kABytes + row * 128);
        const uint32_t bb = smem_u32(sB + s * Cfg::kBStage);
        const uint32_t blo =
            Cfg::kBloInStage ? bb + (uint32_t)kBBytes : smem_u32(sBlo + ja * kBBytes);
        float4 av[8], bv[kBPer];
        if (MULTITAP) {
          // float4 q of the row = channels 4*qq.. of tap block j (dense rows of
          // Cp floats); k-block columns past K = R*S*Cp are zero
          // rows of Cp = 8 / 16 channels arrive with the 32 / 64-byte TMA
          // swizzle: 16-byte chunk c of row r sits at c ^ ((r * Cp * 4) >> 7)
          // within the row (address bits 4-5 XOR bits 7-8)
          const int l = p.Cp == 4 ? 0 : (p.Cp == 8 ? 1 : 2);  // log2(Cp / 4)
          const int mask = (1 << l) - 1;
          const int swz = ((row * p.Cp * 4) >> 7) & mask;
          const uint32_t a0 = smem_u32(sA + s * kABytes) + row * p.Cp * 4;
          const int kvalid = p.R * p.S * p.Cp - kb * kBK;
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            av[q] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (4 * q < kvalid)
              av[q] = lds128(a0 + (q >> l) * (kBM * p.Cp * 4) + (((q & mask) ^ swz) << 4));
          }
        } else if (A_MODE == 4) {
          // MN-major tile: k-row k is 512 bytes (128 m values); this thread's
          // row is one float of each, so a warp reads one 128-byte line per k
          const uint32_t a0 = smem_u32(sA + s * kABytes) + row * 4;
#pragma unroll
          for (int j = 0; j < 8; ++j)
            av[j] = make_float4(lds32(a0 + (4 * j) * 512), lds32(a0 + (4 * j + 1) * 512),
                                lds32(a0 + (4 * j + 2) * 512), lds32(a0 + (4 * j + 3) * 512));
        } else {
#pragma unroll
          for (int j = 0; j < 8; ++j) av[j] = lds128(arow + ((j ^ (row & 7)) << 4));
        }
        if (b_conv) {
#pragma unroll
          for (int i = 0; i < kBPer; ++i) bv[i] = lds128(bb + (ct + 128 * i) * 16);
        }
        uint32_t hi[32], lo[32];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float x[4] = {av[j].x, av[j].y, av[j].z, av[j].w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            uint32_t h;
            if (p.split_trunc) {
              h = __float_as_uint(x[e]) & 0xFFFFE000u;
            } else {
              asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(h) : "f"(x[e]));
            }
            hi[4 * j + e] = h;
            lo[4 * j + e] = __float_as_uint(x[e] - __uint_as_float(h));
          }
        }
        const uint32_t t_a = t_lane + (uint32_t)(Cfg::kAccCols + ja * 2 * kBK);
        tmem_st_32x32b_x32(t_a, hi);
        tmem_st_32x32b_x32(t_a + (uint32_t)kBK, lo);
        if (!b_conv) {
        } else if (p.split_trunc) {
#pragma unroll
          for (int i = 0; i < kBPer; ++i) sts128(blo + (ct + 128 * i) * 16, tf32_trunc_rem4(bv[i]));
        } else {
#pragma unroll
          for (int i = 0; i < kBPer; ++i) {
            const float4 h = tf32_hi4(bv[i]);
            sts128(bb + (ct + 128 * i) * 16, h);
            sts128(blo + (ct + 128 * i) * 16,
                   make_float4(bv[i].x - h.x, bv[i].y - h.y, bv[i].z - h.z, bv[i].w - h.w));
          }
        }
        fence_proxy_async_smem();
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(&conv_bar[ja]);
        if (++s == S) { s = 0; ph ^= 1; }
        if (++ja == kAS) ja = 0;
        if (q >= kAS && ++s_rel == S) { s_rel = 0; ph_rel ^= 1; }
      }
    }
  } else if (GATHER && warp >= Roles::kWarpGather && warp < Roles::kWarpGather + 4) {
    // ------------------------------------------------------------ im2col gather
    // Each thread owns one row (output pixel) of the A tile: 8 x 16-byte
    // cp.async per k-block into the swizzled row, then an asynchronous
    // arrive on the stage's full barrier when its copies land.
    const int r = threadIdx.x - Roles::kWarpGather * 32;  // tile row 0..127
    const int swz = r & 7;
    const int Ktot = p.R * p.S * p.Cp;
    const int HoWo = p.Ho * p.Wo;
    int s = 0;
    uint32_t ph = 0;
    bool ok = true;
    for (int w = blockIdx.x; w < p.num_units && ok && !*abort_flag; w += gridDim.x) {
      const WorkUnit u = work_unit(p, w);
      int tm, tn;
      tile_coords(u.tile, p.tiles_m, p.tiles_n, p.group_m, tm, tn);
      const int m = tm * kBM + r;
      const bool mvalid = m < p.M;
      const int img = mvalid ? m / HoWo : 0;
      const int rem = mvalid ? m - img * HoWo : 0;
      const int oh = rem / p.Wo;
      const int ow = rem - oh * p.Wo;
      const int ih0 = oh * p.sh - p.ph;
      const int iw0 = ow * p.sw - p.pw;
      const float* ximg = p.x + (int64_t)img * p.H * p.W * p.Cp;
      // (tap, channel) of the first 16-byte chunk of the k-block, advanced
      // incrementally (Cp % 4 == 0, so a chunk never straddles a tap).
      int tap = (u.kb0 * kBK) / p.Cp;
      int ci = u.kb0 * kBK - tap * p.Cp;
      for (int kb = u.kb0; kb < u.kb1; ++kb) {
        if (!mbar_wait_bounded(&empty_bar[s], ph ^ 1, abort_flag, p.err, DEV_TIMEOUT_EMPTY,
                               p.timeout_ns)) {
          ok = false;
          break;
        }
        uint8_t* dst_row = sA + s * kABytes + r * 128;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const int k = kb * kBK + c * 4;
          const int rr = tap / p.S;
          const int ss = tap - rr * p.S;
          const int ih = ih0 + rr, iw = iw0 + ss;
          const bool v = mvalid && k < Ktot && ih >= 0 && ih < p.H && iw >= 0 && iw < p.W;
          const float* src = v ? ximg + ((int64_t)ih * p.W + iw) * p.Cp + ci : p.x;
          cp_async_16(dst_row + ((c ^ swz) << 4), src, v ? 16u : 0u);
          ci += 4;
          if (ci == p.Cp) { ci = 0; ++tap; }
        }
        cp_async_mbar_arrive_noinc(&full_bar[s]);
        if (++s == S) { s = 0; ph ^= 1; }
      }
    }
    cp_async_wait<0>();
  }

  // ------------------------------------------------------------ teardown
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (*abort_flag) {
    // Give in-flight TMA / cp.async copies time to land before the CTA's
    // shared memory is released (bounded: ~1 ms).
    const uint64_t t0 = globaltimer_ns();
    while (globaltimer_ns() - t0 < 1000000ull) __nanosleep(1000);
    __syncthreads();
  }
  if (warp == Roles::kWarpMma) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::kTmemCols);
  }
  if (threadIdx.x == 0) trace_stamp(p, 1);
}

}  // namespace rtb
