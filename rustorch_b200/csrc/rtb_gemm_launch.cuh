// Kernel-variant dispatch of the tcgen05 GEMM engine: the template behind the
// per-tile-width translation units rtb_gemm_bn{64,128,256}.cu.
#pragma once
#include "rtb_gemm.cuh"
#include "rtb_internal.h"

namespace rtb {

template <int BN, bool SPLIT, int A_MODE, int B_MN>
int launch_variant(rtb_ctx* ctx, const CUtensorMap& tmA, const CUtensorMap& tmB,
                   const CUtensorMap& tmBlo, const CUtensorMap& tmC, const GemmParams& p,
                   cudaStream_t stream) {
  using Cfg = GemmCfgFor<BN, SPLIT, A_MODE>;
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
                 tmB, tmBlo, tmC, p);
  if (e != cudaSuccess) return cuda_status(e, "gemm kernel launch");
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_status(e, "gemm kernel launch");
  return RTB_OK;
}

template <int BN, bool SPLIT>
int launch_prec(rtb_ctx* ctx, const CUtensorMap& tmA, const CUtensorMap& tmB,
                const CUtensorMap& tmBlo, const CUtensorMap& tmC, const GemmParams& p,
                const GemmDesc& d, cudaStream_t s) {
  if (d.gather == 1) return launch_variant<BN, SPLIT, 1, 0>(ctx, tmA, tmB, tmBlo, tmC, p, s);
  if (d.gather == 2) return launch_variant<BN, SPLIT, 2, 0>(ctx, tmA, tmB, tmBlo, tmC, p, s);
  if (d.gather == 3) {
    if constexpr (SPLIT) return launch_variant<BN, SPLIT, 3, 0>(ctx, tmA, tmB, tmBlo, tmC, p, s);
    else return set_error(RTB_E_INVALID, "multi-tap im2col needs the 3xTF32 converters");
  }
  if (d.a_mn_major) {
    if constexpr (SPLIT) {
      if (d.b_mn_major) return set_error(RTB_E_INVALID, "MN-major A takes a K-major B");
      return launch_variant<BN, SPLIT, 4, 0>(ctx, tmA, tmB, tmBlo, tmC, p, s);
    } else {
      return set_error(RTB_E_INVALID, "MN-major A tiles need the 3xTF32 converters");
    }
  }
  if (d.b_mn_major) return launch_variant<BN, SPLIT, 0, 1>(ctx, tmA, tmB, tmBlo, tmC, p, s);
  return launch_variant<BN, SPLIT, 0, 0>(ctx, tmA, tmB, tmBlo, tmC, p, s);
}

template <int BN>
int launch_bn(rtb_ctx* ctx, const CUtensorMap& tmA, const CUtensorMap& tmB,
              const CUtensorMap& tmBlo, const CUtensorMap& tmC, const GemmParams& p,
              const GemmDesc& d, cudaStream_t s) {
  if (!d.split3) return launch_prec<BN, false>(ctx, tmA, tmB, tmBlo, tmC, p, d, s);
  if constexpr (BN <= 128) {
    return launch_prec<BN, true>(ctx, tmA, tmB, tmBlo, tmC, p, d, s);
  } else {
    return set_error(RTB_E_INVALID, "3xTF32 tiles are at most 128 columns wide");
  }
}

}  // namespace rtb
