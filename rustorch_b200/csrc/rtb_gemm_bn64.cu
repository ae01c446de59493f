// The tcgen05 GEMM engine's 64-column tile variants (every producer mode,
// B layout and precision), instantiated in their own translation unit.
#include "rtb_gemm_launch.cuh"

namespace rtb {

template int launch_bn<64>(rtb_ctx*, const CUtensorMap&, const CUtensorMap&, const CUtensorMap&,
                           const CUtensorMap&, const GemmParams&, const GemmDesc&, cudaStream_t);

}  // namespace rtb
