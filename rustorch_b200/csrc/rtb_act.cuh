// Epilogue activations shared by every kernel that ends in one: the
// reference's Activation enum (rustorch-core/src/backend/mod.rs:1-7) as
// applied by matmul_fused's staged path (rustorch-core/src/ops.rs:1703-1708):
//   RTB_ACT_RELU     f32::max(x, 0)       (ops.rs:449-491; NaN -> 0)
//   RTB_ACT_SIGMOID  1 / (1 + exp(-x))    (ops/activations.rs:47-50)
//   RTB_ACT_TANH     tanh(x)              (ops/activations.rs:213)
// exp and tanh are CUDA's expf / tanhf (their documented error bounds are a
// few ulp; the GPU tests hold the results to the f64 values).
#pragma once
#include "../../include/rustorch_b200.h"

namespace rtb {

__device__ __forceinline__ float activate(float y, int act) {
  if (act == RTB_ACT_RELU) return fmaxf(y, 0.0f);  // NaN -> 0, as f32::max
  if (act == RTB_ACT_SIGMOID) return 1.0f / (1.0f + expf(-y));
  if (act == RTB_ACT_TANH) return tanhf(y);
  return y;
}

// The activation over an array held in registers; the selection is made once
// for the whole array.
template <int N>
__device__ __forceinline__ void activate_n(float (&v)[N], int act) {
  if (act == RTB_ACT_RELU) {
#pragma unroll
    for (int j = 0; j < N; ++j) v[j] = fmaxf(v[j], 0.0f);
  } else if (act == RTB_ACT_SIGMOID) {
#pragma unroll
    for (int j = 0; j < N; ++j) v[j] = 1.0f / (1.0f + expf(-v[j]));
  } else if (act == RTB_ACT_TANH) {
#pragma unroll
    for (int j = 0; j < N; ++j) v[j] = tanhf(v[j]);
  }
}

__device__ __forceinline__ float4 activate4(float4 v, int act) {
  float a[4] = {v.x, v.y, v.z, v.w};
  activate_n<4>(a, act);
  return make_float4(a[0], a[1], a[2], a[3]);
}

}  // namespace rtb
