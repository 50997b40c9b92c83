// Gated-DeltaNet decode-row glue: the gated RMSNorm after the recurrence (the decode row's recurrence with its own glue
// is gdnrec::glue_step_kernel in gdn_recurrent.cuh).
//
// norm_gate_kernel: Qwen3NextRMSNormGated, w * rms_norm(x) then * silu(z) (gdn_cuda.py:200-222): one warp a row.
#pragma once

#include "common.cuh"

namespace lb2 {
namespace glue {

template <typename T>
__global__ void __launch_bounds__(128) norm_gate_kernel(const T* x, const T* z, const T* wt, T* out, int64_t R, int D,
                                                        float eps) {
  const int64_t row = int64_t(blockIdx.x) * 4 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= R) return;
  const T* xr = x + row * D;
  float ns = 0.f;
  for (int e = lane; e < D; e += 32) {
    const float v = to_f<T>(xr[e]);
    ns = fmaf(v, v, ns);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ns += __shfl_xor_sync(0xffffffffu, ns, o);
  ns = rsqrtf(ns / D + eps);
  for (int e = lane; e < D; e += 32) {
    const T n = from_f<T>(to_f<T>(wt[e]) * to_f<T>(from_f<T>(to_f<T>(xr[e]) * ns)));
    const float gz = to_f<T>(z[row * D + e]);
    const float gs = gz * (1.f / (1.f + __expf(-gz)));
    out[row * D + e] = from_f<T>(gs * to_f<T>(n));
  }
}

}  // namespace glue
}  // namespace lb2
