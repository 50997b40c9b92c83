// Gated-DeltaNet decode-row glue (the reference's MOE_CUDA_GDN_GLUE kernels, gdn_cuda.py:102-268).
//
// step_glue_kernel: NR positions of one sequence from the causal conv's output (before silu), for one value head a
// block: silu of the conv output, the q / k RMSNorm (eps = 1e-6 / Dk, then scaled by Dk^-1 / Dk^-0.5 -- the
// normalize_qk of qwen4_exp_vendor.py:471-473), sigmoid(b), g = exp(-exp(A_log) * softplus(a + dt_bias)) and one
// recurrence step per position, the state of the block's value rows held in registers across the NR positions.
// The 16-bit rounding points follow the reference's kernel: silu and the normalised q / k are rounded to the
// activation dtype before use.
// norm_gate_kernel: Qwen3NextRMSNormGated, w * rms_norm(x) then * silu(z) (gdn_cuda.py:200-222): one warp a row.
#pragma once

#include "common.cuh"

namespace lb2 {
namespace glue {

template <typename T>
__device__ __forceinline__ T silu_t(T x) {
  const float xf = to_f<T>(x);
  const T sg = from_f<T>(1.f / (1.f + __expf(-xf)));
  return from_f<T>(xf * to_f<T>(sg));
}

struct StepParams {
  const void* conv;  // [NR, 2 Hk Dk + Hv Dv], activation dtype
  const void* a;     // [NR, Hv] activation dtype
  const void* b;     // [NR, Hv] activation dtype
  const float* A_log;    // [Hv]
  const float* dt_bias;  // [Hv]
  const float* s_in;     // [Hv, Dv, Dk]
  float* s_out;
  void* y;  // [NR, Hv, Dv] activation dtype
  int NR, Hk, Hv, Dv;
  float sq, sk, eps;
};

// A block: RB value rows of one value head over NR positions in order; Dk = 32 * NPT.
template <typename T, int NPT, int RB>
__global__ void __launch_bounds__(RB * 32) step_glue_kernel(const StepParams p) {
  constexpr int DK = 32 * NPT;
  __shared__ T sv[2 * DK];
  __shared__ float qk[2 * DK];
  __shared__ float nrm[2], gb[2];
  const int hv = blockIdx.y;
  const int hk = hv / (p.Hv / p.Hk);
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int t = threadIdx.x;
  const int dv = blockIdx.x * RB + w;
  const bool live = dv < p.Dv;
  const int CD = 2 * p.Hk * DK + p.Hv * p.Dv;
  const T* conv = static_cast<const T*>(p.conv);
  const T* av = static_cast<const T*>(p.a);
  const T* bv = static_cast<const T*>(p.b);
  T* yv = static_cast<T*>(p.y);
  float s[NPT];
  const int64_t so = ((int64_t)hv * p.Dv + (live ? dv : 0)) * DK + lane * NPT;
#pragma unroll
  for (int i = 0; i < NPT; ++i) s[i] = live ? p.s_in[so + i] : 0.f;
  for (int r = 0; r < p.NR; ++r) {
    const T* cv = conv + (int64_t)r * CD;
    for (int e = t; e < 2 * DK; e += RB * 32)
      sv[e] = silu_t(cv[(e < DK ? hk : p.Hk + hk) * DK + (e % DK)]);
    if (t == 0) {
      const float bf = to_f<T>(bv[r * p.Hv + hv]);
      gb[1] = to_f<T>(from_f<T>(1.f / (1.f + __expf(-bf))));
      const float x = to_f<T>(av[r * p.Hv + hv]) + p.dt_bias[hv];
      const float sp = x > 20.f ? x : log1pf(__expf(x));
      gb[0] = __expf(-__expf(p.A_log[hv]) * sp);
    }
    __syncthreads();
    if (w < 2) {  // rms of q (warp 0) and k (warp 1)
      float n = 0.f;
      for (int e = lane; e < DK; e += 32) {
        const float x = to_f<T>(sv[w * DK + e]);
        n = fmaf(x, x, n);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) n += __shfl_xor_sync(0xffffffffu, n, o);
      if (lane == 0) nrm[w] = rsqrtf(n / DK + p.eps);
    }
    __syncthreads();
    for (int e = t; e < 2 * DK; e += RB * 32) {
      const T yn = from_f<T>(to_f<T>(sv[e]) * nrm[e < DK ? 0 : 1]);
      qk[e] = to_f<T>(from_f<T>(to_f<T>(yn) * (e < DK ? p.sq : p.sk)));
    }
    __syncthreads();
    if (live) {
      float qf[NPT], kf[NPT];
#pragma unroll
      for (int i = 0; i < NPT; ++i) {
        qf[i] = qk[lane * NPT + i];
        kf[i] = qk[DK + lane * NPT + i];
      }
      const float vf = to_f<T>(silu_t(cv[2 * p.Hk * DK + hv * p.Dv + dv]));
      const float gf = gb[0], bf = gb[1];
      float kv = 0.f;
#pragma unroll
      for (int i = 0; i < NPT; ++i) {
        s[i] = s[i] * gf;
        kv = fmaf(s[i], kf[i], kv);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) kv += __shfl_xor_sync(0xffffffffu, kv, o);
      const float delta = (vf - kv) * bf;
      float out = 0.f;
#pragma unroll
      for (int i = 0; i < NPT; ++i) {
        s[i] = fmaf(kf[i], delta, s[i]);
        out = fmaf(s[i], qf[i], out);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) out += __shfl_xor_sync(0xffffffffu, out, o);
      if (lane == 0) yv[((int64_t)r * p.Hv + hv) * p.Dv + dv] = from_f<T>(out);
    }
    __syncthreads();  // the next position rewrites sv, qk, nrm and gb
  }
  if (live)
#pragma unroll
    for (int i = 0; i < NPT; ++i) p.s_out[so + i] = s[i];
}

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
