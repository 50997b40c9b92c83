// Gated-DeltaNet recurrence, position by position (decode steps and short passes).
//
// One warp per (sequence b, value head hv, value row dv), lane l holding state[dv][l*NPT, (l+1)*NPT) in fp32
// registers, as the reference's CUDA recurrence lays it out (gdn_cuda.py:18-66); per position:
//   s <- s * g; kv = sum(s * k); delta = (v[dv] - kv) * beta; s <- s + k * delta; y[dv] = sum(s * q).
// Consecutive warps take consecutive value rows of one head, so a block's state rows are one contiguous stretch
// of HBM and its q / k loads are shared through L1. For a decode step (T = 1) the kernel is a streaming pass over
// the state: read and written once, Dv * Dk * 8 bytes per (b, hv).
#pragma once

#include "common.cuh"

namespace lb2 {
namespace gdnrec {

struct Params {
  const void* q;
  const void* k;
  const void* v;
  const void* g;
  const void* beta;
  const uint8_t* mask;
  const float* s_in;
  float* s_out;
  void* y;
  int qdt, vdt, gdt, bdt, g_vec;
  int B, T, Hk, Dk, Hv, Dv;
};

__device__ __forceinline__ float ld_any(const void* p, int64_t i, int dt) {
  switch (dt) {
    case LB2_F32: return static_cast<const float*>(p)[i];
    case LB2_BF16: return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
    default: return __half2float(static_cast<const __half*>(p)[i]);
  }
}

template <typename QT, int NPT>
__device__ __forceinline__ void ld_vec(const QT* p, float* out) {
#pragma unroll
  for (int i = 0; i < NPT; ++i) out[i] = to_f<QT>(p[i]);
}

template <typename QT, int NPT>
__global__ void __launch_bounds__(128) recurrent_kernel(const Params p) {
  const int lane = threadIdx.x & 31;
  const int64_t row = int64_t(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int64_t rows = int64_t(p.B) * p.Hv * p.Dv;
  if (row >= rows) return;
  const int dv = int(row % p.Dv);
  const int64_t bh = row / p.Dv;
  const int hv = int(bh % p.Hv), b = int(bh / p.Hv);
  const int hk = hv / (p.Hv / p.Hk);
  const int Dk = p.Dk;

  float s[NPT];
  const int64_t so = (bh * p.Dv + dv) * Dk + lane * NPT;
#pragma unroll
  for (int i = 0; i < NPT; ++i) s[i] = p.s_in[so + i];

  const QT* qb = static_cast<const QT*>(p.q);
  const QT* kb = static_cast<const QT*>(p.k);
  QT* yb = static_cast<QT*>(p.y);
  for (int t = 0; t < p.T; ++t) {
    const int64_t bt = int64_t(b) * p.T + t;
    const int64_t vo = (bt * p.Hv + hv) * p.Dv + dv;
    if (p.mask && !p.mask[bt]) {
      if (lane == 0) yb[vo] = from_f<QT>(0.f);
      continue;
    }
    const int64_t qo = (bt * p.Hk + hk) * Dk + lane * NPT;
    const int64_t go = bt * p.Hv + hv;
    float kf[NPT], qf[NPT], gf[NPT];
    ld_vec<QT, NPT>(kb + qo, kf);
    ld_vec<QT, NPT>(qb + qo, qf);
    if (p.g_vec) {
#pragma unroll
      for (int i = 0; i < NPT; ++i) gf[i] = ld_any(p.g, go * Dk + lane * NPT + i, p.gdt);
    } else {
      const float gs = ld_any(p.g, go, p.gdt);
#pragma unroll
      for (int i = 0; i < NPT; ++i) gf[i] = gs;
    }
    const float bt_ = ld_any(p.beta, go, p.bdt);
    const float vv = ld_any(p.v, vo, p.vdt);
    float kv = 0.f;
#pragma unroll
    for (int i = 0; i < NPT; ++i) {
      s[i] = s[i] * gf[i];
      kv = fmaf(s[i], kf[i], kv);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) kv += __shfl_xor_sync(0xffffffffu, kv, o);
    const float delta = (vv - kv) * bt_;
    float out = 0.f;
#pragma unroll
    for (int i = 0; i < NPT; ++i) {
      s[i] = fmaf(kf[i], delta, s[i]);
      out = fmaf(s[i], qf[i], out);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) out += __shfl_xor_sync(0xffffffffu, out, o);
    if (lane == 0) yb[vo] = from_f<QT>(out);
  }
#pragma unroll
  for (int i = 0; i < NPT; ++i) p.s_out[so + i] = s[i];
}

}  // namespace gdnrec
}  // namespace lb2
