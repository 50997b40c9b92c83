// Gated-DeltaNet recurrence, position by position (decode steps and short passes).
//
// One warp per R consecutive value rows of one (sequence b, value head hv), lane l holding state[dv][l*NPT,
// (l+1)*NPT) of each row in fp32 registers, as the reference's CUDA recurrence lays a row out (gdn_cuda.py:18-66);
// per position:
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

// NPT consecutive 16-bit values (one 8-byte load for NPT = 4, 16-byte for 8) widened to fp32.
template <typename QT, int NPT>
__device__ __forceinline__ void ld_vec(const QT* p, float* out) {
  if constexpr (NPT == 4) {
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    const QT* h = reinterpret_cast<const QT*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) out[i] = to_f<QT>(h[i]);
  } else if constexpr (NPT == 8) {
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    const QT* h = reinterpret_cast<const QT*>(&u);
#pragma unroll
    for (int i = 0; i < 8; ++i) out[i] = to_f<QT>(h[i]);
  } else {
#pragma unroll
    for (int i = 0; i < NPT; ++i) out[i] = to_f<QT>(p[i]);
  }
}

// R value rows a warp (consecutive rows of one head, so q / k loads are shared and R state rows are in flight at
// once); lane l holds elements [l * NPT, (l + 1) * NPT) of each row. Grid: x = groups of R rows (four warps a
// block), y = (b, hv): no index division.
template <typename QT, int NPT, int R>
__global__ void __launch_bounds__(128) recurrent_kernel(const Params p) {
  const int lane = threadIdx.x & 31;
  const int grp = int(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (grp * R >= p.Dv) return;
  const int dv0 = grp * R;
  const int64_t bh = blockIdx.y;
  const int hv = int(blockIdx.y) % p.Hv, b = int(blockIdx.y) / p.Hv;
  const int hk = hv / (p.Hv / p.Hk);
  const int Dk = p.Dk;

  float s[R][NPT];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int64_t so = (bh * p.Dv + dv0 + r) * Dk + lane * NPT;
    if constexpr (NPT == 4) {
      const float4 x = *reinterpret_cast<const float4*>(p.s_in + so);
      s[r][0] = x.x; s[r][1] = x.y; s[r][2] = x.z; s[r][3] = x.w;
    } else {
#pragma unroll
      for (int i = 0; i < NPT; ++i) s[r][i] = p.s_in[so + i];
    }
  }

  const QT* qb = static_cast<const QT*>(p.q);
  const QT* kb = static_cast<const QT*>(p.k);
  QT* yb = static_cast<QT*>(p.y);
  for (int t = 0; t < p.T; ++t) {
    const int64_t bt = int64_t(b) * p.T + t;
    const int64_t vo = (bt * p.Hv + hv) * p.Dv + dv0;
    if (p.mask && !p.mask[bt]) {
      if (lane < R) yb[vo + lane] = from_f<QT>(0.f);
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
    float vv[R];
#pragma unroll
    for (int r = 0; r < R; ++r) vv[r] = ld_any(p.v, vo + r, p.vdt);
    float kv[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      kv[r] = 0.f;
#pragma unroll
      for (int i = 0; i < NPT; ++i) {
        s[r][i] = s[r][i] * gf[i];
        kv[r] = fmaf(s[r][i], kf[i], kv[r]);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
      for (int r = 0; r < R; ++r) kv[r] += __shfl_xor_sync(0xffffffffu, kv[r], o);
    float out[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const float delta = (vv[r] - kv[r]) * bt_;
      out[r] = 0.f;
#pragma unroll
      for (int i = 0; i < NPT; ++i) {
        s[r][i] = fmaf(kf[i], delta, s[r][i]);
        out[r] = fmaf(s[r][i], qf[i], out[r]);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
      for (int r = 0; r < R; ++r) out[r] += __shfl_xor_sync(0xffffffffu, out[r], o);
    if (lane == 0)
#pragma unroll
      for (int r = 0; r < R; ++r) yb[vo + r] = from_f<QT>(out[r]);
  }
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int64_t so = (bh * p.Dv + dv0 + r) * Dk + lane * NPT;
    if constexpr (NPT == 4) {
      *reinterpret_cast<float4*>(p.s_out + so) = make_float4(s[r][0], s[r][1], s[r][2], s[r][3]);
    } else {
#pragma unroll
      for (int i = 0; i < NPT; ++i) p.s_out[so + i] = s[r][i];
    }
  }
}

}  // namespace gdnrec
}  // namespace lb2
