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

// One position for the R state rows a warp holds (lane l: elements [l NPT, (l + 1) NPT) of each row):
//   s <- s * g; kv = s . k; delta = (v - kv) * beta; s <- s + k * delta; out = s . q,
// the dot products summed over the warp (out valid in every lane), the reference recurrence's arithmetic order per
// element (gdn_cuda.py:39-64).
template <int NPT, int R>
__device__ __forceinline__ void advance(float (&s)[R][NPT], const float* kf, const float* qf, const float* gf,
                                        float beta, const float* vv, float* out) {
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
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const float delta = (vv[r] - kv[r]) * beta;
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
}

template <int NPT, int R>
__device__ __forceinline__ void load_rows(float (&s)[R][NPT], const float* src) {
#pragma unroll
  for (int r = 0; r < R; ++r) {
    if constexpr (NPT == 4) {
      const float4 x = *reinterpret_cast<const float4*>(src + r * 32 * NPT);
      s[r][0] = x.x; s[r][1] = x.y; s[r][2] = x.z; s[r][3] = x.w;
    } else {
#pragma unroll
      for (int i = 0; i < NPT; ++i) s[r][i] = src[r * 32 * NPT + i];
    }
  }
}

template <int NPT, int R>
__device__ __forceinline__ void store_rows(const float (&s)[R][NPT], float* dst) {
#pragma unroll
  for (int r = 0; r < R; ++r) {
    if constexpr (NPT == 4) {
      *reinterpret_cast<float4*>(dst + r * 32 * NPT) = make_float4(s[r][0], s[r][1], s[r][2], s[r][3]);
    } else {
#pragma unroll
      for (int i = 0; i < NPT; ++i) dst[r * 32 * NPT + i] = s[r][i];
    }
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
  const int64_t so = (bh * p.Dv + dv0) * Dk + lane * NPT;  // row dv0's elements of this lane; row r at + r Dk
  load_rows<NPT, R>(s, p.s_in + so);

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
    float out[R];
    advance<NPT, R>(s, kf, qf, gf, bt_, vv, out);
    if (lane == 0)
#pragma unroll
      for (int r = 0; r < R; ++r) yb[vo + r] = from_f<QT>(out[r]);
  }
  store_rows<NPT, R>(s, p.s_out + so);
}

// ------------------------------------------------------------------------------------------------ decode-row glue
//
// qwen3_5's GatedDeltaNet decode rows from the causal conv's output (before silu), the recurrence with its glue in
// one pass: NR positions of one sequence, the state rows in registers across all of them. Per position, every warp
// makes its head's q and k itself (no shared memory, no block barrier): lane l takes elements [l NPT, (l + 1) NPT)
// of the head's q and k columns of the conv row, applies silu (sigmoid rounded to the activation dtype, then the
// product rounded), sums its squares and reduces over the warp, normalises (rsqrt(sum / Dk + eps), rounded), scales
// (sq, sk: Dk^-1 and Dk^-0.5 rounded, the product rounded) -- normalize_qk of qwen4_exp_vendor.py:471-473 at the
// rounding points of the reference's fused kernel (gdn_cuda.py:118-198). Every lane also forms beta = sigmoid(b)
// (rounded) and g = exp(-exp(A_log) softplus(a + dt_bias)) (fp32), and the silu'd v of the warp's R rows; then one
// `advance`. The q / k work is repeated by each warp of a head: 2 Dk values, against the R Dk state values a warp
// streams, so it stays off the memory path.
struct GlueParams {
  const void* conv;  // [NR, 2 Hk Dk + Hv Dv], activation dtype
  const void* a;     // [NR, Hv]
  const void* b;     // [NR, Hv]
  const float* A_log;    // [Hv]
  const float* dt_bias;  // [Hv]
  const float* s_in;     // [Hv, Dv, Dk]
  float* s_out;
  void* y;  // [NR, Hv, Dv]
  int NR, Hk, Hv, Dv;
  float sq, sk, eps;
};

template <typename T>
__device__ __forceinline__ float silu_rounded(float x) {
  const float sg = to_f<T>(from_f<T>(1.f / (1.f + __expf(-x))));
  return to_f<T>(from_f<T>(x * sg));
}

// Grid: x = groups of R rows (four warps a block), y = value head.
template <typename T, int NPT, int R>
__global__ void __launch_bounds__(128) glue_step_kernel(const GlueParams p) {
  constexpr int DK = 32 * NPT;
  const int lane = threadIdx.x & 31;
  const int grp = int(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (grp * R >= p.Dv) return;
  const int dv0 = grp * R;
  const int hv = blockIdx.y;
  const int hk = hv / (p.Hv / p.Hk);
  const int64_t cd = 2 * int64_t(p.Hk) * DK + int64_t(p.Hv) * p.Dv;
  const T* conv = static_cast<const T*>(p.conv);
  const T* av = static_cast<const T*>(p.a);
  const T* bv = static_cast<const T*>(p.b);
  T* yv = static_cast<T*>(p.y);
  const float decay_rate = __expf(p.A_log[hv]);
  const float bias = p.dt_bias[hv];

  float s[R][NPT];
  const int64_t so = (int64_t(hv) * p.Dv + dv0) * DK + lane * NPT;
  load_rows<NPT, R>(s, p.s_in + so);
  for (int pos = 0; pos < p.NR; ++pos) {
    const T* row = conv + pos * cd;
    float qf[NPT], kf[NPT], vv[R], gf[NPT];
    ld_vec<T, NPT>(row + int64_t(hk) * DK + lane * NPT, qf);
    ld_vec<T, NPT>(row + int64_t(p.Hk + hk) * DK + lane * NPT, kf);
    float nq = 0.f, nk = 0.f;
#pragma unroll
    for (int i = 0; i < NPT; ++i) {
      qf[i] = silu_rounded<T>(qf[i]);
      kf[i] = silu_rounded<T>(kf[i]);
      nq = fmaf(qf[i], qf[i], nq);
      nk = fmaf(kf[i], kf[i], nk);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      nq += __shfl_xor_sync(0xffffffffu, nq, o);
      nk += __shfl_xor_sync(0xffffffffu, nk, o);
    }
    const float iq = rsqrtf(nq / DK + p.eps), ik = rsqrtf(nk / DK + p.eps);
#pragma unroll
    for (int i = 0; i < NPT; ++i) {
      qf[i] = to_f<T>(from_f<T>(to_f<T>(from_f<T>(qf[i] * iq)) * p.sq));
      kf[i] = to_f<T>(from_f<T>(to_f<T>(from_f<T>(kf[i] * ik)) * p.sk));
    }
    const float beta = to_f<T>(from_f<T>(1.f / (1.f + __expf(-to_f<T>(bv[pos * p.Hv + hv])))));
    const float x = to_f<T>(av[pos * p.Hv + hv]) + bias;
    const float g = __expf(-decay_rate * (x > 20.f ? x : log1pf(__expf(x))));
#pragma unroll
    for (int i = 0; i < NPT; ++i) gf[i] = g;
#pragma unroll
    for (int r = 0; r < R; ++r) vv[r] = silu_rounded<T>(to_f<T>(row[2 * p.Hk * DK + int64_t(hv) * p.Dv + dv0 + r]));
    float out[R];
    advance<NPT, R>(s, kf, qf, gf, beta, vv, out);
    if (lane < R) {
      float mine = out[0];
#pragma unroll
      for (int r = 1; r < R; ++r)
        if (lane == r) mine = out[r];
      yv[(int64_t(pos) * p.Hv + hv) * p.Dv + dv0 + lane] = from_f<T>(mine);
    }
  }
  store_rows<NPT, R>(s, p.s_out + so);
}

}  // namespace gdnrec
}  // namespace lb2
