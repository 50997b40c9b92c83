// The attention layer's glue on either side of the SDPA (layer_glue.py:578-619, the reference's qk and agate
// kernels at layer_glue.py:241-296), for bf16 rows.
//
// qk_norm_rope: for each row (b, s) and each of the NQ query heads and NK key heads, x = the head's D values (query
// head h: columns [2 h D, 2 h D + D) of q_proj's output, whose other half is the output gate; key head h: columns
// [h D, h D + D) of k_proj's output),
//   inv = 1 / sqrt(sum(x^2) / D + eps)                         (fp32 sum of squares)
//   o_j = bf16(w_j * bf16(x_j * inv))                           (RMSNorm with the norm's bf16 weight)
//   j < R:  r_j = bf16(bf16(o_j * bf16(cos_j)) + bf16(rot_j * bf16(sin_j))),  rot_j = -o_{j+R/2} (j < R/2),
//           o_{j-R/2} (j >= R/2)                                 (rotate-half RoPE on the first R dims)
//   j >= R: r_j = o_j,
// written head-major: q [B, NQ, S, D], k [B, NK, S, D] (the layout the cache update and the SDPA take). cos / sin are
// [S, R] (one row a position, shared by the batch), in fp32, bf16 or fp16.
//
// out_gate: out[b, s, h D + j] = bf16(o[b, s, h D + j] * sig(g)), g = q_proj's gate value [b, s, 2 h D + D + j] and
// sig(g) = bf16(sigmoid(g)), the reference's per-bf16-pattern sigmoid table.
//
// Both are HBM-bound streams: D / 32 consecutive values a lane, 16-byte loads and stores; the grid's x index picks
// the rows and its y index the warp's head group (no 64-bit index division per warp). A warp takes ROWS rows of
// its head and issues their loads before any arithmetic; the RoPE phase runs on all 32 lanes over strided columns
// (coalesced cos / sin reads), through shared memory.
#pragma once

#include "common.cuh"

namespace lb2 {
namespace aglue {

struct QkParams {
  const __nv_bfloat16* qg;  // [B, S, NQ * 2 D]
  const __nv_bfloat16* kr;  // [B, S, NK * D]
  const __nv_bfloat16* qw;  // [D]
  const __nv_bfloat16* kw;  // [D]
  const void* cs;           // [S, R]
  const void* sn;           // [S, R]
  int csdt;
  float eps;
  __nv_bfloat16* q;  // [B, NQ, S, D]
  __nv_bfloat16* k;  // [B, NK, S, D]
  int B, S, NQ, NK, R;
};

__device__ __forceinline__ float bf(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

__device__ __forceinline__ float ld_any(const void* p, int64_t i, int dt) {
  switch (dt) {
    case LB2_F32: return static_cast<const float*>(p)[i];
    case LB2_BF16: return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
    default: return __half2float(static_cast<const __half*>(p)[i]);
  }
}

// E = D / 32 values a lane, loaded and stored as E / 8 16-byte pieces (E / 4 8-byte pieces when E == 4).
template <int E>
__device__ __forceinline__ void ld_row(const __nv_bfloat16* src, float* x) {
  if constexpr (E == 4) {
    const uint2 u = *reinterpret_cast<const uint2*>(src);
    const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) x[i] = __bfloat162float(h[i]);
  } else {
#pragma unroll
    for (int c = 0; c < E / 8; ++c) {
      const uint4 u = *reinterpret_cast<const uint4*>(src + 8 * c);
      const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
      for (int i = 0; i < 8; ++i) x[8 * c + i] = __bfloat162float(h[i]);
    }
  }
}

template <int E>
__device__ __forceinline__ void st_row(__nv_bfloat16* dst, const float* x) {
  if constexpr (E == 4) {
    uint2 u;
    __nv_bfloat16* h = reinterpret_cast<__nv_bfloat16*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __float2bfloat16_rn(x[i]);
    *reinterpret_cast<uint2*>(dst) = u;
  } else {
#pragma unroll
    for (int c = 0; c < E / 8; ++c) {
      uint4 u;
      __nv_bfloat16* h = reinterpret_cast<__nv_bfloat16*>(&u);
#pragma unroll
      for (int i = 0; i < 8; ++i) h[i] = __float2bfloat16_rn(x[8 * c + i]);
      *reinterpret_cast<uint4*>(dst + 8 * c) = u;
    }
  }
}

constexpr int WARPS = 4;
constexpr int ROWS = 2;  // rows a warp takes (one head): their loads are in flight together

template <int D>
__global__ void __launch_bounds__(WARPS * 32) qk_norm_rope_kernel(const QkParams p) {
  constexpr int E = D / 32;
  __shared__ __align__(16) float part[WARPS][ROWS][D];  // the normalised rows; RoPE updates its first R values
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hd = blockIdx.y * WARPS + warp;  // query heads, then key heads
  if (hd >= p.NQ + p.NK) return;
  const bool isq = hd < p.NQ;
  const int h = isq ? hd : hd - p.NQ;
  const int nrows = p.B * p.S;  // < 2^31: checked by the launcher
  const int row0 = blockIdx.x * ROWS;
  const int64_t rstride = isq ? int64_t(p.NQ) * 2 * D : int64_t(p.NK) * D;
  const __nv_bfloat16* src = (isq ? p.qg + int64_t(h) * 2 * D : p.kr + int64_t(h) * D) + lane * E;
  float x[ROWS][E];
#pragma unroll
  for (int r = 0; r < ROWS; ++r) {
    if (row0 + r < nrows) {
      ld_row<E>(src + (row0 + r) * rstride, x[r]);
    } else {
#pragma unroll
      for (int i = 0; i < E; ++i) x[r][i] = 0.f;
    }
  }
  float wv[E];
  ld_row<E>((isq ? p.qw : p.kw) + lane * E, wv);
  // RMSNorm; the rows go to shared memory, where the RoPE phase (all lanes, strided columns) reads its partners
#pragma unroll
  for (int r = 0; r < ROWS; ++r) {
    float acc = 0.f;
#pragma unroll
    for (int i = 0; i < E; ++i) acc = fmaf(x[r][i], x[r][i], acc);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    const float inv = 1.f / sqrtf(acc / float(D) + p.eps);
#pragma unroll
    for (int i = 0; i < E; i += 4)  // (16-byte stores: a lane's E values are consecutive)
      *reinterpret_cast<float4*>(&part[warp][r][lane * E + i]) =
          make_float4(bf(wv[i] * bf(x[r][i] * inv)), bf(wv[i + 1] * bf(x[r][i + 1] * inv)),
                      bf(wv[i + 2] * bf(x[r][i + 2] * inv)), bf(wv[i + 3] * bf(x[r][i + 3] * inv)));
  }
  __syncwarp();
  const int R = p.R, half = R >> 1;
  float rv[ROWS][(D + 31) / 32];  // rotated values of columns lane, lane + 32, ... (< R)
#pragma unroll
  for (int r = 0; r < ROWS; ++r) {
    const int row = row0 + r;
    const int s = row < nrows ? row % p.S : 0;
#pragma unroll
    for (int k = 0; k < D / 32; ++k) {
      const int j = lane + 32 * k;
      if (j < R) {
        const float oj = part[warp][r][j];
        const float rot = j < half ? -part[warp][r][j + half] : part[warp][r][j - half];
        const int64_t c = int64_t(s) * R + j;
        rv[r][k] = bf(bf(oj * bf(ld_any(p.cs, c, p.csdt))) + bf(rot * bf(ld_any(p.sn, c, p.csdt))));
      }
    }
  }
  __syncwarp();  // every partner read before the rotated values replace them
#pragma unroll
  for (int r = 0; r < ROWS; ++r)
#pragma unroll
    for (int k = 0; k < D / 32; ++k)
      if (lane + 32 * k < R) part[warp][r][lane + 32 * k] = rv[r][k];
  __syncwarp();
#pragma unroll
  for (int r = 0; r < ROWS; ++r) {
    const int row = row0 + r;
    if (row >= nrows) break;
    const int b = row / p.S, s = row - b * p.S;
    float o[E];
#pragma unroll
    for (int i = 0; i < E; i += 4) {
      const float4 v = *reinterpret_cast<const float4*>(&part[warp][r][lane * E + i]);
      o[i] = v.x;
      o[i + 1] = v.y;
      o[i + 2] = v.z;
      o[i + 3] = v.w;
    }
    __nv_bfloat16* dst = isq ? p.q + ((int64_t(b) * p.NQ + h) * p.S + s) * D
                              : p.k + ((int64_t(b) * p.NK + h) * p.S + s) * D;
    st_row<E>(dst + lane * E, o);
  }
}

struct GateParams {
  const __nv_bfloat16* o;   // [rows, NQ * D]
  const __nv_bfloat16* qg;  // [rows, NQ * 2 D]
  __nv_bfloat16* out;       // [rows, NQ * D] (may be o itself)
  int64_t rows;
  int NQ;
};

template <int D>
__global__ void __launch_bounds__(WARPS * 32) out_gate_kernel(const GateParams p) {
  constexpr int E = D / 32;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.y * WARPS + warp;
  if (h >= p.NQ) return;
  const int64_t row = blockIdx.x;
  const int64_t oo = row * (int64_t(p.NQ) * D) + int64_t(h) * D + lane * E;
  float x[E], g[E];
  ld_row<E>(p.o + oo, x);
  ld_row<E>(p.qg + row * (int64_t(p.NQ) * 2 * D) + int64_t(h) * 2 * D + D + lane * E, g);
#pragma unroll
  for (int i = 0; i < E; ++i) x[i] = bf(x[i] * bf(1.f / (1.f + expf(-g[i]))));
  st_row<E>(p.out + oo, x);
}

}  // namespace aglue
}  // namespace lb2
