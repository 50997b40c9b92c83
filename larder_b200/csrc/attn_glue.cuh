// The attention layer's glue on either side of the SDPA (layer_glue.py:578-619, the reference's qk and agate
// kernels at layer_glue.py:241-296), for bf16 rows.
//
// qk_norm_rope: for each row (b, s) and each of the NQ query heads and NK key heads, x = the head's D values (query
// head h: columns [2 h D, 2 h D + D) of q_proj's output, whose other half is the output gate; key head h: columns
// [h D, h D + D) of k_proj's output),
//   inv = rsqrt(sum(x^2) / D + eps)        (fp32 sum of squares; rsqrtf, within 2 ulp of the reference's precise rsqrt)
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
// the rows and its y index the warp's head group (no 64-bit index division per warp). A warp takes several rows of
// its head and issues their loads before any arithmetic. For R in {0, 32, 64, 128} the lanes hold strided column pairs
// and RoPE runs on every lane (qk_rope_pair_kernel); other widths go through shared memory over strided columns
// (qk_norm_rope_kernel).
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

// bf16-rounds two values in place: one paired conversion, then bit moves back to fp32.
__device__ __forceinline__ void bf2(float& a, float& b) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  const uint32_t u = *reinterpret_cast<const uint32_t*>(&h);
  a = __uint_as_float(u << 16);
  b = __uint_as_float(u & 0xffff0000u);
}

// Stores E bf16-exact fp32 values (their low 16 bits zero) as bf16: the high halves packed by bit moves.
template <int E>
__device__ __forceinline__ void st_row_exact(__nv_bfloat16* dst, const float* x) {
  uint32_t w[E / 2];
#pragma unroll
  for (int i = 0; i < E / 2; ++i) w[i] = __byte_perm(__float_as_uint(x[2 * i]), __float_as_uint(x[2 * i + 1]), 0x7632);
  if constexpr (E == 4) {
    *reinterpret_cast<uint2*>(dst) = make_uint2(w[0], w[1]);
  } else {
#pragma unroll
    for (int c = 0; c < E / 8; ++c)
      *reinterpret_cast<uint4*>(dst + 8 * c) = make_uint4(w[4 * c], w[4 * c + 1], w[4 * c + 2], w[4 * c + 3]);
  }
}

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
    const float inv = rsqrtf(acc / float(D) + p.eps);
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

// qk_norm_rope in a pair-strided layout: lane l holds the column pairs (64 k + 2 l, 64 k + 2 l + 1), k < D / 64, so
// the rotated columns of a row are spread over all 32 lanes, and a column's rotate-half partner is in lane
// l ^ (R / 4), same pair (MODE 1: R = 32 or 64), or in this lane's other pair (MODE 2: R = 128); MODE 0 has no RoPE.
// A block takes QROWS rows and WARPS heads (a warp a head); the rows' cos / sin are read once a block into shared
// memory (rounded to bf16 as every use takes them, sin negated where the partner enters negated) while the warps' row
// loads are in flight. Roundings go two values a paired conversion; the results, bf16-exact, are packed for the stores
// by bit moves. The arithmetic and its roundings are those of qk_norm_rope_kernel.
constexpr int QROWS = 4;

// A table value as fp32 (cos / sin come as fp32, bf16 or f16).
__device__ __forceinline__ float tab_f(float x) { return x; }
__device__ __forceinline__ float tab_f(__nv_bfloat16 x) { return __bfloat162float(x); }
__device__ __forceinline__ float tab_f(__half x) { return __half2float(x); }

// The bf16 pair of two values, packed (low half a), and its two values back as fp32.
__device__ __forceinline__ uint32_t bf2w(float a, float b) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}
__device__ __forceinline__ float lo_f(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float hi_f(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

template <int D, int MODE, typename CT>
__global__ void __launch_bounds__(WARPS * 32) qk_rope_pair_kernel(const QkParams p) {
  constexpr int NP = D / 64;  // column pairs a lane
  __shared__ __align__(16) float2 trig[2][QROWS][64];  // (cos, sin) pairs of the block's rows, R / 2 <= 64 pairs
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hd = blockIdx.y * WARPS + warp;  // query heads, then key heads
  const bool live = hd < p.NQ + p.NK;
  const bool isq = hd < p.NQ;
  const int h = isq ? hd : hd - p.NQ;
  const int nrows = p.B * p.S;  // < 2^31: checked by the launcher
  const int row0 = blockIdx.x * QROWS;
  const int64_t rstride = isq ? int64_t(p.NQ) * 2 * D : int64_t(p.NK) * D;
  const __nv_bfloat16* src =
      (isq ? p.qg + int64_t(h) * 2 * D : p.kr + int64_t(h) * D) + int64_t(row0) * rstride + 2 * lane;
  uint32_t raw[QROWS][NP], wraw[NP];
  if (live) {
#pragma unroll
    for (int r = 0; r < QROWS; ++r) {
      const bool in = row0 + r < nrows;
#pragma unroll
      for (int k = 0; k < NP; ++k)
        raw[r][k] = in ? *reinterpret_cast<const uint32_t*>(src + r * rstride + 64 * k) : 0u;
    }
    const __nv_bfloat16* w = (isq ? p.qw : p.kw) + 2 * lane;
#pragma unroll
    for (int k = 0; k < NP; ++k) wraw[k] = *reinterpret_cast<const uint32_t*>(w + 64 * k);
  }
  // the block's first row as (sequence, position); later rows step the position (rows past the end take the
  // positions that follow, inside the table)
  const int b0 = row0 / p.S, s0 = row0 - b0 * p.S;
  const int R = p.R;
  if (MODE != 0) {
    const int q = threadIdx.x;  // q < R / 2: cos pairs, else sin pairs (R <= 128: one per thread)
    if (q < R) {
      const int w = 2 * q >= R, qq = q - w * (R >> 1);
      const CT* tab = static_cast<const CT*>(w ? p.sn : p.cs) + 2 * qq;
      const bool neg = w && 4 * qq < R;
      int s = s0;
#pragma unroll
      for (int r = 0; r < QROWS; ++r) {
        const CT* e = tab + int64_t(s) * R;
        float a = tab_f(e[0]), b = tab_f(e[1]);
        bf2(a, b);
        if (neg) a = -a, b = -b;
        trig[w][r][qq] = make_float2(a, b);
        if (++s == p.S) s = 0;
      }
    }
  }
  __syncthreads();
  if (!live) return;
  float wv[2 * NP];
#pragma unroll
  for (int k = 0; k < NP; ++k) wv[2 * k] = lo_f(wraw[k]), wv[2 * k + 1] = hi_f(wraw[k]);
  const int NH = isq ? p.NQ : p.NK;
  __nv_bfloat16* const obase = (isq ? p.q : p.k) + 2 * lane;
  int b = b0, s = s0;
  int64_t orow = (int64_t(b) * NH + h) * p.S + s;  // output row of (b, h, s)
#pragma unroll
  for (int r = 0; r < QROWS; ++r) {
    float x[2 * NP];
#pragma unroll
    for (int k = 0; k < NP; ++k) x[2 * k] = lo_f(raw[r][k]), x[2 * k + 1] = hi_f(raw[r][k]);
    float acc = 0.f;
#pragma unroll
    for (int i = 0; i < 2 * NP; ++i) acc = fmaf(x[i], x[i], acc);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    const float inv = rsqrtf(acc / float(D) + p.eps);
    // bf16(bf16(x inv) w), packed: the stored words of the pairs RoPE leaves alone
    uint32_t ow[NP];
#pragma unroll
    for (int k = 0; k < NP; ++k) {
      float u = x[2 * k] * inv, v = x[2 * k + 1] * inv;
      bf2(u, v);
      ow[k] = bf2w(u * wv[2 * k], v * wv[2 * k + 1]);
    }
    if (MODE == 1) {  // pair 0 of lanes 2 lane < R: partner in lane ^ (R / 4)
      const float x0 = lo_f(ow[0]), x1 = hi_f(ow[0]);
      const float p0 = __shfl_xor_sync(0xffffffffu, x0, R >> 2), p1 = __shfl_xor_sync(0xffffffffu, x1, R >> 2);
      if (2 * lane < R) {
        const float2 c = trig[0][r][lane], sg = trig[1][r][lane];
        float a0 = x0 * c.x, a1 = x1 * c.y, q0 = p0 * sg.x, q1 = p1 * sg.y;
        bf2(a0, a1);
        bf2(q0, q1);
        ow[0] = bf2w(a0 + q0, a1 + q1);
      }
    } else if (MODE == 2) {  // pairs 0 and 1 (R = 128): each the other's partner
      const float xs[4] = {lo_f(ow[0]), hi_f(ow[0]), lo_f(ow[1]), hi_f(ow[1])};
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const float2 c = trig[0][r][32 * k + lane], sg = trig[1][r][32 * k + lane];
        float a0 = xs[2 * k] * c.x, a1 = xs[2 * k + 1] * c.y, q0 = xs[2 * (1 - k)] * sg.x,
              q1 = xs[2 * (1 - k) + 1] * sg.y;
        bf2(a0, a1);
        bf2(q0, q1);
        ow[k] = bf2w(a0 + q0, a1 + q1);
      }
    }
    if (row0 + r < nrows) {
      __nv_bfloat16* dst = obase + orow * D;
#pragma unroll
      for (int k = 0; k < NP; ++k) *reinterpret_cast<uint32_t*>(dst + 64 * k) = ow[k];
    }
    if (++s == p.S) {
      s = 0, ++b;
      orow = (int64_t(b) * NH + h) * p.S;
    } else {
      ++orow;
    }
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
  for (int i = 0; i < E; i += 2) {
    float s0 = 1.f / (1.f + expf(-g[i])), s1 = 1.f / (1.f + expf(-g[i + 1]));
    bf2(s0, s1);
    float a = x[i] * s0, b = x[i + 1] * s1;
    bf2(a, b);
    x[i] = a, x[i + 1] = b;
  }
  st_row_exact<E>(p.out + oo, x);
}

}  // namespace aglue
}  // namespace lb2
