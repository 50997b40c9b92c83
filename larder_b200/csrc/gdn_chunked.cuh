// Gated-DeltaNet chunked prefill: the recurrence of gdn_cuda.py:18-66 (scalar gate, no mask) computed in chunks
// of C = 64 positions, Dk = Dv = 128.
//
// Within a chunk with cumulative log-decay gamma_t = sum_{i<=t} log g_i and Gam_t = exp(gamma_t), the state after
// position t is  S_t = Gam_t S_0 + sum_{j<=t} exp(gamma_t - gamma_j) u_j k_j^T,  where the deltas u_j solve the
// unit lower-triangular system  (I + A) U = diag(beta) V - diag(beta Gam) K S_0^T,
//   A[t][j] = beta_t exp(gamma_t - gamma_j) (k_t . k_j)  (j < t).
// With T = (I + A)^{-1}, W = T diag(beta Gam) K and U' = T diag(beta) V this is U = U' - W S_0^T, and
//   Y = diag(Gam) Q S_0^T + M U,  M[t][j] = exp(gamma_t - gamma_j) (q_t . k_j)  (j <= t),
//   S_C = Gam_C S_0 + U^T diag(exp(gamma_C - gamma)) K.
// Decay ratios are always formed as exp(gamma_t - gamma_j) with j <= t (never a division by a small Gam), so no
// intermediate overflows however strong the decay.
//
// Two launches:
//   prep (grid: chunks x v-heads x batch, independent): K K^T and Q K^T on bf16 mma.sync (fp32 accumulate), the
//        decay / beta weighting, T by blocked inversion (16 x 16 diagonal blocks by substitution, then 32 and 64
//        by the 2 x 2 block formula) in fp32, and W, U' on TF32 mma.sync with their B operands (beta Gam K,
//        beta V) formed from the 16-bit tiles on the fly; writes W, U', M, gamma, Gam to the workspace.
//   scan (grid: Dv / 32 value-row blocks x v-heads x batch, 8 warps): the state slice S[32 x 128] in fp32
//        registers (a TF32 copy in shared memory for the products that read all of it), chunks in order, each
//        chunk's tiles prefetched by bulk copies (the workspace is laid out as the shared-memory tiles) while the
//        previous chunk computes; U, Y and the state update on TF32 mma.sync with fp32 accumulation. W and M are
//        stored already rounded to TF32 by prep.
#pragma once

#include "common.cuh"

namespace lb2 {
namespace gdnchunk {

constexpr int C = 64;
constexpr int DK = 128;
constexpr int DV = 128;
constexpr int DVB = 32;   // value rows a scan CTA owns
constexpr int KP = 136;   // bf16 row stride of K / Q tiles (conflict-free ldmatrix and scalar reads)
constexpr int AP = 68;    // fp32 row stride of A / T / M tiles
constexpr int RP = 136;   // fp32 row stride of 128-wide fp32 tiles (B operands)
constexpr int WP = 132;   // fp32 row stride of W / S tiles (A operands and S^T reads)
constexpr int UP = 36;    // fp32 row stride of 32-wide U tiles
// Workspace of one (batch, head, chunk) in floats, laid out as the scan's shared-memory tiles (padded rows included)
// so that a scan CTA fetches a chunk with two bulk copies: W [C][WP] and M [C][AP] (TF32 values) and gamma, Gam
// [2 C] as one block, then U' as DV / DVB slices [C][UP] of 32 value columns each.
constexpr int WS_W = 0;
constexpr int WS_M = WS_W + C * WP;
constexpr int WS_G = WS_M + C * AP;
constexpr int WS_U = WS_G + 2 * C;
constexpr int UNIT = WS_U + (DV / DVB) * C * UP;
constexpr int WMG_BYTES = WS_U * 4;  // W, M and the gates: one copy
static_assert(WS_M % 4 == 0 && WS_G % 4 == 0 && WS_U % 4 == 0 && UNIT % 4 == 0, "16-byte aligned workspace tiles");

struct Params {
  const void* q;
  const void* k;
  const void* v;
  const void* g;
  const void* beta;
  int qdt, vdt, gdt, bdt;
  const float* s_in;
  float* s_out;
  void* y;
  int B, T, Hk, Hv, nchunks;
  float* ws;
};

__device__ __forceinline__ float ldf(const void* p, int64_t i, int dt) {
  switch (dt) {
    case LB2_F32: return static_cast<const float*>(p)[i];
    case LB2_BF16: return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
    default: return __half2float(static_cast<const __half*>(p)[i]);
  }
}

__device__ __forceinline__ uint32_t tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return r;
}

// A 16-bit value's exact TF32 bit pattern (bf16 and fp16 mantissas fit TF32's 10 bits).
template <typename T>
__device__ __forceinline__ uint32_t tf32_of(T x) {
  return __float_as_uint(to_f<T>(x));
}

__device__ __forceinline__ void mma_tf32(float* c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

template <typename T>
__device__ __forceinline__ void mma_16816(float* c, const uint32_t* a, uint32_t b0, uint32_t b1);
template <>
__device__ __forceinline__ void mma_16816<__nv_bfloat16>(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
template <>
__device__ __forceinline__ void mma_16816<__half>(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldsm4(uint32_t addr, uint32_t* r) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

// 16-byte cp.async, zero-filling the destination when `in` is false (nothing is read then).
__device__ __forceinline__ void cp_async16_zfill(void* dst, const void* src, bool in) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(in ? 16 : 0)
               : "memory");
}

// acc (a 16 x 8 m16n8k8 accumulator) += L R over K = 8 ksteps, with L's rows at Lp (row stride ldl, columns from
// Lp) and R's rows k at Rp + k ldr, in three TF32 products per step (hi hi + hi lo + lo hi of each fp32 operand
// split into TF32 high and low parts), so that the block products of the inversion keep close to fp32 accuracy.
__device__ __forceinline__ void mma3_tile(const float* Lp, int ldl, const float* Rp, int ldr, int ksteps, float* acc,
                                          int lane) {
  const int r = lane >> 2, cq = lane & 3;
  for (int ks = 0; ks < ksteps; ++ks) {
    const int k0 = ks * 8;
    const float a[4] = {Lp[r * ldl + k0 + cq], Lp[(r + 8) * ldl + k0 + cq], Lp[r * ldl + k0 + cq + 4],
                        Lp[(r + 8) * ldl + k0 + cq + 4]};
    const float bb[2] = {Rp[(k0 + cq) * ldr + r], Rp[(k0 + cq + 4) * ldr + r]};
    uint32_t ah[4], al[4], bh[2], bl[2];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      ah[i] = tf32(a[i]);
      al[i] = tf32(a[i] - __uint_as_float(ah[i]));
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      bh[i] = tf32(bb[i]);
      bl[i] = tf32(bb[i] - __uint_as_float(bh[i]));
    }
    mma_tf32(acc, al[0], al[1], al[2], al[3], bh[0], bh[1]);
    mma_tf32(acc, ah[0], ah[1], ah[2], ah[3], bl[0], bl[1]);
    mma_tf32(acc, ah[0], ah[1], ah[2], ah[3], bh[0], bh[1]);
  }
}

// Workspace tiles of one (batch, head, chunk).
__device__ __forceinline__ float* unit_ptr(const Params& p, int b, int h, int c) {
  return p.ws + ((int64_t(b) * p.Hv + h) * p.nchunks + c) * UNIT;
}

// ------------------------------------------------------------------------------------------------ prep

struct PrepSmem {
  static constexpr int KB = 0;                              // bf16 [C][KP]
  static constexpr int QB = KB + C * KP * 2;                // bf16 [C][KP]
  static constexpr int VB = QB + C * KP * 2;                // bf16 [C][KP]
  static constexpr int AF = VB + C * KP * 2;                // f32 [C][AP]  A, then T
  static constexpr int XS = AF + C * AP * 4;                // f32 [32][XP] inversion scratch
  static constexpr int GAM = XS + 32 * 40 * 4;              // f32 [C] gamma, [C] Gam, [C] beta
  static constexpr int BYTES = GAM + 3 * C * 4;
};

template <typename T>
__global__ void __launch_bounds__(128) prep_kernel(const Params p) {
  const int c = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int hk = h / (p.Hv / p.Hk);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int t0 = c * C;
  extern __shared__ __align__(16) uint8_t sm[];
  T* Kb = reinterpret_cast<T*>(sm + PrepSmem::KB);
  T* Qb = reinterpret_cast<T*>(sm + PrepSmem::QB);
  T* Vb = reinterpret_cast<T*>(sm + PrepSmem::VB);
  float* Af = reinterpret_cast<float*>(sm + PrepSmem::AF);
  float* Xs = reinterpret_cast<float*>(sm + PrepSmem::XS);
  float* gam = reinterpret_cast<float*>(sm + PrepSmem::GAM);
  float* Gam = gam + C;
  float* bet = Gam + C;

  // 1. K, Q and V tiles (16-bit) by cp.async, zero past T: they land while the gates are formed
  {
    const T* kg = static_cast<const T*>(p.k);
    const T* qg = static_cast<const T*>(p.q);
    const T* vg = static_cast<const T*>(p.v);
#pragma unroll
    for (int i = 0; i < C * (DK / 8) / 128; ++i) {
      const int e = tid + 128 * i, r = e / (DK / 8), u = e % (DK / 8);
      const bool in = t0 + r < p.T;
      const int64_t row = int64_t(b) * p.T + (in ? t0 + r : 0);  // (a row of the sequence even when not read)
      cp_async16_zfill(Kb + r * KP + u * 8, kg + (row * p.Hk + hk) * DK + u * 8, in);
      cp_async16_zfill(Qb + r * KP + u * 8, qg + (row * p.Hk + hk) * DK + u * 8, in);
      cp_async16_zfill(Vb + r * KP + u * 8, vg + (row * p.Hv + h) * DV + u * 8, in);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  }
  // 2. gates: gamma = inclusive prefix sum of log g over the chunk (positions past T: g = 1, beta = 0)
  if (warp == 0) {
    float x[2], bt[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int pos = t0 + lane + 32 * u;
      const bool in = pos < p.T;
      const int64_t go = (int64_t(b) * p.T + pos) * p.Hv + h;
      x[u] = in ? __logf(ldf(p.g, go, p.gdt)) : 0.f;
      bt[u] = in ? ldf(p.beta, go, p.bdt) : 0.f;
    }
#pragma unroll
    for (int u = 0; u < 2; ++u)
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float y = __shfl_up_sync(0xffffffffu, x[u], o);
        if (lane >= o) x[u] += y;
      }
    x[1] += __shfl_sync(0xffffffffu, x[0], 31);
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      gam[lane + 32 * u] = x[u];
      Gam[lane + 32 * u] = __expf(x[u]);
      bet[lane + 32 * u] = bt[u];
    }
  }
  asm volatile("cp.async.wait_all;" ::: "memory");
  __syncthreads();

  // 3. K K^T and Q K^T for rows 16 w .. 16 w + 15 (bf16 mma, fp32 accumulate), then decay / beta weighting
  {
    float kk[8][4], qk[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) kk[n][e] = qk[n][e] = 0.f;
    const uint32_t kb_addr = smem_u32(Kb), qb_addr = smem_u32(Qb);
#pragma unroll
    for (int ks = 0; ks < DK / 16; ++ks) {
      uint32_t ak[4], aq[4];
      const int ar = warp * 16 + (lane & 15), ac = ks * 16 + (lane >> 4) * 8;
      ldsm4(kb_addr + (ar * KP + ac) * 2, ak);
      ldsm4(qb_addr + (ar * KP + ac) * 2, aq);
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t bk[4];
        const int br = np * 16 + (lane & 7) + 8 * (lane >> 4), bc = ks * 16 + ((lane >> 3) & 1) * 8;
        ldsm4(kb_addr + (br * KP + bc) * 2, bk);
        mma_16816<T>(kk[2 * np], ak, bk[0], bk[1]);
        mma_16816<T>(kk[2 * np + 1], ak, bk[2], bk[3]);
        mma_16816<T>(qk[2 * np], aq, bk[0], bk[1]);
        mma_16816<T>(qk[2 * np + 1], aq, bk[2], bk[3]);
      }
    }
    float* Mg = unit_ptr(p, b, h, c) + WS_M;
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {  // columns j, j + 1 of row t
        const int t = warp * 16 + (lane >> 2) + 8 * hh;
        const int j = n * 8 + 2 * (lane & 3);
        const float d0 = j <= t ? __expf(gam[t] - gam[j]) : 0.f, d1 = j + 1 <= t ? __expf(gam[t] - gam[j + 1]) : 0.f;
        *reinterpret_cast<float2*>(&Af[t * AP + j]) =
            make_float2(j < t ? bet[t] * d0 * kk[n][2 * hh] : 0.f, j + 1 < t ? bet[t] * d1 * kk[n][2 * hh + 1] : 0.f);
        // an MMA operand of the scan: rounded once here
        *reinterpret_cast<float2*>(&Mg[t * AP + j]) = make_float2(__uint_as_float(tf32(d0 * qk[n][2 * hh])),
                                                                  __uint_as_float(tf32(d1 * qk[n][2 * hh + 1])));
      }
  }
  __syncthreads();

  // 4. T = (I + A)^{-1}, in place over A's lower triangle (diagonal 1, upper 0)
  // level 0: each warp inverts its 16 x 16 diagonal block by forward substitution, lane i holding column i
  {
    const int base = warp * 16;
    float tc[16];
    const int i = lane & 15;
#pragma unroll
    for (int r = 0; r < 16; ++r) {
      float s = 0.f;
#pragma unroll
      for (int j = 0; j < r; ++j) s = fmaf(Af[(base + r) * AP + base + j], tc[j], s);
      tc[r] = i < r ? -s : (i == r ? 1.f : 0.f);
    }
    __syncwarp();
    if (lane < 16)
#pragma unroll
      for (int r = 0; r < 16; ++r) Af[(base + r) * AP + base + i] = tc[r];
  }
  __syncthreads();
  // level 1: T[hi][lo] = -T[hi][hi] A[hi][lo] T[lo][lo] for the block pairs (0, 1) and (2, 3) (16 x 16 blocks):
  // warp w takes pair w / 2 and output columns 8 (w % 2) .. + 7, first of X = A[hi][lo] T[lo][lo], then of the block
  constexpr int XP = 40;  // row stride of the scratch X (conflict-free B fragment reads)
  {
    const int pr = warp >> 1, n0 = (warp & 1) * 8;
    const int lo = 32 * pr, hi = lo + 16;
    float* X = Xs + pr * 16 * XP;
    const int r = lane >> 2, cq = lane & 3;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    mma3_tile(Af + hi * AP + lo, AP, Af + lo * AP + lo + n0, AP, 2, acc, lane);
    X[r * XP + n0 + 2 * cq] = acc[0];
    X[r * XP + n0 + 2 * cq + 1] = acc[1];
    X[(r + 8) * XP + n0 + 2 * cq] = acc[2];
    X[(r + 8) * XP + n0 + 2 * cq + 1] = acc[3];
    __syncthreads();
    float t[4] = {0.f, 0.f, 0.f, 0.f};
    mma3_tile(Af + hi * AP + hi, AP, X + n0, XP, 2, t, lane);
    Af[(hi + r) * AP + lo + n0 + 2 * cq] = -t[0];
    Af[(hi + r) * AP + lo + n0 + 2 * cq + 1] = -t[1];
    Af[(hi + r + 8) * AP + lo + n0 + 2 * cq] = -t[2];
    Af[(hi + r + 8) * AP + lo + n0 + 2 * cq + 1] = -t[3];
  }
  __syncthreads();
  // level 2: T[32:64][0:32] = -T[32:64][32:64] A[32:64][0:32] T[0:32][0:32] (32 x 32 blocks): warp w takes the two
  // 16 x 8 output tiles 2 w, 2 w + 1 (row tile = index / 4, column tile = index % 4) of each product
  {
    const int r = lane >> 2, cq = lane & 3;
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int ti = warp * 2 + u, m0 = (ti >> 2) * 16, n0 = (ti & 3) * 8;
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
      mma3_tile(Af + (32 + m0) * AP, AP, Af + n0, AP, 4, acc, lane);
      Xs[(m0 + r) * XP + n0 + 2 * cq] = acc[0];
      Xs[(m0 + r) * XP + n0 + 2 * cq + 1] = acc[1];
      Xs[(m0 + r + 8) * XP + n0 + 2 * cq] = acc[2];
      Xs[(m0 + r + 8) * XP + n0 + 2 * cq + 1] = acc[3];
    }
    __syncthreads();
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int ti = warp * 2 + u, m0 = (ti >> 2) * 16, n0 = (ti & 3) * 8;
      float t[4] = {0.f, 0.f, 0.f, 0.f};
      mma3_tile(Af + (32 + m0) * AP + 32, AP, Xs + n0, XP, 4, t, lane);
      Af[(32 + m0 + r) * AP + n0 + 2 * cq] = -t[0];
      Af[(32 + m0 + r) * AP + n0 + 2 * cq + 1] = -t[1];
      Af[(32 + m0 + r + 8) * AP + n0 + 2 * cq] = -t[2];
      Af[(32 + m0 + r + 8) * AP + n0 + 2 * cq + 1] = -t[3];
    }
  }
  __syncthreads();
  // 5. U' = T diag(beta) V, then W = T diag(beta Gam) K (TF32 mma). Warp w takes output columns 32 w .. 32 w + 31 of
  // all four 16-row blocks (T is lower triangular, so row block m reads k < 16 (m + 1): split by rows, the last
  // warp would do four times the first's work). The column factors (beta, then Gam on top) are folded into T first,
  // warp w scaling rows 16 w .., so that the B fragments are the 16-bit tiles' exact TF32 values.
  {
    float* Wg = unit_ptr(p, b, h, c) + WS_W;
    float* Ug = unit_ptr(p, b, h, c) + WS_U;
    const int r = lane >> 2, cq = lane & 3, nw = warp * 32;
#pragma unroll 1
    for (int which = 1; which >= 0; --which) {
      const T* R = which ? Vb : Kb;
      {  // lane l scales columns l and l + 32 of rows 16 w .. 16 w + 15 (the lower triangle: columns < 16 w + 16)
        const int m0 = warp * 16;
        const float f0 = which ? bet[lane] : Gam[lane], f1 = which ? bet[lane + 32] : Gam[lane + 32];
#pragma unroll
        for (int rr = 0; rr < 16; ++rr) {
          Af[(m0 + rr) * AP + lane] *= f0;
          if (m0 >= 16) Af[(m0 + rr) * AP + lane + 32] *= f1;
        }
      }
      __syncthreads();
#pragma unroll 1
      for (int mt = 0; mt < 4; ++mt) {
        const int m0 = mt * 16;
        float acc[4][4];
#pragma unroll
        for (int n = 0; n < 4; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.f;
        for (int k0 = 0; k0 < m0 + 16; k0 += 8) {
          const uint32_t a0 = tf32(Af[(m0 + r) * AP + k0 + cq]), a1 = tf32(Af[(m0 + r + 8) * AP + k0 + cq]);
          const uint32_t a2 = tf32(Af[(m0 + r) * AP + k0 + cq + 4]), a3 = tf32(Af[(m0 + r + 8) * AP + k0 + cq + 4]);
#pragma unroll
          for (int n = 0; n < 4; ++n) {
            const int n0 = nw + n * 8;
            mma_tf32(acc[n], a0, a1, a2, a3, tf32_of(R[(k0 + cq) * KP + n0 + r]),
                     tf32_of(R[(k0 + cq + 4) * KP + n0 + r]));
          }
        }
        if (!which)  // W is an MMA operand of the scan: stored rounded to TF32; U' stays fp32
#pragma unroll
          for (int n = 0; n < 4; ++n)
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[n][e] = __uint_as_float(tf32(acc[n][e]));
#pragma unroll
        for (int n = 0; n < 4; ++n) {  // W rows of stride WP; U' in slices of DVB columns, rows of stride UP
          const int col = nw + n * 8 + 2 * cq;
          float* g0 = which ? Ug + ((col / DVB) * C + m0 + r) * UP + col % DVB : Wg + (m0 + r) * WP + col;
          float* g1 = g0 + 8 * (which ? UP : WP);
          *reinterpret_cast<float2*>(g0) = make_float2(acc[n][0], acc[n][1]);
          *reinterpret_cast<float2*>(g1) = make_float2(acc[n][2], acc[n][3]);
        }
      }
      __syncthreads();  // every warp has read T before it is scaled again
    }
  }
  // 7. gamma and Gam for the scan
  if (tid < C) {
    float* gg = unit_ptr(p, b, h, c) + WS_G;
    gg[tid] = gam[tid];
    gg[C + tid] = Gam[tid];
  }
}

// ------------------------------------------------------------------------------------------------ scan

constexpr int SCAN_THREADS = 256;  // warps 0-3: U = U' - W S^T and the state update; warps 4-7: Q S^T and M U
constexpr int UQ = 68;             // u32 row stride of the transposed U tiles [DVB][C] (conflict-free ldmatrix)

struct ScanSmem {
  // one prefetch buffer; W, M and G in the workspace's order (one bulk copy)
  static constexpr int W = 0;                         // tf32 [C][WP]
  static constexpr int M = W + (WS_M - WS_W) * 4;     // tf32 [C][AP]
  static constexpr int G = W + (WS_G - WS_W) * 4;     // f32 [C] gamma, [C] Gam
  static constexpr int U = W + (WS_U - WS_W) * 4;     // f32 [C][UP]   U' columns of this block
  // Q and K tiles as the tiled TMA lands them: two boxes of [64 positions][64 columns] (128-byte rows, 128-byte
  // swizzle: the 16-byte piece j of row r sits at piece j ^ (r % 8)), 1024-byte aligned
  static constexpr int QK_TILE = 2 * C * 64 * 2;
  static constexpr int Q = (U + C * UP * 4 + 1023) / 1024 * 1024;
  static constexpr int K = Q + QK_TILE;
  static constexpr int BUF = K + QK_TILE;
  // persistent
  static constexpr int ST = 2 * BUF;                  // tf32 [DVB][WP] the state slice, rounded for the MMAs
  static constexpr int UB = ST + DVB * WP * 4;        // tf32 [DVB][UQ] this chunk's U, transposed
  static constexpr int UD = UB + DVB * UQ * 4;        // tf32 [DVB][UQ] (diag(exp(gamma_C - gamma)) U)^T
  static constexpr int BAR = UD + DVB * UQ * 4;       // 2 mbarriers: buffer b's copies landed
  static constexpr int BYTES = BAR + 16 + 1024;  // (+ alignment of the dynamic shared memory base to 1024)
};
static_assert(ScanSmem::BUF % 1024 == 0 && ScanSmem::U % 16 == 0 && ScanSmem::Q % 1024 == 0, "copy alignment");
static_assert(ScanSmem::BYTES <= 232448, "scan shared memory");

// Element (row, col) of a Q / K tile (see ScanSmem) as its exact TF32 bit pattern.
template <typename T>
__device__ __forceinline__ uint32_t qk_tf32(const uint8_t* tile, int row, int col) {
  const int off = (col >> 6) * (C * 128) + row * 128 + ((((col & 63) >> 3) ^ (row & 7)) << 4) + ((col & 7) << 1);
  return tf32_of(*reinterpret_cast<const T*>(tile + off));
}

// TF32 m16n8k8 fragments by ldmatrix (an 8 x 4 block of 32-bit values is an 8 x 8 block of 16-bit halves; thread
// g * 4 + t receives the 32-bit value at row g, column t, the fragments' layout). `base` is the shared address of
// element (0, 0) of a row-major fp32 / TF32 tile with `ld` values a row (ld * 4 % 128 == 16: conflict-free rows).
// A: rows m0 .. m0 + 15, columns k0 .. k0 + 7.
__device__ __forceinline__ void frag_a(uint32_t base, int ld, int m0, int k0, int lane, uint32_t* a) {
  ldsm4(base + ((m0 + (lane & 7) + ((lane >> 3) & 1) * 8) * ld + k0 + (lane >> 4) * 4) * 4, a);
}
// B of two n-tiles from a tile stored n-major ([n][k]): n0 .. n0 + 15, k0 .. k0 + 7; b[0], b[1] for n-tile n0,
// b[2], b[3] for n0 + 8.
__device__ __forceinline__ void frag_b2(uint32_t base, int ld, int n0, int k0, int lane, uint32_t* b) {
  ldsm4(base + ((n0 + (lane & 7) + (lane >> 4) * 8) * ld + k0 + ((lane >> 3) & 1) * 4) * 4, b);
}


// The tiles of chunk c into one buffer, completing on its mbarrier (thread 0 issues all): W, M and the gates in one
// bulk copy, this block's U' slice in another, and the Q and K tiles by tiled TMA, two 64-column boxes each (rows
// past T arrive as zeros).
__device__ __forceinline__ void scan_prefetch(const Params& p, const CUtensorMap* qmap, const CUtensorMap* kmap,
                                              uint8_t* buf, uint64_t* full, int b, int h, int hk, int c, int blk) {
  const float* u = unit_ptr(p, b, h, c);
  fence_proxy_async_shared();  // the buffer's reads two chunks back precede these writes
  mbar_arrive_expect_tx(full, uint32_t(WMG_BYTES + C * UP * 4 + 2 * ScanSmem::QK_TILE));
  bulk_g2s(buf + ScanSmem::W, u + WS_W, WMG_BYTES, full);
  bulk_g2s(buf + ScanSmem::U, u + WS_U + blk * C * UP, C * UP * 4, full);
#pragma unroll
  for (int db = 0; db < DK / 64; ++db) {
    tma_load_4d(buf + ScanSmem::Q + db * C * 128, qmap, db * 64, c * C, hk, b, full);
    tma_load_4d(buf + ScanSmem::K + db * C * 128, kmap, db * 64, c * C, hk, b, full);
  }
}

// Named barriers (ids 1-4; 0 is __syncthreads): wait until `count` threads arrived, or arrive without waiting. The
// arriving threads' earlier shared-memory writes are visible to the threads that waited.
__device__ __forceinline__ void nbar_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}
__device__ __forceinline__ void nbar_arrive(int id, int count) {
  asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(count) : "memory");
}
// bar.sync that also ORs a flag over the participating threads.
__device__ __forceinline__ bool nbar_sync_or(int id, int count, bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\tbar.red.or.pred q, %2, %3, p;\n\tselp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(uint32_t(v)), "r"(id), "r"(count)
      : "memory");
  return r != 0;
}
constexpr int BAR_A = 1;   // all 256: U of the chunk written, every read of the state copy done
constexpr int BAR_S = 2;   // warps 0-3 arrive, warps 4-7 wait: the state copy updated
constexpr int BAR_U = 3;   // warps 4-7 arrive, warps 0-3 wait: M U read the chunk's U and its buffer is done with
constexpr int BAR_S0 = 4;  // warps 0-3: the state copy updated, before their next W S^T

// One CTA: value rows dv0 .. dv0 + 31 of one (batch, v-head), all chunks in order. Two roles, so that Y stays off the
// chain from one chunk's state to the next:
//   warps 0-3 own the fp32 state slice in registers (warp w: key columns 32 w .. 32 w + 31 of all 32 rows; a TF32
//     copy in shared memory feeds the products that read the whole slice). Per chunk: U = U' - W S^T (16 positions
//     each), then the state update S <- Gam_C S + (diag(exp(gamma_C - gamma)) U)^T K on their columns;
//   warps 4-7 form Gam Q S^T beside W S^T, then M U and the Y store while warps 0-3 update the state, and wait for
//     the updated copy before the next chunk's Q S^T.
// Barrier order a chunk: warps 0-3 wait BAR_U (M U of the chunk before is done, so U and that chunk's buffer are
// free: the next chunk's copies are issued), W S^T, write U, BAR_A, update, arrive BAR_S, sync BAR_S0; warps 4-7 wait
// BAR_S (the state copy of this chunk is complete), Q S^T, BAR_A, M U, store Y, arrive BAR_U. A wait that gave up in
// any thread is ORed at BAR_A and every warp leaves the loop there.
template <typename T>
__global__ void __launch_bounds__(SCAN_THREADS, 1) scan_kernel(const __grid_constant__ CUtensorMap qmap,
                                                                const __grid_constant__ CUtensorMap kmap,
                                                                const Params p) {
  const int blk = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int hk = h / (p.Hv / p.Hk);
  const int dv0 = blk * DVB;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int r = lane >> 2, cq = lane & 3;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint32_t* St = reinterpret_cast<uint32_t*>(sm + ScanSmem::ST);
  uint32_t* Ub = reinterpret_cast<uint32_t*>(sm + ScanSmem::UB);
  uint32_t* Ud = reinterpret_cast<uint32_t*>(sm + ScanSmem::UD);
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + ScanSmem::BAR);
  if (tid == 0) {
    prefetch_tensormap(&qmap);
    prefetch_tensormap(&kmap);
    mbar_init(&full[0], 1);
    mbar_init(&full[1], 1);
    fence_barrier_init();
  }

  // warps 0-3: the state tile of this warp, rows mt * 16 + r (+ 8), columns 32 warp + 8 n + 2 cq (+ 1)
  const bool chain = warp < 4;
  float sreg[2][4][4];
  const float* sin = p.s_in + (int64_t(b) * p.Hv + h) * DV * DK;
  if (chain) {
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int n = 0; n < 4; ++n)
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const int i = mt * 16 + r + 8 * hh, d = warp * 32 + n * 8 + 2 * cq;
          const float2 v = *reinterpret_cast<const float2*>(sin + int64_t(dv0 + i) * DK + d);
          sreg[mt][n][2 * hh] = v.x;
          sreg[mt][n][2 * hh + 1] = v.y;
          St[i * WP + d] = tf32(v.x);
          St[i * WP + d + 1] = tf32(v.y);
        }
  }
  __syncthreads();  // barriers initialised, the state copy written
  if (p.nchunks > 0 && tid == 0) scan_prefetch(p, &qmap, &kmap, sm, &full[0], b, h, hk, 0, blk);

  bool ok = true;
  int issued = p.nchunks > 0 ? 1 : 0;  // chunks whose copies were issued (thread 0)
  const int m0 = (warp & 3) * 16;
  for (int c = 0; c < p.nchunks; ++c) {
    const bool last = c + 1 == p.nchunks;
    uint8_t* buf = sm + (c & 1) * ScanSmem::BUF;
    const uint32_t* W = reinterpret_cast<const uint32_t*>(buf + ScanSmem::W);
    const float* U = reinterpret_cast<const float*>(buf + ScanSmem::U);
    const uint32_t* M = reinterpret_cast<const uint32_t*>(buf + ScanSmem::M);
    const uint8_t* Q = buf + ScanSmem::Q;
    const uint8_t* K = buf + ScanSmem::K;
    const float* G = reinterpret_cast<const float*>(buf + ScanSmem::G);
    float acc[4][4];
#pragma unroll
    for (int n = 0; n < 4; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[n][e] = 0.f;
    if (chain) {
      if (c > 0) nbar_sync(BAR_U, SCAN_THREADS);  // M U of chunk c - 1 done: U and that chunk's buffer are free
      if (!last && tid == 0) {
        scan_prefetch(p, &qmap, &kmap, sm + ((c + 1) & 1) * ScanSmem::BUF, &full[(c + 1) & 1], b, h, hk, c + 1, blk);
        issued = c + 2;
      }
      ok = mbar_wait(&full[c & 1], (c >> 1) & 1, 71);
      // (1) acc = W S^T: rows m0 .. m0 + 15, all 32 value columns
#pragma unroll 4
      for (int k0 = 0; k0 < DK; k0 += 8) {
        uint32_t a[4], b01[4], b23[4];
        frag_a(smem_u32(W), WP, m0, k0, lane, a);
        frag_b2(smem_u32(St), WP, 0, k0, lane, b01);
        frag_b2(smem_u32(St), WP, 16, k0, lane, b23);
        mma_tf32(acc[0], a[0], a[1], a[2], a[3], b01[0], b01[1]);
        mma_tf32(acc[1], a[0], a[1], a[2], a[3], b01[2], b01[3]);
        mma_tf32(acc[2], a[0], a[1], a[2], a[3], b23[0], b23[1]);
        mma_tf32(acc[3], a[0], a[1], a[2], a[3], b23[2], b23[3]);
      }
      // U = U' - W S^T, stored rounded for the products that read it, plain and scaled by exp(gamma_C - gamma_t)
      const float gl = G[C - 1];
      const float dl = __expf(gl - G[m0 + r]), dh = __expf(gl - G[m0 + r + 8]);
#pragma unroll
      for (int n = 0; n < 4; ++n)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int t = m0 + r + 8 * (e >> 1), col = n * 8 + 2 * cq + (e & 1);
          const float u = U[t * UP + col] - acc[n][e];
          Ub[col * UQ + t] = tf32(u);
          Ud[col * UQ + t] = tf32((e >> 1 ? dh : dl) * u);
        }
    } else {
      if (c > 0) nbar_sync(BAR_S, SCAN_THREADS);  // the state copy of chunk c is complete
      ok = mbar_wait(&full[c & 1], (c >> 1) & 1, 71);
      // (1) acc = Gam Q S^T: rows m0 .. m0 + 15, all 32 value columns
#pragma unroll 4
      for (int k0 = 0; k0 < DK; k0 += 8) {
        const uint32_t a0 = qk_tf32<T>(Q, m0 + r, k0 + cq), a1 = qk_tf32<T>(Q, m0 + r + 8, k0 + cq);
        const uint32_t a2 = qk_tf32<T>(Q, m0 + r, k0 + cq + 4), a3 = qk_tf32<T>(Q, m0 + r + 8, k0 + cq + 4);
        uint32_t b01[4], b23[4];
        frag_b2(smem_u32(St), WP, 0, k0, lane, b01);
        frag_b2(smem_u32(St), WP, 16, k0, lane, b23);
        mma_tf32(acc[0], a0, a1, a2, a3, b01[0], b01[1]);
        mma_tf32(acc[1], a0, a1, a2, a3, b01[2], b01[3]);
        mma_tf32(acc[2], a0, a1, a2, a3, b23[0], b23[1]);
        mma_tf32(acc[3], a0, a1, a2, a3, b23[2], b23[3]);
      }
      const float gl = G[C + m0 + r], gh = G[C + m0 + r + 8];
#pragma unroll
      for (int n = 0; n < 4; ++n) {
        acc[n][0] *= gl;
        acc[n][1] *= gl;
        acc[n][2] *= gh;
        acc[n][3] *= gh;
      }
    }
    if (nbar_sync_or(BAR_A, SCAN_THREADS, !ok)) {  // U complete; every read of the state copy done
      ok = false;
      break;
    }
    if (chain) {
      // (2) S <- Gam_C S + (diag(dec) U)^T K on this warp's 32 key columns (all 32 value rows)
      const float gc = G[C + C - 1];
#pragma unroll
      for (int mt = 0; mt < 2; ++mt)
#pragma unroll
        for (int n = 0; n < 4; ++n)
#pragma unroll
          for (int e = 0; e < 4; ++e) sreg[mt][n][e] *= gc;
#pragma unroll 2
      for (int k0 = 0; k0 < C; k0 += 8) {
        uint32_t a[2][4];
#pragma unroll
        for (int mt = 0; mt < 2; ++mt) frag_a(smem_u32(Ud), UQ, mt * 16, k0, lane, a[mt]);
#pragma unroll
        for (int n = 0; n < 4; ++n) {
          const int col = warp * 32 + n * 8 + r;
          const uint32_t b0 = qk_tf32<T>(K, k0 + cq, col), b1 = qk_tf32<T>(K, k0 + cq + 4, col);
#pragma unroll
          for (int mt = 0; mt < 2; ++mt) mma_tf32(sreg[mt][n], a[mt][0], a[mt][1], a[mt][2], a[mt][3], b0, b1);
        }
      }
#pragma unroll
      for (int mt = 0; mt < 2; ++mt)
#pragma unroll
        for (int n = 0; n < 4; ++n)
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            const int i = mt * 16 + r + 8 * hh, d = warp * 32 + n * 8 + 2 * cq;
            St[i * WP + d] = tf32(sreg[mt][n][2 * hh]);
            St[i * WP + d + 1] = tf32(sreg[mt][n][2 * hh + 1]);
          }
      if (!last) {
        nbar_arrive(BAR_S, SCAN_THREADS);
        nbar_sync(BAR_S0, 128);
      }
    } else {
      // (3) Y = Gam Q S^T + M U (M lower triangular: k < m0 + 16), stored
      for (int k0 = 0; k0 < m0 + 16; k0 += 8) {
        uint32_t a[4], b01[4], b23[4];
        frag_a(smem_u32(M), AP, m0, k0, lane, a);
        frag_b2(smem_u32(Ub), UQ, 0, k0, lane, b01);
        frag_b2(smem_u32(Ub), UQ, 16, k0, lane, b23);
        mma_tf32(acc[0], a[0], a[1], a[2], a[3], b01[0], b01[1]);
        mma_tf32(acc[1], a[0], a[1], a[2], a[3], b01[2], b01[3]);
        mma_tf32(acc[2], a[0], a[1], a[2], a[3], b23[0], b23[1]);
        mma_tf32(acc[3], a[0], a[1], a[2], a[3], b23[2], b23[3]);
      }
      if (!last) nbar_arrive(BAR_U, SCAN_THREADS);  // done with U and with this chunk's buffer
      T* yg = static_cast<T*>(p.y);
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int t = m0 + r + 8 * hh, pos = c * C + t;
        if (pos < p.T) {
          T* yr = yg + ((int64_t(b) * p.T + pos) * p.Hv + h) * DV + dv0;
#pragma unroll
          for (int n = 0; n < 4; ++n) {
            yr[n * 8 + 2 * cq] = from_f<T>(acc[n][2 * hh]);
            yr[n * 8 + 2 * cq + 1] = from_f<T>(acc[n][2 * hh + 1]);
          }
        }
      }
    }
  }
  if (!ok) {  // a wait gave up (status word set): let the copies still in flight land (bounded), write nothing
    if (tid == 0)
      for (int c2 = max(0, issued - 2); c2 < issued; ++c2) mbar_wait(&full[c2 & 1], (c2 >> 1) & 1, 72);
    return;
  }
  if (chain) {
    float* sout = p.s_out + (int64_t(b) * p.Hv + h) * DV * DK;
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int n = 0; n < 4; ++n)
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const int i = mt * 16 + r + 8 * hh, d = warp * 32 + n * 8 + 2 * cq;
          *reinterpret_cast<float2*>(sout + int64_t(dv0 + i) * DK + d) =
              make_float2(sreg[mt][n][2 * hh], sreg[mt][n][2 * hh + 1]);
        }
  }
}

}  // namespace gdnchunk
}  // namespace lb2
