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
//        chunk's workspace tiles prefetched with cp.async while the previous chunk computes; U, Y and the state
//        update on TF32 mma.sync with fp32 accumulation. W and M are stored already rounded to TF32 by prep.
#pragma once

#include "common.cuh"

namespace lb2 {
namespace gdnchunk {

constexpr int C = 64;
constexpr int DK = 128;
constexpr int DV = 128;
constexpr int DVB = 32;   // value rows a scan CTA owns
constexpr int UNIT = C * DK + C * DV + C * C + 2 * C;  // workspace floats a (batch, head, chunk)
constexpr int KP = 136;   // bf16 row stride of K / Q tiles (conflict-free ldmatrix and scalar reads)
constexpr int AP = 68;    // fp32 row stride of A / T / M tiles
constexpr int RP = 136;   // fp32 row stride of 128-wide fp32 tiles (B operands)
constexpr int WP = 132;   // fp32 row stride of W / S tiles (A operands and S^T reads)
constexpr int UP = 36;    // fp32 row stride of 32-wide U tiles

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

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
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
  static constexpr int XS = AF + C * AP * 4;                // f32 [32][33] inversion scratch
  static constexpr int GAM = XS + 32 * 33 * 4;              // f32 [C] gamma, [C] Gam, [C] beta
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

  // 1. gates: gamma = inclusive prefix sum of log g over the chunk (positions past T: g = 1, beta = 0)
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
  // 2. K, Q and V tiles (16-bit, vector loads), zero past T
  {
    const T* kg = static_cast<const T*>(p.k);
    const T* qg = static_cast<const T*>(p.q);
    const T* vg = static_cast<const T*>(p.v);
#pragma unroll 4
    for (int e = tid; e < C * (DK / 8); e += 128) {
      const int r = e / (DK / 8), u = e % (DK / 8);
      const int pos = t0 + r;
      uint4 kv = make_uint4(0, 0, 0, 0), qv = make_uint4(0, 0, 0, 0), vv = make_uint4(0, 0, 0, 0);
      if (pos < p.T) {
        const int64_t off = ((int64_t(b) * p.T + pos) * p.Hk + hk) * DK + u * 8;
        kv = *reinterpret_cast<const uint4*>(kg + off);
        qv = *reinterpret_cast<const uint4*>(qg + off);
        vv = *reinterpret_cast<const uint4*>(vg + ((int64_t(b) * p.T + pos) * p.Hv + h) * DV + u * 8);
      }
      *reinterpret_cast<uint4*>(Kb + r * KP + u * 8) = kv;
      *reinterpret_cast<uint4*>(Qb + r * KP + u * 8) = qv;
      *reinterpret_cast<uint4*>(Vb + r * KP + u * 8) = vv;
    }
  }
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
    float* Mg = unit_ptr(p, b, h, c) + C * DK + C * DV;
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int t = warp * 16 + (lane >> 2) + 8 * (e >> 1);
        const int j = n * 8 + 2 * (lane & 3) + (e & 1);
        const float dec = j <= t ? __expf(gam[t] - gam[j]) : 0.f;
        Af[t * AP + j] = j < t ? bet[t] * dec * kk[n][e] : 0.f;
        Mg[t * C + j] = __uint_as_float(tf32(dec * qk[n][e]));  // an MMA operand of the scan: rounded once here
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
  // level 1: T[hi][lo] = -T[hi][hi] A[hi][lo] T[lo][lo] for block pairs (0, 1) and (2, 3)
  {
    const int pr = tid >> 6, t = tid & 63;  // 64 threads a pair, 4 outputs each
    const int lo = 32 * pr, hi = lo + 16;
    float* X = Xs + pr * 16 * 17;
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int o = t + 64 * u, r = o >> 4, cc = o & 15;
      float s = 0.f;
#pragma unroll
      for (int j = 0; j < 16; ++j) s = fmaf(Af[(hi + r) * AP + lo + j], Af[(lo + j) * AP + lo + cc], s);
      X[r * 17 + cc] = s;
    }
    __syncthreads();
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int o = t + 64 * u, r = o >> 4, cc = o & 15;
      float s = 0.f;
#pragma unroll
      for (int j = 0; j < 16; ++j) s = fmaf(Af[(hi + r) * AP + hi + j], X[j * 17 + cc], s);
      Af[(hi + r) * AP + lo + cc] = -s;
    }
  }
  __syncthreads();
  // level 2: T[32:64][0:32] = -T[32:64][32:64] A[32:64][0:32] T[0:32][0:32]
  {
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int o = tid + 128 * u, r = o >> 5, cc = o & 31;
      float s = 0.f;
#pragma unroll 8
      for (int j = 0; j < 32; ++j) s = fmaf(Af[(32 + r) * AP + j], Af[j * AP + cc], s);
      Xs[r * 33 + cc] = s;
    }
    __syncthreads();
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int o = tid + 128 * u, r = o >> 5, cc = o & 31;
      float s = 0.f;
#pragma unroll 8
      for (int j = 0; j < 32; ++j) s = fmaf(Af[(32 + r) * AP + 32 + j], Xs[j * 33 + cc], s);
      Af[(32 + r) * AP + cc] = -s;
    }
  }
  __syncthreads();
  // 5. W = T diag(beta Gam) K and U' = T diag(beta) V (TF32 mma), rows 16 w .. 16 w + 15; the B fragments are
  // formed from the 16-bit tiles on the fly. T is lower triangular, so only k < 16 (w + 1) contributes.
  {
    float* Wg = unit_ptr(p, b, h, c);
    float* Ug = Wg + C * DK;
    const int r = lane >> 2, cq = lane & 3, m0 = warp * 16;
#pragma unroll 1
    for (int which = 0; which < 2; ++which) {
      const T* R = which ? Vb : Kb;
      float* G = which ? Ug : Wg;
#pragma unroll 1
      for (int nh = 0; nh < 2; ++nh) {  // two halves of 64 columns, to bound registers
        float acc[8][4];
#pragma unroll
        for (int n = 0; n < 8; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.f;
        for (int k0 = 0; k0 < 16 * (warp + 1); k0 += 8) {
          const uint32_t a0 = tf32(Af[(m0 + r) * AP + k0 + cq]), a1 = tf32(Af[(m0 + r + 8) * AP + k0 + cq]);
          const uint32_t a2 = tf32(Af[(m0 + r) * AP + k0 + cq + 4]), a3 = tf32(Af[(m0 + r + 8) * AP + k0 + cq + 4]);
          const float s0 = which ? bet[k0 + cq] : bet[k0 + cq] * Gam[k0 + cq];
          const float s1 = which ? bet[k0 + cq + 4] : bet[k0 + cq + 4] * Gam[k0 + cq + 4];
#pragma unroll
          for (int n = 0; n < 8; ++n) {
            const int n0 = nh * 64 + n * 8;
            mma_tf32(acc[n], a0, a1, a2, a3, tf32(s0 * to_f<T>(R[(k0 + cq) * KP + n0 + r])),
                     tf32(s1 * to_f<T>(R[(k0 + cq + 4) * KP + n0 + r])));
          }
        }
        if (!which)  // W is an MMA operand of the scan: stored rounded to TF32; U' stays fp32
#pragma unroll
          for (int n = 0; n < 8; ++n)
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[n][e] = __uint_as_float(tf32(acc[n][e]));
#pragma unroll
        for (int n = 0; n < 8; ++n) {
          const int col = nh * 64 + n * 8 + 2 * cq;
          *reinterpret_cast<float2*>(&G[(m0 + r) * DK + col]) = make_float2(acc[n][0], acc[n][1]);
          *reinterpret_cast<float2*>(&G[(m0 + r + 8) * DK + col]) = make_float2(acc[n][2], acc[n][3]);
        }
      }
    }
  }
  // 7. gamma and Gam for the scan
  if (tid < C) {
    float* gg = unit_ptr(p, b, h, c) + C * DK + C * DV + C * C;
    gg[tid] = gam[tid];
    gg[C + tid] = Gam[tid];
  }
}

// ------------------------------------------------------------------------------------------------ scan

constexpr int SCAN_THREADS = 256;  // warps 0-3: U = U' - W S^T; warps 4-7: Q S^T and M U; all 8: the state update
constexpr int UQ = 40;             // u32 row stride of the U tiles read as MMA operands (conflict-free fragments)

struct ScanSmem {
  // one prefetch buffer
  static constexpr int W = 0;                         // tf32 [C][WP]
  static constexpr int U = W + C * WP * 4;            // f32 [C][UP]   U' columns of this block
  static constexpr int M = U + C * UP * 4;            // tf32 [C][AP]
  static constexpr int Q = M + C * AP * 4;            // 16-bit [C][KP]
  static constexpr int K = Q + C * KP * 2;            // 16-bit [C][KP]
  static constexpr int G = K + C * KP * 2;            // f32 [C] gamma, [C] Gam
  static constexpr int BUF = G + 2 * C * 4;
  // persistent
  static constexpr int ST = 2 * BUF;                  // tf32 [DVB][WP] the state slice, rounded for the MMAs
  static constexpr int UB = ST + DVB * WP * 4;        // tf32 [C][UQ] this chunk's U
  static constexpr int UD = UB + C * UQ * 4;          // tf32 [C][UQ] diag(exp(gamma_C - gamma)) U
  static constexpr int BYTES = UD + C * UQ * 4;
};
static_assert(ScanSmem::BYTES <= 232448, "scan shared memory");

// A 16-bit value's exact TF32 bit pattern (bf16 and fp16 mantissas fit TF32's 10 bits).
template <typename T>
__device__ __forceinline__ uint32_t tf32_of(T x) {
  return __float_as_uint(to_f<T>(x));
}

template <typename T>
__device__ __forceinline__ void scan_prefetch(const Params& p, uint8_t* buf, int b, int h, int hk, int c, int dv0,
                                              int tid) {
  const float* u = unit_ptr(p, b, h, c);
  float* W = reinterpret_cast<float*>(buf + ScanSmem::W);
  float* U = reinterpret_cast<float*>(buf + ScanSmem::U);
  float* M = reinterpret_cast<float*>(buf + ScanSmem::M);
  T* Q = reinterpret_cast<T*>(buf + ScanSmem::Q);
  T* K = reinterpret_cast<T*>(buf + ScanSmem::K);
  float* G = reinterpret_cast<float*>(buf + ScanSmem::G);
#pragma unroll
  for (int e = tid; e < C * (DK / 4); e += SCAN_THREADS) {  // W: 64 rows x 32 pieces of 16 B
    const int r = e >> 5, q = e & 31;
    cp_async16(W + r * WP + q * 4, u + r * DK + q * 4);
  }
#pragma unroll
  for (int e = tid; e < C * (DVB / 4); e += SCAN_THREADS) {  // U' columns dv0 .. dv0 + 31
    const int r = e >> 3, q = e & 7;
    cp_async16(U + r * UP + q * 4, u + C * DK + r * DV + dv0 + q * 4);
  }
#pragma unroll
  for (int e = tid; e < C * (C / 4); e += SCAN_THREADS) {  // M
    const int r = e >> 4, q = e & 15;
    cp_async16(M + r * AP + q * 4, u + C * DK + C * DV + r * C + q * 4);
  }
  if (tid < 2 * C / 4) cp_async16(G + tid * 4, u + C * DK + C * DV + C * C + tid * 4);
  const T* qg = static_cast<const T*>(p.q);
  const T* kg = static_cast<const T*>(p.k);
#pragma unroll
  for (int e = tid; e < C * (DK / 8); e += SCAN_THREADS) {  // Q, K rows (zero past T)
    const int r = e >> 4, q = e & 15;
    const int pos = c * C + r;
    if (pos < p.T) {
      const int64_t off = ((int64_t(b) * p.T + pos) * p.Hk + hk) * DK + q * 8;
      cp_async16(Q + r * KP + q * 8, qg + off);
      cp_async16(K + r * KP + q * 8, kg + off);
    } else {
      *reinterpret_cast<uint4*>(Q + r * KP + q * 8) = make_uint4(0, 0, 0, 0);
      *reinterpret_cast<uint4*>(K + r * KP + q * 8) = make_uint4(0, 0, 0, 0);
    }
  }
}

// One CTA: value rows dv0 .. dv0 + 31 of one (batch, v-head), all chunks in order. The fp32 state slice lives in
// registers, warp w owning key columns 16 w .. 16 w + 15 of all 32 rows; a TF32 copy in shared memory feeds the
// products that read the whole slice. Per chunk: (1) warps 0-3 form U = U' - W S^T (16 positions each) while warps
// 4-7 form Gam Q S^T; (2) all warps update their state columns with U^T diag(exp(gamma_C - gamma)) K while warps
// 4-7 add M U to Y and store it.
template <typename T>
__global__ void __launch_bounds__(SCAN_THREADS, 1) scan_kernel(const Params p) {
  const int blk = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int hk = h / (p.Hv / p.Hk);
  const int dv0 = blk * DVB;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int r = lane >> 2, cq = lane & 3;
  extern __shared__ __align__(16) uint8_t sm[];
  uint32_t* St = reinterpret_cast<uint32_t*>(sm + ScanSmem::ST);
  uint32_t* Ub = reinterpret_cast<uint32_t*>(sm + ScanSmem::UB);
  uint32_t* Ud = reinterpret_cast<uint32_t*>(sm + ScanSmem::UD);

  // the state tile of this warp: rows mt * 16 + r (+ 8), columns 16 warp + 8 n + 2 cq (+ 1)
  float sreg[2][2][4];
  const float* sin = p.s_in + (int64_t(b) * p.Hv + h) * DV * DK;
#pragma unroll
  for (int mt = 0; mt < 2; ++mt)
#pragma unroll
    for (int n = 0; n < 2; ++n)
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int i = mt * 16 + r + 8 * hh, d = warp * 16 + n * 8 + 2 * cq;
        const float2 v = *reinterpret_cast<const float2*>(sin + int64_t(dv0 + i) * DK + d);
        sreg[mt][n][2 * hh] = v.x;
        sreg[mt][n][2 * hh + 1] = v.y;
        St[i * WP + d] = tf32(v.x);
        St[i * WP + d + 1] = tf32(v.y);
      }
  scan_prefetch<T>(p, sm, b, h, hk, 0, dv0, tid);
  cp_async_commit();

  for (int c = 0; c < p.nchunks; ++c) {
    uint8_t* buf = sm + (c & 1) * ScanSmem::BUF;
    if (c + 1 < p.nchunks) scan_prefetch<T>(p, sm + ((c + 1) & 1) * ScanSmem::BUF, b, h, hk, c + 1, dv0, tid);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    const uint32_t* W = reinterpret_cast<const uint32_t*>(buf + ScanSmem::W);
    const float* U = reinterpret_cast<const float*>(buf + ScanSmem::U);
    const uint32_t* M = reinterpret_cast<const uint32_t*>(buf + ScanSmem::M);
    const T* Q = reinterpret_cast<const T*>(buf + ScanSmem::Q);
    const T* K = reinterpret_cast<const T*>(buf + ScanSmem::K);
    const float* G = reinterpret_cast<const float*>(buf + ScanSmem::G);
    const int m0 = (warp & 3) * 16;

    // (1) warps 0-3: acc = W S^T; warps 4-7: acc = Q S^T. Rows m0 .. m0 + 15, all 32 value columns.
    float acc[4][4];
#pragma unroll
    for (int n = 0; n < 4; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[n][e] = 0.f;
    if (warp < 4) {
#pragma unroll 4
      for (int k0 = 0; k0 < DK; k0 += 8) {
        const uint32_t a0 = W[(m0 + r) * WP + k0 + cq], a1 = W[(m0 + r + 8) * WP + k0 + cq];
        const uint32_t a2 = W[(m0 + r) * WP + k0 + cq + 4], a3 = W[(m0 + r + 8) * WP + k0 + cq + 4];
#pragma unroll
        for (int n = 0; n < 4; ++n)
          mma_tf32(acc[n], a0, a1, a2, a3, St[(n * 8 + r) * WP + k0 + cq], St[(n * 8 + r) * WP + k0 + cq + 4]);
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
          Ub[t * UQ + col] = tf32(u);
          Ud[t * UQ + col] = tf32((e >> 1 ? dh : dl) * u);
        }
    } else {
#pragma unroll 4
      for (int k0 = 0; k0 < DK; k0 += 8) {
        const uint32_t a0 = tf32_of(Q[(m0 + r) * KP + k0 + cq]), a1 = tf32_of(Q[(m0 + r + 8) * KP + k0 + cq]);
        const uint32_t a2 = tf32_of(Q[(m0 + r) * KP + k0 + cq + 4]);
        const uint32_t a3 = tf32_of(Q[(m0 + r + 8) * KP + k0 + cq + 4]);
#pragma unroll
        for (int n = 0; n < 4; ++n)
          mma_tf32(acc[n], a0, a1, a2, a3, St[(n * 8 + r) * WP + k0 + cq], St[(n * 8 + r) * WP + k0 + cq + 4]);
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
    __syncthreads();  // U complete; every read of the state copy done

    // (2) S <- Gam_C S + (diag(dec) U)^T K on this warp's 16 key columns (all 32 value rows)
    {
      const float gc = G[C + C - 1];
#pragma unroll
      for (int mt = 0; mt < 2; ++mt)
#pragma unroll
        for (int n = 0; n < 2; ++n)
#pragma unroll
          for (int e = 0; e < 4; ++e) sreg[mt][n][e] *= gc;
#pragma unroll 2
      for (int k0 = 0; k0 < C; k0 += 8) {
        uint32_t a[2][4];
#pragma unroll
        for (int mt = 0; mt < 2; ++mt) {
          a[mt][0] = Ud[(k0 + cq) * UQ + mt * 16 + r];
          a[mt][1] = Ud[(k0 + cq) * UQ + mt * 16 + r + 8];
          a[mt][2] = Ud[(k0 + cq + 4) * UQ + mt * 16 + r];
          a[mt][3] = Ud[(k0 + cq + 4) * UQ + mt * 16 + r + 8];
        }
#pragma unroll
        for (int n = 0; n < 2; ++n) {
          const int col = warp * 16 + n * 8 + r;
          const uint32_t b0 = tf32_of(K[(k0 + cq) * KP + col]), b1 = tf32_of(K[(k0 + cq + 4) * KP + col]);
#pragma unroll
          for (int mt = 0; mt < 2; ++mt) mma_tf32(sreg[mt][n], a[mt][0], a[mt][1], a[mt][2], a[mt][3], b0, b1);
        }
      }
#pragma unroll
      for (int mt = 0; mt < 2; ++mt)
#pragma unroll
        for (int n = 0; n < 2; ++n)
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            const int i = mt * 16 + r + 8 * hh, d = warp * 16 + n * 8 + 2 * cq;
            St[i * WP + d] = tf32(sreg[mt][n][2 * hh]);
            St[i * WP + d + 1] = tf32(sreg[mt][n][2 * hh + 1]);
          }
    }
    // (3) warps 4-7: Y = Gam Q S^T + M U (M lower triangular: k < m0 + 16), stored
    if (warp >= 4) {
      for (int k0 = 0; k0 < m0 + 16; k0 += 8) {
        const uint32_t a0 = M[(m0 + r) * AP + k0 + cq], a1 = M[(m0 + r + 8) * AP + k0 + cq];
        const uint32_t a2 = M[(m0 + r) * AP + k0 + cq + 4], a3 = M[(m0 + r + 8) * AP + k0 + cq + 4];
#pragma unroll
        for (int n = 0; n < 4; ++n)
          mma_tf32(acc[n], a0, a1, a2, a3, Ub[(k0 + cq) * UQ + n * 8 + r], Ub[(k0 + cq + 4) * UQ + n * 8 + r]);
      }
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
    __syncthreads();  // the state copy complete and this chunk's buffer free before the next prefetch
  }
  float* sout = p.s_out + (int64_t(b) * p.Hv + h) * DV * DK;
#pragma unroll
  for (int mt = 0; mt < 2; ++mt)
#pragma unroll
    for (int n = 0; n < 2; ++n)
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int i = mt * 16 + r + 8 * hh, d = warp * 16 + n * 8 + 2 * cq;
        *reinterpret_cast<float2*>(sout + int64_t(dv0 + i) * DK + d) =
            make_float2(sreg[mt][n][2 * hh], sreg[mt][n][2 * hh + 1]);
      }
}

}  // namespace gdnchunk
}  // namespace lb2
