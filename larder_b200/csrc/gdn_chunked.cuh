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
// Two launches, every product on the tcgen05 tensor cores (kind::f16, fp32 accumulators in TMEM), fp32 values that
// feed a product passed as a 16-bit hi / lo pair (hi = round(x), lo = round(x - hi): about 16 mantissa bits):
//   prep (grid: chunks x v-heads x batch, independent): K K^T and Q K^T, the decay / beta weighting, T by blocked
//        inversion in fp32 on the CUDA cores, then W and U'; writes W, U', M, gamma, Gam to the workspace in the
//        scan's shared-memory layout.
//   scan (grid: Dv / 32 value columns x v-heads x batch): the state slice in fp32 registers, chunks in order, each
//        chunk's workspace pieces and Q / K tiles prefetched a chunk ahead; U, Y and the state update per chunk.
#pragma once

#include <type_traits>

#include "attn_prefill.cuh"
#include "common.cuh"

namespace lb2 {
namespace gdnchunk {

constexpr int C = 64;
constexpr int DK = 128;
constexpr int DV = 128;
constexpr int DVB = 32;   // value rows a scan CTA owns
constexpr int AP = 68;    // fp32 row stride of prep's A / T tiles
constexpr int UP = 36;    // fp32 row stride of the U' slices (32 value columns)
// Workspace of one (batch, head, chunk), in bytes, laid out as the scan's shared-memory operands so that a chunk
// arrives by four bulk copies. W and M are stored as 16-bit hi / lo pairs (hi = round(x), lo = round(x - hi): their
// sum carries about 16 mantissa bits) in the tensor cores' 128-byte-swizzled K-major form: row r of a 64-column
// block at r * 128 bytes, its 16-byte piece j at piece j ^ (r % 8).
//   W_hi, W_lo [64 positions][128 keys]: two column blocks of 8 KB each;  M_hi, M_lo [64][64]: 8 KB each;
//   gamma, Gam [64] fp32;  U' as DV / DVB slices [64][UP] fp32 of 32 value columns each.
constexpr int WS_WHI = 0;
constexpr int WS_WLO = WS_WHI + 2 * C * 128;
constexpr int WS_MHI = WS_WLO + 2 * C * 128;
constexpr int WS_MLO = WS_MHI + C * 128;
constexpr int WS_G = WS_MLO + C * 128;
constexpr int WS_U = WS_G + 2 * C * 4;
constexpr int USLICE = C * UP * 4;
constexpr int UNIT_BYTES = WS_U + (DV / DVB) * USLICE;
static_assert(WS_G % 16 == 0 && WS_U % 16 == 0 && UNIT_BYTES % 16 == 0, "16-byte aligned workspace pieces");

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

// Workspace of one (batch, head, chunk).
__device__ __forceinline__ uint8_t* unit_ptr(const Params& p, int b, int h, int c) {
  return reinterpret_cast<uint8_t*>(p.ws) + ((int64_t(b) * p.Hv + h) * p.nchunks + c) * int64_t(UNIT_BYTES);
}

// ------------------------------------------------------------------------------------------------ prep
//
// One CTA of 4 warps a (chunk, v-head), its products on tcgen05 (kind::f16, accumulators in TMEM, M = 64 MMAs: an
// accumulator's row m sits in TMEM lane m % 16 + 32 (m / 16) from the lane the MMA names, so two M = 64 products
// written at lane 0 and lane 16 share 32 x 4 lanes, and warp w's lanes 0-15 read rows 16 w .. of the first and its
// lanes 16-31 rows 16 w .. of the second):
//   P_A  K K^T (lane 0) and Q K^T (lane 16), N = 64, from the K / Q tiles as TMA lands them;
//   A = diag(beta) (decay x K K^T) strictly below the diagonal, M = decay x Q K^T on and below it (M as a hi / lo pair
//   straight to the workspace); T = (I + A)^{-1} in fp32 on the CUDA cores (16 x 16 diagonal blocks by substitution,
//   then the 2 x 2 block formula at 32 and 64);
//   P_W  W = (T diag(beta Gam)) K (lane 0), then U' = (T diag(beta)) V (lane 16), N = 128: A = the scaled T as a hi /
//   lo pair, B = the K / V tile read MN-major (positions are the products' K).

constexpr int PREP_TMEM_COLS = 128;
constexpr int XP = 36;  // row stride of the inversion scratch (conflict-free float4 rows)

// Regions reused as the steps go, so that four CTAs fit an SM (with 128 TMEM columns each, the SM's 512): the Q tile
// is dead once P_A has committed, and its region then holds A and T (fp32, 1 KB more than the tile), then T diag(beta
// Gam) once every thread has its row of T in registers; the K tile is dead once W's products have committed, and its
// region then holds T diag(beta), kept in registers until then.
struct PrepSmem {
  static constexpr int K0 = 0;                  // K tile: two TMA boxes [64 positions][64 keys]; later T diag(beta)
  static constexpr int V0 = K0 + 2 * C * 128;   // V tile, the same (64 value columns a box)
  static constexpr int Q0 = V0 + 2 * C * 128;   // Q tile; later A / T, then T diag(beta Gam)
  static constexpr int AF = Q0;                 // f32 [C][AP]: A, then T
  static constexpr int TBG = Q0;                // hi, lo: [64][64] 16-bit, 8 KB each
  static constexpr int TB = K0;
  static constexpr int XS = AF + C * AP * 4;    // f32 [32][XP], the inversion scratch
  static constexpr int GAM = XS + 32 * XP * 4;  // f32 [C] gamma, [C] Gam, [C] beta
  static constexpr int BAR = GAM + 3 * C * 4;   // 2 mbarriers: loads landed, MMAs done
  static constexpr int SLOT = BAR + 16;         // TMEM base address
  static constexpr int BYTES = SLOT + 16 + 1024;
};
static_assert(PrepSmem::Q0 % 1024 == 0 && PrepSmem::XS % 16 == 0 && PrepSmem::BYTES + 1024 <= 228 * 1024 / 4,
              "four prep CTAs an SM");


// Writes 64 values of row `row` of a 16-bit K-major operand pair (128-byte swizzle) as hi / lo: eight 16-byte pieces.
// The 16-bit hi / lo pairs of two values (hi = round(x), lo = round(x - hi)), packed two a word, with one paired
// conversion for the two hi halves and one for the two lo halves: the single-value conversions go through a narrow
// pipe and were the largest cost of the scan's epilogues.
template <typename T>
__device__ __forceinline__ void split2(float a, float b, uint32_t& h, uint32_t& l);
template <>
__device__ __forceinline__ void split2<__nv_bfloat16>(float a, float b, uint32_t& h, uint32_t& l) {
  h = pack2<__nv_bfloat16>(a, b);
  l = pack2<__nv_bfloat16>(a - __uint_as_float(h << 16), b - __uint_as_float(h & 0xffff0000u));
}
template <>
__device__ __forceinline__ void split2<__half>(float a, float b, uint32_t& h, uint32_t& l) {
  h = pack2<__half>(a, b);
  const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&h));
  l = pack2<__half>(a - f.x, b - f.y);
}

template <typename T>
__device__ __forceinline__ void put_row_pair(uint8_t* hi, uint8_t* lo, int row, const float* x) {
#pragma unroll
  for (int j8 = 0; j8 < 8; ++j8) {
    uint32_t h[4], l[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      split2<T>(x[8 * j8 + 2 * e], x[8 * j8 + 2 * e + 1], h[e], l[e]);
    }
    const int off = row * 128 + (((j8 ^ row) & 7) << 4);
    *reinterpret_cast<uint4*>(hi + off) = make_uint4(h[0], h[1], h[2], h[3]);
    *reinterpret_cast<uint4*>(lo + off) = make_uint4(l[0], l[1], l[2], l[3]);
  }
}

template <typename T>
__global__ void __launch_bounds__(128, 4) prep_kernel(const __grid_constant__ CUtensorMap qmap,
                                                   const __grid_constant__ CUtensorMap kmap,
                                                   const __grid_constant__ CUtensorMap vmap, const Params p) {
  constexpr uint32_t AB = std::is_same<T, __nv_bfloat16>::value ? 1 : 0;
  constexpr uint32_t IDESC_A = prefill::idesc_f16(AB, 0, 0, 64, 64);   // K K^T, Q K^T
  constexpr uint32_t IDESC_W = prefill::idesc_f16(AB, 0, 1, 64, 128);  // W, U' (B: the K / V tile, MN-major)
  constexpr uint32_t LANE16 = 16u << 16;
  const int c = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int hk = h / (p.Hv / p.Hk);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int t0 = c * C;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* Af = reinterpret_cast<float*>(sm + PrepSmem::AF);
  float* Xs = reinterpret_cast<float*>(sm + PrepSmem::XS);
  float* gam = reinterpret_cast<float*>(sm + PrepSmem::GAM);
  float* Gam = gam + C;
  float* bet = Gam + C;
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + PrepSmem::BAR);
  uint32_t* slot = reinterpret_cast<uint32_t*>(sm + PrepSmem::SLOT);
  uint8_t* unit = unit_ptr(p, b, h, c);

  // The scan (this grid's programmatic dependent) may launch once every prep CTA has started; it waits for this
  // grid's completion before reading anything.
  // 1. the K and Q tiles by TMA (rows past T land as zeros) while the gates are formed; TMEM. (The V tile, read only
  // by U''s products, comes after M has left through its region.)
  if (tid == 0) {
    mbar_init(&bar[0], 1);
    mbar_init(&bar[1], 1);
    fence_barrier_init();
    prefetch_tensormap(&qmap);
    prefetch_tensormap(&kmap);
    prefetch_tensormap(&vmap);
    mbar_arrive_expect_tx(&bar[0], 2 * 2 * C * 128);
#pragma unroll
    for (int db = 0; db < 2; ++db) {
      tma_load_4d(sm + PrepSmem::K0 + db * C * 128, &kmap, db * 64, t0, hk, b, &bar[0]);
      tma_load_4d(sm + PrepSmem::Q0 + db * C * 128, &qmap, db * 64, t0, hk, b, &bar[0]);
    }
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)),
                 "r"(PREP_TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    // gates: gamma = inclusive prefix sum of log g over the chunk (positions past T: g = 1, beta = 0)
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
  prefill::tc_fence_before();
  __syncthreads();
  prefill::tc_fence_after();
  const uint32_t tmem = *slot;
  const uint32_t lq = uint32_t(32 * warp) << 16;
  bool ok = mbar_wait(&bar[0], 0, 75);

  // 2. P_A: K K^T (lane 0) and Q K^T (lane 16), K = 128 keys in two 64-key blocks of four steps
  if (tid == 0 && ok) {
    prefill::tc_fence_after();
    const uint32_t k0 = smem_u32(sm + PrepSmem::K0), q0 = smem_u32(sm + PrepSmem::Q0);
#pragma unroll
    for (int kb = 0; kb < 2; ++kb)
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        const uint64_t ak = prefill::sdesc(k0 + kb * C * 128 + ks * 32, 16, 1024);
        const uint64_t aq = prefill::sdesc(q0 + kb * C * 128 + ks * 32, 16, 1024);
        prefill::umma_ss(tmem, ak, ak, IDESC_A, (kb | ks) ? 1u : 0u);
        prefill::umma_ss(tmem + LANE16, aq, ak, IDESC_A, (kb | ks) ? 1u : 0u);
      }
    prefill::umma_commit(&bar[1]);
  }
  ok = __all_sync(0xffffffffu, ok && mbar_wait(&bar[1], 0, 76));
  // 3. A (lanes 0-15: row t of K K^T) into shared memory; M (lanes 16-31: row t of Q K^T) staged in the V tile's
  // region, then to the workspace by one bulk copy, after which the V tile is loaded there
  {
    const int t = 16 * warp + (lane & 15);
    float x[C];
    if (ok) {
      prefill::tc_fence_after();
      prefill::tmem_ld32(tmem + lq, x);
      prefill::tmem_ld32(tmem + lq + 32, x + 32);
      prefill::tmem_wait_ld();
    } else {
#pragma unroll
      for (int j = 0; j < C; ++j) x[j] = 0.f;
    }
    // the decays exp(gamma_t - gamma_j) (j <= t), shared by the lane pair (l, l ^ 16) that has row t: this lane forms
    // those of the j with parity `half`, the other lane's come by a shuffle; columns past the warp's last row are zero
    const float gt = gam[t];
    const int half = lane >> 4;
    const int ilim = 8 * (warp + 1);  // j <= 16 warp + 15 covers every row of the warp
#pragma unroll
    for (int i = 0; i < C / 2; ++i) {
      float own = 0.f;
      if (i < ilim) {
        const int j = 2 * i + half;
        own = j <= t ? __expf(gt - gam[j]) : 0.f;
      }
      const float other = __shfl_xor_sync(0xffffffffu, own, 16);
      x[2 * i] *= half ? other : own;
      x[2 * i + 1] *= half ? own : other;
    }
    if (lane < 16) {  // A: strictly lower, weighted by beta_t
      const float bt = bet[t];
#pragma unroll
      for (int j = 0; j < C; j += 4) {
        float4 a;
        a.x = j < t ? bt * x[j] : 0.f;
        a.y = j + 1 < t ? bt * x[j + 1] : 0.f;
        a.z = j + 2 < t ? bt * x[j + 2] : 0.f;
        a.w = j + 3 < t ? bt * x[j + 3] : 0.f;
        *reinterpret_cast<float4*>(Af + t * AP + j) = a;
      }
    } else {  // M: lower with the diagonal (the decay is zero above it)
      put_row_pair<T>(sm + PrepSmem::V0, sm + PrepSmem::V0 + C * 128, t, x);
    }
  }
  fence_proxy_async_shared();
  prefill::tc_fence_before();
  __syncthreads();
  if (tid == 0 && ok) {  // (M_hi, M_lo: 16 KB, adjacent in the workspace as in the stage)
    bulk_s2g(unit + WS_MHI, sm + PrepSmem::V0, 2 * C * 128);
    bulk_commit();
    bulk_wait_read();
    mbar_arrive_expect_tx(&bar[0], 2 * C * 128);
#pragma unroll
    for (int db = 0; db < 2; ++db)
      tma_load_4d(sm + PrepSmem::V0 + db * C * 128, &vmap, db * 64, t0, h, b, &bar[0]);
  }


  // 4. T = (I + A)^{-1}, in place over A's lower triangle (diagonal 1, upper 0), fp32 on the CUDA cores
  // level 0: each warp inverts its 16 x 16 diagonal block by forward substitution, lane i holding column i
  {
    const int base = warp * 16;
    float tc[16];
    const int i = lane & 15;
#pragma unroll
    for (int r = 0; r < 16; ++r) {
      float sum = 0.f;
#pragma unroll
      for (int j = 0; j < r; ++j) sum = fmaf(Af[(base + r) * AP + base + j], tc[j], sum);
      tc[r] = i < r ? -sum : (i == r ? 1.f : 0.f);
    }
    __syncwarp();
    if (lane < 16)
#pragma unroll
      for (int r = 0; r < 16; ++r) Af[(base + r) * AP + base + i] = tc[r];
  }
  __syncthreads();
  // level 1: T[hi][lo] = -T[hi][hi] (A[hi][lo] T[lo][lo]) for the 16 x 16 block pairs (lo, hi) = (0, 16), (32, 48):
  // threads 64 p .. 64 p + 63 take pair p, the thread row r = (tid % 64) / 4 and columns c0 .. c0 + 3 of the block
  // (float4 operands: a quarter warp reads two rows of A and four column groups of one row of T, conflict-free)
  {
    const int pr = tid >> 6, r = (tid & 63) >> 2, c0 = (tid & 3) * 4;
    const int lo = 32 * pr, hi = lo + 16;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int k = 0; k < 16; k += 4) {
      const float4 a = *reinterpret_cast<const float4*>(Af + (hi + r) * AP + lo + k);
      const float av[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const float4 bq = *reinterpret_cast<const float4*>(Af + (lo + k + kk) * AP + lo + c0);
        acc[0] = fmaf(av[kk], bq.x, acc[0]);
        acc[1] = fmaf(av[kk], bq.y, acc[1]);
        acc[2] = fmaf(av[kk], bq.z, acc[2]);
        acc[3] = fmaf(av[kk], bq.w, acc[3]);
      }
    }
    *reinterpret_cast<float4*>(Xs + (16 * pr + r) * XP + c0) = make_float4(acc[0], acc[1], acc[2], acc[3]);
    __syncthreads();
    float t4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int k = 0; k < 16; k += 4) {
      const float4 a = *reinterpret_cast<const float4*>(Af + (hi + r) * AP + hi + k);
      const float av[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const float4 xq = *reinterpret_cast<const float4*>(Xs + (16 * pr + k + kk) * XP + c0);
        t4[0] = fmaf(av[kk], xq.x, t4[0]);
        t4[1] = fmaf(av[kk], xq.y, t4[1]);
        t4[2] = fmaf(av[kk], xq.z, t4[2]);
        t4[3] = fmaf(av[kk], xq.w, t4[3]);
      }
    }
    *reinterpret_cast<float4*>(Af + (hi + r) * AP + lo + c0) = make_float4(-t4[0], -t4[1], -t4[2], -t4[3]);
  }
  __syncthreads();
  // level 2: T[32:64][0:32] = -T[32:64][32:64] (A[32:64][0:32] T[0:32][0:32]) (32 x 32 blocks): thread row
  // r = tid / 4, columns c0 .. c0 + 7
  {
    const int r = tid >> 2, c0 = (tid & 3) * 8;
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int k = 0; k < 32; k += 4) {
      const float4 a = *reinterpret_cast<const float4*>(Af + (32 + r) * AP + k);
      const float av[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const float4 b0 = *reinterpret_cast<const float4*>(Af + (k + kk) * AP + c0);
        const float4 b1 = *reinterpret_cast<const float4*>(Af + (k + kk) * AP + c0 + 4);
        acc[0] = fmaf(av[kk], b0.x, acc[0]);
        acc[1] = fmaf(av[kk], b0.y, acc[1]);
        acc[2] = fmaf(av[kk], b0.z, acc[2]);
        acc[3] = fmaf(av[kk], b0.w, acc[3]);
        acc[4] = fmaf(av[kk], b1.x, acc[4]);
        acc[5] = fmaf(av[kk], b1.y, acc[5]);
        acc[6] = fmaf(av[kk], b1.z, acc[6]);
        acc[7] = fmaf(av[kk], b1.w, acc[7]);
      }
    }
    *reinterpret_cast<float4*>(Xs + r * XP + c0) = make_float4(acc[0], acc[1], acc[2], acc[3]);
    *reinterpret_cast<float4*>(Xs + r * XP + c0 + 4) = make_float4(acc[4], acc[5], acc[6], acc[7]);
    __syncthreads();
    float t8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int k = 0; k < 32; k += 4) {
      const float4 a = *reinterpret_cast<const float4*>(Af + (32 + r) * AP + 32 + k);
      const float av[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const float4 x0 = *reinterpret_cast<const float4*>(Xs + (k + kk) * XP + c0);
        const float4 x1 = *reinterpret_cast<const float4*>(Xs + (k + kk) * XP + c0 + 4);
        t8[0] = fmaf(av[kk], x0.x, t8[0]);
        t8[1] = fmaf(av[kk], x0.y, t8[1]);
        t8[2] = fmaf(av[kk], x0.z, t8[2]);
        t8[3] = fmaf(av[kk], x0.w, t8[3]);
        t8[4] = fmaf(av[kk], x1.x, t8[4]);
        t8[5] = fmaf(av[kk], x1.y, t8[5]);
        t8[6] = fmaf(av[kk], x1.z, t8[6]);
        t8[7] = fmaf(av[kk], x1.w, t8[7]);
      }
    }
    *reinterpret_cast<float4*>(Af + (32 + r) * AP + c0) = make_float4(-t8[0], -t8[1], -t8[2], -t8[3]);
    *reinterpret_cast<float4*>(Af + (32 + r) * AP + c0 + 4) = make_float4(-t8[4], -t8[5], -t8[6], -t8[7]);
  }
  __syncthreads();
  // 5. W = T diag(beta Gam) K (lane 0): every thread takes a row of T into registers (threads 0-63 row tid scaled by
  // beta Gam, threads 64-127 row tid - 64 scaled by beta, for U'), then threads 0-63 write their row of W's A operand
  // (a hi / lo pair) over T; K = 64 positions in four steps of 16 rows of the K tile (B MN-major: its two 64-key boxes
  // 8 KB apart)
  float tx[C];
  {
    const int r = tid & (C - 1);
    const bool w_row = tid < C;
#pragma unroll
    for (int j = 0; j < C; j += 4) {
      const float4 a = *reinterpret_cast<const float4*>(Af + r * AP + j);
      tx[j] = a.x * (w_row ? bet[j] * Gam[j] : bet[j]);
      tx[j + 1] = a.y * (w_row ? bet[j + 1] * Gam[j + 1] : bet[j + 1]);
      tx[j + 2] = a.z * (w_row ? bet[j + 2] * Gam[j + 2] : bet[j + 2]);
      tx[j + 3] = a.w * (w_row ? bet[j + 3] * Gam[j + 3] : bet[j + 3]);
    }
  }
  __syncthreads();  // T is read: its region takes T diag(beta Gam)
  if (tid < C) put_row_pair<T>(sm + PrepSmem::TBG, sm + PrepSmem::TBG + C * 128, tid, tx);
  fence_proxy_async_shared();
  prefill::tc_fence_before();
  __syncthreads();
  if (tid == 0 && ok) {
    prefill::tc_fence_after();
    const uint32_t k0 = smem_u32(sm + PrepSmem::K0), tg = smem_u32(sm + PrepSmem::TBG);
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
      const uint64_t bk = prefill::sdesc(k0 + ks * 16 * 128, C * 128, 1024);
      prefill::umma_ss(tmem, prefill::sdesc(tg + ks * 32, 16, 1024), bk, IDESC_W, ks ? 1u : 0u);
      prefill::umma_ss(tmem, prefill::sdesc(tg + C * 128 + ks * 32, 16, 1024), bk, IDESC_W, 1u);
    }
    prefill::umma_commit(&bar[1]);
  }
  ok = __all_sync(0xffffffffu, ok && mbar_wait(&bar[1], 1, 77));
  // 6. U' = T diag(beta) V (lane 16): threads 64-127 write its A operand from their registers where the K tile was
  // (W's products are done with it), then while those MMAs run every warp takes W out of TMEM (lanes 0-15: row t) as
  // hi / lo pairs
  if (tid >= C) put_row_pair<T>(sm + PrepSmem::TB, sm + PrepSmem::TB + C * 128, tid - C, tx);
  ok = __all_sync(0xffffffffu, ok && mbar_wait(&bar[0], 1, 79));  // the V tile has landed (long since)
  fence_proxy_async_shared();
  prefill::tc_fence_before();
  __syncthreads();
  if (tid == 0 && ok) {
    prefill::tc_fence_after();
    const uint32_t v0 = smem_u32(sm + PrepSmem::V0), tb = smem_u32(sm + PrepSmem::TB);
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
      const uint64_t bv = prefill::sdesc(v0 + ks * 16 * 128, C * 128, 1024);
      prefill::umma_ss(tmem + LANE16, prefill::sdesc(tb + ks * 32, 16, 1024), bv, IDESC_W, ks ? 1u : 0u);
      prefill::umma_ss(tmem + LANE16, prefill::sdesc(tb + C * 128 + ks * 32, 16, 1024), bv, IDESC_W, 1u);
    }
    prefill::umma_commit(&bar[1]);
  }
  // W and U' leave through shared memory by bulk copies: written there by rows, they reach the workspace as whole
  // lines (row-by-row 16-byte global stores touch sixteen lines a warp instruction and held the load / store unit).
  // W, a half (64 key columns, hi and lo: 16 KB) at a time, is staged where T diag(beta Gam) was (free once W's
  // products have committed).
  const int t = 16 * warp + (lane & 15);
  uint8_t* wst = sm + PrepSmem::TBG;
  if (ok) prefill::tc_fence_after();
#pragma unroll 1
  for (int half = 0; half < 2; ++half) {
    float x[C];
    if (ok) {
      prefill::tmem_ld32(tmem + lq + half * C, x);
      prefill::tmem_ld32(tmem + lq + half * C + 32, x + 32);
      prefill::tmem_wait_ld();
    }
    if (half) {  // the first half's copies have read the stage
      if (tid == 0) bulk_wait_read();
      __syncthreads();
    }
    if (lane < 16 && ok) put_row_pair<T>(wst, wst + C * 128, t, x);
    fence_proxy_async_shared();
    __syncthreads();
    if (tid == 0 && ok) {
      bulk_s2g(unit + WS_WHI + half * C * 128, wst, C * 128);
      bulk_s2g(unit + WS_WLO + half * C * 128, wst + C * 128, C * 128);
      bulk_commit();
    }
  }
  // 7. U' (lanes 16-31: row t) in fp32 slices of 32 value columns, staged as the workspace holds them (all four slices,
  // 36 KB from the K tile's region on: free once U''s products have committed, and past W's stage once its copies
  // have read it)
  ok = __all_sync(0xffffffffu, ok && mbar_wait(&bar[1], 0, 78));
  if (ok) prefill::tc_fence_after();
  uint8_t* ust = sm + PrepSmem::K0;
  static_assert(PrepSmem::K0 + (DV / DVB) * USLICE <= PrepSmem::XS, "U' stage inside the tile regions");
  if (tid == 0) bulk_wait_read();
  __syncthreads();
#pragma unroll 1
  for (int half = 0; half < 2; ++half) {
    float x[C];
    if (ok) {
      prefill::tmem_ld32(tmem + lq + half * C, x);
      prefill::tmem_ld32(tmem + lq + half * C + 32, x + 32);
      prefill::tmem_wait_ld();
    }
    if (lane >= 16 && ok)
#pragma unroll
      for (int s2 = 0; s2 < 2; ++s2) {  // value columns 64 half + 32 s2 ..: slice 2 half + s2
        float4* g = reinterpret_cast<float4*>(ust + (2 * half + s2) * USLICE + t * UP * 4);
#pragma unroll
        for (int q4 = 0; q4 < DVB / 4; ++q4)
          g[q4] = make_float4(x[32 * s2 + 4 * q4], x[32 * s2 + 4 * q4 + 1], x[32 * s2 + 4 * q4 + 2],
                              x[32 * s2 + 4 * q4 + 3]);
      }
  }
  fence_proxy_async_shared();
  __syncthreads();
  if (tid == 0 && ok) {
    bulk_s2g(unit + WS_U, ust, (DV / DVB) * USLICE);
    bulk_commit();
  }
  // 8. gamma and Gam for the scan
  if (tid < C) {
    float* gg = reinterpret_cast<float*>(unit + WS_G);
    gg[tid] = gam[tid];
    gg[C + tid] = Gam[tid];
  }
  if (tid == 0) bulk_wait_all();  // the bulk copies have read their stages and written the workspace
  prefill::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    prefill::tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(PREP_TMEM_COLS));
  }
}

// ------------------------------------------------------------------------------------------------ scan
//
// One CTA: value columns dv0 .. dv0 + 31 of one (batch, v-head), all chunks in order, every product on the tensor
// cores (tcgen05.mma kind::f16, accumulators in TMEM). The state slice S [32 value rows x 128 keys] is kept in fp32
// registers of the eight epilogue warps (two threads a key k, one with S[0 .. 15][k], one with S[16 .. 31][k]) and
// given to the MMAs as a 16-bit hi / lo pair in shared memory. Every B operand is MN-major with N = 64: the 32 value
// rows' hi halves, then their lo halves, so one MMA reads its A tile once for both halves and an epilogue thread writes
// its row with four 16-byte stores. Per chunk:
//   P1  D1 = [W_hi ; Q] [S_hi | S_lo]^T   (M = 128: rows 0-63 W, rows 64-127 Q; K = 128)
//       D4 = W_lo [S_hi | S_lo]^T           (rows 0-63 used)      -> W S^T = D1[0:64] + D4[0:64], both halves summed
//   E-U U = U' - W S^T (TMEM lanes 0-63: thread = position, half the columns), Ud = diag(exp(gamma_C - gamma)) U,
//       both as hi / lo pairs
//   P2  D2 = K^T [Ud_hi | Ud_lo]           (M = 128 keys, A = the K tile as the TMA loads it, MN-major; K = 64)
//   P3  D3 = (M_hi + M_lo) [U_hi | U_lo]^T  (rows 64-127 used)
//   E-S S <- Gam_C S + D2 (all eight warps, thread = key, half the columns) -> the next P1's operand
//   E-Y Y = Gam (D1[64:128]) + D3[64:128] (lanes 64-127: thread = position) -> y
// The chain from one chunk to the next is P1 -> E-U -> P2 -> E-S; P3 and E-Y run beside it (D1 / D3 / D4 are
// double-buffered by chunk parity, so E-Y may lag a chunk). Chunk c's W, M, gates and U' slice arrive by bulk copies
// and its Q and K tiles by tiled TMA, into one of two buffers, a chunk ahead.
//
// Rows past T in the last chunk: Q and K arrive as zeros and prep left W, U' zero there, so they add nothing; their
// y is not stored.

// warps 0-7 epilogue: warp w reads TMEM lane quarter w % 4 and takes value columns 16 (w / 4) .. + 15 of the
// slice; warp 8 loads, warp 9 issues the MMAs
constexpr int TC_EPI = 8, TC_LOAD = 8, TC_MMA = 9;
constexpr int TC_THREADS = 320;
constexpr int VH = DVB / 2;      // value columns a thread
constexpr int TC_TMEM_COLS = 512;

struct TcSmem {
  // one chunk buffer (two of them): the shared-memory images of the workspace pieces, each operand 1024-aligned
  static constexpr int A1 = 0;                 // [W_hi kb0 | Q kb0 | W_hi kb1 | Q kb1], 8 KB each: P1's A
  static constexpr int WLO = 4 * C * 128;      // W_lo kb0, kb1 (8 KB each); then M_hi, M_lo, gates in workspace order
  static constexpr int MHI = WLO + 2 * C * 128;
  static constexpr int MLO = MHI + C * 128;
  static constexpr int G = MLO + C * 128;      // gamma [64], Gam [64] fp32
  static constexpr int U = G + 2 * C * 4;      // U' slice [64][UP] fp32
  static constexpr int K = (U + USLICE + 1023) / 1024 * 1024;  // K tile: two TMA boxes [64 positions][64 keys]
  static constexpr int BUF = K + 2 * C * 128;
  // persistent operands (16-bit, 128-byte swizzle, K-major)
  // B operands of the chain, MN-major (N = 64: the 32 value rows' hi halves, then their lo halves, a 128-byte row):
  // S^T [128 keys][hi 32 | lo 32] (16 KB), Ud [64 positions][hi 32 | lo 32] (8 KB), U the same
  static constexpr int SOP = 2 * BUF;
  static constexpr int UDOP = SOP + DK * 128;
  static constexpr int UOP = UDOP + C * 128;
  static constexpr int BAR = UOP + C * 128;    // mbarriers
  static constexpr int NBAR = 16;
  static constexpr int SLOT = BAR + NBAR * 8;  // TMEM base address; abort flag
  static constexpr int BYTES = SLOT + 16 + 1024;  // (+ alignment of the dynamic shared memory base)
  // bytes that land in a buffer a chunk
  static constexpr uint32_t TX = 2 * C * 128 + (WS_U - WS_WLO) + USLICE + 4 * C * 128;
};
static_assert(TcSmem::WLO - TcSmem::A1 == 4 * 8192 && TcSmem::G - TcSmem::WLO == WS_G - WS_WLO, "copy layout");
static_assert(TcSmem::BUF % 1024 == 0 && TcSmem::SOP % 1024 == 0 && TcSmem::BYTES <= 232448, "scan shared memory");

// barrier slots
constexpr int B_FULL = 0;     // [2] a buffer's copies landed
constexpr int B_EMPTY = 2;    // [2] a buffer is free: its MMAs committed and the eight epilogue warps done with it
constexpr int B_SREADY = 4;   // the state operand of the next chunk written (eight warps)
constexpr int B_D1 = 5;       // [2] P1 done
constexpr int B_UREADY = 7;   // U operands written (warps 0, 1, 4, 5)
constexpr int B_D2 = 8;       // P2 done
constexpr int B_D3 = 9;       // [2] P3 done
constexpr int B_YDONE = 11;   // [2] E-Y read D1 / D3 of that parity (warps 2, 3, 6, 7)
constexpr int B_DRAIN = 13;   // every MMA issued has completed (the MMA thread's exit)
constexpr int B_UDREADY = 14; // Ud operands written (warps 0, 1, 4, 5): P2 may start

// TMEM columns
// D1 = [W_hi ; Q] [S_hi | S_lo]^T, D4 = W_lo [S_hi | S_lo]^T and D3 = (M_hi + M_lo) [U_hi | U_lo]^T: two 64-column
// buffers each (the products with the hi and the lo halves side by side); D2 = K^T [Ud_hi | Ud_lo]: 64 columns
constexpr uint32_t T_D1 = 0, T_D3 = 128, T_D4 = 256, T_D2 = 384;


// Writes the 16 values x (value rows r0 .. r0 + 15) into row `row` (a key or a position) of an MN-major operand
// [rows][hi 32 | lo 32]: the hi halves at elements r0 .., the lo halves at 32 + r0 .., four 16-byte stores.
template <typename T>
__device__ __forceinline__ void put_row16(uint8_t* op, int row, int r0, const float* x) {
  uint32_t h[8], l[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) split2<T>(x[2 * e], x[2 * e + 1], h[e], l[e]);
  uint8_t* r = op + row * 128;
  const int c0 = r0 >> 3, sw = row & 7;
  *reinterpret_cast<uint4*>(r + (((c0) ^ sw) << 4)) = make_uint4(h[0], h[1], h[2], h[3]);
  *reinterpret_cast<uint4*>(r + (((c0 + 1) ^ sw) << 4)) = make_uint4(h[4], h[5], h[6], h[7]);
  *reinterpret_cast<uint4*>(r + (((c0 + 4) ^ sw) << 4)) = make_uint4(l[0], l[1], l[2], l[3]);
  *reinterpret_cast<uint4*>(r + (((c0 + 5) ^ sw) << 4)) = make_uint4(l[4], l[5], l[6], l[7]);
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
  uint32_t* r = reinterpret_cast<uint32_t*>(v);
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

template <typename T>
__global__ void __launch_bounds__(TC_THREADS, 1) scan_kernel(const __grid_constant__ CUtensorMap qmap,
                                                              const __grid_constant__ CUtensorMap kmap,
                                                              const Params p) {
  constexpr uint32_t AB = std::is_same<T, __nv_bfloat16>::value ? 1 : 0;
  // B always MN-major [K rows][hi 32 | lo 32] (N = 64); A K-major, or MN-major for the K tile read as K^T
  constexpr uint32_t IDESC_K2 = prefill::idesc_f16(AB, 0, 1, 128, 2 * DVB);
  constexpr uint32_t IDESC_MN2 = prefill::idesc_f16(AB, 1, 1, 128, 2 * DVB);
  const int blk = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int hk = h / (p.Hv / p.Hk);
  const int dv0 = blk * DVB;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n = p.nchunks;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + TcSmem::BAR);
  uint32_t* slot = reinterpret_cast<uint32_t*>(sm + TcSmem::SLOT);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sm + TcSmem::SLOT + 4);

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bar[B_FULL + i], 1);
      mbar_init(&bar[B_EMPTY + i], 1 + TC_EPI);  // the MMA commit + one arrive per epilogue warp
      mbar_init(&bar[B_D1 + i], 1);
      mbar_init(&bar[B_D3 + i], 1);
      mbar_init(&bar[B_YDONE + i], TC_EPI / 2);
    }
    mbar_init(&bar[B_SREADY], TC_EPI);
    mbar_init(&bar[B_UREADY], TC_EPI / 2);
    mbar_init(&bar[B_UDREADY], TC_EPI / 2);
    mbar_init(&bar[B_D2], 1);
    mbar_init(&bar[B_DRAIN], 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == TC_MMA) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)),
                 "r"(TC_TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  prefill::tc_fence_before();
  __syncthreads();
  prefill::tc_fence_after();
  const uint32_t tmem = *slot;
  // Launched as a programmatic dependent of prep: the set-up above touched only this CTA's shared memory and TMEM;
  // every global read below waits for prep's grid to complete.

  if (warp < TC_EPI) {
    // ------------------------------------------------------------------------------------ epilogue warps
    const int quarter = warp & 3, vh = warp >> 2;
    const int k = 32 * quarter + lane;                // this thread's key column of S (and TMEM lane)
    const int r0 = VH * vh;                           // its value rows r0 .. r0 + 15 of the slice
    const uint32_t lq = uint32_t(32 * quarter) << 16;  // the warp's TMEM lane quarter
    float s[VH];
    const float* sin = p.s_in + (int64_t(b) * p.Hv + h) * DV * DK + int64_t(dv0 + r0) * DK + k;
#pragma unroll
    for (int j = 0; j < VH; ++j) s[j] = sin[int64_t(j) * DK];
    if (n > 0) {
      put_row16<T>(sm + TcSmem::SOP, k, r0, s);
      fence_proxy_async_shared();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar[B_SREADY]);
    }
    bool ok = true;
    for (int c = 0; c < n && ok; ++c) {
      const int par = c & 1;
      uint8_t* buf = sm + par * TcSmem::BUF;
      const float* gam = reinterpret_cast<const float*>(buf + TcSmem::G);
      const float* Gam = gam + C;
      // the chunk's buffer has landed (it did before P1 could run): gates and U' are read off the chain
      ok = __all_sync(0xffffffffu, mbar_wait(&bar[B_FULL + par], (c >> 1) & 1, 80) && !*abort_flag);
      if (!ok) break;
      if (quarter < 2) {  // E-U: positions t = k (0 .. 63)
        const int t = k;
        const float dec = __expf(gam[C - 1] - gam[t]);
        float u[VH];
        {
          const float4* up = reinterpret_cast<const float4*>(buf + TcSmem::U + t * UP * 4 + r0 * 4);
#pragma unroll
          for (int q4 = 0; q4 < VH / 4; ++q4) {
            const float4 x = up[q4];
            u[4 * q4] = x.x, u[4 * q4 + 1] = x.y, u[4 * q4 + 2] = x.z, u[4 * q4 + 3] = x.w;
          }
        }
        ok = __all_sync(0xffffffffu, mbar_wait(&bar[B_D1 + par], (c >> 1) & 1, 81) && !*abort_flag);
        if (!ok) break;
        prefill::tc_fence_after();
        {
          float d[VH], dl[VH], d4[VH], d4l[VH];
          tmem_ld16(tmem + lq + T_D1 + par * 64 + r0, d);
          tmem_ld16(tmem + lq + T_D1 + par * 64 + DVB + r0, dl);
          tmem_ld16(tmem + lq + T_D4 + par * 64 + r0, d4);
          tmem_ld16(tmem + lq + T_D4 + par * 64 + DVB + r0, d4l);
          prefill::tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < VH; ++j) u[j] -= (d[j] + dl[j]) + (d4[j] + d4l[j]);
        }
        prefill::tc_fence_before();
        {  // Ud first: the state update (P2) waits for it; U (P3, off the chain) after
          float ud[VH];
#pragma unroll
          for (int j = 0; j < VH; ++j) ud[j] = dec * u[j];
          put_row16<T>(sm + TcSmem::UDOP, t, r0, ud);
        }
        fence_proxy_async_shared();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bar[B_UDREADY]);
        put_row16<T>(sm + TcSmem::UOP, t, r0, u);
        fence_proxy_async_shared();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bar[B_UREADY]);
      }
      const float gc = Gam[C - 1];  // read before the wait: the buffer stays until this warp releases it
      // E-S: S <- Gam_C S + K^T Ud on this thread's key column
      ok = __all_sync(0xffffffffu, mbar_wait(&bar[B_D2], c & 1, 82) && !*abort_flag);
      if (!ok) break;
      prefill::tc_fence_after();
      {
        float d2[VH], d2l[VH];
        tmem_ld16(tmem + lq + T_D2 + r0, d2);
        tmem_ld16(tmem + lq + T_D2 + DVB + r0, d2l);
        prefill::tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < VH; ++j) s[j] = fmaf(gc, s[j], d2[j] + d2l[j]);
      }
      if (c + 1 < n) {
        put_row16<T>(sm + TcSmem::SOP, k, r0, s);
        fence_proxy_async_shared();
      }
      prefill::tc_fence_before();
      __syncwarp();
      if (lane == 0 && c + 1 < n) mbar_arrive(&bar[B_SREADY]);
      if (quarter >= 2) {  // E-Y: positions t = k - 64
        ok = __all_sync(0xffffffffu, mbar_wait(&bar[B_D3 + par], (c >> 1) & 1, 83) && !*abort_flag);
        if (!ok) break;
        prefill::tc_fence_after();
        float qs[VH], mu[VH];
        {
          float ql[VH], ml[VH];
          tmem_ld16(tmem + lq + T_D1 + par * 64 + r0, qs);
          tmem_ld16(tmem + lq + T_D1 + par * 64 + DVB + r0, ql);
          tmem_ld16(tmem + lq + T_D3 + par * 64 + r0, mu);
          tmem_ld16(tmem + lq + T_D3 + par * 64 + DVB + r0, ml);
          prefill::tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < VH; ++j) qs[j] += ql[j], mu[j] += ml[j];
        }
        const int t = k - C;
        const int pos = c * C + t;
        const float gt = Gam[t];
        prefill::tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bar[B_YDONE + par]);
        if (pos < p.T) {
          uint4* yr = reinterpret_cast<uint4*>(static_cast<T*>(p.y) + ((int64_t(b) * p.T + pos) * p.Hv + h) * DV +
                                               dv0 + r0);
#pragma unroll
          for (int q8 = 0; q8 < VH / 8; ++q8) {
            uint32_t w4[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int j = 8 * q8 + 2 * e;
              w4[e] = pack2<T>(fmaf(gt, qs[j], mu[j]), fmaf(gt, qs[j + 1], mu[j + 1]));
            }
            yr[q8] = make_uint4(w4[0], w4[1], w4[2], w4[3]);
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar[B_EMPTY + par]);  // this warp is done with the chunk's buffer
    }
    if (!ok) {
      *abort_flag = 1;
    } else {
      float* sout = p.s_out + (int64_t(b) * p.Hv + h) * DV * DK + int64_t(dv0 + r0) * DK + k;
#pragma unroll
      for (int j = 0; j < VH; ++j) sout[int64_t(j) * DK] = s[j];
    }
  } else if (warp == TC_LOAD) {
    // ------------------------------------------------------------------------------------ loads
    if (lane == 0 && n > 0) {
      prefetch_tensormap(&qmap);
      prefetch_tensormap(&kmap);
      int issued = 0;
      for (int c = 0; c < n; ++c) {
        const int par = c & 1;
        if (c >= 2 && !mbar_wait(&bar[B_EMPTY + par], ((c >> 1) - 1) & 1, 84)) {
          *abort_flag = 1;
          break;
        }
        if (*abort_flag) break;
        uint8_t* buf = sm + par * TcSmem::BUF;
        const uint8_t* u = unit_ptr(p, b, h, c);
        fence_proxy_async_shared();
        mbar_arrive_expect_tx(&bar[B_FULL + par], TcSmem::TX);
        bulk_g2s(buf + TcSmem::A1, u + WS_WHI, C * 128, &bar[B_FULL + par]);
        bulk_g2s(buf + TcSmem::A1 + 2 * C * 128, u + WS_WHI + C * 128, C * 128, &bar[B_FULL + par]);
        bulk_g2s(buf + TcSmem::WLO, u + WS_WLO, WS_U - WS_WLO, &bar[B_FULL + par]);
        bulk_g2s(buf + TcSmem::U, u + WS_U + blk * USLICE, USLICE, &bar[B_FULL + par]);
#pragma unroll
        for (int db = 0; db < DK / 64; ++db) {
          tma_load_4d(buf + TcSmem::A1 + db * 2 * C * 128 + C * 128, &qmap, db * 64, c * C, hk, b, &bar[B_FULL + par]);
          tma_load_4d(buf + TcSmem::K + db * C * 128, &kmap, db * 64, c * C, hk, b, &bar[B_FULL + par]);
        }
        issued = c + 1;
      }
      // what was issued has landed before the CTA may leave (bounded)
      for (int c = max(0, issued - 2); c < issued; ++c) mbar_wait(&bar[B_FULL + (c & 1)], (c >> 1) & 1, 85);
    }
  } else {
    // ------------------------------------------------------------------------------------ MMA issuer
    if (elect_one() && n > 0) {
      bool ok = true;
      const uint32_t sop = smem_u32(sm + TcSmem::SOP);
      const uint32_t uop = smem_u32(sm + TcSmem::UOP), udop = smem_u32(sm + TcSmem::UDOP);
      for (int c = 0; c < n && ok; ++c) {
        const int par = c & 1;
        const uint32_t base = smem_u32(sm + par * TcSmem::BUF);
        ok = mbar_wait(&bar[B_FULL + par], (c >> 1) & 1, 86) && mbar_wait(&bar[B_SREADY], c & 1, 87) &&
             (c < 2 || mbar_wait(&bar[B_YDONE + par], ((c >> 1) - 1) & 1, 88)) && !*abort_flag;
        if (!ok) break;
        prefill::tc_fence_after();
        // P1: D1 = [W_hi ; Q] [S_hi | S_lo]^T, D4 = W_lo [S_hi | S_lo]^T (N = 64: each A tile read once for both
        // halves; K = 128 keys: two 64-key blocks of A, 4 steps each, and 16 rows of S^T a step)
#pragma unroll
        for (int kb = 0; kb < 2; ++kb)
#pragma unroll
          for (int ks = 0; ks < 4; ++ks) {
            const uint32_t acc = (kb | ks) ? 1u : 0u;
            const uint64_t a = prefill::sdesc(base + TcSmem::A1 + kb * 2 * C * 128 + ks * 32, 16, 1024);
            const uint64_t al = prefill::sdesc(base + TcSmem::WLO + kb * C * 128 + ks * 32, 16, 1024);
            const uint64_t bs = prefill::sdesc(sop + (kb * 4 + ks) * 16 * 128, DK * 128, 1024);
            prefill::umma_ss(tmem + T_D1 + par * 64, a, bs, IDESC_K2, acc);
            prefill::umma_ss(tmem + T_D4 + par * 64, al, bs, IDESC_K2, acc);
          }
        prefill::umma_commit(&bar[B_D1 + par]);
        ok = mbar_wait(&bar[B_UDREADY], c & 1, 89) && !*abort_flag;
        if (!ok) break;
        prefill::tc_fence_after();
        // P2: D2 = K^T [Ud_hi | Ud_lo]: A = the K tile [64 positions][128 keys] read as M = keys (MN-major: the two
        // 64-key boxes 8 KB apart), K = positions in steps of 16 rows
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
          const uint64_t a = prefill::sdesc(base + TcSmem::K + ks * 16 * 128, C * 128, 1024);
          prefill::umma_ss(tmem + T_D2, a, prefill::sdesc(udop + ks * 16 * 128, C * 128, 1024), IDESC_MN2, ks ? 1u : 0u);
        }
        prefill::umma_commit(&bar[B_D2]);
        ok = mbar_wait(&bar[B_UREADY], c & 1, 91) && !*abort_flag;
        if (!ok) break;
        prefill::tc_fence_after();
        // P3: D3[64:128] = (M_hi + M_lo) [U_hi | U_lo]^T; the A rows 0-63 are whatever precedes M_hi / M_lo in the
        // buffer (D3 rows 0-63 unused)
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
          const uint64_t ahi = prefill::sdesc(base + TcSmem::MHI - C * 128 + ks * 32, 16, 1024);
          const uint64_t alo = prefill::sdesc(base + TcSmem::MHI + ks * 32, 16, 1024);
          const uint64_t bu = prefill::sdesc(uop + ks * 16 * 128, C * 128, 1024);
          prefill::umma_ss(tmem + T_D3 + par * 64, ahi, bu, IDESC_K2, ks ? 1u : 0u);
          prefill::umma_ss(tmem + T_D3 + par * 64, alo, bu, IDESC_K2, 1u);
        }
        prefill::umma_commit(&bar[B_D3 + par]);
        prefill::umma_commit(&bar[B_EMPTY + par]);
      }
      if (!ok) *abort_flag = 1;
      prefill::umma_commit(&bar[B_DRAIN]);  // every MMA issued has completed before TMEM is freed
      mbar_wait(&bar[B_DRAIN], 0, 90);
    }
    __syncwarp();
  }
  prefill::tc_fence_before();
  __syncthreads();
  if (warp == TC_MMA) {
    prefill::tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TC_TMEM_COLS));
  }
}

}  // namespace gdnchunk
}  // namespace lb2
