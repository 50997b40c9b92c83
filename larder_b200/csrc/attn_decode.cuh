// Split-KV decode attention for a few query rows over a long KV cache (HBM-bandwidth bound).
//
// Work unit: one CTA per (key split s, KV head hk, sequence b). The G*T query rows sharing KV head hk are folded
// into 16-row tiles (the fold of foldattn.py:230-259), so every K/V byte is read from HBM once per decode call.
// A producer warp streams 64-key K and V tiles with TMA (128-byte swizzled boxes of 64 head-dim elements) into a
// STAGES-deep mbarrier ring; four consumer warps each take 16 of a tile's 64 keys and run S = Q K^T and O += P V
// on mma.sync m16n8k16 (fp32 accumulate) with an fp32 online softmax in base 2. The four warps' (max, sum, O) are
// merged in shared memory, and the split's partial is merged with the other splits of (b, hk) by log-sum-exp in
// the last CTA to finish (an atomic ticket per (b, hk)), the same combine as foldattn_merge (foldattn.py:188-211)
// and CpuAttn's range merge (cpu_ext/cpu_kern.cpp:607-628).
#pragma once

#include "common.cuh"

namespace lb2 {
namespace decode {

constexpr int BK = 64;         // keys per tile
constexpr int CONSUMERS = 4;   // consumer warps, 16 keys of each tile apiece
constexpr int THREADS = (CONSUMERS + 1) * 32;

template <int D>
struct Cfg {
  static constexpr int STAGES = D == 64 ? 4 : D == 128 ? 3 : 2;
  static constexpr int TILE_BYTES = BK * D * 2;             // one K (or V) tile, bf16/f16
  static constexpr int STAGE_BYTES = 2 * TILE_BYTES;        // K + V
  static constexpr int RING_BYTES = STAGES * STAGE_BYTES;
  static constexpr int SMEM_BYTES = RING_BYTES + 1024 /*align*/ + 256 /*barriers*/;
};

struct Params {
  const void* q;
  int64_t q_st[3];
  void* o;
  int64_t o_st[3];
  float* part_o;    // emit mode: normalised fp32 o, [B, Hq, T, D] contiguous
  float* part_lse;  // emit mode: natural-log lse, [B, Hq, T]
  const int32_t* kv_len;
  float* ws_o;      // [B, Hkv, nsplit, rows_pad, D] unnormalised partial O
  float* ws_ml;     // [B, Hkv, nsplit, rows_pad, 2] (max in log2 units, sum)
  int* ws_cnt;      // [B * Hkv] tickets, zero between calls
  int B, Hq, Hkv, T, N, G, rows;
  int split, nsplit;
  int causal, emit;
  float scale_log2;  // softmax scale * log2(e)
};

template <typename T>
__device__ __forceinline__ void mma16816(float* c, const uint32_t* a, uint32_t b0, uint32_t b1);
template <>
__device__ __forceinline__ void mma16816<__nv_bfloat16>(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
template <>
__device__ __forceinline__ void mma16816<__half>(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t* r) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t* r) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

// Byte offset of (key row r, 16-byte chunk c of head-dim block db) in a tile of 128-byte swizzled TMA boxes laid
// out [D / 64][BK][64 elements]: chunk c of row r sits at chunk c ^ (r & 7).
__device__ __forceinline__ uint32_t swz(int db, int r, int c) {
  return uint32_t(db * BK * 128 + r * 128 + ((c ^ (r & 7)) << 4));
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <typename T, int D, int MT>
__global__ void __launch_bounds__(THREADS) decode_kernel(const __grid_constant__ CUtensorMap kmap,
                                                          const __grid_constant__ CUtensorMap vmap, const Params p) {
  using C = Cfg<D>;
  constexpr int STAGES = C::STAGES;
  constexpr int ND = D / 8;  // 8-wide head-dim tiles of the output
  constexpr int KD = D / 16; // 16-wide k-steps of Q K^T
  const int s = blockIdx.x, hk = blockIdx.y, b = blockIdx.z;
  const int len = p.kv_len ? min(max(p.kv_len[b], 0), p.N) : p.N;
  const int nsplit_b = max(1, (len + p.split - 1) / p.split);
  if (s >= nsplit_b) return;  // the whole CTA: nothing of this sequence lies in this split
  const int n0 = s * p.split, n1 = min(len, n0 + p.split);
  const int ntiles = n1 > n0 ? (n1 - n0 + BK - 1) / BK : 0;

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(ring + C::RING_BYTES);
  uint64_t* empty = full + STAGES;
  __shared__ int s_last;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], CONSUMERS);
    }
    fence_barrier_init();
  }
  __syncthreads();

  // ------------------------------------------------------------------ producer warp: TMA K/V tiles into the ring
  if (warp == CONSUMERS) {
    if (lane == 0) {
      prefetch_tensormap(&kmap);
      prefetch_tensormap(&vmap);
      int issued = 0;
      for (int i = 0; i < ntiles; ++i) {
        const int st = i % STAGES;
        if (i >= STAGES && !mbar_wait(&empty[st], ((i / STAGES) - 1) & 1, 1)) break;
        uint8_t* kt = ring + st * C::STAGE_BYTES;
        uint8_t* vt = kt + C::TILE_BYTES;
        mbar_arrive_expect_tx(&full[st], C::STAGE_BYTES);
        const int key0 = n0 + i * BK;
#pragma unroll
        for (int db = 0; db < D / 64; ++db) {
          tma_load_4d(kt + db * BK * 128, &kmap, db * 64, key0, hk, b, &full[st]);
          tma_load_4d(vt + db * BK * 128, &vmap, db * 64, key0, hk, b, &full[st]);
        }
        issued = i + 1;
      }
      // Before the CTA may exit: the last tiles issued have landed (normally already consumed; bounded).
      for (int i = max(0, issued - STAGES); i < issued; ++i) mbar_wait(&full[i % STAGES], (i / STAGES) & 1, 2);
    }
    __syncthreads();
    __syncthreads();
    if (p.nsplit > 1 && nsplit_b > 1) __syncthreads();
    return;
  }

  // ------------------------------------------------------------------ consumer warps
  const int quad = lane >> 2, qid = lane & 3;
  // Q fragments (A operand, row-major 16 x 16 per k-step): rows are folded (g, t) pairs, row = g * T + t.
  uint32_t qa[MT][KD][4];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const int r = mt * 16 + quad + 8 * hh;
      const bool live = r < p.rows;
      const int g = live ? r / p.T : 0, t = live ? r % p.T : 0;
      const T* qrow = reinterpret_cast<const T*>(p.q) + b * p.q_st[0] + int64_t(hk * p.G + g) * p.q_st[1] +
                      int64_t(t) * p.q_st[2];
#pragma unroll
      for (int kk = 0; kk < KD; ++kk) {
        const int d = kk * 16 + 2 * qid;
        qa[mt][kk][hh] = live ? *reinterpret_cast<const uint32_t*>(qrow + d) : 0u;
        qa[mt][kk][hh + 2] = live ? *reinterpret_cast<const uint32_t*>(qrow + d + 8) : 0u;
      }
    }
  }
  // Causal limit of each of this thread's rows: the last visible key (bottom-right over this sequence's length).
  int lim[MT][2];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const int r = mt * 16 + quad + 8 * hh;
      lim[mt][hh] = r >= p.rows ? -1 : (p.causal ? len - p.T + (r % p.T) : len - 1);
    }

  float m_run[MT][2], l_run[MT][2];
  float acc[MT][ND][4];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) {
    m_run[mt][0] = m_run[mt][1] = -INFINITY;
    l_run[mt][0] = l_run[mt][1] = 0.f;
#pragma unroll
    for (int j = 0; j < ND; ++j) acc[mt][j][0] = acc[mt][j][1] = acc[mt][j][2] = acc[mt][j][3] = 0.f;
  }

  bool ok = true;
  for (int i = 0; i < ntiles && ok; ++i) {
    const int st = i % STAGES;
    if (!mbar_wait(&full[st], (i / STAGES) & 1, 3)) {
      ok = false;
      break;
    }
    const uint32_t kt = smem_u32(ring + st * C::STAGE_BYTES);
    const uint32_t vt = kt + C::TILE_BYTES;
    const int kbase = n0 + i * BK + warp * 16;  // this warp's first key
    // Rows of this warp's 16 keys that lie past the sequence (capacity padding may hold anything): zero V there
    // so that P = 0 never meets a non-finite value.
    const int nvalid = min(16, max(0, n1 - kbase));
    if (nvalid < 16) {
      uint8_t* vrow = ring + st * C::STAGE_BYTES + C::TILE_BYTES;
      for (int e = lane; e < (16 - nvalid) * (D / 8); e += 32) {
        const int r = warp * 16 + nvalid + e / (D / 8), c = e % (D / 8);
        *reinterpret_cast<uint4*>(vrow + swz(c / 8, r, c % 8)) = make_uint4(0, 0, 0, 0);
      }
      __syncwarp();
    }

    // S = Q K^T over this warp's 16 keys: two 8-key n-tiles.
    float sc[MT][2][4];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) sc[mt][nt][0] = sc[mt][nt][1] = sc[mt][nt][2] = sc[mt][nt][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < KD; ++kk) {
      uint32_t kb[4];
      const int r = warp * 16 + (lane & 7) + 8 * (lane >> 4);
      const int c = (kk * 16) / 8 + ((lane >> 3) & 1);
      ldsm_x4(kt + swz(c / 8, r, c % 8), kb);
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        mma16816<T>(sc[mt][0], qa[mt][kk], kb[0], kb[1]);
        mma16816<T>(sc[mt][1], qa[mt][kk], kb[2], kb[3]);
      }
    }

    // Online softmax (base 2) per row; each thread holds rows quad and quad + 8 of every m-tile.
    uint32_t pa[MT][4];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        float mx = -INFINITY;
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int key = kbase + nt * 8 + 2 * qid + e;
            float& x = sc[mt][nt][2 * hh + e];
            x = (key < n1 && key <= lim[mt][hh]) ? x * p.scale_log2 : -INFINITY;
            mx = fmaxf(mx, x);
          }
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        const float m_new = fmaxf(m_run[mt][hh], mx);
        const float m_use = m_new == -INFINITY ? 0.f : m_new;
        const float corr = ex2(m_run[mt][hh] - m_use);
        m_run[mt][hh] = m_new;
        float ls = 0.f;
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            float& x = sc[mt][nt][2 * hh + e];
            x = ex2(x - m_use);
            ls += x;
          }
        l_run[mt][hh] = l_run[mt][hh] * corr + ls;
#pragma unroll
        for (int j = 0; j < ND; ++j) {
          acc[mt][j][2 * hh] *= corr;
          acc[mt][j][2 * hh + 1] *= corr;
        }
      }
      pa[mt][0] = pack2<T>(sc[mt][0][0], sc[mt][0][1]);
      pa[mt][1] = pack2<T>(sc[mt][0][2], sc[mt][0][3]);
      pa[mt][2] = pack2<T>(sc[mt][1][0], sc[mt][1][1]);
      pa[mt][3] = pack2<T>(sc[mt][1][2], sc[mt][1][3]);
    }

    // O += P V over this warp's 16 keys: V^T fragments by transposed ldmatrix, two 8-wide d-tiles a load.
#pragma unroll
    for (int j = 0; j < ND; j += 2) {
      uint32_t vb[4];
      const int r = warp * 16 + (lane & 7) + 8 * ((lane >> 3) & 1);
      const int c = j + (lane >> 4);
      ldsm_x4_t(vt + swz(c / 8, r, c % 8), vb);
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        mma16816<T>(acc[mt][j], pa[mt], vb[0], vb[1]);
        mma16816<T>(acc[mt][j + 1], pa[mt], vb[2], vb[3]);
      }
    }
    if (nvalid < 16) fence_proxy_async_shared();  // generic writes above precede the next TMA into this stage
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[st]);
  }

  // ------------------------------------------------------------------ merge the four warps (shared memory)
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      l_run[mt][hh] += __shfl_xor_sync(0xffffffffu, l_run[mt][hh], 1);
      l_run[mt][hh] += __shfl_xor_sync(0xffffffffu, l_run[mt][hh], 2);
    }
  __syncthreads();  // (1) every warp is done with the ring: reuse it for the merge
  constexpr int RP = MT * 16;  // padded rows
  float* wo = reinterpret_cast<float*>(ring);          // [CONSUMERS][RP][D]
  float* wml = wo + CONSUMERS * RP * D;                // [CONSUMERS][RP][2]
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const int r = mt * 16 + quad + 8 * hh;
      if (qid == 0) {
        wml[(warp * RP + r) * 2] = m_run[mt][hh];
        wml[(warp * RP + r) * 2 + 1] = l_run[mt][hh];
      }
#pragma unroll
      for (int j = 0; j < ND; ++j)
        *reinterpret_cast<float2*>(&wo[(warp * RP + r) * D + j * 8 + 2 * qid]) =
            make_float2(acc[mt][j][2 * hh], acc[mt][j][2 * hh + 1]);
    }
  // named barrier over the consumer warps only (the producer waits at the block barriers below)
  asm volatile("bar.sync 1, %0;" ::"r"(CONSUMERS * 32));

  const int ct = threadIdx.x;  // 0 .. 127
  const bool single = nsplit_b == 1;
  float* so = p.ws_o + ((size_t(b) * p.Hkv + hk) * p.nsplit + s) * RP * D;
  float* sml = p.ws_ml + ((size_t(b) * p.Hkv + hk) * p.nsplit + s) * RP * 2;
  for (int e = ct; e < p.rows * D; e += CONSUMERS * 32) {
    const int r = e / D, d = e % D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < CONSUMERS; ++w) M = fmaxf(M, wml[(w * RP + r) * 2]);
    const float Mu = M == -INFINITY ? 0.f : M;
    float L = 0.f, O = 0.f;
#pragma unroll
    for (int w = 0; w < CONSUMERS; ++w) {
      const float wgt = ex2(wml[(w * RP + r) * 2] - Mu);
      L += wml[(w * RP + r) * 2 + 1] * wgt;
      O += wo[(w * RP + r) * D + d] * wgt;
    }
    if (single) {
      const int g = r / p.T, t = r % p.T, h = hk * p.G + g;
      const float val = L > 0.f ? O / L : 0.f;
      if (p.emit) {
        const size_t ro = (size_t(b) * p.Hq + h) * p.T + t;
        p.part_o[ro * D + d] = val;
        if (d == 0) p.part_lse[ro] = L > 0.f ? (M + __log2f(L)) * 0.69314718055994531f : -INFINITY;
      } else {
        reinterpret_cast<T*>(p.o)[b * p.o_st[0] + int64_t(h) * p.o_st[1] + int64_t(t) * p.o_st[2] + d] =
            from_f<T>(val);
      }
    } else {
      so[r * D + d] = O;
      if (d == 0) {
        sml[r * 2] = M;
        sml[r * 2 + 1] = L;
      }
    }
  }
  __syncthreads();  // (2)
  if (p.nsplit > 1 && nsplit_b > 1) {
    // ---------------------------------------------------------------- the last split of (b, hk) merges them all
    if (threadIdx.x == 0) {
      __threadfence();
      const int prev = atomicAdd(&p.ws_cnt[b * p.Hkv + hk], 1);
      s_last = prev == nsplit_b - 1;
      if (s_last) {
        p.ws_cnt[b * p.Hkv + hk] = 0;  // ready for the next call
        __threadfence();
      }
    }
    __syncthreads();  // (3)
    if (!s_last) return;
    const float* bo = p.ws_o + (size_t(b) * p.Hkv + hk) * p.nsplit * RP * D;
    const float* bml = p.ws_ml + (size_t(b) * p.Hkv + hk) * p.nsplit * RP * 2;
    for (int e = ct; e < p.rows * D; e += CONSUMERS * 32) {
      const int r = e / D, d = e % D;
      float M = -INFINITY;
      for (int w = 0; w < nsplit_b; ++w) M = fmaxf(M, __ldcg(&bml[(w * RP + r) * 2]));
      const float Mu = M == -INFINITY ? 0.f : M;
      float L = 0.f, O = 0.f;
      for (int w = 0; w < nsplit_b; ++w) {
        const float wgt = ex2(__ldcg(&bml[(w * RP + r) * 2]) - Mu);
        L += __ldcg(&bml[(w * RP + r) * 2 + 1]) * wgt;
        O += __ldcg(&bo[(size_t(w) * RP + r) * D + d]) * wgt;
      }
      const int g = r / p.T, t = r % p.T, h = hk * p.G + g;
      const float val = L > 0.f ? O / L : 0.f;
      if (p.emit) {
        const size_t ro = (size_t(b) * p.Hq + h) * p.T + t;
        p.part_o[ro * D + d] = val;
        if (d == 0) p.part_lse[ro] = L > 0.f ? (M + __log2f(L)) * 0.69314718055994531f : -INFINITY;
      } else {
        reinterpret_cast<T*>(p.o)[b * p.o_st[0] + int64_t(h) * p.o_st[1] + int64_t(t) * p.o_st[2] + d] =
            from_f<T>(val);
      }
    }
  }
  (void)ok;
}

// Merges R rank partials (normalised o, natural-log lse) row by row: one warp per row.
template <typename T>
__global__ void combine_kernel(const float* __restrict__ part_o, const float* __restrict__ part_lse, int R,
                               int rows, int Hq, int Tq, int D, void* o, int64_t o0, int64_t o1, int64_t o2) {
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  float M = -INFINITY;
  for (int r = 0; r < R; ++r) M = fmaxf(M, part_lse[size_t(r) * rows + row]);
  const float Mu = M == -INFINITY ? 0.f : M;
  float wsum = 0.f;
  for (int r = 0; r < R; ++r) wsum += __expf(part_lse[size_t(r) * rows + row] - Mu);
  const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
  const int t = row % Tq, h = (row / Tq) % Hq, b = row / (Tq * Hq);
  T* orow = reinterpret_cast<T*>(o) + b * o0 + int64_t(h) * o1 + int64_t(t) * o2;
  for (int d = lane; d < D; d += 32) {
    float x = 0.f;
    for (int r = 0; r < R; ++r)
      x += __expf(part_lse[size_t(r) * rows + row] - Mu) * part_o[(size_t(r) * rows + row) * D + d];
    orow[d] = from_f<T>(x * inv);
  }
}

}  // namespace decode
}  // namespace lb2
