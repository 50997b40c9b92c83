// Split-KV decode attention for a few query rows over a long KV cache (HBM-bandwidth bound).
//
// Persistent kernel: one CTA per SM walks a static round-robin share of equal-sized work units, a unit being
// (sequence b, one `split`-key range of it, KV head hk). The G*T query rows sharing KV head hk are folded into
// 16-row tiles (the fold of foldattn.py:230-259), so every K/V byte is read from HBM once per call.
// A producer warp streams, unit after unit without a pause, the unit's folded Q tile (a 2-slot ring) and its
// 64-key K and V tiles (a STAGES-deep ring), all with TMA into 128-byte swizzled boxes of 64 head-dim elements;
// four consumer warps each take 16 of a tile's 64 keys and run S = Q K^T and O += P V on mma.sync m16n8k16 (fp32
// accumulate) with an fp32 online softmax in base 2. At a unit's end each consumer warp drops its partial (max, sum,
// unnormalised O) into shared memory and goes on to the next unit while the producer keeps streaming; a merger warp
// folds the four into the unit's partial in the workspace; split_combine_kernel, launched right behind as a
// programmatic dependent, merges the splits of each (b, hk, row) by log-sum-exp -- the combine of foldattn_merge
// (foldattn.py:188-211) and CpuAttn's range merge (cpu_ext/cpu_kern.cpp:607-628).
#pragma once

#include "common.cuh"

namespace lb2 {
namespace decode {

constexpr int BK = 64;         // keys per tile
constexpr int CONSUMERS = 4;   // consumer warps, 16 keys of each tile apiece
constexpr int PRODUCER = CONSUMERS;     // warp index of the TMA producer
constexpr int MERGER = CONSUMERS + 1;   // warp index of the partial merger
constexpr int THREADS = (CONSUMERS + 2) * 32;
constexpr int MAX_B = 1024;    // sequences a call (the per-CTA unit table)

template <int D, int MT>
struct Cfg {
  static constexpr int RP = MT * 16;                          // folded rows, padded
  static constexpr int STAGES = D == 64 ? 6 : D == 128 ? 4 : 2;
  static constexpr int TILE_BYTES = BK * D * 2;               // one K (or V) tile, bf16/f16
  static constexpr int STAGE_BYTES = 2 * TILE_BYTES;          // K + V
  static constexpr int RING_BYTES = STAGES * STAGE_BYTES;
  static constexpr int QSLOT = (D / 64) * RP * 128;           // one folded Q tile
  static constexpr int Q_OFF = RING_BYTES;
  static constexpr int PART_OFF = Q_OFF + 2 * QSLOT;         // [CONSUMERS][RP][D] O + [CONSUMERS][RP][2] (m, l)
  static constexpr int PART_BYTES = CONSUMERS * RP * D * 4 + CONSUMERS * RP * 2 * 4;
  static constexpr int PREFIX_OFF = PART_OFF + PART_BYTES;   // [MAX_B + 1] ints
  static constexpr int LENS_OFF = PREFIX_OFF + (MAX_B + 1) * 4;  // [MAX_B] ints
  static constexpr int META_OFF = LENS_OFF + MAX_B * 4;
  static constexpr int PMETA_OFF = META_OFF + 2 * 32;        // (b, hk, s, nsplit_b) of the unit in the part area
  static constexpr int BAR_OFF = (PMETA_OFF + 16 + 15) / 16 * 16;
  static constexpr int SMEM_BYTES = BAR_OFF + 256 + 1024 /*align*/;
  static_assert(SMEM_BYTES <= 232448, "shared memory budget");
};

struct Params {
  void* o;
  int64_t o_st[3];
  float* part_o;    // emit mode: normalised fp32 o, [B, Hq, T, D] contiguous
  float* part_lse;  // emit mode: natural-log lse, [B, Hq, T]
  const int32_t* kv_len;
  float* ws_o;      // [B, Hkv, nsplit, rows, D] unnormalised partial O of each split
  float* ws_ml;     // [B, Hkv, nsplit, rows, 2] (max in log2 units, sum)
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

// Unit u of the call -> (b, s, hk) through the prefix table of per-sequence split counts.
__device__ __forceinline__ void unit_coords(const int* prefix, int B, int Hkv, int u, int& b, int& s, int& hk) {
  const int pidx = u / Hkv;
  hk = u - pidx * Hkv;
  int lo = 0, hi = B;  // largest b with prefix[b] <= pidx
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (prefix[mid] <= pidx) lo = mid; else hi = mid;
  }
  b = lo;
  s = pidx - prefix[b];
}

template <typename T, int D, int MT>
__global__ void __launch_bounds__(THREADS, 1) decode_kernel(const __grid_constant__ CUtensorMap qmap,
                                                             const __grid_constant__ CUtensorMap kmap,
                                                             const __grid_constant__ CUtensorMap vmap,
                                                             const Params p) {
  using C = Cfg<D, MT>;
  constexpr int STAGES = C::STAGES;
  constexpr int RP = C::RP;
  constexpr int ND = D / 8;   // 8-wide head-dim tiles of the output
  constexpr int KD = D / 16;  // 16-wide k-steps of Q K^T

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  int* prefix = reinterpret_cast<int*>(sm + C::PREFIX_OFF);
  int* meta = reinterpret_cast<int*>(sm + C::META_OFF);  // [2 slots][8]: b, hk, s, n0, n1, len
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + C::BAR_OFF);
  uint64_t* empty = full + STAGES;
  uint64_t* q_full = empty + STAGES;
  uint64_t* q_empty = q_full + 2;
  uint64_t* part_full = q_empty + 2;   // the four consumer warps' partials of a unit are in the part area
  uint64_t* part_empty = part_full + 1;  // the merger has read them
  int* pmeta = reinterpret_cast<int*>(sm + C::PMETA_OFF);
  float* pwo = reinterpret_cast<float*>(sm + C::PART_OFF);  // [CONSUMERS][RP][D]
  float* pwml = pwo + CONSUMERS * RP * D;                  // [CONSUMERS][RP][2]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int* lens = reinterpret_cast<int*>(sm + C::LENS_OFF);
  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], CONSUMERS);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], CONSUMERS);
    }
    mbar_init(part_full, CONSUMERS);
    mbar_init(part_empty, 1);
    fence_barrier_init();
  }
  // per-sequence lengths and split counts (loaded in parallel), then warp 0 scans the counts into a prefix table
  for (int b = threadIdx.x; b < p.B; b += THREADS) {
    const int len = p.kv_len ? min(max(p.kv_len[b], 0), p.N) : p.N;
    lens[b] = len;
    prefix[b + 1] = max(1, (len + p.split - 1) / p.split);
  }
  __syncthreads();
  if (warp == 0) {
    int run = 0;
    for (int base = 0; base < p.B; base += 32) {
      int x = base + lane < p.B ? prefix[base + lane + 1] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
      }
      if (base + lane < p.B) prefix[base + lane + 1] = run + x;
      run += __shfl_sync(0xffffffffu, x, 31);
    }
    if (lane == 0) prefix[0] = 0;
  }
  __syncthreads();
  const int units = prefix[p.B] * p.Hkv;
  // The split combine (launched as this grid's programmatic dependent) may start its prologue now; it waits for
  // this grid's completion before reading any partial.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  // ------------------------------------------------------------------ producer warp: Q tiles and K/V tiles
  if (warp == PRODUCER) {
    if (lane == 0) {
      prefetch_tensormap(&qmap);
      prefetch_tensormap(&kmap);
      prefetch_tensormap(&vmap);
      int gt = 0, uc = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < units && ok; u += gridDim.x, ++uc) {
        int b, s, hk;
        unit_coords(prefix, p.B, p.Hkv, u, b, s, hk);
        const int len = lens[b];
        const int n0 = s * p.split, n1 = min(len, n0 + p.split);
        const int ntiles = n1 > n0 ? (n1 - n0 + BK - 1) / BK : 0;
        const int qs = uc & 1;
        if (uc >= 2 && !mbar_wait(&q_empty[qs], ((uc >> 1) - 1) & 1, 1)) break;
        int* m = meta + qs * 8;
        m[0] = b; m[1] = hk; m[2] = s; m[3] = n0; m[4] = n1; m[5] = len;
        mbar_arrive_expect_tx(&q_full[qs], (D / 64) * p.rows * 128);
#pragma unroll
        for (int db = 0; db < D / 64; ++db)
          tma_load_4d(sm + C::Q_OFF + qs * C::QSLOT + db * RP * 128, &qmap, db * 64, 0, hk * p.G, b, &q_full[qs]);
        for (int i = 0; i < ntiles; ++i, ++gt) {
          const int st = gt % STAGES;
          if (gt >= STAGES && !mbar_wait(&empty[st], ((gt / STAGES) - 1) & 1, 2)) {
            ok = false;
            break;
          }
          uint8_t* kt = sm + st * C::STAGE_BYTES;
          uint8_t* vt = kt + C::TILE_BYTES;
          mbar_arrive_expect_tx(&full[st], C::STAGE_BYTES);
          const int key0 = n0 + i * BK;
#pragma unroll
          for (int db = 0; db < D / 64; ++db) {
            tma_load_4d(kt + db * BK * 128, &kmap, db * 64, key0, hk, b, &full[st]);
            tma_load_4d(vt + db * BK * 128, &vmap, db * 64, key0, hk, b, &full[st]);
          }
        }
      }
      // Drain: the last loads issued have landed before the CTA may finish (normally already consumed).
      for (int g2 = max(0, gt - STAGES); g2 < gt; ++g2) mbar_wait(&full[g2 % STAGES], (g2 / STAGES) & 1, 3);
      for (int q2 = max(0, uc - 2); q2 < uc; ++q2) mbar_wait(&q_full[q2 & 1], (q2 >> 1) & 1, 4);
    }
    return;  // the producer takes part in no block-wide barrier after the setup
  }

  // ------------------------------------------------------------------ merger warp: one partial per unit
  if (warp == MERGER) {
    int uc = 0;
    for (int u = blockIdx.x; u < units; u += gridDim.x, ++uc) {
      if (!mbar_wait(part_full, uc & 1, 7)) break;
      const int b = pmeta[0], hk = pmeta[1], s = pmeta[2];
      const size_t part = ((size_t(b) * p.Hkv + hk) * p.nsplit + s) * p.rows;
      for (int e = lane; e < p.rows * D; e += 32) {
        const int r = e / D, d = e % D;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < CONSUMERS; ++w) M = fmaxf(M, pwml[(w * RP + r) * 2]);
        const float Mu = M == -INFINITY ? 0.f : M;
        float L = 0.f, O = 0.f;
#pragma unroll
        for (int w = 0; w < CONSUMERS; ++w) {
          const float wgt = ex2(pwml[(w * RP + r) * 2] - Mu);
          L += pwml[(w * RP + r) * 2 + 1] * wgt;
          O += pwo[(w * RP + r) * D + d] * wgt;
        }
        p.ws_o[(part + r) * D + d] = O;
        if (d == 0) *reinterpret_cast<float2*>(&p.ws_ml[(part + r) * 2]) = make_float2(M, L);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(part_empty);
    }
    return;
  }

  // ------------------------------------------------------------------ consumer warps
  const int quad = lane >> 2, qid = lane & 3;
  int gt = 0, uc = 0;
  bool ok = true;
  for (int u = blockIdx.x; u < units && ok; u += gridDim.x, ++uc) {
    const int qs = uc & 1;
    // No named barrier joins the consumer warps: a warp whose (time-bounded) wait gives up leaves the loop, the
    // producer then stops at its own bounded waits, and the other warps' waits end the same way.
    if (!mbar_wait(&q_full[qs], (uc >> 1) & 1, 5)) break;
    const int* m = meta + qs * 8;
    const int b = m[0], hk = m[1], s = m[2], n0 = m[3], n1 = m[4], len = m[5];
    const int ntiles = n1 > n0 ? (n1 - n0 + BK - 1) / BK : 0;
    const int nsplit_b = max(1, (len + p.split - 1) / p.split);
    // Q fragments (A operand, row-major 16 x 16 a k-step) from the swizzled Q tile; rows are folded (g, t).
    uint32_t qa[MT][KD][4];
    const uint32_t qaddr = smem_u32(sm + C::Q_OFF + qs * C::QSLOT);
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int kk = 0; kk < KD; ++kk) {
        const int r = mt * 16 + (lane & 15), c = kk * 2 + (lane >> 4);
        ldsm_x4(qaddr + (c / 8) * RP * 128 + swz(0, r, c % 8), qa[mt][kk]);
      }
    __syncwarp();
    if (lane == 0) mbar_arrive(&q_empty[qs]);

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

    for (int i = 0; i < ntiles; ++i, ++gt) {
      const int st = gt % STAGES;
      if (!mbar_wait(&full[st], (gt / STAGES) & 1, 6)) {
        ok = false;
        break;
      }
      const uint32_t kt = smem_u32(sm + st * C::STAGE_BYTES);
      const uint32_t vt = kt + C::TILE_BYTES;
      const int kbase = n0 + i * BK + warp * 16;  // this warp's first key
      // Rows of this warp's 16 keys past the sequence (capacity padding may hold anything): zero V there so that
      // P = 0 never meets a non-finite value.
      const int nvalid = min(16, max(0, n1 - kbase));
      if (nvalid < 16) {
        uint8_t* vrow = sm + st * C::STAGE_BYTES + C::TILE_BYTES;
        for (int e = lane; e < (16 - nvalid) * (D / 8); e += 32) {
          const int r = warp * 16 + nvalid + e / (D / 8), c = e % (D / 8);
          *reinterpret_cast<uint4*>(vrow + swz(c / 8, r, c % 8)) = make_uint4(0, 0, 0, 0);
        }
        __syncwarp();
      }
      float sc[MT][2][4];
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) sc[mt][nt][0] = sc[mt][nt][1] = sc[mt][nt][2] = sc[mt][nt][3] = 0.f;
#pragma unroll
      for (int kk = 0; kk < KD; ++kk) {
        uint32_t kb[4];
        const int r = warp * 16 + (lane & 7) + 8 * (lane >> 4);
        const int c = kk * 2 + ((lane >> 3) & 1);
        ldsm_x4(kt + swz(c / 8, r, c % 8), kb);
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
          mma16816<T>(sc[mt][0], qa[mt][kk], kb[0], kb[1]);
          mma16816<T>(sc[mt][1], qa[mt][kk], kb[2], kb[3]);
        }
      }
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

    // -------------------------------------------------------------- unit epilogue: this warp's partial
    // Each warp drops its (max, sum, unnormalised O) for the unit's rows into the part area and goes on to the next
    // unit while the producer keeps streaming; the merger warp folds the four into the unit's one partial in the
    // workspace (split_combine_kernel then merges the splits of each (b, hk, row)).
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        l_run[mt][hh] += __shfl_xor_sync(0xffffffffu, l_run[mt][hh], 1);
        l_run[mt][hh] += __shfl_xor_sync(0xffffffffu, l_run[mt][hh], 2);
      }
    if (uc >= 1 && !mbar_wait(part_empty, (uc - 1) & 1, 8)) break;  // the merger has read the previous unit's
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int r = mt * 16 + quad + 8 * hh;
        if (r >= p.rows) continue;
        if (qid == 0) {
          pwml[(warp * RP + r) * 2] = m_run[mt][hh];
          pwml[(warp * RP + r) * 2 + 1] = l_run[mt][hh];
        }
#pragma unroll
        for (int j = 0; j < ND; ++j)
          *reinterpret_cast<float2*>(&pwo[(warp * RP + r) * D + j * 8 + 2 * qid]) =
              make_float2(acc[mt][j][2 * hh], acc[mt][j][2 * hh + 1]);
      }
    if (warp == 0 && lane == 0) {
      pmeta[0] = b;
      pmeta[1] = hk;
      pmeta[2] = s;
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(part_full);
  }
}

// Merges the splits of every (b, hk, folded row) of a decode call: one warp per row, lanes across the head dim
// (float4 loads), several splits' loads in flight at once. Rows of single-split sequences were written by the
// decode kernel and are skipped.
template <typename T, int D>
__global__ void __launch_bounds__(256) split_combine_kernel(const Params p) {
  // One block per (b, hk, folded row): the row's nsplit_b partials (one per split). Pass 1: every (max, sum) pair, the
  // block max and the total sum, and each partial's weight in shared memory. Pass 2: threads split the head dim into
  // float4 groups and the partials into interleaved sets, so every thread has its few loads in flight at once; the
  // sets are summed in shared memory.
  asm volatile("griddepcontrol.wait;" ::: "memory");  // the decode grid has completed and its writes are visible
  constexpr int CG = D / 4;          // float4 column groups
  constexpr int PG = 256 / CG;       // partial sets
  __shared__ float wts[2 * D];  // a sequence has at most 2 D splits
  __shared__ float red[PG][D];
  __shared__ float s_red[8];
  const int r = blockIdx.x % p.rows;
  const int bh = blockIdx.x / p.rows;
  const int b = bh / p.Hkv, hk = bh % p.Hkv;
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const int len = p.kv_len ? min(max(p.kv_len[b], 0), p.N) : p.N;
  const int nparts = max(1, (len + p.split - 1) / p.split);
  const size_t base = size_t(bh) * p.nsplit * p.rows;  // partial index of (b, hk, split 0, row 0)
  // pass 1
  float M = -INFINITY;
  for (int q = tid; q < nparts; q += 256) {
    const float m = __ldcg(&p.ws_ml[(base + size_t(q) * p.rows + r) * 2]);
    wts[q] = m;
    M = fmaxf(M, m);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
  if (lane == 0) s_red[w] = M;
  __syncthreads();
  M = s_red[0];
#pragma unroll
  for (int i = 1; i < 8; ++i) M = fmaxf(M, s_red[i]);
  const float Mu = M == -INFINITY ? 0.f : M;
  __syncthreads();
  float L = 0.f;
  for (int q = tid; q < nparts; q += 256) {
    const float wq = ex2(wts[q] - Mu);
    wts[q] = wq;
    L += wq * __ldcg(&p.ws_ml[(base + size_t(q) * p.rows + r) * 2 + 1]);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
  if (lane == 0) s_red[w] = L;
  __syncthreads();
  L = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) L += s_red[i];
  // pass 2
  const int cg = tid % CG, pg = tid / CG;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 8
  for (int q = pg; q < nparts; q += PG) {
    const float wq = wts[q];
    const float4 x = __ldcg(reinterpret_cast<const float4*>(p.ws_o + (base + size_t(q) * p.rows + r) * D) + cg);
    acc.x += wq * x.x;
    acc.y += wq * x.y;
    acc.z += wq * x.z;
    acc.w += wq * x.w;
  }
  *reinterpret_cast<float4*>(&red[pg][cg * 4]) = acc;
  __syncthreads();
  if (tid < D) {
    float o = 0.f;
#pragma unroll
    for (int i = 0; i < PG; ++i) o += red[i][tid];
    const float val = L > 0.f ? o / L : 0.f;
    const int g = r / p.T, t = r % p.T, h = hk * p.G + g;
    if (p.emit) {
      const size_t ro = (size_t(b) * p.Hq + h) * p.T + t;
      p.part_o[ro * D + tid] = val;
      if (tid == 0) p.part_lse[ro] = L > 0.f ? (M + __log2f(L)) * 0.69314718055994531f : -INFINITY;
    } else {
      reinterpret_cast<T*>(p.o)[b * p.o_st[0] + int64_t(h) * p.o_st[1] + int64_t(t) * p.o_st[2] + tid] =
          from_f<T>(val);
    }
  }
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
