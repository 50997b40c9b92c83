// Prefill / multi-row causal GQA attention on the 5th-generation tensor cores (tcgen05, TMEM accumulators).
//
// One CTA computes one 128-row query tile of one head: O = softmax(scale Q K^T + mask) V [* sigmoid(gate)].
// Warp roles (320 threads):
//   warps 0-7  softmax + epilogue: query row r = 32 (w % 4) + lane is TMEM lane r of S and O; warps w and w + 4
//              split the row's columns, exchanging the row max through shared memory. They read S with
//              tcgen05.ld, keep the running max / sum in base 2, write P (bf16/f16) into a double-buffered
//              128-byte swizzled shared tile, rescale the O row in TMEM only when the max grew by more than 2^8,
//              and finally normalise O, apply the optional sigmoid gate and store the row.
//   warp 8     TMA producer: Q once, then K and V tiles (128-byte swizzled boxes of 64 head-dim elements) into
//              two-stage rings.
//   warp 9     MMA issuer (one elected thread): S_j = Q K_j^T (SS operands, M=128, N=BN) into one of two S
//              buffers in TMEM, then O += P_{j-1} V_{j-1} (M=128, N=D, V read MN-major), so S_{j+1} runs while
//              the softmax warps work on S_j. Completion is signalled with tcgen05.commit on mbarriers.
// Causal is bottom-right (row t sees keys 0 .. N - T + t, chunkattn.py:359-365); a tile reads only the KV tiles
// up to its last row's limit, and only tiles crossing a row's limit are masked element by element. Every mbarrier
// wait is time-bounded; a wait that gives up sets the CTA's abort flag, every role drains what it issued, TMEM is
// released and the launch ends with the device status word set.
#pragma once

#include "common.cuh"

namespace lb2 {
namespace prefill {

constexpr int BM = 128;
constexpr int THREADS = 320;
constexpr int SOFTMAX_WARPS = 8;  // two per SM sub-partition: warps w and w + 4 share rows, split the columns
constexpr int PRODUCER_WARP = 8;
constexpr int MMA_WARP = 9;
constexpr int TMEM_COLS = 512;

template <int D>
struct Cfg {
  static constexpr int BN = D == 256 ? 64 : 128;
  static constexpr int QBYTES = BM * D * 2;
  static constexpr int KBYTES = BN * D * 2;  // one K tile; a V tile is the same size
  static constexpr int PBYTES = BM * BN * 2;
  static constexpr int STAGES = 2;
  static constexpr int Q_OFF = 0;
  static constexpr int K_OFF = Q_OFF + QBYTES;
  static constexpr int V_OFF = K_OFF + STAGES * KBYTES;
  static constexpr int P_OFF = V_OFF + STAGES * KBYTES;
  static constexpr int BAR_OFF = P_OFF + 2 * PBYTES;  // P double-buffered: P_j is written while PV_{j-1} runs
  // at least ~120 KB so that one CTA holds an SM (its TMEM allocation is all 512 columns)
  static constexpr int RED_OFF = BAR_OFF + 256;  // [2 halves][128 rows] fp32: a row's partial max / sum
  static constexpr int SMEM_RAW = RED_OFF + 2 * BM * 4;
  static constexpr int SMEM_BYTES = (SMEM_RAW < 120 * 1024 ? 120 * 1024 : SMEM_RAW) + 1024;
  static constexpr int S_COL = 0;       // S buffers at columns [0, BN) and [BN, 2 BN)
  static constexpr int O_COL = 2 * BN;  // O at [2 BN, 2 BN + D)
  static_assert(O_COL + D <= TMEM_COLS, "TMEM budget");
  static_assert(SMEM_BYTES <= 232448, "shared memory budget");
};

struct Params {
  void* o;
  int64_t o_st[3];
  const void* gate;
  int64_t g_st[3];
  const uint8_t* mask;
  int64_t m_st[2];
  int B, Hq, Hkv, T, N, G;
  int mask_kind;
  int mtiles;  // ceil(T / BM)
  float scale_log2;
};

// ---------------------------------------------------------------------------------------------- tcgen05 helpers

// Shared-memory matrix descriptor (sm100 format): start, leading / stride byte offsets (16-byte units),
// version 1, 128-byte swizzle.
__device__ __forceinline__ uint64_t sdesc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= uint64_t((addr >> 4) & 0x3FFFu);
  d |= uint64_t((lbo >> 4) & 0x3FFFu) << 16;
  d |= uint64_t((sbo >> 4) & 0x3FFFu) << 32;
  d |= uint64_t(1) << 46;
  d |= uint64_t(2) << 61;
  return d;
}

// Instruction descriptor for kind::f16: fp32 accumulate, A/B bf16 (ab = 1) or f16 (ab = 0), majors (0 = K-major,
// 1 = MN-major), M x N.
__host__ __device__ constexpr uint32_t idesc_f16(int ab, int a_mn, int b_mn, int M, int N) {
  return (1u << 4) | (uint32_t(ab) << 7) | (uint32_t(ab) << 10) | (uint32_t(a_mn) << 15) | (uint32_t(b_mn) << 16) |
         (uint32_t(N >> 3) << 17) | (uint32_t(M >> 4) << 24);
}

__device__ __forceinline__ void umma_ss(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc));
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
  uint32_t* r = reinterpret_cast<uint32_t*>(v);
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,"
      "%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float* v) {
  const uint32_t* r = reinterpret_cast<const uint32_t*>(v);
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
      "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ float ex2f(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Number of BN-key tiles query tile mt reads.
template <int D>
__device__ __forceinline__ int kv_tiles(const Params& p, int mt) {
  constexpr int BN = Cfg<D>::BN;
  int last = p.N;  // keys [0, last) may be visible to some row of the tile
  if (p.mask_kind == LB2_MASK_CAUSAL) {
    const int rmax = min(p.T, (mt + 1) * BM) - 1;
    last = min(p.N, p.N - p.T + rmax + 1);
  }
  return last <= 0 ? 0 : (last + BN - 1) / BN;
}

template <typename T, int D>
__global__ void __launch_bounds__(THREADS, 1) fmha_kernel(const __grid_constant__ CUtensorMap qmap,
                                                           const __grid_constant__ CUtensorMap kmap,
                                                           const __grid_constant__ CUtensorMap vmap,
                                                           const Params p) {
  using C = Cfg<D>;
  constexpr int BN = C::BN;
  constexpr int AB = std::is_same<T, __nv_bfloat16>::value ? 1 : 0;
  constexpr uint32_t IDESC_S = idesc_f16(AB, 0, 0, BM, BN);
  constexpr uint32_t IDESC_PV = idesc_f16(AB, 0, 1, BM, D);

  // Heaviest query tiles first (causal tiles late in the sequence read the most keys); heads vary fastest so that
  // neighbouring CTAs share their KV head's tiles in L2.
  const int bh = blockIdx.x % (p.B * p.Hq);
  const int mt = p.mtiles - 1 - int(blockIdx.x / (p.B * p.Hq));
  const int b = bh / p.Hq, h = bh % p.Hq, hk = h / p.G;
  const int r0 = mt * BM;
  const int ntiles = kv_tiles<D>(p, mt);

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + C::BAR_OFF);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;   // [2]
  uint64_t* k_empty = bars + 3;  // [2]
  uint64_t* v_full = bars + 5;   // [2]
  uint64_t* v_empty = bars + 7;  // [2]
  uint64_t* s_full = bars + 9;   // [2]
  uint64_t* s_free = bars + 11;  // [2]
  uint64_t* p_full = bars + 13;  // [2] P_j written into buffer j & 1
  uint64_t* o_done = bars + 15;  // [2] PV_j complete, committed to o_done[j & 1]
  uint64_t* drain = bars + 17;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 18);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 19);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], SOFTMAX_WARPS * 32);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&p_full[i], SOFTMAX_WARPS * 32);
      mbar_init(&o_done[i], 1);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == MMA_WARP) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == PRODUCER_WARP) {
    // ------------------------------------------------------------------------------------ TMA producer
    if (lane == 0 && ntiles > 0) {
      prefetch_tensormap(&qmap);
      prefetch_tensormap(&kmap);
      prefetch_tensormap(&vmap);
      mbar_arrive_expect_tx(q_full, C::QBYTES);
#pragma unroll
      for (int db = 0; db < D / 64; ++db)
        tma_load_4d(sm + C::Q_OFF + db * BM * 128, &qmap, db * 64, r0, h, b, q_full);
      int issued = 0;
      for (int j = 0; j < ntiles && !*abort_flag; ++j) {
        const int st = j & 1;
        if (j >= 2 && !mbar_wait(&k_empty[st], ((j >> 1) - 1) & 1, 11)) {
          *abort_flag = 1;
          break;
        }
        mbar_arrive_expect_tx(&k_full[st], C::KBYTES);
#pragma unroll
        for (int db = 0; db < D / 64; ++db)
          tma_load_4d(sm + C::K_OFF + st * C::KBYTES + db * BN * 128, &kmap, db * 64, j * BN, hk, b, &k_full[st]);
        if (j >= 2 && !mbar_wait(&v_empty[st], ((j >> 1) - 1) & 1, 12)) {
          *abort_flag = 1;
          issued = 2 * j + 1;
          break;
        }
        mbar_arrive_expect_tx(&v_full[st], C::KBYTES);
#pragma unroll
        for (int db = 0; db < D / 64; ++db)
          tma_load_4d(sm + C::V_OFF + st * C::KBYTES + db * BN * 128, &vmap, db * 64, j * BN, hk, b, &v_full[st]);
        issued = 2 * j + 2;
      }
      // Drain: every load issued has landed before the CTA may finish (already true on the normal path).
      mbar_wait(q_full, 0, 13);
      for (int u = max(0, issued - 4); u < issued; ++u) {
        const int j = u >> 1;
        mbar_wait((u & 1) ? &v_full[j & 1] : &k_full[j & 1], (j >> 1) & 1, 14);
      }
    }
  } else if (warp == MMA_WARP) {
    // ------------------------------------------------------------------------------------ MMA issuer
    if (ntiles > 0) {
      const bool leader = elect_one();
      const uint32_t q_addr = smem_u32(sm + C::Q_OFF);
      const uint32_t p_addr = smem_u32(sm + C::P_OFF);
      bool ok = !leader || mbar_wait(q_full, 0, 21);
      int pv_done = 0;
      auto issue_pv = [&](int i) -> bool {
        const int st = i & 1;
        if (!mbar_wait(&v_full[st], (i >> 1) & 1, 22)) return false;
        if (!mbar_wait(&p_full[st], (i >> 1) & 1, 23)) return false;
        tc_fence_after();
        const uint32_t v_addr = smem_u32(sm + C::V_OFF + st * C::KBYTES);
        const uint32_t pb = p_addr + st * C::PBYTES;
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk) {
          const uint64_t a = sdesc(pb + (kk >> 2) * BM * 128 + (kk & 3) * 32, 16, 1024);
          const uint64_t bd = sdesc(v_addr + kk * 16 * 128, BN * 128, 1024);
          umma_ss(tmem + C::O_COL, a, bd, IDESC_PV, (i > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&o_done[st]);
        umma_commit(&v_empty[st]);
        return true;
      };
      if (leader) {
        for (int j = 0; j < ntiles && ok; ++j) {
          const int st = j & 1;
          if (!mbar_wait(&k_full[st], (j >> 1) & 1, 24) || (j >= 2 && !mbar_wait(&s_free[st], ((j >> 1) - 1) & 1, 25))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t k_addr = smem_u32(sm + C::K_OFF + st * C::KBYTES);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint64_t a = sdesc(q_addr + (kk >> 2) * BM * 128 + (kk & 3) * 32, 16, 1024);
            const uint64_t bd = sdesc(k_addr + (kk >> 2) * BN * 128 + (kk & 3) * 32, 16, 1024);
            umma_ss(tmem + C::S_COL + st * BN, a, bd, IDESC_S, kk > 0 ? 1u : 0u);
          }
          umma_commit(&s_full[st]);
          umma_commit(&k_empty[st]);
          if (j >= 1) {
            if (!issue_pv(j - 1)) {
              ok = false;
              break;
            }
            pv_done = j;
          }
        }
        if (ok && pv_done < ntiles) ok = issue_pv(ntiles - 1);
        if (!ok) *abort_flag = 1;
        // Drain: everything this thread issued has completed before TMEM may be released.
        umma_commit(drain);
        mbar_wait(drain, 0, 26);
      }
      __syncwarp();
    }
  } else {
    // ------------------------------------------------------------------------------------ softmax warps
    constexpr int HC = BN / 2;  // S columns a thread owns
    constexpr int HD = D / 2;   // O columns a thread owns
    const int r = 32 * (warp & 3) + lane;  // row in the tile == TMEM lane
    const int hf = warp >> 2;              // which half of the columns
    const int row = r0 + r;
    const uint32_t lane_base = tmem + (uint32_t(32 * (warp & 3)) << 16);
    const uint32_t pair_bar = 2 + (warp & 3);  // named barrier of warps w and w + 4 (ids 2..5)
    float* red = reinterpret_cast<float*>(sm + C::RED_OFF);
    const int lim = p.mask_kind == LB2_MASK_CAUSAL ? p.N - p.T + row : p.N - 1;
    const uint8_t* mrow = (p.mask_kind == LB2_MASK_ARRAY && row < p.T) ? p.mask + int64_t(row) * p.m_st[0] : nullptr;
    float m_run = -INFINITY, l_run = 0.f;
    uint8_t* prow = sm + C::P_OFF;
    bool ok = true;
    for (int j = 0; j < ntiles; ++j) {
      const int st = j & 1;
      // A failed wait never leaves a warp alone at a barrier: the decision to stop is made warp-uniform before
      // the warp-collective TMEM loads and pair-uniform at the max exchange (bar.red.and), where both warps of a
      // row pair leave the loop together.
      bool okj = ok && !*abort_flag && mbar_wait(&s_full[st], (j >> 1) & 1, 31);
      okj = __all_sync(0xffffffffu, okj);
      float s[HC];
      if (okj) {
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < HC; c += 32) tmem_ld32(lane_base + C::S_COL + st * BN + hf * HC + c, s + c);
        tmem_wait_ld();
        tc_fence_before();
        mbar_arrive(&s_free[st]);
      } else {
#pragma unroll
        for (int c = 0; c < HC; ++c) s[c] = -INFINITY;
      }

      const int key0 = j * BN + hf * HC;
      const bool full_tile = j * BN + BN - 1 <= lim && j * BN + BN <= p.N && !mrow;
      float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
      if (full_tile) {
#pragma unroll
        for (int c = 0; c < HC; ++c) mx4[c & 3] = fmaxf(mx4[c & 3], s[c]);
      } else {
#pragma unroll
        for (int c = 0; c < HC; ++c) {
          const int key = key0 + c;
          bool vis = key <= lim && key < p.N;
          if (mrow && vis) vis = mrow[int64_t(key) * p.m_st[1]] != 0;
          s[c] = vis ? s[c] : -INFINITY;
          mx4[c & 3] = fmaxf(mx4[c & 3], s[c]);
        }
      }
      float tmax = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3]));  // raw score units (scale > 0)
      red[hf * BM + r] = tmax;
      uint32_t pair_ok;
      asm volatile(
          "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\t"
          "bar.red.and.pred q, %2, 64, p;\n\tselp.u32 %0, 1, 0, q;\n\t}"
          : "=r"(pair_ok)
          : "r"(uint32_t(okj)), "r"(pair_bar)
          : "memory");
      tmax = fmaxf(tmax, red[(1 - hf) * BM + r]);
      asm volatile("bar.sync %0, 64;" ::"r"(pair_bar));  // both read before the next tile rewrites
      if (!pair_ok) {
        ok = false;
        break;
      }
      const float tmax2 = tmax * p.scale_log2;  // base-2 units
      // The running max moves only when it grew by more than 2^8 (fp32 O and the 16-bit P absorb the rest); O is
      // rescaled in TMEM then, after PV_{j-1} has completed. tcgen05.ld / st are warp-collective, so a warp rescales
      // when any of its rows must (factor 1 for the others); both warps of a row pair decide alike.
      const bool move = tmax2 > m_run + 8.f;
      const float factor = move ? ex2f(m_run - tmax2) : 1.f;
      if (__any_sync(0xffffffffu, move && j > 0 && l_run > 0.f)) {
        if (!mbar_wait(&o_done[(j - 1) & 1], ((j - 1) >> 1) & 1, 32)) ok = false;
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < HD; c += 32) {
          float ov[32];
          tmem_ld32(lane_base + C::O_COL + hf * HD + c, ov);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) ov[e] *= factor;
          tmem_st32(lane_base + C::O_COL + hf * HD + c, ov);
        }
        tmem_wait_st();
      }
      if (move) {
        l_run *= factor;
        m_run = tmax2;
      }
      // P buffer j & 1 was last read by PV_{j-2}.
      if (j >= 2 && !mbar_wait(&o_done[j & 1], ((j >> 1) - 1) & 1, 34)) ok = false;
      const float nm = m_run == -INFINITY ? 0.f : -m_run;
      uint8_t* pbuf = prow + (j & 1) * C::PBYTES;
      float ls4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int c = 0; c < HC; c += 8) {
        float e[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          e[u] = ex2f(fmaf(s[c + u], p.scale_log2, nm));
          ls4[u & 3] += e[u];
        }
        uint4 pk;
        pk.x = pack2<T>(e[0], e[1]);
        pk.y = pack2<T>(e[2], e[3]);
        pk.z = pack2<T>(e[4], e[5]);
        pk.w = pack2<T>(e[6], e[7]);
        const int cc = hf * HC + c;
        const int box = cc >> 6, ch = (cc & 63) >> 3;
        *reinterpret_cast<uint4*>(pbuf + box * BM * 128 + r * 128 + ((ch ^ (r & 7)) << 4)) = pk;
      }
      l_run += (ls4[0] + ls4[1]) + (ls4[2] + ls4[3]);
      fence_proxy_async_shared();
      tc_fence_before();
      mbar_arrive(&p_full[j & 1]);
    }
    if (ok && ntiles > 0) {
      if (!mbar_wait(&o_done[(ntiles - 1) & 1], ((ntiles - 1) >> 1) & 1, 33)) ok = false;
      tc_fence_after();
    }
    // ---------------------------------------------------------------------------------- epilogue
    // Warp-uniform from here on: every lane takes part in the TMEM loads, only rows inside T store. The row sum is
    // the two halves' partial sums.
    ok = __all_sync(0xffffffffu, ok);
    red[hf * BM + r] = l_run;
    asm volatile("bar.sync %0, 64;" ::"r"(pair_bar));
    const float l_tot = l_run + red[(1 - hf) * BM + r];
    const bool have_o = ntiles > 0 && ok;
    const bool store = row < p.T;
    T* orow = reinterpret_cast<T*>(p.o) + b * p.o_st[0] + int64_t(h) * p.o_st[1] + int64_t(row) * p.o_st[2] + hf * HD;
    const T* grow = p.gate ? reinterpret_cast<const T*>(p.gate) + b * p.g_st[0] + int64_t(h) * p.g_st[1] +
                                 int64_t(row) * p.g_st[2] + hf * HD
                           : nullptr;
    const float inv = (have_o && l_tot > 0.f) ? 1.f / l_tot : 0.f;
#pragma unroll 1
    for (int c = 0; c < HD; c += 32) {
      float ov[32];
      if (have_o) {
        tmem_ld32(lane_base + C::O_COL + hf * HD + c, ov);
        tmem_wait_ld();
      } else {
#pragma unroll
        for (int e = 0; e < 32; ++e) ov[e] = 0.f;
      }
      if (!store) continue;
#pragma unroll
      for (int e = 0; e < 32; e += 8) {
        float x[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) x[u] = ov[e + u] * inv;
        if (grow) {
          const uint4 gv = *reinterpret_cast<const uint4*>(grow + c + e);
          const T* gh = reinterpret_cast<const T*>(&gv);
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            const float z = to_f<T>(gh[u]);
            x[u] = x[u] / (1.f + __expf(-z));
          }
        }
        uint4 pk;
        pk.x = pack2<T>(x[0], x[1]);
        pk.y = pack2<T>(x[2], x[3]);
        pk.z = pack2<T>(x[4], x[5]);
        pk.w = pack2<T>(x[6], x[7]);
        *reinterpret_cast<uint4*>(orow + c + e) = pk;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == MMA_WARP) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS));
  }
}

}  // namespace prefill
}  // namespace lb2
