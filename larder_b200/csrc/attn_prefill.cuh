// Prefill / multi-row causal GQA attention on the 5th-generation tensor cores (tcgen05, TMEM accumulators).
//
// One CTA computes one 128-row query tile of one head: O = softmax(scale Q K^T + mask) V [* sigmoid(gate)].
// Warp roles (320 threads):
//   warps 0-7  softmax + epilogue: query row r = 32 (w % 4) + lane is TMEM lane r of S and O; warps w and w + 4
//              split the row's columns, exchanging the row max through shared memory. They read S_j with
//              tcgen05.ld, keep the running max / sum in base 2, write P_j (bf16/f16, key pairs packed a column) into
//              TMEM buffer j % 2 once PV_{j-2} has finished reading it, rescale the O row in TMEM only when the max
//              grew by more than 2^8, and finally normalise O, apply the optional sigmoid gate and store the row.
//   warp 8     TMA producers: lane 0 loads Q once, then K tiles into a three-stage ring; lane 1 loads V tiles into
//              a two-stage ring (128-byte swizzled boxes of 64 head-dim elements). Each ring refills as soon as its
//              own stage frees.
//   warp 9     MMA issuer (one elected thread): S_j = Q K_j^T (SS operands, M=128, N=BN) into S buffer j % 2, and
//              O += P_j V_j (A = P_j from TMEM, B = V_j MN-major from shared memory, M=128, N=D). It polls the
//              barriers and issues whichever is ready: S_{j+2} as soon as K_{j+2} has landed and the softmax warps
//              have loaded S_j, so the next scores are computed while the softmax of tile j still runs; PV_j as soon
//              as P_j and V_j are in. Completion is signalled with tcgen05.commit on mbarriers. S and P have separate
//              TMEM buffers, so no MMA writes TMEM that an earlier one may still be reading.
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
  static constexpr int KSTAGES = 3;  // K_{j+3} loads while S_j.. S_{j+2} are still ahead of it
  static constexpr int VSTAGES = 2;
  static constexpr int SBUF = 2;  // S buffers in TMEM (fp32), and as many P buffers (16-bit, BN / 2 columns each)
  static constexpr int Q_OFF = 0;
  static constexpr int K_OFF = Q_OFF + QBYTES;
  static constexpr int V_OFF = K_OFF + KSTAGES * KBYTES;
  static constexpr int BAR_OFF = V_OFF + VSTAGES * KBYTES;
  // at least ~120 KB so that one CTA holds an SM (its TMEM allocation is all 512 columns)
  static constexpr int RED_OFF = BAR_OFF + 256;  // [2 halves][128 rows] fp32: a row's partial max / sum
  static constexpr int SMEM_RAW = RED_OFF + 2 * BM * 4;
  static constexpr int SMEM_BYTES = (SMEM_RAW < 120 * 1024 ? 120 * 1024 : SMEM_RAW) + 1024;
  static constexpr int S_COL = 0;                // S buffers at columns [b BN, (b + 1) BN)
  static constexpr int P_COL = SBUF * BN;        // P buffers at [P_COL + b BN / 2, ...)
  static constexpr int O_COL = P_COL + SBUF * BN / 2;  // O at [3 BN, 3 BN + D)
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
  // Optional key-tile lists (array masks): row block m reads tl[m * tl_ld + 0 .. tn[m]) instead of every tile up to
  // its horizon -- the tiles in which some row of the block keeps a key (a block is BM rows here, 2 BM rows in the
  // CTA-pair kernel). NULL: every tile.
  const int32_t* tl;
  const int32_t* tn;
  int tl_ld;
};

// Applies a row's mask to its scores s of keys key0 .. key0 + HC - 1: -inf past lim (the causal limit) or N, and,
// with an array mask row mrow, where the mask byte is 0. A contiguous mask row is read in 16-byte pieces when
// aligned (one load for 16 keys instead of 16 byte loads).
template <int HC>
__device__ __forceinline__ void mask_scores(float* s, const uint8_t* mrow, int64_t mst1, int key0, int lim, int N) {
  if (mrow && mst1 == 1 && key0 + HC <= N && (reinterpret_cast<uintptr_t>(mrow + key0) & 15) == 0) {
#pragma unroll
    for (int c = 0; c < HC; c += 16) {
      const uint4 m4 = *reinterpret_cast<const uint4*>(mrow + key0 + c);
      const uint32_t w[4] = {m4.x, m4.y, m4.z, m4.w};
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        const bool keep = ((w[e >> 2] >> (8 * (e & 3))) & 0xFFu) != 0 && key0 + c + e <= lim;
        s[c + e] = keep ? s[c + e] : -INFINITY;
      }
    }
    return;
  }
#pragma unroll
  for (int c = 0; c < HC; ++c) {
    const int key = key0 + c;
    bool vis = key <= lim && key < N;
    if (mrow && vis) vis = mrow[int64_t(key) * mst1] != 0;
    s[c] = vis ? s[c] : -INFINITY;
  }
}

// The index of the j-th key tile row block m reads.
__device__ __forceinline__ int key_tile(const Params& p, int m, int j) { return p.tl ? p.tl[int64_t(m) * p.tl_ld + j] : j; }

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

// D (TMEM) [+]= A (TMEM, M rows x 16 elements a column pair) x B (shared memory descriptor).
__device__ __forceinline__ void umma_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
      "r"(tmem_a), "l"(b), "r"(idesc), "r"(acc));
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

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ float ex2f(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 2^x on the FMA and integer pipes instead of the multi-function unit, for a share of the softmax's exponentials
// (the split FlashAttention-4 describes for Blackwell): x = j + f with j = round(x) through the 1.5 * 2^23 rounding
// constant, 2^f by a degree-4 polynomial whose coefficients were fitted for relative error on [-1/2, 1/2] (at most
// 2.7e-6, about 18.5 bits: finer than the bf16 rounding P gets), 2^j added into the exponent field. x below -125
// gives 0 (as ex2.approx.ftz gives 0 below -126; masked scores are -inf).
__device__ __forceinline__ float ex2_fma(float x) {
  const float xc = fmaxf(x, -125.f);
  const float t = xc + 12582912.f;
  const float f = xc - (t - 12582912.f);
  float p = fmaf(0.009570101276040077f, f, 0.05591785907745361f);
  p = fmaf(p, f, 0.240247443318367f);
  p = fmaf(p, f, 0.6931217908859253f);
  p = fmaf(p, f, 0.9999992847442627f);
  const float r = __int_as_float(__float_as_int(p) + (__float_as_int(t) << 23));
  return x < -125.f ? 0.f : r;
}

// Number of BN-key tiles query tile mt reads.
template <int D>
__device__ __forceinline__ int kv_tiles(const Params& p, int mt) {
  constexpr int BN = Cfg<D>::BN;
  if (p.tn) return p.tn[mt];
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
  constexpr int KS = C::KSTAGES, VS = C::VSTAGES, SB = C::SBUF;
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
  uint64_t* q_full = bars;               // [1]
  uint64_t* k_full = q_full + 1;         // [KS]
  uint64_t* k_empty = k_full + KS;       // [KS]
  uint64_t* v_full = k_empty + KS;       // [VS]
  uint64_t* v_empty = v_full + VS;       // [VS]
  uint64_t* s_full = v_empty + VS;       // [SB] S_j complete in S buffer j % SB
  uint64_t* s_free = s_full + SB;        // [SB] the softmax warps have loaded S_j
  uint64_t* p_full = s_free + SB;        // [SB] P_j written into P buffer j % SB
  uint64_t* o_done = p_full + SB;        // [SB] PV_j complete (P buffer j % SB read), committed to o_done[j % SB]
  uint64_t* drain = o_done + SB;         // [1]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(drain + 2);
  static_assert((1 + 2 * KS + 2 * VS + 4 * SB + 1) * 8 + 16 <= 256, "barrier area");

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < KS; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
    }
    for (int i = 0; i < VS; ++i) {
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    for (int i = 0; i < SB; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], SOFTMAX_WARPS * 32);
      mbar_init(&p_full[i], SOFTMAX_WARPS * 32);
    }
    for (int i = 0; i < SB; ++i) mbar_init(&o_done[i], 1);
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
    // ------------------------------------------------------------------------------------ TMA producers
    // Lane 0 loads Q, then K tiles; lane 1 loads V tiles. Each ring refills as soon as its own stage frees, so K_{j+2}
    // (needed for S_{j+2}, which the MMA issuer runs before PV_j) never waits behind a V tile.
    if (lane < 2 && ntiles > 0) {
      if (lane == 0) {
        prefetch_tensormap(&qmap);
        prefetch_tensormap(&kmap);
        mbar_arrive_expect_tx(q_full, C::QBYTES);
#pragma unroll
        for (int db = 0; db < D / 64; ++db)
          tma_load_4d(sm + C::Q_OFF + db * BM * 128, &qmap, db * 64, r0, h, b, q_full);
      } else {
        prefetch_tensormap(&vmap);
      }
      const int NS = lane == 0 ? KS : VS;
      uint64_t* fullb = lane == 0 ? k_full : v_full;
      uint64_t* emptyb = lane == 0 ? k_empty : v_empty;
      const CUtensorMap* map = lane == 0 ? &kmap : &vmap;
      const int off = lane == 0 ? C::K_OFF : C::V_OFF;
      int issued = 0;
      for (int j = 0; j < ntiles && !*abort_flag; ++j) {
        const int st = j % NS;
        if (j >= NS && !mbar_wait(&emptyb[st], ((j / NS) - 1) & 1, 11 + lane)) {
          *abort_flag = 1;
          break;
        }
        mbar_arrive_expect_tx(&fullb[st], C::KBYTES);
#pragma unroll
        for (int db = 0; db < D / 64; ++db)
          tma_load_4d(sm + off + st * C::KBYTES + db * BN * 128, map, db * 64, key_tile(p, mt, j) * BN, hk, b,
                      &fullb[st]);
        issued = j + 1;
      }
      // Drain: every load this lane issued has landed before the CTA may finish (already true normally).
      if (lane == 0) mbar_wait(q_full, 0, 13);
      for (int j = max(0, issued - NS); j < issued; ++j) mbar_wait(&fullb[j % NS], (j / NS) & 1, 14);
    }
  } else if (warp == MMA_WARP) {
    // ------------------------------------------------------------------------------------ MMA issuer
    if (ntiles > 0) {
      const bool leader = elect_one();
      const uint32_t q_addr = smem_u32(sm + C::Q_OFF);
      bool ok = !leader || mbar_wait(q_full, 0, 21);
      // S_j = Q K_j^T into S buffer j % SB (K_j landed; the softmax warps have loaded S_{j-SB}).
      auto issue_s = [&](int j) {
        const int st = j % KS, sb = j % SB;
        tc_fence_after();
        const uint32_t k_addr = smem_u32(sm + C::K_OFF + st * C::KBYTES);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint64_t a = sdesc(q_addr + (kk >> 2) * BM * 128 + (kk & 3) * 32, 16, 1024);
          const uint64_t bd = sdesc(k_addr + (kk >> 2) * BN * 128 + (kk & 3) * 32, 16, 1024);
          umma_ss(tmem + C::S_COL + sb * BN, a, bd, IDESC_S, kk > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[sb]);
        umma_commit(&k_empty[st]);
      };
      // O += P_i V_i: A = P_i from TMEM (16 keys = 8 columns a k-step), B = V_i MN-major.
      auto issue_pv = [&](int i) {
        const int st = i % VS, sb = i % SB;
        tc_fence_after();
        const uint32_t v_addr = smem_u32(sm + C::V_OFF + st * C::KBYTES);
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk) {
          const uint64_t bd = sdesc(v_addr + kk * 16 * 128, BN * 128, 1024);
          umma_ts(tmem + C::O_COL, tmem + C::P_COL + sb * (BN / 2) + kk * 8, bd, IDESC_PV, (i > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&o_done[i % SB]);
        umma_commit(&v_empty[st]);
      };
      if (leader) {
        // Issue whichever of S_js and PV_jp is ready first (PV first when both are), polling the barriers without
        // blocking: a late K tile then never holds back a PV whose P and V are in, nor a late V tile the next S.
        // PV_jp needs S_jp issued. The whole loop is time-bounded.
        int js = 0, jp = 0;
        uint64_t t0 = 0;
        for (uint32_t it = 1; ok && jp < ntiles; ++it) {
          if (jp < js && mbar_test_wait(&v_full[jp % VS], (jp / VS) & 1) &&
              mbar_test_wait(&p_full[jp % SB], (jp / SB) & 1)) {
            issue_pv(jp++);
            t0 = 0;
            continue;
          }
          if (js < ntiles && mbar_test_wait(&k_full[js % KS], (js / KS) & 1) &&
              (js < SB || mbar_test_wait(&s_free[js % SB], ((js / SB) - 1) & 1))) {
            issue_s(js++);
            t0 = 0;
            continue;
          }
          // Nothing ready: back off briefly, so that this polling thread does not take issue slots and MIO
          // bandwidth from the softmax warps that share its SM sub-partition.
          __nanosleep(20);
          if ((it & 15) == 0) {
            if (*abort_flag) {
              ok = false;
              break;
            }
            const uint64_t now = globaltimer_ns();
            if (t0 == 0) {
              t0 = now;
            } else if (now - t0 > kWaitNs) {
              report_timeout(27);
              ok = false;
              break;
            }
          }
        }
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
    bool ok = true;
    for (int j = 0; j < ntiles; ++j) {
      const int sb = j % SB;
      const uint32_t scol = C::S_COL + sb * BN;
      // A failed wait never leaves a warp alone at a barrier: the decision to stop is made warp-uniform before
      // the warp-collective TMEM loads and pair-uniform at the max exchange (bar.red.and), where both warps of a
      // row pair leave the loop together.
      bool okj = ok && !*abort_flag && mbar_wait(&s_full[sb], (j / SB) & 1, 31);
      okj = __all_sync(0xffffffffu, okj);
      float s[HC];
      if (okj) {
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < HC; c += 32) tmem_ld32(lane_base + scol + hf * HC + c, s + c);
        tmem_wait_ld();
        tc_fence_before();
        mbar_arrive(&s_free[sb]);
      } else {
#pragma unroll
        for (int c = 0; c < HC; ++c) s[c] = -INFINITY;
      }

      const int kt = key_tile(p, mt, j);
      const int key0 = kt * BN + hf * HC;
      const bool full_tile = kt * BN + BN - 1 <= lim && kt * BN + BN <= p.N && !mrow;
      float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
      if (full_tile) {
#pragma unroll
        for (int c = 0; c < HC; ++c) mx4[c & 3] = fmaxf(mx4[c & 3], s[c]);
      } else {
        mask_scores<HC>(s, mrow, p.m_st[1], key0, lim, p.N);
#pragma unroll
        for (int c = 0; c < HC; ++c) mx4[c & 3] = fmaxf(mx4[c & 3], s[c]);
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
      // both read before the next tile rewrites red
      asm volatile("bar.sync %0, 64;" ::"r"(pair_bar));
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
        if (!mbar_wait(&o_done[(j - 1) % SB], ((j - 1) / SB) & 1, 32)) ok = false;
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
      // P_j (16-bit, key pairs packed a 32-bit column) into P buffer j % SB, this half's HC keys at columns
      // hf HC / 2 ...; the buffer was last read by PV_{j-SB}.
      if (j >= SB && !mbar_wait(&o_done[sb], ((j / SB) - 1) & 1, 34)) ok = false;
      tc_fence_after();
      const float nm = m_run == -INFINITY ? 0.f : -m_run;
      float ls4[4] = {0.f, 0.f, 0.f, 0.f};
      uint32_t pk[HC / 2];
#pragma unroll
      for (int c = 0; c < HC; c += 2) {
        const float e0 = ex2f(fmaf(s[c], p.scale_log2, nm));
        const float e1 = ex2f(fmaf(s[c + 1], p.scale_log2, nm));
        ls4[c & 3] += e0;
        ls4[(c + 1) & 3] += e1;
        pk[c / 2] = pack2<T>(e0, e1);
      }
#pragma unroll
      for (int c = 0; c < HC / 2; c += 16) tmem_st16(lane_base + C::P_COL + sb * (BN / 2) + hf * (HC / 2) + c, pk + c);
      l_run += (ls4[0] + ls4[1]) + (ls4[2] + ls4[3]);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&p_full[sb]);
    }
    if (ok && ntiles > 0) {
      if (!mbar_wait(&o_done[(ntiles - 1) % SB], ((ntiles - 1) / SB) & 1, 33)) ok = false;
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
