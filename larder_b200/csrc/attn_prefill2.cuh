// Prefill attention on a pair of CTAs (a 2-CTA cluster sharing each MMA: tcgen05 cta_group::2), head dims 128, 256.
//
// The single-CTA kernel (attn_prefill.cuh) reads every K and V byte once per 128 query rows; at head dim 256 each
// SM then streams 64 KB of K/V from L2 per 64-key tile and the L2 -> shared memory transfer, not the tensor cores,
// sets the pace. Here the two CTAs of a cluster take 256 consecutive rows of one head (128 each) and one MMA
// instruction covers both (M = 256): matrix A (Q for the scores, P for the output) stays split by rows, one half in
// each CTA, and matrix B is split along N, so each CTA loads only HALF of every K tile (64 of its 128 keys) and HALF
// of every V tile (D / 2 of its D columns). Per SM that halves the K/V bytes per FLOP. Tiles of 128 keys make the
// score MMAs N = 128 wide and halve the per-tile handshakes of the softmax; at head dim 256 TMEM then holds one S
// buffer (128 columns), two P buffers (64 each) and O (256); at head dim 128, two S buffers, two P buffers and O.
//
// Roles (576 threads a CTA):
//   warps 0-15 softmax + epilogue on the CTA's own 128 rows (TMEM lane r = row r of its S, P and O): warp w serves
//              the rows of lane quarter w % 4 and the key group w / 4 (32 of a tile's 128 keys, 64 of O's columns),
//              so four warps share each row. The running max moves only when a group's tile max exceeds it by more
//              than 2^8: one barrier of the four warps checks that, and only then do they swap maxima through shared
//              memory. After loading S_j and after writing P_j each warp arrives once on the LEADER CTA's s_free /
//              p_full barrier.
//   warp 16    TMA producers of the CTA's halves: lane 0 Q then K, lane 1 V. Loads complete on the leader's
//              barriers (the 2-CTA form of the bulk tensor copy); the leader's lanes announce the byte counts of both
//              halves. Each CTA refills a stage when its own k_empty / v_empty says the pair's MMA has finished it.
//   warp 17    in the leader (rank 0) only, one elected thread issues every MMA of the pair: S_j = Q K_j^T into the S
//              buffer and O += P_j V_j (A = P_j from TMEM), whichever is ready first, and commits completion to
//              the barriers of both CTAs (one commit each). In both CTAs warp 17 allocates and frees the TMEM.
// The grid is persistent: as many clusters as fit at once, each taking 256-row items (heaviest first) in turn; the
// next item's Q, K and V loads and its first score MMA overlap the current item's last tiles and epilogue.
// Causal is bottom-right as in the single-CTA kernel; the pair loops over the KV tiles its later rows need, the
// earlier CTA's rows masking the last tile or two. Every wait is time-bounded; a wait that gives up sets the CTA's
// abort flag, the roles drain what they issued, and both CTAs meet at a final cluster barrier before TMEM is freed.
#pragma once

#include "attn_prefill.cuh"

namespace lb2 {
namespace prefill2 {

using prefill::BM;
using prefill::TMEM_COLS;
using prefill::Params;

constexpr int NG = 4;                         // softmax warps a lane quarter (key / O column groups)
constexpr int SOFTMAX_WARPS = 4 * NG;
constexpr int PRODUCER_WARP = SOFTMAX_WARPS;
constexpr int MMA_WARP = SOFTMAX_WARPS + 1;
constexpr int THREADS = (SOFTMAX_WARPS + 2) * 32;

template <int D>
struct Cfg {
  static constexpr int BN = 128;                // keys a tile (the pair)
  static constexpr int HN = BN / 2;             // K rows (keys) a CTA holds
  static constexpr int HD = D / 2;              // V columns a CTA holds
  static constexpr int QBYTES = BM * D * 2;
  static constexpr int KHBYTES = HN * D * 2;    // a CTA's half of a K tile
  static constexpr int VHBYTES = BN * HD * 2;   // a CTA's half of a V tile
  static constexpr int KS = D == 256 ? 2 : 4;   // K / V stages (32 KB halves at head dim 256, 16 KB at 128)
  static constexpr int VS = KS;
  static constexpr int Q_OFF = 0;
  static constexpr int K_OFF = Q_OFF + QBYTES;
  static constexpr int V_OFF = K_OFF + KS * KHBYTES;
  static constexpr int BAR_OFF = V_OFF + VS * VHBYTES;
  static constexpr int RED_OFF = BAR_OFF + 256;  // [NG groups][128 rows] fp32
  static constexpr int SMEM_BYTES = RED_OFF + NG * BM * 4 + 1024;
  // S buffers: the softmax copies S_j to registers at once, so S_{j+1} can overwrite it while P_j is still being
  // formed; at head dim 128 O leaves TMEM room for a second buffer, and S_{j+1} no longer waits for that copy.
  static constexpr int SB = D == 256 ? 1 : 2;
  static constexpr int PB = 2;                    // P buffers
  static constexpr int S_COL = 0;                 // S buffers [b BN, (b + 1) BN), b < SB
  static constexpr int P_COL = SB * BN;           // P buffers [P_COL + b BN / 2, ...), b < PB
  static constexpr int O_COL = P_COL + PB * BN / 2;  // O [O_COL, O_COL + D)
  static_assert(O_COL + D <= TMEM_COLS, "TMEM budget");
  static_assert(SMEM_BYTES <= 232448, "shared memory budget");
  static_assert(D == 128 || D == 256, "the pair kernel is built for head dims 128 and 256");
};

// The softmax's exponential of column c of a thread's 32: at head dim 256 a quarter of them (c % 8 in {6, 7}) on the
// FMA pipe, the rest on the multi-function unit. At head dim 128 all go to the multi-function unit: that kernel is
// bound by instruction issue, and the polynomial's nine instructions cost more than the unit's queue (measured 2.7 %
// slower with the split).
template <int D>
__device__ __forceinline__ float ex2_mix(int c, float x) {
  return (D == 256 && (c & 7) >= 6) ? prefill::ex2_fma(x) : prefill::ex2f(x);
}

// ---------------------------------------------------------------------------------------------- cluster helpers

// Arrive on an mbarrier anywhere in the cluster. The arriving warps order their tcgen05 loads / stores before it
// with tcgen05.fence::before_thread_sync, the MMA thread orders its MMAs after the wait with
// tcgen05.fence::after_thread_sync.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

__device__ __forceinline__ bool mbar_test_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// 4-D tiled TMA load into this CTA's shared memory, completing on the leader CTA's copy of the mbarrier (the 2-CTA
// form of the copy, whose barrier may sit in either CTA of the pair).
__device__ __forceinline__ void tma_load_4d_pair(void* dst, const CUtensorMap* map, int c0, int c1, int c2, int c3,
                                                 uint64_t* bar) {
  const uint32_t b = mapa(smem_u32(bar), 0);
  asm volatile(
      "cp.async.bulk.tensor.4d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(dst)),
      "l"(map), "r"(b), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

__device__ __forceinline__ void umma2_ss(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5, %5, %5, %5, %5}, p;\n\t}" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc), "r"(0u));
}

__device__ __forceinline__ void umma2_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, {%5, %5, %5, %5, %5, %5, %5, %5}, p;\n\t}" ::"r"(
          tmem_d),
      "r"(tmem_a), "l"(b), "r"(idesc), "r"(acc), "r"(0u));
}

// Completion of this thread's prior pair MMAs, signalled on the barrier at this shared-memory offset in both CTAs
// (one commit a CTA).
__device__ __forceinline__ void umma2_commit_both(uint64_t* bar) {
  const uint32_t local = smem_u32(bar);
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(local) : "memory");
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(mapa(local, 1))
               : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
  uint32_t* r = reinterpret_cast<uint32_t*>(v);
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

// Number of BN-key tiles the pair of row tiles mt2 (rows [256 mt2, 256 mt2 + 256)) reads.
template <int D>
__device__ __forceinline__ int kv_tiles2(const Params& p, int mt2) {
  constexpr int BN = Cfg<D>::BN;
  if (p.tn) return p.tn[mt2];
  int last = p.N;
  if (p.mask_kind == LB2_MASK_CAUSAL) {
    const int rmax = min(p.T, (mt2 + 1) * 2 * BM) - 1;
    last = min(p.N, p.N - p.T + rmax + 1);
  }
  return last <= 0 ? 0 : (last + BN - 1) / BN;
}

// Work item k of a pass, heaviest first; heads vary fastest so that neighbouring clusters share their KV head's
// tiles in L2: the 256-row pair mt2 of (batch, query head) b, h. (A sequence-major order, one sequence's K and V at a
// time, measured 5 % slower on 8 sequences of 8192 rows.)
struct Item {
  int b, h, hk, r0, ntiles, mt2;
};

__device__ __forceinline__ int item_mt2(const Params& p, int k) { return p.mtiles - 1 - k / (p.B * p.Hq); }

template <int D>
__device__ __forceinline__ Item item_of(const Params& p, int k, uint32_t rank) {
  Item it;
  const int bh = k % (p.B * p.Hq);
  const int mt2 = item_mt2(p, k);
  it.b = bh / p.Hq;
  it.h = bh % p.Hq;
  it.hk = it.h / p.G;
  it.r0 = mt2 * 2 * BM + int(rank) * BM;  // this CTA's first row
  it.ntiles = kv_tiles2<D>(p, mt2);
  it.mt2 = mt2;
  return it;
}

// The items of cluster c of nc: round r takes item r nc + c, every other round in reverse order (a snake over the
// heaviest-first list), so that the clusters' totals even out.
__device__ __forceinline__ int item_index(int r, int c, int nc) { return r * nc + ((r & 1) ? nc - 1 - c : c); }

// Persistent: the grid holds as many clusters as fit at once, each looping over its items. Every role walks the same
// item sequence; the K / V stage rings, the S and P buffers and their barriers run on counters that continue across
// items. Two barriers hand resources from one item to the next: q_empty (the item's last score MMA has read Q, so
// the next Q may land) and o_free (the epilogue has read O out of TMEM, so the next item's first PV may overwrite
// it). Both count only items that have keys, so that no waiter can fall two phases behind.
template <typename T, int D>
__global__ void __launch_bounds__(THREADS, 1) fmha2_kernel(const __grid_constant__ CUtensorMap qmap,
                                                            const __grid_constant__ CUtensorMap kmap,
                                                            const __grid_constant__ CUtensorMap vmap,
                                                            const Params p) {
  using C = Cfg<D>;
  constexpr int BN = C::BN, HN = C::HN, HD = C::HD;
  constexpr int KS = C::KS, VS = C::VS;
  constexpr int AB = std::is_same<T, __nv_bfloat16>::value ? 1 : 0;
  constexpr uint32_t IDESC_S = prefill::idesc_f16(AB, 0, 0, 2 * BM, BN);
  constexpr uint32_t IDESC_PV = prefill::idesc_f16(AB, 0, 1, 2 * BM, D);

  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  const int cl = blockIdx.x >> 1, ncl = gridDim.x >> 1;
  const int total = p.B * p.Hq * p.mtiles;

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + C::BAR_OFF);
  uint64_t* q_full = bars;            // [1]  leader: both Q halves of the item landed
  uint64_t* q_empty = q_full + 1;     // [1]  both CTAs: the item's score MMAs are done with Q
  uint64_t* k_full = q_empty + 1;     // [KS] leader: both K halves of the stage landed
  uint64_t* k_empty = k_full + KS;    // [KS] both CTAs: the pair's MMA has read the stage
  uint64_t* v_full = k_empty + KS;    // [VS] leader
  uint64_t* v_empty = v_full + VS;    // [VS] both CTAs
  uint64_t* s_full = v_empty + VS;    // [SB] both CTAs: S_j complete in S buffer j % SB
  uint64_t* s_free = s_full + C::SB;  // [SB] leader: all softmax warps of the pair have loaded S_j
  uint64_t* p_full = s_free + C::SB;  // [PB] leader: all softmax warps have written P_j into P buffer j % PB
  uint64_t* o_done = p_full + C::PB;  // [PB] both CTAs: PV_j complete (P buffer j % PB read)
  uint64_t* o_free = o_done + C::PB;  // [1]  leader: all softmax warps of the pair have read the item's O
  uint64_t* drain = o_free + 1;       // [1]  leader
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(drain + 2);
  static_assert((2 + 2 * KS + 2 * VS + 2 * C::SB + 2 * C::PB + 2) * 8 + 16 <= 256, "barrier area");

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int i = 0; i < KS; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
    }
    for (int i = 0; i < VS; ++i) {
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    for (int i = 0; i < C::SB; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 2 * SOFTMAX_WARPS);
    }
    for (int i = 0; i < C::PB; ++i) {
      mbar_init(&p_full[i], 2 * SOFTMAX_WARPS);
      mbar_init(&o_done[i], 1);
    }
    mbar_init(o_free, 2 * SOFTMAX_WARPS);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == MMA_WARP) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
  }
  prefill::tc_fence_before();
  __syncthreads();
  cluster_sync();  // both CTAs' barriers are initialised before any remote arrive or load completion
  prefill::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == PRODUCER_WARP) {
    // ------------------------------------------------------------------------------------ TMA producers
    if (lane < 2) {
      if (lane == 0) {
        prefetch_tensormap(&qmap);
        prefetch_tensormap(&kmap);
      } else {
        prefetch_tensormap(&vmap);
      }
      const int NS = lane == 0 ? KS : VS;
      const int bytes = lane == 0 ? C::KHBYTES : C::VHBYTES;
      uint64_t* fullb = lane == 0 ? k_full : v_full;
      uint64_t* emptyb = lane == 0 ? k_empty : v_empty;
      int jg = 0, qi = 0, q_issued = -1;  // tiles issued on this lane's ring; items with keys so far; last Q item
      bool stop = false;
      for (int rr = 0; rr * ncl < total && !stop; ++rr) {
        const int kidx = item_index(rr, cl, ncl);
        if (kidx >= total) continue;
        const Item itm = item_of<D>(p, kidx, rank);
        if (itm.ntiles == 0) continue;
        if (lane == 0) {  // Q of this item, once the previous item's score MMAs are done with the buffer
          if (qi > 0 && !mbar_wait(q_empty, (qi - 1) & 1, 45)) {
            *abort_flag = 1;
            break;
          }
          if (leader) mbar_arrive_expect_tx(q_full, 2 * C::QBYTES);
#pragma unroll
          for (int db = 0; db < D / 64; ++db)
            tma_load_4d_pair(sm + C::Q_OFF + db * BM * 128, &qmap, db * 64, itm.r0, itm.h, itm.b, q_full);
          q_issued = qi;
        }
        for (int j = 0; j < itm.ntiles; ++j, ++jg) {
          if (*abort_flag) {
            stop = true;
            break;
          }
          const int st = jg % NS;
          if (jg >= NS && !mbar_wait(&emptyb[st], ((jg / NS) - 1) & 1, 41 + lane)) {
            *abort_flag = 1;
            stop = true;
            break;
          }
          if (leader) mbar_arrive_expect_tx(&fullb[st], 2 * bytes);
          if (lane == 0) {  // keys [j BN + rank HN, + HN), all D columns: D / 64 boxes of (64, HN)
            uint8_t* dst = sm + C::K_OFF + st * C::KHBYTES;
#pragma unroll
            for (int db = 0; db < D / 64; ++db)
              tma_load_4d_pair(dst + db * HN * 128, &kmap, db * 64, prefill::key_tile(p, itm.mt2, j) * BN + int(rank) * HN, itm.hk, itm.b,
                               &fullb[st]);
          } else {  // keys [j BN, + BN), columns [rank HD, + HD): HD / 64 boxes of (64, BN)
            uint8_t* dst = sm + C::V_OFF + st * C::VHBYTES;
#pragma unroll
            for (int db = 0; db < HD / 64; ++db)
              tma_load_4d_pair(dst + db * BN * 128, &vmap, int(rank) * HD + db * 64, prefill::key_tile(p, itm.mt2, j) * BN, itm.hk, itm.b,
                               &fullb[st]);
          }
        }
        ++qi;
      }
      // Drain (leader only: the loads of both CTAs complete on its barriers): everything issued has landed.
      if (leader) {
        if (lane == 0 && q_issued >= 0) mbar_wait(q_full, q_issued & 1, 43);
        for (int g = max(0, jg - NS); g < jg; ++g) mbar_wait(&fullb[g % NS], (g / NS) & 1, 44);
      }
    }
  } else if (warp == MMA_WARP) {
    // ------------------------------------------------------------------------------------ MMA issuer (leader)
    if (leader) {
      const bool elected = elect_one();
      if (elected) {
        const uint32_t q_addr = smem_u32(sm + C::Q_OFF);
        auto issue_s = [&](int g) {
          const int st = g % KS, sb = g % C::SB;
          prefill::tc_fence_after();
          const uint32_t k_addr = smem_u32(sm + C::K_OFF + st * C::KHBYTES);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint64_t a = prefill::sdesc(q_addr + (kk >> 2) * BM * 128 + (kk & 3) * 32, 16, 1024);
            const uint64_t bd = prefill::sdesc(k_addr + (kk >> 2) * HN * 128 + (kk & 3) * 32, 16, 1024);
            umma2_ss(tmem + C::S_COL + sb * BN, a, bd, IDESC_S, kk > 0 ? 1u : 0u);
          }
          umma2_commit_both(&s_full[sb]);
          umma2_commit_both(&k_empty[st]);
        };
        auto issue_pv = [&](int g, bool first) {
          const int st = g % VS, pb = g % C::PB;
          prefill::tc_fence_after();
          const uint32_t v_addr = smem_u32(sm + C::V_OFF + st * C::VHBYTES);
#pragma unroll
          for (int kk = 0; kk < BN / 16; ++kk) {
            const uint64_t bd = prefill::sdesc(v_addr + kk * 16 * 128, BN * 128, 1024);
            umma2_ts(tmem + C::O_COL, tmem + C::P_COL + pb * (BN / 2) + kk * 8, bd, IDESC_PV,
                     (!first || kk > 0) ? 1u : 0u);
          }
          umma2_commit_both(&o_done[pb]);  // PV_g read P buffer g % PB
          umma2_commit_both(&v_empty[st]);
        };
        bool ok = true;
        int js_g = 0, jp_g = 0, qi = 0;  // S and PV tiles issued; items with keys so far
        for (int rr = 0; ok && rr * ncl < total; ++rr) {
          const int kidx = item_index(rr, cl, ncl);
          if (kidx >= total) continue;
          const int nt = kv_tiles2<D>(p, item_mt2(p, kidx));
          if (nt == 0) continue;
          ok = mbar_wait(q_full, qi & 1, 51);
          bool o_ok = qi == 0;  // O may be overwritten by this item's first PV
          int js = 0, jp = 0;
          uint64_t t0 = 0;
          for (uint32_t it = 1; ok && jp < nt; ++it) {
            if (jp < js && (jp > 0 || o_ok || (o_ok = mbar_test_wait_cluster(o_free, (qi - 1) & 1))) &&
                mbar_test_wait_cluster(&v_full[jp_g % VS], (jp_g / VS) & 1) &&
                mbar_test_wait_cluster(&p_full[jp_g % C::PB], (jp_g / C::PB) & 1)) {
              issue_pv(jp_g++, jp++ == 0);
              t0 = 0;
              continue;
            }
            if (js < nt && mbar_test_wait_cluster(&k_full[js_g % KS], (js_g / KS) & 1) &&
                (js_g < C::SB || mbar_test_wait_cluster(&s_free[js_g % C::SB], ((js_g / C::SB) - 1) & 1))) {
              issue_s(js_g++);
              if (++js == nt) umma2_commit_both(q_empty);  // the item's score MMAs are done with Q
              t0 = 0;
              continue;
            }
            // Nothing ready: sleep on the barrier that gates the next MMA in the usual order (S_{j+SB} needs the
            // softmax to have loaded S_j, which precedes P_j), so that this thread takes no issue slots from the
            // softmax warps sharing its SM sub-partition and still wakes the moment that barrier completes.
            if (jp < js && (js >= nt || js - jp > C::SB)) {
              if (!mbar_test_wait_cluster(&p_full[jp_g % C::PB], (jp_g / C::PB) & 1))
                mbar_try_wait_hint(&p_full[jp_g % C::PB], (jp_g / C::PB) & 1, 1000);
              else
                mbar_try_wait_hint(&v_full[jp_g % VS], (jp_g / VS) & 1, 1000);
            } else if (js < nt) {
              if (js_g >= C::SB && !mbar_test_wait_cluster(&s_free[js_g % C::SB], ((js_g / C::SB) - 1) & 1))
                mbar_try_wait_hint(&s_free[js_g % C::SB], ((js_g / C::SB) - 1) & 1, 1000);
              else
                mbar_try_wait_hint(&k_full[js_g % KS], (js_g / KS) & 1, 1000);
            }
            if ((it & 15) == 0) {
              if (*abort_flag) {
                ok = false;
                break;
              }
              const uint64_t now = globaltimer_ns();
              if (t0 == 0) {
                t0 = now;
              } else if (now - t0 > kWaitNs) {
                report_timeout(52);
                ok = false;
                break;
              }
            }
          }
          ++qi;
        }
        if (!ok) *abort_flag = 1;
        asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                         smem_u32(drain))
                     : "memory");
        mbar_wait(drain, 0, 53);
      }
      __syncwarp();
    }
  } else {
    // ------------------------------------------------------------------------------------ softmax warps
    constexpr int HC = BN / NG;  // S columns (keys) a thread owns
    constexpr int DH = D / NG;   // O columns a thread owns
    static_assert(HC == 32, "a softmax thread loads 32 S columns");
    const int r = 32 * (warp & 3) + lane;
    const int grp = warp >> 2;
    const uint32_t lane_base = tmem + (uint32_t(32 * (warp & 3)) << 16);
    const uint32_t grp_bar = 2 + (warp & 3);  // named barrier of the NG warps of a lane quarter (ids 2..5)
    float* red = reinterpret_cast<float*>(sm + C::RED_OFF);
    const uint32_t s_free_l = mapa(smem_u32(s_free), 0), p_full_l = mapa(smem_u32(p_full), 0);
    const uint32_t o_free_l = mapa(smem_u32(o_free), 0);
    bool ok = true;
    int jg = 0;  // S tiles consumed so far (the MMA issuer's S and PV counters follow the same sequence)
    for (int rr = 0; ok && rr * ncl < total; ++rr) {
      const int kidx = item_index(rr, cl, ncl);
      if (kidx >= total) continue;
      const Item itm = item_of<D>(p, kidx, rank);
      const int ntiles = itm.ntiles;
      const int row = itm.r0 + r;
      const int lim = p.mask_kind == LB2_MASK_CAUSAL ? p.N - p.T + row : p.N - 1;
      const uint8_t* mrow =
          (p.mask_kind == LB2_MASK_ARRAY && row < p.T) ? p.mask + int64_t(row) * p.m_st[0] : nullptr;
      float m_run = -INFINITY, l_run = 0.f;
      for (int j = 0; j < ntiles; ++j) {
        const int g = jg + j;
        const int sb = g % C::SB;
        bool okj = ok && !*abort_flag && mbar_wait(&s_full[sb], (g / C::SB) & 1, 61);
        okj = __all_sync(0xffffffffu, okj);
        float s[HC];
        if (okj) {
          prefill::tc_fence_after();
          prefill::tmem_ld32(lane_base + C::S_COL + sb * BN + grp * HC, s);
          prefill::tmem_wait_ld();
          prefill::tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster(s_free_l + 8u * sb);
        } else {
#pragma unroll
          for (int c = 0; c < HC; ++c) s[c] = -INFINITY;
        }
        const int kt = prefill::key_tile(p, itm.mt2, j);
        const int key0 = kt * BN + grp * HC;
        const bool full_tile = kt * BN + BN - 1 <= lim && kt * BN + BN <= p.N && !mrow;
        if (!full_tile) prefill::mask_scores<HC>(s, mrow, p.m_st[1], key0, lim, p.N);
        // P_j with the running max. The running max moves only when a row's tile max exceeds it by more than 2^8,
        // i.e. when some P of the row exceeds 2^8; P >= 0, so a thread whose P sum is at most 2^8 has no such
        // element and skips the max altogether. Otherwise (or before the row's first key) the exact check below
        // runs, and the rows that move recompute their P.
        float nm = m_run == -INFINITY ? 0.f : -m_run;
        float ls4[4] = {0.f, 0.f, 0.f, 0.f};
        uint32_t pk[HC / 2];
#pragma unroll
        for (int c = 0; c < HC; c += 2) {
          const float e0 = ex2_mix<D>(c, fmaf(s[c], p.scale_log2, nm));
          const float e1 = ex2_mix<D>(c, fmaf(s[c + 1], p.scale_log2, nm));
          ls4[c & 3] += e0;
          ls4[(c + 1) & 3] += e1;
          pk[c / 2] = pack2<T>(e0, e1);
        }
        // one barrier of the quarter's NG warps: does any of their rows want to move its max (or did a wait fail)?
        const bool want = !okj || m_run == -INFINITY || !((ls4[0] + ls4[1]) + (ls4[2] + ls4[3]) <= 256.f);
        uint32_t any_want;
        asm volatile(
            "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\t"
            "bar.red.or.pred q, %2, %3, p;\n\tselp.u32 %0, 1, 0, q;\n\t}"
            : "=r"(any_want)
            : "r"(uint32_t(want)), "r"(grp_bar), "n"(NG * 32)
            : "memory");
        if (any_want) {
          float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
          for (int c = 0; c < HC; ++c) mx4[c & 3] = fmaxf(mx4[c & 3], s[c]);
          float tmax = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3]));
          red[grp * BM + r] = tmax;
          uint32_t all_ok;
          asm volatile(
              "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\t"
              "bar.red.and.pred q, %2, %3, p;\n\tselp.u32 %0, 1, 0, q;\n\t}"
              : "=r"(all_ok)
              : "r"(uint32_t(okj)), "r"(grp_bar), "n"(NG * 32)
              : "memory");
#pragma unroll
          for (int g2 = 0; g2 < NG; ++g2) tmax = fmaxf(tmax, red[g2 * BM + r]);
          asm volatile("bar.sync %0, %1;" ::"r"(grp_bar), "n"(NG * 32));
          if (!all_ok) {
            ok = false;
            break;
          }
          const float tmax2 = tmax * p.scale_log2;
          const bool move = tmax2 > m_run + 8.f;
          const float factor = move ? prefill::ex2f(m_run - tmax2) : 1.f;
          if (__any_sync(0xffffffffu, move && j > 0 && l_run > 0.f)) {
            if (!mbar_wait(&o_done[(g - 1) % C::PB], ((g - 1) / C::PB) & 1, 62)) ok = false;
            prefill::tc_fence_after();
#pragma unroll 1
            for (int c = 0; c < DH; c += 16) {  // (16 columns at a time: S and P stay in registers meanwhile)
              float ov[16];
              tmem_ld16(lane_base + C::O_COL + grp * DH + c, ov);
              prefill::tmem_wait_ld();
#pragma unroll
              for (int e = 0; e < 16; ++e) ov[e] *= factor;
              prefill::tmem_st16(lane_base + C::O_COL + grp * DH + c, reinterpret_cast<const uint32_t*>(ov));
            }
            prefill::tmem_wait_st();
          }
          if (move) {  // this row's P with its new max
            l_run *= factor;
            m_run = tmax2;
            nm = -m_run;
#pragma unroll
            for (int c = 0; c < 4; ++c) ls4[c] = 0.f;
#pragma unroll
            for (int c = 0; c < HC; c += 2) {
              const float e0 = ex2_mix<D>(c, fmaf(s[c], p.scale_log2, nm));
              const float e1 = ex2_mix<D>(c, fmaf(s[c + 1], p.scale_log2, nm));
              ls4[c & 3] += e0;
              ls4[(c + 1) & 3] += e1;
              pk[c / 2] = pack2<T>(e0, e1);
            }
          }
        }
        // P_j into P buffer g % PB (last read by PV_{g-PB}): this group's HC keys at columns grp HC / 2 ...
        const int pbuf = g % C::PB;
        if (g >= C::PB && !mbar_wait(&o_done[pbuf], ((g / C::PB) - 1) & 1, 64)) ok = false;
        prefill::tc_fence_after();
        prefill::tmem_st16(lane_base + C::P_COL + pbuf * (BN / 2) + grp * (HC / 2), pk);
        l_run += (ls4[0] + ls4[1]) + (ls4[2] + ls4[3]);
        prefill::tmem_wait_st();
        prefill::tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(p_full_l + 8u * pbuf);
      }
      if (ok && ntiles > 0) {
        const int gl = jg + ntiles - 1;  // the item's last PV
        if (!mbar_wait(&o_done[gl % C::PB], (gl / C::PB) & 1, 63)) ok = false;
        prefill::tc_fence_after();
      }
      // -------------------------------------------------------------------------------- epilogue of the item
      ok = __all_sync(0xffffffffu, ok);
      float l_tot = 0.f;
      if (ntiles > 0) {  // (an item without keys skips the exchange, whose buffer the quarter may still be reading)
        red[grp * BM + r] = l_run;
        // the quarter's warps agree on ok, so that all of them leave the item loop together or none does
        uint32_t all_ok;
        asm volatile(
            "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\t"
            "bar.red.and.pred q, %2, %3, p;\n\tselp.u32 %0, 1, 0, q;\n\t}"
            : "=r"(all_ok)
            : "r"(uint32_t(ok)), "r"(grp_bar), "n"(NG * 32)
            : "memory");
        ok = all_ok != 0;
#pragma unroll
        for (int g2 = 0; g2 < NG; ++g2) l_tot += red[g2 * BM + r];
      }
      const bool have_o = ntiles > 0 && ok;
      const bool store = row < p.T;
      T* orow = reinterpret_cast<T*>(p.o) + itm.b * p.o_st[0] + int64_t(itm.h) * p.o_st[1] + int64_t(row) * p.o_st[2] +
                grp * DH;
      const T* grow = p.gate ? reinterpret_cast<const T*>(p.gate) + itm.b * p.g_st[0] + int64_t(itm.h) * p.g_st[1] +
                                   int64_t(row) * p.g_st[2] + grp * DH
                             : nullptr;
      const float inv = (have_o && m_run != -INFINITY && l_tot > 0.f) ? 1.f / l_tot : 0.f;
#pragma unroll 1
      for (int c = 0; c < DH; c += 32) {
        float ov[32];
        if (have_o) {
          prefill::tmem_ld32(lane_base + C::O_COL + grp * DH + c, ov);
          prefill::tmem_wait_ld();
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
          uint4 pk4;
          pk4.x = pack2<T>(x[0], x[1]);
          pk4.y = pack2<T>(x[2], x[3]);
          pk4.z = pack2<T>(x[4], x[5]);
          pk4.w = pack2<T>(x[6], x[7]);
          *reinterpret_cast<uint4*>(orow + c + e) = pk4;
        }
      }
      if (ntiles > 0) {  // O is read: the next item's first PV may overwrite it
        prefill::tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(o_free_l);
      }
      jg += ntiles;
    }
    if (!ok) *abort_flag = 1;
  }

  // The leader's MMAs read this CTA's shared memory and TMEM: neither CTA frees anything before both are done.
  prefill::tc_fence_before();
  __syncthreads();
  cluster_sync();
  if (warp == MMA_WARP) {
    prefill::tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS));
  }
}

}  // namespace prefill2
}  // namespace lb2
