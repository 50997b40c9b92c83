// Split-KV decode attention for a few query rows over a long KV cache (HBM-bandwidth bound).
//
// Persistent kernel: one CTA per SM walks its share of the call's work items, an item being (sequence b, KV head hk,
// a key range of b). The G*T query rows sharing KV head hk are folded into 16-row tiles (the fold of
// foldattn.py:230-259), so every K/V byte is read from HBM once per call. Two schedules:
//  - balanced (split = 0): the call's 64-key tiles, ordered (b, hk, tile), are cut into gridDim.x equal runs and CTA c
//    takes run c, cut again where a (b, hk) pair ends. Every CTA streams the same number of tiles whatever the
//    per-sequence lengths, and CTA c's item of pair p writes partial slot c + p: unique (a later CTA starts at or
//    after an earlier CTA's last pair) and contiguous per pair, so the combine finds a pair's partials by arithmetic;
//  - split (split > 0): equal `split`-key units (b, s, hk) dealt round-robin, partial slot (b Hkv + hk) nsplit + s.
// A producer warp streams, item after item without a pause, the item's folded Q tile (a 2-slot ring) and its 64-key
// K and V tiles (a STAGES-deep ring), all with TMA into 128-byte swizzled boxes of 64 head-dim elements; four
// consumer warps each take 16 of a tile's 64 keys and run S = Q K^T and O += P V on mma.sync m16n8k16 (fp32
// accumulate) with an fp32 online softmax in base 2. At an item's end each consumer warp drops its partial (max, sum,
// unnormalised O) into shared memory and goes on to the next item while the producer keeps streaming; a merger warp
// folds the four into the item's partial in the workspace; split_combine_kernel, launched right behind as a
// programmatic dependent, merges the partials of each (b, hk, row) by log-sum-exp -- the combine of foldattn_merge
// (foldattn.py:188-211) and CpuAttn's range merge (cpu_ext/cpu_kern.cpp:607-628).
#pragma once

#include "common.cuh"

namespace lb2 {
namespace decode {

constexpr int BK = 64;         // keys per tile
constexpr int MAX_B = 1024;    // sequences a call (the per-CTA prefix table)
constexpr int MAX_PARTS = 512; // partials of one (b, hk) pair the combine can merge

// NT: 8-row tiles of folded query rows (rows <= 8 NT). With one row tile, two groups of four consumer warps take
// alternate K/V tiles (eight consumer warps, two a scheduler, so one hides the other's latency); otherwise one
// group of four. The K/V ring gets as many stages as shared memory holds (at most 8).
template <int D, int NT>
struct Cfg {
  static constexpr int RP = NT * 8;                           // folded rows, padded
  static constexpr int GROUPS = NT == 1 ? 2 : 1;
  static constexpr int CONSUMERS = 4 * GROUPS;                // consumer warps, 16 keys of a tile apiece
  static constexpr int PRODUCER = CONSUMERS;                  // warp index of the TMA producer
  static constexpr int MERGER = CONSUMERS + 1;                // warp index of the partial merger
  static constexpr int THREADS = (CONSUMERS + 2) * 32;
  static constexpr bool Q_REGS = NT * (D / 16) <= 16;         // Q^T fragments held in registers for the item
  static constexpr int TILE_BYTES = BK * D * 2;               // one K (or V) tile, bf16/f16
  static constexpr int STAGE_BYTES = 2 * TILE_BYTES;          // K + V
  static constexpr int QSLOT = (D / 64) * RP * 128;           // one folded Q tile
  static constexpr int PART_BYTES = CONSUMERS * RP * D * 4 + CONSUMERS * RP * 2 * 4;
  static constexpr int FIXED = 2 * QSLOT + PART_BYTES + (2 * MAX_B + 1) * 4 + 16 + 256 + 1024;
  static constexpr int STAGES_FIT = (232448 - FIXED) / STAGE_BYTES;
  // With two groups the stage count is even, so that stage st only ever holds tiles of group st % 2: a warp then waits
  // on every phase of its stages in order. (With an odd count the tile STAGES back in the same stage is the other
  // group's; a wait for phase k could run while phase k - 1 is still open, and parity k & 1 would match phase k - 2.)
  static constexpr int STAGES = (STAGES_FIT > 8 ? 8 : STAGES_FIT) / GROUPS * GROUPS;
  static constexpr int RING_BYTES = STAGES * STAGE_BYTES;
  static constexpr int Q_OFF = RING_BYTES;
  static constexpr int PART_OFF = Q_OFF + 2 * QSLOT;         // [CONSUMERS][RP][D] O + [CONSUMERS][RP][2] (m, l)
  static constexpr int PREFIX_OFF = PART_OFF + PART_BYTES;   // [MAX_B + 1] ints
  static constexpr int LENS_OFF = PREFIX_OFF + (MAX_B + 1) * 4;  // [MAX_B] ints
  static constexpr int BAR_OFF = (LENS_OFF + MAX_B * 4 + 15) / 16 * 16;
  static constexpr int SMEM_BYTES = BAR_OFF + 256 + 1024 /*align*/;
  static_assert(STAGES >= 2 && STAGES % GROUPS == 0 && SMEM_BYTES <= 232448, "shared memory budget");
  static_assert((2 * STAGES + 6) * 8 <= 256, "barrier area");
};

struct Params {
  void* o;
  int64_t o_st[3];
  float* part_o;    // emit mode: normalised fp32 o, [B, Hq, T, D] contiguous
  float* part_lse;  // emit mode: natural-log lse, [B, Hq, T]
  const int32_t* kv_len;
  float* ws_o;      // [slots, rows, D] unnormalised partial O of each item
  float* ws_ml;     // [slots, rows, 2] (max in log2 units, sum)
  int B, Hq, Hkv, T, N, G, rows;
  int balanced;     // 1: balanced tile runs; 0: split units
  int split, nsplit;  // split mode: keys a unit, slots a (b, hk) pair
  int grid;         // CTAs of the decode grid (the balanced schedule's run count)
  int causal, emit;
  float scale_log2;  // softmax scale * log2(e)
  // push mode (npush > 0): the emitted partial goes to npush places at once -- this rank's slot in every rank's
  // exchange buffer, peers' through NVLink -- instead of part_o / part_lse (same offsets in each; the o rows as
  // bf16 at the start of the o area)
  int npush;
  float* push_o[8];
  float* push_lse[8];
  // and the call is announced by the block that finishes last: it stores push_epoch into every rank's flag of this
  // rank (push_flag[i]), once push_count (this rank's, in its own buffer) shows every block done
  uint32_t* push_count;
  uint32_t* push_flag[8];
  uint32_t push_epoch;
  // pick mode (picks != nullptr; one sequence): the call's keys are the gathered rows of a QSA decode step -- key g is
  // row tb[g / cr] cr + g % cr of the cache view for g < nsel cr, then the view's trailing partial block -- read
  // straight from the view (pk / pv, head and position strides in bytes, view length pick_n) by the producer warp
  const int32_t* picks;
  int nsel, cr, pick_n;
  const uint8_t* pk;
  const uint8_t* pv;
  int64_t pk_hst, pk_pst, pv_hst, pv_pst;
};

// The cache-view row of gathered key g in pick mode (out-of-range picks read row 0, recorded in the status word).
__device__ __forceinline__ int pick_row(const Params& p, int g) {
  const int j = g / p.cr;
  const int r = j < p.nsel ? p.picks[j] * p.cr + (g - j * p.cr) : p.pick_n / p.cr * p.cr + (g - p.nsel * p.cr);
  if (r < 0 || r >= p.pick_n) {
    report_bad_index(98);
    return 0;
  }
  return r;
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}

// Arrives on the mbarrier once this thread's earlier cp.async copies have landed (raising the phase's expected count
// by one first, so the arrival is neutral to it).
__device__ __forceinline__ void cp_async_arrive(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.shared.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}

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

// Transposes an 8 x 8 matrix of 16-bit values held a row pair a lane (lane l: row l / 4, columns 2 (l % 4) and
// 2 (l % 4) + 1) across the warp, in the same layout.
__device__ __forceinline__ uint32_t movm_t(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}

// One work item: KV head hk of sequence b (length len), keys [n0, n1), partial slot `slot`.
struct Item {
  int b, hk, n0, n1, len, slot;
};

// The CTA's work items in order. prefix[b] counts, for one head, the split units (split mode) or the key tiles
// (balanced mode) of sequences before b; lens[b] is b's length. Every role of the CTA walks the same sequence.
struct Sched {
  const int* prefix;
  const int* lens;
  int B, Hkv, split, nsplit, balanced;
  int cur, end, step;

  __device__ __forceinline__ Sched(const Params& p, const int* prefix_, const int* lens_)
      : prefix(prefix_), lens(lens_), B(p.B), Hkv(p.Hkv), split(p.split), nsplit(p.nsplit), balanced(p.balanced) {
    const int total = prefix[p.B] * p.Hkv;  // units or tiles of the call
    if (balanced) {
      cur = int(int64_t(blockIdx.x) * total / gridDim.x);
      end = int(int64_t(blockIdx.x + 1) * total / gridDim.x);
      step = 0;
    } else {
      cur = blockIdx.x;
      end = total;
      step = gridDim.x;
    }
  }

  __device__ __forceinline__ bool more() const { return cur < end; }

  __device__ __forceinline__ bool next(Item& it) {
    if (cur >= end) return false;
    const int key = cur / Hkv;
    int lo = 0, hi = B;  // the largest b with prefix[b] <= key, i.e. prefix[b] * Hkv <= cur
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (prefix[mid] <= key) lo = mid; else hi = mid;
    }
    const int b = lo;
    it.b = b;
    it.len = lens[b];
    if (balanced) {  // tiles ordered (b, hk, tile); b has nt >= 1 tiles, since cur < the call's total
      const int base = prefix[b] * Hkv, nt = prefix[b + 1] - prefix[b];
      const int hk = (cur - base) / nt, i0 = cur - base - hk * nt;
      const int seg_end = min(end, base + (hk + 1) * nt);
      it.hk = hk;
      it.n0 = i0 * BK;
      it.n1 = min(it.len, (i0 + seg_end - cur) * BK);
      it.slot = int(blockIdx.x) + b * Hkv + hk;
      cur = seg_end;
    } else {  // units ordered (b, s, hk)
      const int hk = cur - key * Hkv, s = key - prefix[b];
      it.hk = hk;
      it.n0 = s * split;
      it.n1 = min(it.len, it.n0 + split);
      it.slot = (b * Hkv + hk) * nsplit + s;
      cur += step;
    }
    return true;
  }
};

template <typename T, int D, int NT>
__global__ void __launch_bounds__(Cfg<D, NT>::THREADS, 1) decode_kernel(const __grid_constant__ CUtensorMap qmap,
                                                                       const __grid_constant__ CUtensorMap kmap,
                                                                       const __grid_constant__ CUtensorMap vmap,
                                                                       const Params p) {
  using C = Cfg<D, NT>;
  constexpr int STAGES = C::STAGES;
  constexpr int RP = C::RP;
  constexpr int CONSUMERS = C::CONSUMERS;
  constexpr int THREADS = C::THREADS;
  constexpr int KD = D / 16;  // 16-wide k-steps of K Q^T, and 16-row head-dim blocks of O^T

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  int* prefix = reinterpret_cast<int*>(sm + C::PREFIX_OFF);
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + C::BAR_OFF);
  uint64_t* empty = full + STAGES;
  uint64_t* q_full = empty + STAGES;
  uint64_t* q_empty = q_full + 2;
  uint64_t* part_full = q_empty + 2;   // the consumer warps' partials of an item are in the part area
  uint64_t* part_empty = part_full + 1;  // the merger has read them
  float* pwo = reinterpret_cast<float*>(sm + C::PART_OFF);  // [CONSUMERS][RP][D]
  float* pwml = pwo + CONSUMERS * RP * D;                  // [CONSUMERS][RP][2]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int* lens = reinterpret_cast<int*>(sm + C::LENS_OFF);
  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 4);  // the four warps of the group that takes the tile
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], CONSUMERS);
    }
    mbar_init(part_full, CONSUMERS);
    mbar_init(part_empty, 1);
    fence_barrier_init();
    prefetch_tensormap(&qmap);  // kernel parameters: no dependency on the previous kernel
    prefetch_tensormap(&kmap);
    prefetch_tensormap(&vmap);
  }
  // Launched as a programmatic dependent of the previous kernel in the stream: everything above touched only this
  // CTA's shared memory; every global read below waits for that kernel to complete.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  // per-sequence lengths and unit or tile counts (loaded in parallel), then warp 0 scans the counts into a prefix
  // table
  for (int b = threadIdx.x; b < p.B; b += THREADS) {
    const int len = p.kv_len ? min(max(p.kv_len[b], 0), p.N) : p.N;
    lens[b] = len;
    prefix[b + 1] = p.balanced ? (len + BK - 1) / BK : max(1, (len + p.split - 1) / p.split);
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
  // The split combine (launched as this grid's programmatic dependent) may start its prologue now; it waits for
  // this grid's completion before reading any partial.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  // Pick mode: every thread of the CTA copies the CTA's first tiles (as many as the ring holds) before the roles part,
  // so that those loads have the whole CTA's copy capacity behind them (one warp's 16-byte copies keep too few bytes
  // in flight); the producer goes on from the next tile. Each thread's arrival follows its copies; thread 0's plain
  // arrival, after a barrier, completes each stage's phase once all of them have landed.
  constexpr int CPR = D / 8;  // 16-byte chunks a K / V row
  int pre = 0;
  if (p.picks) {
    Sched s0(p, prefix, lens);
    Item i0;
    while (pre < STAGES && s0.next(i0)) {
      const int nt = i0.n1 > i0.n0 ? (i0.n1 - i0.n0 + BK - 1) / BK : 0;
      const uint8_t* kh = p.pk + i0.hk * p.pk_hst;
      const uint8_t* vh = p.pv + i0.hk * p.pv_hst;
      for (int i = 0; i < nt && pre < STAGES; ++i, ++pre) {
        const uint32_t kt = smem_u32(sm + pre * C::STAGE_BYTES), vt = kt + C::TILE_BYTES;
        const int key0 = i0.n0 + i * BK;
        for (int e = threadIdx.x; e < BK * CPR; e += THREADS) {
          const int r = e / CPR, c = e - r * CPR;
          const int src = pick_row(p, min(key0 + r, i0.len - 1));
          const uint32_t off = swz(c >> 3, r, c & 7);
          cp_async16(kt + off, kh + src * p.pk_pst + c * 16);
          cp_async16(vt + off, vh + src * p.pv_pst + c * 16);
        }
        cp_async_arrive(&full[pre]);
      }
    }
    __syncthreads();
    if (threadIdx.x == 0)
      for (int i = 0; i < pre; ++i) mbar_arrive(&full[i]);
  }

  // ------------------------------------------------------------------ producer warp: Q tiles and K/V tiles
  if (warp == C::PRODUCER && p.picks) {
    // Pick mode: lane 0 loads the Q tiles by TMA as below; the whole warp fills each K / V tile with 16-byte cp.async
    // copies of the gathered rows, into the layout the TMA boxes give (128-byte swizzle, [D / 64][BK][64]). Lane l
    // resolves the rows l and l + 32 of a tile (rows past the call's length repeat its last row, which the consumers
    // mask), and every lane's arrival on the stage's full barrier follows its copies. The CTA's first `pre` tiles
    // were copied above by all its threads.
    int gt = 0, uc = 0;
    bool ok = true;
    Sched sched(p, prefix, lens);
    Item it;
    for (; ok && sched.next(it); ++uc) {
      const int b = it.b, hk = it.hk, n0 = it.n0;
      const int ntiles = it.n1 > n0 ? (it.n1 - n0 + BK - 1) / BK : 0;
      const int qs = uc & 1;
      if (lane == 0) {
        ok = uc < 2 || mbar_wait(&q_empty[qs], ((uc >> 1) - 1) & 1, 1);
        if (ok) {
          mbar_arrive_expect_tx(&q_full[qs], (D / 64) * p.rows * 128);
#pragma unroll
          for (int db = 0; db < D / 64; ++db)
            tma_load_4d(sm + C::Q_OFF + qs * C::QSLOT + db * RP * 128, &qmap, db * 64, 0, hk * p.G, b, &q_full[qs]);
        }
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      const uint8_t* kh = p.pk + hk * p.pk_hst;
      const uint8_t* vh = p.pv + hk * p.pv_hst;
      for (int i = 0; ok && i < ntiles; ++i, ++gt) {
        if (gt < pre) continue;
        const int st = gt % STAGES;
        bool w = true;
        if (lane == 0 && gt >= STAGES) w = mbar_wait(&empty[st], ((gt / STAGES) - 1) & 1, 2);
        if (!__shfl_sync(0xffffffffu, w, 0)) {
          ok = false;
          break;
        }
        const uint32_t kt = smem_u32(sm + st * C::STAGE_BYTES), vt = kt + C::TILE_BYTES;
        const int key0 = n0 + i * BK;
        const int row_lo = pick_row(p, min(key0 + lane, it.len - 1));
        const int row_hi = pick_row(p, min(key0 + 32 + lane, it.len - 1));
#pragma unroll 4
        for (int t = 0; t < BK * CPR / 32; ++t) {
          const int e = lane + 32 * t, r = e / CPR, c = e - r * CPR;
          const int src = (32 * t) / CPR < 32 ? __shfl_sync(0xffffffffu, row_lo, r & 31)
                                               : __shfl_sync(0xffffffffu, row_hi, r & 31);
          const uint32_t off = swz(c >> 3, r, c & 7);
          cp_async16(kt + off, kh + src * p.pk_pst + c * 16);
          cp_async16(vt + off, vh + src * p.pv_pst + c * 16);
        }
        cp_async_arrive(&full[st]);
        __syncwarp();
        if (lane == 0) mbar_arrive(&full[st]);
      }
    }
    // Drain: the last copies issued have landed before the CTA may finish (normally already consumed).
    if (lane == 0) {
      for (int g2 = max(0, gt - STAGES); g2 < gt; ++g2) mbar_wait(&full[g2 % STAGES], (g2 / STAGES) & 1, 3);
      for (int q2 = max(0, uc - 2); q2 < uc; ++q2) mbar_wait(&q_full[q2 & 1], (q2 >> 1) & 1, 4);
    }
    return;
  }
  if (warp == C::PRODUCER) {
    if (lane == 0) {
      int gt = 0, uc = 0;
      bool ok = true;
      Sched sched(p, prefix, lens);
      Item it;
      for (; ok && sched.next(it); ++uc) {
        const int b = it.b, hk = it.hk, n0 = it.n0;
        const int ntiles = it.n1 > n0 ? (it.n1 - n0 + BK - 1) / BK : 0;
        const int qs = uc & 1;
        if (uc >= 2 && !mbar_wait(&q_empty[qs], ((uc >> 1) - 1) & 1, 1)) break;
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

  // ------------------------------------------------------------------ merger warp: one partial per item
  // (all but the CTA's last item, which the consumer warps merge themselves, a row each, once the stream has ended)
  if (warp == C::MERGER) {
    int uc = 0;
    Sched sched(p, prefix, lens);
    Item it;
    for (; sched.next(it) && sched.more(); ++uc) {
      if (!mbar_wait(part_full, uc & 1, 7)) break;
      const size_t part = size_t(it.slot) * p.rows;
      for (int r = 0; r < p.rows; ++r) {
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < CONSUMERS; ++w) M = fmaxf(M, pwml[(w * RP + r) * 2]);
        const float Mu = M == -INFINITY ? 0.f : M;
        float wgt[CONSUMERS], L = 0.f;
#pragma unroll
        for (int w = 0; w < CONSUMERS; ++w) {
          wgt[w] = ex2(pwml[(w * RP + r) * 2] - Mu);
          L += pwml[(w * RP + r) * 2 + 1] * wgt[w];
        }
        for (int c = lane; c < D / 4; c += 32) {
          float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
          for (int w = 0; w < CONSUMERS; ++w) {
            const float4 x = *reinterpret_cast<const float4*>(&pwo[(w * RP + r) * D + 4 * c]);
            o.x += wgt[w] * x.x;
            o.y += wgt[w] * x.y;
            o.z += wgt[w] * x.z;
            o.w += wgt[w] * x.w;
          }
          reinterpret_cast<float4*>(&p.ws_o[(part + r) * D])[c] = o;
        }
        if (lane == 0) *reinterpret_cast<float2*>(&p.ws_ml[(part + r) * 2]) = make_float2(M, L);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(part_empty);
    }
    return;
  }

  // ------------------------------------------------------------------ consumer warps
  // Keys sit in the M dimension of the MMAs: S^T = K Q^T (m16n8k16: 16 keys x 8 folded rows, k over the head dim)
  // and O^T += V^T P^T (16 head-dim rows x 8 folded rows, k over the keys), so a tile of 8 rows wastes no MMA rows.
  // The S^T accumulators turn into the B operand of the second product with one movmatrix transpose each.
  const int quad = lane >> 2, qid = lane & 3;
  const int grp = warp >> 2, wq = warp & 3;  // group (takes tiles gt with gt % GROUPS == grp), warp in the group
  int gt = 0, uc = 0;
  bool ok = true;
  Sched sched(p, prefix, lens);
  Item it;
  for (; ok && sched.next(it); ++uc) {
    const int qs = uc & 1;
    // No named barrier joins the consumer warps: a warp whose (time-bounded) wait gives up leaves the loop, the
    // producer then stops at its own bounded waits, and the other warps' waits end the same way.
    if (!mbar_wait(&q_full[qs], (uc >> 1) & 1, 5)) {
      ok = false;
      break;
    }
    const int n0 = it.n0, n1 = it.n1, len = it.len;
    const int ntiles = n1 > n0 ? (n1 - n0 + BK - 1) / BK : 0;
    // Q^T fragments (B operand, 16 head-dim x 8 rows a k-step): one ldmatrix.x4 gives two k-steps of a row tile.
    const uint32_t qaddr = smem_u32(sm + C::Q_OFF + qs * C::QSLOT);
    auto q_frag = [&](int nt, int k2, uint32_t* x) {
      const int r = nt * 8 + (lane & 7), c = k2 * 4 + (lane >> 3);
      ldsm_x4(qaddr + (c / 8) * RP * 128 + swz(0, r, c % 8), x);
    };
    uint32_t qb[C::Q_REGS ? NT : 1][C::Q_REGS ? KD / 2 : 1][4];
    if constexpr (C::Q_REGS) {
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int k2 = 0; k2 < KD / 2; ++k2) q_frag(nt, k2, qb[nt][k2]);
      __syncwarp();
      if (lane == 0) mbar_arrive(&q_empty[qs]);
    }

    int lim[NT][2];  // last visible key of rows nt 8 + 2 qid + e; -1 for padding rows
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int r = nt * 8 + 2 * qid + e;
        lim[nt][e] = r >= p.rows ? -1 : (p.causal ? len - p.T + (r % p.T) : len - 1);
      }
    float m_run[NT][2], l_run[NT][2];
    float acc[NT][KD][4];  // O^T: (head dim 16 j + quad (+8), rows nt 8 + 2 qid (+1))
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      m_run[nt][0] = m_run[nt][1] = -INFINITY;
      l_run[nt][0] = l_run[nt][1] = 0.f;
#pragma unroll
      for (int j = 0; j < KD; ++j) acc[nt][j][0] = acc[nt][j][1] = acc[nt][j][2] = acc[nt][j][3] = 0.f;
    }

    for (int i = 0; i < ntiles; ++i, ++gt) {
      if (C::GROUPS > 1 && (gt & 1) != grp) continue;  // the other group's tile
      const int st = gt % STAGES;
      if (!mbar_wait(&full[st], (gt / STAGES) & 1, 6)) {
        ok = false;
        break;
      }
      const uint32_t kt = smem_u32(sm + st * C::STAGE_BYTES);
      const uint32_t vt = kt + C::TILE_BYTES;
      const int kbase = n0 + i * BK + wq * 16;  // this warp's first key
      // Rows of this warp's 16 keys past the sequence (capacity padding may hold anything): zero V there so that
      // P = 0 never meets a non-finite value.
      const int nvalid = min(16, max(0, n1 - kbase));
      if (nvalid < 16) {
        uint8_t* vrow = sm + st * C::STAGE_BYTES + C::TILE_BYTES;
        for (int e = lane; e < (16 - nvalid) * (D / 8); e += 32) {
          const int r = wq * 16 + nvalid + e / (D / 8), c = e % (D / 8);
          *reinterpret_cast<uint4*>(vrow + swz(c / 8, r, c % 8)) = make_uint4(0, 0, 0, 0);
        }
        __syncwarp();
      }
      // S^T = K Q^T: (keys quad, quad + 8) x (rows 2 qid, 2 qid + 1) a lane
      float sc[NT][4];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.f;
#pragma unroll
      for (int kk = 0; kk < KD; ++kk) {
        uint32_t ka[4];
        const int r = wq * 16 + (lane & 15), c = kk * 2 + (lane >> 4);
        ldsm_x4(kt + swz(c / 8, r, c % 8), ka);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          if constexpr (C::Q_REGS) {
            mma16816<T>(sc[nt], ka, qb[nt][kk >> 1][2 * (kk & 1)], qb[nt][kk >> 1][2 * (kk & 1) + 1]);
          } else {
            uint32_t x[4];
            q_frag(nt, kk >> 1, x);
            mma16816<T>(sc[nt], ka, x[2 * (kk & 1)], x[2 * (kk & 1) + 1]);
          }
        }
      }
      // online softmax over this warp's 16 keys (a row's keys are spread over the lanes of equal qid)
      uint32_t pb[NT][2];
      const int key0 = kbase + quad, key1 = key0 + 8;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          float& x0 = sc[nt][e];
          float& x1 = sc[nt][2 + e];
          x0 = (key0 < n1 && key0 <= lim[nt][e]) ? x0 * p.scale_log2 : -INFINITY;
          x1 = (key1 < n1 && key1 <= lim[nt][e]) ? x1 * p.scale_log2 : -INFINITY;
          float mx = fmaxf(x0, x1);
          mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
          mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
          mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
          const float m_new = fmaxf(m_run[nt][e], mx);
          const float m_use = m_new == -INFINITY ? 0.f : m_new;
          const float corr = ex2(m_run[nt][e] - m_use);
          m_run[nt][e] = m_new;
          x0 = ex2(x0 - m_use);
          x1 = ex2(x1 - m_use);
          l_run[nt][e] = l_run[nt][e] * corr + x0 + x1;
#pragma unroll
          for (int j = 0; j < KD; ++j) {
            acc[nt][j][e] *= corr;
            acc[nt][j][2 + e] *= corr;
          }
        }
        // P^T as the B operand (16 keys x 8 rows): transpose the two 8 x 8 (key, row) blocks
        pb[nt][0] = movm_t(pack2<T>(sc[nt][0], sc[nt][1]));
        pb[nt][1] = movm_t(pack2<T>(sc[nt][2], sc[nt][3]));
      }
      // O^T += V^T P^T: V^T fragments (A operand, 16 head-dim x 16 keys) by transposing loads of V rows
#pragma unroll
      for (int j = 0; j < KD; ++j) {
        uint32_t va[4];
        const int r = wq * 16 + (lane & 7) + 8 * (lane >> 4);
        const int c = 2 * j + ((lane >> 3) & 1);
        ldsm_x4_t(vt + swz(c / 8, r, c % 8), va);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) mma16816<T>(acc[nt][j], va, pb[nt][0], pb[nt][1]);
      }
      if (nvalid < 16) fence_proxy_async_shared();  // generic writes above precede the next TMA into this stage
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);
    }
    if constexpr (!C::Q_REGS) {
      __syncwarp();
      if (lane == 0) mbar_arrive(&q_empty[qs]);
    }

    // -------------------------------------------------------------- item epilogue: this warp's partial
    // Each warp drops its (max, sum, unnormalised O) for the item's rows into the part area and goes on to the next
    // item while the producer keeps streaming; the merger warp folds them into the item's one partial in the
    // workspace (split_combine_kernel then merges the partials of each (b, hk, row)).
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        l_run[nt][e] += __shfl_xor_sync(0xffffffffu, l_run[nt][e], 4);
        l_run[nt][e] += __shfl_xor_sync(0xffffffffu, l_run[nt][e], 8);
        l_run[nt][e] += __shfl_xor_sync(0xffffffffu, l_run[nt][e], 16);
      }
    if (!ok) break;
    if (uc >= 1 && !mbar_wait(part_empty, (uc - 1) & 1, 8)) {  // the merger has read the previous item's
      ok = false;
      break;
    }
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int r = nt * 8 + 2 * qid + e;
        if (r >= p.rows) continue;
        if (quad == 0) {
          pwml[(warp * RP + r) * 2] = m_run[nt][e];
          pwml[(warp * RP + r) * 2 + 1] = l_run[nt][e];
        }
        float* orow = pwo + (warp * RP + r) * D + quad;
#pragma unroll
        for (int j = 0; j < KD; ++j) {
          orow[16 * j] = acc[nt][j][e];
          orow[16 * j + 8] = acc[nt][j][2 + e];
        }
      }
    __syncwarp();
    if (lane == 0) mbar_arrive(part_full);
    if (!sched.more()) {
      // the CTA's last item: every consumer warp's partial is in the part area once part_full completes; the
      // consumer warps merge them, warp w the rows w, w + CONSUMERS, ...
      if (!mbar_wait(part_full, uc & 1, 11)) {
        ok = false;
        break;
      }
      const size_t part = size_t(it.slot) * p.rows;
      for (int r = warp; r < p.rows; r += CONSUMERS) {
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < CONSUMERS; ++w) M = fmaxf(M, pwml[(w * RP + r) * 2]);
        const float Mu = M == -INFINITY ? 0.f : M;
        float wgt[CONSUMERS], L = 0.f;
#pragma unroll
        for (int w = 0; w < CONSUMERS; ++w) {
          wgt[w] = ex2(pwml[(w * RP + r) * 2] - Mu);
          L += pwml[(w * RP + r) * 2 + 1] * wgt[w];
        }
        for (int c = lane; c < D / 4; c += 32) {
          float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
          for (int w = 0; w < CONSUMERS; ++w) {
            const float4 x = *reinterpret_cast<const float4*>(&pwo[(w * RP + r) * D + 4 * c]);
            o.x += wgt[w] * x.x;
            o.y += wgt[w] * x.y;
            o.z += wgt[w] * x.z;
            o.w += wgt[w] * x.w;
          }
          reinterpret_cast<float4*>(&p.ws_o[(part + r) * D])[c] = o;
        }
        if (lane == 0) *reinterpret_cast<float2*>(&p.ws_ml[(part + r) * 2]) = make_float2(M, L);
      }
    }
  }
}

// Merges the partials of every (b, hk, folded row) of a decode call by log-sum-exp.
template <typename T, int D>
__global__ void __launch_bounds__(256) split_combine_kernel(const Params p) {
  // One block per (b, hk); warp w merges folded rows w, w + 8, ..., lane l the float4 columns l, l + 32, ... Its
  // partials sit in consecutive slots: split mode, (b Hkv + hk) nsplit + s for the nsplit_b splits of b; balanced
  // mode, c + (b Hkv + hk) for the CTAs c whose tile runs meet the pair, found from the pair's first and last tile.
  // After the grid dependency, each lane issues its (max, sum) load and the O loads of the first HELD partials at
  // once (one round trip to L2); a longer span loads the rest once the weights are known.
  constexpr int CW = D / 4;  // float4 columns of a row
  constexpr int CL = (CW + 31) / 32;  // columns a lane
  constexpr int HELD = 8;
  __shared__ int s_tiles[2][8];
  const int bh = blockIdx.x;
  const int b = bh / p.Hkv, hk = bh % p.Hkv;
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const int len = p.kv_len ? min(max(p.kv_len[b], 0), p.N) : p.N;
  int first, nparts;
  if (p.balanced) {
    // tiles (one head) of the sequences before b and of all sequences; kv_len is an input of the call, so this
    // runs before the wait for the decode grid
    int before = 0, total = 0;
    for (int i = tid; i < p.B; i += 256) {
      const int li = p.kv_len ? min(max(p.kv_len[i], 0), p.N) : p.N;
      const int t = (li + BK - 1) / BK;
      total += t;
      if (i < b) before += t;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      before += __shfl_xor_sync(0xffffffffu, before, o);
      total += __shfl_xor_sync(0xffffffffu, total, o);
    }
    if (lane == 0) {
      s_tiles[0][w] = before;
      s_tiles[1][w] = total;
    }
    __syncthreads();
    before = total = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      before += s_tiles[0][i];
      total += s_tiles[1][i];
    }
    const int nt = (len + BK - 1) / BK;
    if (nt == 0) {
      first = 0;
      nparts = 0;
    } else {  // CTA of tile t: the largest c with floor(c total / grid) <= t, i.e. ((t + 1) grid - 1) / total
      const int64_t tt = int64_t(total) * p.Hkv, t0 = int64_t(before) * p.Hkv + int64_t(hk) * nt;
      const int c0 = int(((t0 + 1) * p.grid - 1) / tt), c1 = int(((t0 + nt) * p.grid - 1) / tt);
      first = c0 + bh;
      nparts = c1 - c0 + 1;
    }
  } else {
    first = bh * p.nsplit;
    nparts = max(1, (len + p.split - 1) / p.split);
  }
  // the next kernel of the stream (the next decode, a programmatic dependent) may begin its launch now
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");  // the decode grid has completed and its writes are visible
  const float2* ml = reinterpret_cast<const float2*>(p.ws_ml);
  const float4* wo = reinterpret_cast<const float4*>(p.ws_o);
  for (int r = w; r < p.rows; r += 8) {
    const size_t base = size_t(first) * p.rows + r;  // partial index of (first slot, row r); slot stride p.rows
    float4 xs[HELD][CL];
#pragma unroll
    for (int k = 0; k < HELD; ++k)
#pragma unroll
      for (int j = 0; j < CL; ++j) {
        const int c = lane + 32 * j;
        xs[k][j] = (k < nparts && c < CW) ? __ldcg(wo + (base + size_t(k) * p.rows) * CW + c)
                                          : make_float4(0.f, 0.f, 0.f, 0.f);
      }
    float2 mine = make_float2(-INFINITY, 0.f);  // lane q < 32: partial q's (max, sum)
    if (lane < nparts) mine = __ldcg(ml + base + size_t(lane) * p.rows);
    float M = mine.x;
    for (int q = lane + 32; q < nparts; q += 32) M = fmaxf(M, __ldcg(ml + base + size_t(q) * p.rows).x);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    const float Mu = M == -INFINITY ? 0.f : M;
    float L = lane < nparts ? mine.y * ex2(mine.x - Mu) : 0.f;
    for (int q = lane + 32; q < nparts; q += 32) {
      const float2 x = __ldcg(ml + base + size_t(q) * p.rows);
      L += x.y * ex2(x.x - Mu);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
    float4 acc[CL];
#pragma unroll
    for (int j = 0; j < CL; ++j) acc[j] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int k = 0; k < HELD; ++k) {
      const float mk = __shfl_sync(0xffffffffu, mine.x, k);
      if (k < nparts) {
        const float wk = ex2(mk - Mu);
#pragma unroll
        for (int j = 0; j < CL; ++j) {
          acc[j].x += wk * xs[k][j].x;
          acc[j].y += wk * xs[k][j].y;
          acc[j].z += wk * xs[k][j].z;
          acc[j].w += wk * xs[k][j].w;
        }
      }
    }
    for (int q = HELD; q < nparts; ++q) {
      const float wq = ex2(__ldcg(ml + base + size_t(q) * p.rows).x - Mu);
#pragma unroll
      for (int j = 0; j < CL; ++j) {
        const int c = lane + 32 * j;
        if (c < CW) {
          const float4 x = __ldcg(wo + (base + size_t(q) * p.rows) * CW + c);
          acc[j].x += wq * x.x;
          acc[j].y += wq * x.y;
          acc[j].z += wq * x.z;
          acc[j].w += wq * x.w;
        }
      }
    }
    const float inv = L > 0.f ? 1.f / L : 0.f;
    const int g = r / p.T, t = r % p.T, h = hk * p.G + g;
#pragma unroll
    for (int j = 0; j < CL; ++j) {
      const int c = lane + 32 * j;
      if (c >= CW) continue;
      const float4 v = make_float4(acc[j].x * inv, acc[j].y * inv, acc[j].z * inv, acc[j].w * inv);
      if (p.emit) {
        const size_t ro = (size_t(b) * p.Hq + h) * p.T + t;
        const float lse = L > 0.f ? (M + __log2f(L)) * 0.69314718055994531f : -INFINITY;
        if (p.npush) {
#pragma unroll 1
          for (int i = 0; i < p.npush; ++i) {
            // o rows travel as bf16 (half the NVLink bytes; the merged output is 16-bit anyway), lse as fp32
            uint2 h;
            h.x = pack2<__nv_bfloat16>(v.x, v.y);
            h.y = pack2<__nv_bfloat16>(v.z, v.w);
            reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(p.push_o[i]) + ro * D)[c] = h;
            if (c == 0) p.push_lse[i][ro] = lse;
          }
        } else {
          reinterpret_cast<float4*>(p.part_o + ro * D)[c] = v;
          if (c == 0) p.part_lse[ro] = lse;
        }
      } else {
        T* dst = reinterpret_cast<T*>(p.o) + b * p.o_st[0] + int64_t(h) * p.o_st[1] + int64_t(t) * p.o_st[2] + 4 * c;
        dst[0] = from_f<T>(v.x);
        dst[1] = from_f<T>(v.y);
        dst[2] = from_f<T>(v.z);
        dst[3] = from_f<T>(v.w);
      }
    }
  }
  if (p.npush) {  // the last block to finish announces the call to every rank (release at system scope)
    __threadfence_system();  // this thread's pushed rows reach the peers before the call is announced
    __syncthreads();
    if (threadIdx.x == 0) {
      const uint32_t done = atomicAdd(p.push_count, 1u) + 1u;
      if (done == p.push_epoch * gridDim.x) {
        __threadfence_system();
        for (int i = 0; i < p.npush; ++i)
          asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p.push_flag[i]), "r"(p.push_epoch) : "memory");
      }
    }
  }
}

// Merges R rank partials (normalised o, natural-log lse) row by row: one warp per row. Partial r's o rows start at
// part_o + r so, its lse values at part_lse + r sl (floats).
template <typename T>
__global__ void combine_kernel(const float* __restrict__ part_o, const float* __restrict__ part_lse, int R,
                               int64_t so, int64_t sl, int rows, int Hq, int Tq, int D, void* o, int64_t o0,
                               int64_t o1, int64_t o2) {
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  float M = -INFINITY;
  for (int r = 0; r < R; ++r) M = fmaxf(M, part_lse[r * sl + row]);
  const float Mu = M == -INFINITY ? 0.f : M;
  float wsum = 0.f;
  for (int r = 0; r < R; ++r) wsum += __expf(part_lse[r * sl + row] - Mu);
  const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
  const int t = row % Tq, h = (row / Tq) % Hq, b = row / (Tq * Hq);
  T* orow = reinterpret_cast<T*>(o) + b * o0 + int64_t(h) * o1 + int64_t(t) * o2;
  for (int d = lane; d < D; d += 32) {
    float x = 0.f;
    for (int r = 0; r < R; ++r)
      x += __expf(part_lse[r * sl + row] - Mu) * part_o[r * so + int64_t(row) * D + d];
    orow[d] = from_f<T>(x * inv);
  }
}

}  // namespace decode
}  // namespace lb2
