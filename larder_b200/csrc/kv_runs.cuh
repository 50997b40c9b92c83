// The rows a QSA decode step attends to, gathered run by run, and the paged KV home with its VRAM LRU.
//
// Row layout of a gathered step (the order the reference's QSA decode attends in, stream_fast.py:6448-6491): the
// picked blocks tb[0 .. nsel) in order, CR positions each (gathered rows j CR .. j CR + CR - 1 are positions
// tb[j] CR ..), then the trailing partial block, positions own0 .. n - 1 with own0 = n / CR * CR, as rows
// nsel CR ..; m = nsel CR + n - own0 rows in all, [Hk, m, D] per K and V.
//
// Such a step is nsel + 1 runs of consecutive positions. In every source this file reads -- a cache view with a
// position stride, a chunk of the paged home ([K / V][head][2^logc][D], so a CR-aligned block never straddles
// chunks), a pool slot ([K / V][head][CR][D]) -- one run of one head is `len` rows of D values at a fixed row stride,
// and in the output it is len * D contiguous values. So the grid is one CTA a (run, K or V): the CTA resolves the
// run's source once (home, pool slot, victim slot to fill) and moves the run for every head as units spread over its
// threads, unit u of a head's run being row u / upr, column unit u % upr (upr units a row). Positions outside [0, n)
// are never read: their rows are written as zeros and the status word reports the bad index.
//
// Data moves as raw bits: U is uint4 (16-byte units) when every base, stride and row allows it, else the element's
// own width (unsigned short for 16-bit values, unsigned int for fp32), one element a unit. Home chunks must be
// 16-byte aligned for 16-byte units; a run whose chunk is not is written as zeros and reported, never read.
//
// The home may be pinned host memory rewritten after a trim, so home reads bypass the caches (ld.global.cv).
#pragma once

#include "common.cuh"

namespace lb2 {
namespace kvr {

constexpr int RUN_THREADS = 128;

template <typename U>
__device__ __forceinline__ U ld_bypass(const U* p);
template <>
__device__ __forceinline__ uint4 ld_bypass<uint4>(const uint4* p) { return __ldcv(p); }
template <>
__device__ __forceinline__ unsigned int ld_bypass<unsigned int>(const unsigned int* p) { return __ldcv(p); }
template <>
__device__ __forceinline__ unsigned short ld_bypass<unsigned short>(const unsigned short* p) { return __ldcv(p); }

// A source of rows: row r of head h at base + h * hs + r * rs, unit c of a row at + c * us (all in units U).
template <typename U>
struct Rows {
  const U* base;
  int64_t hs, rs, us;
  __device__ __forceinline__ const U* at(int h, int64_t r, int c) const { return base + h * hs + r * rs + c * us; }
};

// The home run starting at pos (K or V, head h), or nullptr (status word set) when its chunk cannot hold units U.
template <typename U>
__device__ __forceinline__ U* home_run(const uint64_t* tbl, int64_t pos, int kv, int h, int Hk, int upr, int logc,
                                       int where) {
  const uint64_t chunk = tbl[pos >> logc];
  if (chunk % alignof(U)) {
    if (threadIdx.x == 0) report_bad_index(where);
    return nullptr;
  }
  const int64_t within = pos & ((int64_t(1) << logc) - 1);
  return reinterpret_cast<U*>(chunk) + (((int64_t(kv) * Hk + h) << logc) + within) * upr;
}

// Run j of a step: its first position, its length and its first gathered row.
struct Run {
  int64_t p0;
  int len, out0;
};
__device__ __forceinline__ Run run_of(const int32_t* tb, int nsel, int cr, int n, int j) {
  const int own0 = n / cr * cr;
  if (j < nsel) return Run{int64_t(tb[j]) * cr, cr, j * cr};
  return Run{own0, n - own0, nsel * cr};
}

// One (run, K or V) of a QSA step from a cache view: gathered rows <- positions of the view (rows of the view:
// positions 0 .. n - 1). Runs 0 .. nsel - 1 are the picked blocks, run nsel the tail.
template <typename U>
__global__ void __launch_bounds__(RUN_THREADS) view_runs_kernel(Rows<U> k, Rows<U> v, const int32_t* tb, int nsel,
                                                                int cr, int n, U* kg, U* vg, int Hk, int upr) {
  const int j = blockIdx.x, kv = blockIdx.y;
  const int m = nsel * cr + n - n / cr * cr;
  const Run run = run_of(tb, nsel, cr, n, j);
  const Rows<U> src = kv ? v : k;
  U* out = kv ? vg : kg;
  const bool inside = run.p0 >= 0 && run.p0 + run.len <= n;
  if (!inside && threadIdx.x == 0) report_bad_index(94);
  const int units = run.len * upr;
  // up to HB heads' loads go out before any store (a store may alias a later load as far as the compiler knows, so
  // a head-by-head loop would wait a round trip a head)
  constexpr int HB = 4;
  for (int h0 = 0; h0 < Hk; h0 += HB)
    for (int u = threadIdx.x; u < units; u += RUN_THREADS) {
      const int r = u / upr, c = u - r * upr;
      U x[HB];
#pragma unroll
      for (int i = 0; i < HB; ++i) x[i] = (inside && h0 + i < Hk) ? *src.at(h0 + i, run.p0 + r, c) : U{};
#pragma unroll
      for (int i = 0; i < HB; ++i)
        if (h0 + i < Hk) out[(int64_t(h0 + i) * m + run.out0) * upr + u] = x[i];
    }
}

// The same rows read from the paged home (table of chunk addresses), n = the sequence length.
template <typename U>
__global__ void __launch_bounds__(RUN_THREADS) home_runs_kernel(const uint64_t* tbl, const int32_t* tb, int nsel,
                                                                int cr, int n, U* kg, U* vg, int Hk, int upr,
                                                                int logc) {
  const int j = blockIdx.x, kv = blockIdx.y;
  const int m = nsel * cr + n - n / cr * cr;
  const Run run = run_of(tb, nsel, cr, n, j);
  U* out = kv ? vg : kg;
  const bool inside = run.p0 >= 0 && run.p0 + run.len <= n;
  if (!inside && threadIdx.x == 0) report_bad_index(95);
  const int units = run.len * upr;
  constexpr int HB = 4;  // heads whose loads go out before any store, as view_runs_kernel
  for (int h0 = 0; h0 < Hk; h0 += HB) {
    const U* src[HB];
#pragma unroll
    for (int i = 0; i < HB; ++i)  // one chunk a run
      src[i] = inside && run.len && h0 + i < Hk ? home_run<U>(tbl, run.p0, kv, h0 + i, Hk, upr, logc, 96) : nullptr;
    for (int u = threadIdx.x; u < units; u += RUN_THREADS) {
      U x[HB];
#pragma unroll
      for (int i = 0; i < HB; ++i) x[i] = src[i] ? ld_bypass(src[i] + u) : U{};
#pragma unroll
      for (int i = 0; i < HB; ++i)
        if (h0 + i < Hk) out[(int64_t(h0 + i) * m + run.out0) * upr + u] = x[i];
    }
  }
}

// Writes s new positions pos0 .. pos0 + s - 1 of k / v (views [Hk, s, D]) into the home. One CTA a (tile of 32
// positions, K or V): the tile's rows of every head as units over the CTA; a tile may cross a chunk boundary, so the
// destination is resolved a row.
template <typename U>
__global__ void __launch_bounds__(RUN_THREADS) home_put_kernel(const uint64_t* tbl, Rows<U> k, Rows<U> v,
                                                               int64_t pos0, int s, int Hk, int upr, int logc) {
  const int kv = blockIdx.y;
  const int r0 = blockIdx.x * 32;
  const int rows = min(32, s - r0);
  const Rows<U> src = kv ? v : k;
  for (int h = 0; h < Hk; ++h)
    for (int u = threadIdx.x; u < rows * upr; u += RUN_THREADS) {
      const int r = u / upr, c = u - r * upr;
      U* row = home_run<U>(tbl, pos0 + r0 + r, kv, h, Hk, upr, logc, 97);
      if (row) row[c] = *src.at(h, r0 + r, c);
    }
}

// ---------------------------------------------------------------------------------------------- VRAM LRU
//
// A pool of ns slots in device memory in front of the home: slot x holds block bo[x]'s CR positions of K and V for
// every head ([slot][K / V][head][CR][D]). State (int32, device): so[block] = its slot or -1, bo[slot] = its block or
// -1, st[slot] = the token that last used it (-1 at first), rf[slot] = its reference bit, mt = {hand, tokens, hits,
// misses}. The replacement policy is CLOCK with second chances and is observable (which slot a block lands in), so it
// is fixed exactly; see lru_plan_kernel.

constexpr int LRU_MAX_NSEL = 1024;

// One token's plan for its distinct picks tb[0 .. nsel), by a single warp.
//  1. Hits: a pick whose block has a slot stamps the slot with this token (t = mt[1] + 1) and sets its reference bit.
//     The other in-range picks are the misses, ranked in pick order.
//  2. Victims: a CLOCK sweep from the hand, 32 slots a step (lane i at slot (hand + swept + i) mod ns; ns >= 32, so
//     no slot appears twice in a step). A slot stamped this token is passed over untouched; one with a clear bit is a
//     victim (stamped with t); one with its bit set loses it. Victims are taken in slot order until every miss has
//     one, and the sweep ends right after the last victim taken (slots after it keep their bits). The sweep gives up
//     after L slots, L the first multiple of NT = ceil32(nsel) at or above 2 ns + NT, so that a token whose misses
//     outnumber the slots it may evict leaves the rest uncached. Stepping slot by slot this way takes the same
//     victims and clears the same bits as a sweep taken in rounds of NT slots with the same bound (each slot is seen
//     once in a round, and a round only ends early at its last victim).
//  3. The i-th miss takes the i-th victim: the victim's old block (never a pick of this token: a slot holding one is
//     stamped t) loses its slot. sl[j] = the hit's slot, -2 - victim for a miss with one, -1 otherwise (read from the
//     home uncached). A pick outside [0, max_blocks) is neither (sl -1, status word set).
__global__ void __launch_bounds__(32) lru_plan_kernel(const int32_t* tb, int nsel, int32_t* so, int max_blocks,
                                                      int32_t* bo, int32_t* st, int32_t* rf, int32_t* mt, int ns,
                                                      int32_t* sl) {
  __shared__ int victim[LRU_MAX_NSEL];
  const int lane = threadIdx.x;
  const unsigned below = (1u << lane) - 1u;
  const int t = mt[1] + 1;
  const int hand = mt[0];
  int misses = 0;
  for (int j0 = 0; j0 < nsel; j0 += 32) {
    const int j = j0 + lane;
    int b = -1, s = -1;
    if (j < nsel) {
      b = tb[j];
      if (b < 0 || b >= max_blocks) {
        report_bad_index(91);
        b = -1;
      } else {
        s = so[b];
      }
    }
    if (s >= 0) {
      st[s] = t;
      rf[s] = 1;
    }
    misses += __popc(__ballot_sync(0xffffffffu, b >= 0 && s < 0));
  }
  __syncwarp();  // the hits' stamps are seen by the sweep
  const int nt = (nsel + 31) & ~31;
  const int limit = (2 * ns + nt + nt - 1) / nt * nt;
  int found = 0, swept = 0;
  while (found < misses && swept < limit) {
    const int x = (hand + swept + lane) % ns;
    const bool used = st[x] == t;
    const bool free_ = !used && rf[x] == 0;
    const unsigned fm = __ballot_sync(0xffffffffu, free_);
    const int need = misses - found;
    const int e = __popc(fm & below);
    int take = __popc(fm), last = 31;
    if (take >= need) {
      take = need;
      last = __ffs(__ballot_sync(0xffffffffu, free_ && e == need - 1)) - 1;
    }
    if (free_ && e < take) {
      victim[found + e] = x;
      st[x] = t;
    }
    if (lane <= last && !used && !free_) rf[x] = 0;
    found += take;
    swept += last + 1;
    __syncwarp();
  }
  __syncwarp();
  int rank0 = 0;
  for (int j0 = 0; j0 < nsel; j0 += 32) {
    const int j = j0 + lane;
    int b = -1, s = -1;
    if (j < nsel) {
      b = tb[j];
      if (b < 0 || b >= max_blocks) b = -1;
      else s = so[b];  // as step 1 saw it: only this lane writes so[b] below
    }
    const bool miss = b >= 0 && s < 0;
    const unsigned mm = __ballot_sync(0xffffffffu, miss);
    const int rank = rank0 + __popc(mm & below);
    rank0 += __popc(mm);
    if (j >= nsel) continue;
    if (s >= 0) {
      sl[j] = s;
    } else if (miss && rank < found) {
      const int x = victim[rank];
      const int old = bo[x];
      if (old >= 0) so[old] = -1;
      bo[x] = b;
      so[b] = x;
      rf[x] = 0;
      sl[j] = -2 - x;
    } else {
      sl[j] = -1;
    }
  }
  if (lane == 0) {
    mt[0] = (hand + swept) % ns;
    mt[1] = t;
    mt[2] += nsel - misses;
    mt[3] += misses;
  }
}

// One token's QSA rows through the LRU, a CTA a (run, K or V) as home_runs_kernel: run j < nsel reads its block from
// the pool slot on a hit, else from the home, and a miss with a victim writes the rows it read into the victim's
// slot too; run nsel is the tail, read from the home. Position n - 1 (the new one) comes from kn / vn ([Hk, D] rows)
// wherever it falls, and the tail's CTA also writes that new row into the home.
template <typename U>
__global__ void __launch_bounds__(RUN_THREADS) lru_runs_kernel(const uint64_t* tbl, U* pool, int ns, const int32_t* tb,
                                                               const int32_t* sl, int nsel, int cr, int n, Rows<U> kn,
                                                               Rows<U> vn, U* kg, U* vg, int Hk, int upr, int logc) {
  const int j = blockIdx.x, kv = blockIdx.y;
  const int m = nsel * cr + n - n / cr * cr;
  const Run run = run_of(tb, nsel, cr, n, j);
  int slot = -1, vic = -1;
  if (j < nsel) {
    const int c = sl[j];
    slot = c >= 0 ? c : -1;
    vic = c <= -2 ? -2 - c : -1;
    if (slot >= ns || vic >= ns) {
      if (threadIdx.x == 0) report_bad_index(92);
      slot = vic = -1;
    }
  }
  const Rows<U> fresh = kv ? vn : kn;
  U* out = kv ? vg : kg;
  const bool inside = run.p0 >= 0 && run.p0 + run.len <= n;
  if (!inside && threadIdx.x == 0) report_bad_index(93);
  const int64_t newest = int64_t(n) - 1 - run.p0;  // the run's row holding position n - 1 (none if outside [0, len))
  const int units = inside ? run.len * upr : 0;
  const int64_t slot_units = int64_t(2) * Hk * cr * upr;
  for (int h = 0; h < Hk; ++h) {
    U* dst = out + (int64_t(h) * m + run.out0) * upr;
    const int64_t in_slot = (int64_t(kv) * Hk + h) * cr * upr;
    const U* from_pool = slot >= 0 ? pool + slot * slot_units + in_slot : nullptr;
    U* fill = vic >= 0 ? pool + vic * slot_units + in_slot : nullptr;
    const U* from_home = units && !from_pool ? home_run<U>(tbl, run.p0, kv, h, Hk, upr, logc, 98) : nullptr;
    for (int u = threadIdx.x; u < units; u += RUN_THREADS) {
      const int r = u / upr, c = u - r * upr;
      U x{};
      if (r == newest) x = *fresh.at(h, 0, c);
      else if (from_pool) x = from_pool[u];
      else if (from_home) x = ld_bypass(from_home + u);
      dst[u] = x;
      if (fill) fill[u] = x;
    }
    if (!inside)  // the run's rows are zeros
      for (int u = threadIdx.x; u < run.len * upr; u += RUN_THREADS) dst[u] = U{};
    if (j == nsel) {  // the new position into the home
      U* row = home_run<U>(tbl, int64_t(n) - 1, kv, h, Hk, upr, logc, 99);
      if (row)
        for (int c = threadIdx.x; c < upr; c += RUN_THREADS) row[c] = *fresh.at(h, 0, c);
    }
  }
}

// A trim to lim blocks: every slot holding a block at or past lim gives it up (the positions from lim * CR on are
// about to be rewritten). One warp walks the pool.
__global__ void __launch_bounds__(32) lru_trim_kernel(int32_t* so, int32_t* bo, int32_t* rf, int ns, int lim) {
  for (int x = threadIdx.x; x < ns; x += 32) {
    const int b = bo[x];
    if (b >= lim) {  // (an empty slot holds -1, and lim >= 0)
      so[b] = -1;
      bo[x] = -1;
      rf[x] = 0;
    }
  }
}

}  // namespace kvr
}  // namespace lb2
