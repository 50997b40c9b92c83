// Gathers for QSA decode over picked KV blocks, and the paged KV home.
//
// pick rows: the reference's QSA decode attends to the sorted picked blocks tb (block size CR) and the sequence's
// trailing partial block (stream_fast.py:6448-6491): gathered row r < NSEL * CR is position tb[r / CR] * CR + r % CR,
// row r >= NSEL * CR is position own0 + r - NSEL * CR with own0 = n / CR * CR; m = NSEL * CR + n - own0 rows.
//
// paged home: the reference's kv_host keeps positions in chunks of 2^LOGC (4096) positions, each chunk laid out
// [K / V][head][2^LOGC][D] and reached through a table of chunk addresses (kv_host.py:17-18, :36-41). The chunks may
// be device memory or pinned, GPU-mapped host memory: the kernels read and write through the table either way.
//
// One warp copies one (row, K or V, head) with 16-byte loads when the row is 16-byte aligned and contiguous.
//
// VRAM LRU (below): the reference's pool of recently picked blocks in device memory, in front of the home.
#pragma once

#include "common.cuh"

namespace lb2 {
namespace kvg {

// CV: bypass the caches on the load (the home may be host memory rewritten after a trim, so a cached copy could be
// stale; the reference's kv_host reads with ld.global.cv for the same reason, kv_host.py:30-34).
template <bool CV, typename T>
__device__ __forceinline__ void copy_row(T* dst, const T* src, int64_t s_st, int D, int lane) {
  constexpr int VEC = 16 / sizeof(T);
  if (s_st == 1 && D % VEC == 0 && ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 15) == 0) {
    for (int c = lane; c < D / VEC; c += 32) {
      const uint4* sp = reinterpret_cast<const uint4*>(src) + c;
      reinterpret_cast<uint4*>(dst)[c] = CV ? __ldcv(sp) : __ldg(sp);
    }
  } else {
    for (int c = lane; c < D; c += 32) dst[c] = src[c * s_st];
  }
}

__device__ __forceinline__ int64_t pick_pos(const int32_t* tb, int nsel, int cr, int own0, int row) {
  return row < nsel * cr ? int64_t(tb[row / cr]) * cr + row % cr : int64_t(own0 + row - nsel * cr);
}

// kg / vg [Hk, m, D] contiguous <- picked rows of k / v [Hk, n, D] (strides k_st / v_st: head, position, dim).
template <typename T>
__global__ void __launch_bounds__(256) gather_picks_kernel(const T* k, int64_t kh, int64_t kn, int64_t kd, const T* v,
                                                           int64_t vh, int64_t vn, int64_t vd, const int32_t* tb,
                                                           int nsel, int cr, int n, T* kg, T* vg, int Hk, int D) {
  const int lane = threadIdx.x & 31;
  const int own0 = n / cr * cr;
  const int m = nsel * cr + n - own0;
  const int row = int((blockIdx.x * int64_t(blockDim.x) + threadIdx.x) >> 5);
  const int h = blockIdx.y;
  if (row >= m) return;
  const int64_t pos = pick_pos(tb, nsel, cr, own0, row);
  if (blockIdx.z == 0)
    copy_row<false>(kg + (int64_t(h) * m + row) * D, k + h * kh + pos * kn, kd, D, lane);
  else
    copy_row<false>(vg + (int64_t(h) * m + row) * D, v + h * vh + pos * vn, vd, D, lane);
}

// Address of position pos of K (kv 0) or V (kv 1), head h, in the paged home.
template <typename T>
__device__ __forceinline__ T* home_row(const uint64_t* tbl, int64_t pos, int kv, int h, int Hk, int D, int logc) {
  const int64_t i = pos & ((int64_t(1) << logc) - 1);
  return reinterpret_cast<T*>(tbl[pos >> logc]) + ((((int64_t(kv) * Hk + h) << logc) + i) * D);
}

// Writes s new positions pos0 .. pos0 + s - 1 of k_new / v_new [Hk, s, D] (strides) into the home.
template <typename T>
__global__ void __launch_bounds__(256) home_put_kernel(const uint64_t* tbl, const T* k, int64_t kh, int64_t kn,
                                                       int64_t kd, const T* v, int64_t vh, int64_t vn, int64_t vd,
                                                       int64_t pos0, int s, int Hk, int D, int logc) {
  const int lane = threadIdx.x & 31;
  const int row = int((blockIdx.x * int64_t(blockDim.x) + threadIdx.x) >> 5);
  const int h = blockIdx.y;
  if (row >= s) return;
  const int kv = blockIdx.z;
  T* dst = home_row<T>(tbl, pos0 + row, kv, h, Hk, D, logc);
  if (kv == 0)
    copy_row<false>(dst, k + h * kh + int64_t(row) * kn, kd, D, lane);
  else
    copy_row<false>(dst, v + h * vh + int64_t(row) * vn, vd, D, lane);
}

// kg / vg [Hk, m, D] <- the picked rows (as gather_picks_kernel) read from the paged home; n = the sequence length.
template <typename T>
__global__ void __launch_bounds__(256) home_gather_kernel(const uint64_t* tbl, const int32_t* tb, int nsel, int cr,
                                                          int n, T* kg, T* vg, int Hk, int D, int logc) {
  const int lane = threadIdx.x & 31;
  const int own0 = n / cr * cr;
  const int m = nsel * cr + n - own0;
  const int row = int((blockIdx.x * int64_t(blockDim.x) + threadIdx.x) >> 5);
  const int h = blockIdx.y;
  if (row >= m) return;
  const int64_t pos = pick_pos(tb, nsel, cr, own0, row);
  const int kv = blockIdx.z;
  copy_row<true>((kv ? vg : kg) + (int64_t(h) * m + row) * D, home_row<T>(tbl, pos, kv, h, Hk, D, logc), 1, D, lane);
}

// ---------------------------------------------------------------------------------------------- VRAM LRU
//
// The reference's kv_host keeps a pool of recently picked blocks in device memory, slot x holding block bo[x]'s CR
// positions of K and V for every head ([slot][K / V][head][CR][D]), and chooses victims for missed blocks by CLOCK
// (kv_host.py:116-185). State, all int32 on the device: so[block] (slot or -1), bo[slot] (block or -1), st[slot]
// (token stamp of the slot's last use, -1 at first), rf[slot] (reference bit), mt = {hand, token, hits, misses}.

constexpr int LRU_MAX_NSEL = 1024;  // picks a token at most: the plan is one block of NT = ceil32(nsel) threads

// Exclusive rank of f among the block's threads and, in *total, how many threads have f (every thread calls it).
__device__ __forceinline__ int block_rank(bool f, int* wcnt, int* total) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const unsigned m = __ballot_sync(0xffffffffu, f);
  if (lane == 0) wcnt[w] = __popc(m);
  __syncthreads();
  int before = 0, all = 0;
  for (int i = 0; i < nw; ++i) {
    const int c = wcnt[i];
    all += c;
    if (i < w) before += c;
  }
  __syncthreads();  // wcnt reusable
  *total = all;
  return before + __popc(m & ((1u << lane) - 1u));
}

// One token's plan for the sorted, distinct picks tb[0 .. nsel): thread j < nsel owns pick j. A resident block is a
// hit (its slot gets this token's stamp and its reference bit). The misses take victims in CLOCK order from the hand:
// rounds of NT consecutive slots, a slot eligible when not stamped this token and its bit is clear; the eligible ones
// are taken in slot order as needed, and the slots passed over before the last one taken lose their bit (a round
// that takes none clears all the bits it passed). The hand stops after the last victim, or after 2 NS + NT slots when
// fewer were eligible; a miss without a victim reads its rows from the home uncached. sl[j] = the hit's slot,
// -2 - victim, or -1. A pick outside [0, max_blocks) is no hit and no miss (sl -1, status word set).
__global__ void __launch_bounds__(LRU_MAX_NSEL) lru_plan_kernel(const int32_t* tb, int nsel, int32_t* so,
                                                                int max_blocks, int32_t* bo, int32_t* st, int32_t* rf,
                                                                int32_t* mt, int ns, int32_t* sl) {
  __shared__ int wcnt[32];
  __shared__ int vict[LRU_MAX_NSEL];
  __shared__ int cut;
  const int j = threadIdx.x, nt = blockDim.x;
  const int t = mt[1] + 1;
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
  __syncthreads();
  int M;
  const int rank = block_rank(b >= 0 && s < 0, wcnt, &M);
  const int hand = mt[0];
  int found = 0, scanned = 0;
  while (found < M && scanned < 2 * ns + nt) {  // found, scanned: the same in every thread
    const int x = int((int64_t(hand) + scanned + j) % ns);
    const bool prot = st[x] == t;
    const bool el = !prot && rf[x] == 0;
    int E;
    const int e = block_rank(el, wcnt, &E);
    const int take = min(E, M - found);
    if (j == 0) cut = nt - 1;
    __syncthreads();
    if (el && take == M - found && e == take - 1) cut = j;  // the last victim this token needs
    if (el && e < take) {
      vict[found + e] = x;
      st[x] = t;
    }
    __syncthreads();
    if (j <= cut && !prot && !el) rf[x] = 0;  // a second chance used up
    found += take;
    scanned += cut + 1;
    __syncthreads();  // this round's writes and reads of cut before the next round
  }
  if (j < nsel) {
    if (s >= 0) {
      sl[j] = s;
    } else if (b >= 0 && rank < found) {
      const int x = vict[rank];
      const int old = bo[x];
      if (old >= 0) so[old] = -1;  // evicted (a resident block: never one of this token's misses)
      bo[x] = b;
      so[b] = x;
      rf[x] = 0;
      sl[j] = -2 - x;
    } else {
      sl[j] = -1;
    }
  }
  if (j == 0) {
    mt[0] = int((int64_t(hand) + scanned) % ns);
    mt[1] = t;
    mt[2] += nsel - M;
    mt[3] += M;
  }
}

// The QSA decode rows of one token over the home with the LRU (kv_host.py:187-257): rows r < m as home_gather_kernel
// (m = nsel * cr + n - own0), plus row m, the new position n - 1. Each row's source: the new k / v row (kn / vn,
// [Hk, D] with strides) for position n - 1 wherever it falls, else the pool for a hit, else the home (cache-bypassing
// loads); a miss with a victim also writes its rows into the victim's slot, and row m writes the new row into the
// home. A row whose position falls outside [0, n) is written as zeros (status word set).
template <typename T>
__global__ void __launch_bounds__(256) lru_gather_kernel(const uint64_t* tbl, T* pool, int ns, const int32_t* tb,
                                                         const int32_t* sl, int nsel, int cr, int n, const T* kn,
                                                         int64_t knh, int64_t knd, const T* vn, int64_t vnh,
                                                         int64_t vnd, T* kg, T* vg, int Hk, int D, int logc) {
  const int lane = threadIdx.x & 31;
  const int own0 = n / cr * cr;
  const int m = nsel * cr + n - own0;
  const int row = int((blockIdx.x * int64_t(blockDim.x) + threadIdx.x) >> 5);
  const int h = blockIdx.y, kv = blockIdx.z;
  if (row > m) return;
  int64_t pos;
  int slot = -1, vic = -1;
  if (row == m) {
    pos = n - 1;
  } else if (row >= nsel * cr) {
    pos = own0 + row - nsel * cr;
  } else {
    const int jj = row / cr;
    pos = int64_t(tb[jj]) * cr + row % cr;
    const int c = sl[jj];
    slot = c >= 0 ? c : -1;
    vic = c <= -2 ? -2 - c : -1;
    if (slot >= ns || vic >= ns) {
      report_bad_index(92);
      slot = vic = -1;
    }
  }
  T* out = (kv ? vg : kg) + (int64_t(h) * m + row) * D;
  if (pos < 0 || pos >= n) {
    report_bad_index(93);
    if (row < m)
      for (int c = lane; c < D; c += 32) out[c] = from_f<T>(0.f);
    return;
  }
  T* dst = row == m ? home_row<T>(tbl, pos, kv, h, Hk, D, logc) : out;
  T* fill = vic >= 0 ? pool + ((int64_t(vic) * 2 + kv) * Hk + h) * int64_t(cr) * D + int64_t(row % cr) * D : nullptr;
  if (pos == n - 1) {
    const T* src = kv ? vn + h * vnh : kn + h * knh;
    copy_row<false>(dst, src, kv ? vnd : knd, D, lane);
    if (fill) copy_row<false>(fill, src, kv ? vnd : knd, D, lane);
  } else if (slot >= 0) {
    copy_row<false>(dst, pool + ((int64_t(slot) * 2 + kv) * Hk + h) * int64_t(cr) * D + int64_t(row % cr) * D, 1,
                    D, lane);
  } else {
    const T* src = home_row<T>(tbl, pos, kv, h, Hk, D, logc);
    copy_row<true>(dst, src, 1, D, lane);
    if (fill) copy_row<true>(fill, src, 1, D, lane);
  }
}

// Slots holding a block at or past lim drop it (kv_host.py:259-276): a trim rewrites those positions.
__global__ void __launch_bounds__(256) lru_inval_kernel(int32_t* so, int32_t* bo, int32_t* rf, int ns, int lim) {
  const int x = int(blockIdx.x * blockDim.x + threadIdx.x);
  if (x >= ns) return;
  const int b = bo[x];
  if (b >= 0 && b >= lim) {
    so[b] = -1;
    bo[x] = -1;
    rf[x] = 0;
  }
}

}  // namespace kvg
}  // namespace lb2
