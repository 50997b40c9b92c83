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

}  // namespace kvg
}  // namespace lb2
