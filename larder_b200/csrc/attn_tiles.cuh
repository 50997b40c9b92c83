// Kept-tile lists of an array mask, for the prefill kernels' tile skipping (the B200 form of qsa_tiles.py's
// per-group tile flags and plan, qsa_tiles.py:28-42, :144-190, :351-359).
//
// A QSA mask keeps few keys of each row, in blocks, so most (row block, key tile) pairs of a prefill chunk hold no
// kept key at all. flag_kernel marks the pairs where some row of the block keeps some key of the tile; compact_kernel
// turns each row block's flags into the ascending list of its kept tiles and their count. The prefill kernels then
// walk a block's list instead of every tile up to its horizon: the producer loads only those K / V tiles, the MMA
// warp issues only their products, and the softmax masks them element by element as before, so the result is the
// masked attention's, with the work proportional to the kept tiles.
#pragma once

#include "common.cuh"

namespace lb2 {
namespace tiles {

// flags[rb * nkt + kt] = 1 when a row of [rb RB, rb RB + RB) and a key of [kt BN, kt BN + BN) (clipped to T x N) are
// kept. One CTA a (key tile, row block); each thread stops at its first kept element. With `vec` (rows of unit key
// stride, 16-byte aligned, BN a multiple of 16) a thread reads 16 keys a load; otherwise one byte at a time.
__global__ void __launch_bounds__(256) flag_kernel(const uint8_t* mask, int64_t ms0, int64_t ms1, int T, int N, int RB,
                                                   int BN, int nkt, uint8_t* flags, int vec) {
  const int kt = blockIdx.x, rb = blockIdx.y;
  const int r0 = rb * RB, rows = min(T, r0 + RB) - r0, k0 = kt * BN, w = min(N, k0 + BN) - k0;
  int any = 0;
  if (vec) {
    const int cpr = (w + 15) >> 4;  // 16-byte pieces a row (the last may be short)
    for (int i = threadIdx.x; i < rows * cpr && !any; i += blockDim.x) {
      const int r = i / cpr, j = i - r * cpr;
      const uint8_t* pc = mask + int64_t(r0 + r) * ms0 + k0 + 16 * j;
      if (16 * j + 16 <= w) {
        const uint4 u = *reinterpret_cast<const uint4*>(pc);
        any = (u.x | u.y | u.z | u.w) != 0u;
      } else {
        for (int e = 0; e < w - 16 * j; ++e) any |= pc[e] != 0;
      }
    }
  } else {
    for (int i = threadIdx.x; i < rows * w && !any; i += blockDim.x) {
      const int r = r0 + i / w, c = k0 + i % w;
      any = mask[int64_t(r) * ms0 + int64_t(c) * ms1] != 0;
    }
  }
  any = __syncthreads_or(any);
  if (threadIdx.x == 0) flags[int64_t(rb) * nkt + kt] = uint8_t(any);
}

// list[rb * nkt + i] = the i-th kept tile of row block rb, ascending; count[rb] = how many. One warp a row block.
__global__ void __launch_bounds__(128) compact_kernel(const uint8_t* flags, int nrb, int nkt, int32_t* list,
                                                      int32_t* count) {
  const int rb = blockIdx.x * 4 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (rb >= nrb) return;
  int n = 0;
  for (int k0 = 0; k0 < nkt; k0 += 32) {
    const int kt = k0 + lane;
    const bool f = kt < nkt && flags[int64_t(rb) * nkt + kt];
    const unsigned m = __ballot_sync(0xffffffffu, f);
    if (f) list[int64_t(rb) * nkt + n + __popc(m & ((1u << lane) - 1u))] = kt;
    n += __popc(m);
  }
  if (lane == 0) count[rb] = n;
}

}  // namespace tiles
}  // namespace lb2
