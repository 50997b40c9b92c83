// KV-range-sharded decode's exchange over NVLink peer memory: the log-sum-exp merge of every rank's partial
// (foldattn.py:188-211's merge taken across GPUs) reading the peers' partials in place, without a collective.
//
// Each rank owns one exchange buffer in its device memory, shared with the other ranks through CUDA IPC:
//   [parity 0: o rows (rows x D fp32) | lse (rows fp32)] [parity 1: the same] [flags: XCH_MAX_RANKS uint32]
// Call e (e = 1, 2, ...) of a rank writes its partial into half e % 2 of its own buffer (the decode-partial kernel,
// before this one on the stream), then peer_combine_kernel
//   1. publishes: every block's thread 0 stores e into flags[rank] of every peer's buffer (a release at system scope,
//      so the partial's writes are visible to a peer that sees the flag; all blocks publish, so no block waits on a
//      block that has not run);
//   2. waits until its own flags[r] >= e for every peer r (acquire, bounded: 2 s of %globaltimer, then the status word
//      is set and the block writes nothing);
//   3. merges the R partials of its rows, reading the peers' halves e % 2 over NVLink (cache-bypassing loads).
// A rank is at most one call ahead of any peer (its call e + 1 needs every peer's flag e + 1, set after the peer's
// call e ended), so a half is rewritten (call e + 2) only after every peer has finished reading it (call e).
//
// Push mode: a rank's buffer holds every rank's partial (R slots a half; o rows as bf16, half the bytes over NVLink),
// and the decode partial of call e writes this rank's rows into slot `rank` of half e % 2 of EVERY rank's buffer (peer stores over NVLink, fenced at system
// scope). The combine then publishes and waits exactly as above, and merges the R slots of its OWN buffer -- local
// reads only. A peer writes half e % 2 of this buffer for call e + 2 only after it has seen this rank's flag e + 1,
// published when this rank's merge of call e was done.
#pragma once

#include "common.cuh"

namespace lb2 {
namespace xch {

constexpr int XCH_MAX_RANKS = 8;

struct PeerParams {
  const float* bufs[XCH_MAX_RANKS];  // every rank's exchange buffer as mapped in this process (bufs[rank]: its own)
  int R, rank, parity;
  uint32_t epoch;
  int64_t half;  // floats in one parity half: rows * (D + 1), or R slots of that in push mode
  int pushed;    // push mode: every rank's partial is in this rank's own buffer, slot r at parity half + r rows (D + 1)
  int rows, Hq, Tq, D;
  int vec;  // the vector merge (every slot 16-byte aligned: rows % 4 == 0; D = 64, 128 or 256), else the scalar one
  void* o;
  int64_t o0, o1, o2;
};

__host__ __device__ constexpr int64_t flags_offset(int64_t half) { return 2 * half; }  // in floats

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// E consecutive values of a partial's o row (lane `lane` of the row's warp): bf16 in push mode, fp32 otherwise.
template <int E>
__device__ __forceinline__ void load_part(const float* src, int64_t o_at, bool pushed, float* v) {
  if (pushed) {
    const unsigned short* s16 = reinterpret_cast<const unsigned short*>(src) + o_at;
    uint32_t w[E / 2];
    if constexpr (E == 2) {
      w[0] = __ldcv(reinterpret_cast<const unsigned int*>(s16));
    } else if constexpr (E == 4) {
      const uint2 u = __ldcv(reinterpret_cast<const uint2*>(s16));
      w[0] = u.x, w[1] = u.y;
    } else {
      const uint4 u = __ldcv(reinterpret_cast<const uint4*>(s16));
      w[0] = u.x, w[1] = u.y, w[2] = u.z, w[3] = u.w;
    }
#pragma unroll
    for (int i = 0; i < E / 2; ++i) v[2 * i] = __uint_as_float(w[i] << 16), v[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  } else {
    const float* s32 = src + o_at;
#pragma unroll
    for (int i = 0; i < E; i += 2) {
      const float2 u = __ldcv(reinterpret_cast<const float2*>(s32 + i));
      v[i] = u.x, v[i + 1] = u.y;
    }
  }
}

// The merge of one row: every rank's o values (E a lane) and lse are loaded before any arithmetic, so that all the
// loads are in flight at once (one round trip), then weighted by exp(lse_r - max) and normalised.
template <typename T, int E>
__device__ __forceinline__ void merge_row(const PeerParams& p, const float* const* src, int row, int lane) {
  const int64_t lse_at = int64_t(p.rows) * p.D + row;
  const int64_t o_at = int64_t(row) * p.D + lane * E;
  float v[XCH_MAX_RANKS][E];
  float lse[XCH_MAX_RANKS];
#pragma unroll
  for (int r = 0; r < XCH_MAX_RANKS; ++r) {
    if (r < p.R) {
      load_part<E>(src[r], o_at, p.pushed != 0, v[r]);
      lse[r] = __ldcv(src[r] + lse_at);
    } else {
#pragma unroll
      for (int e = 0; e < E; ++e) v[r][e] = 0.f;
      lse[r] = -INFINITY;
    }
  }
  float M = -INFINITY;
#pragma unroll
  for (int r = 0; r < XCH_MAX_RANKS; ++r) M = fmaxf(M, lse[r]);
  const float Mu = M == -INFINITY ? 0.f : M;
  float wsum = 0.f;
#pragma unroll
  for (int r = 0; r < XCH_MAX_RANKS; ++r) {
    lse[r] = r < p.R ? __expf(lse[r] - Mu) : 0.f;  // the weights
    wsum += lse[r];
  }
  const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
  const int t = row % p.Tq, h = (row / p.Tq) % p.Hq, b = row / (p.Tq * p.Hq);
  T* orow = reinterpret_cast<T*>(p.o) + b * p.o0 + int64_t(h) * p.o1 + int64_t(t) * p.o2 + lane * E;
#pragma unroll
  for (int e = 0; e < E; ++e) {
    float x = 0.f;
#pragma unroll
    for (int r = 0; r < XCH_MAX_RANKS; ++r)
      if (r < p.R) x += lse[r] * v[r][e];
    orow[e] = from_f<T>(x * inv);
  }
}

// The same merge a value at a time (any D, any slot alignment).
template <typename T>
__device__ __forceinline__ void merge_row_scalar(const PeerParams& p, const float* const* src, int row, int lane) {
  const int64_t lse_at = int64_t(p.rows) * p.D + row;
  float lse[XCH_MAX_RANKS];
  float M = -INFINITY;
#pragma unroll
  for (int r = 0; r < XCH_MAX_RANKS; ++r) {
    lse[r] = r < p.R ? __ldcv(src[r] + lse_at) : -INFINITY;
    M = fmaxf(M, lse[r]);
  }
  const float Mu = M == -INFINITY ? 0.f : M;
  float wsum = 0.f;
#pragma unroll
  for (int r = 0; r < XCH_MAX_RANKS; ++r) {
    lse[r] = r < p.R ? __expf(lse[r] - Mu) : 0.f;
    wsum += lse[r];
  }
  const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
  const int t = row % p.Tq, h = (row / p.Tq) % p.Hq, b = row / (p.Tq * p.Hq);
  T* orow = reinterpret_cast<T*>(p.o) + b * p.o0 + int64_t(h) * p.o1 + int64_t(t) * p.o2;
  const int64_t o_at = int64_t(row) * p.D;
  for (int d = lane; d < p.D; d += 32) {
    float x = 0.f;
#pragma unroll
    for (int r = 0; r < XCH_MAX_RANKS; ++r)
      if (r < p.R)
        x += lse[r] * (p.pushed ? __bfloat162float(__ushort_as_bfloat16(__ldcv(
                                      reinterpret_cast<const unsigned short*>(src[r]) + o_at + d)))
                                : __ldcv(src[r] + o_at + d));
    orow[d] = from_f<T>(x * inv);
  }
}

template <typename T>
__global__ void __launch_bounds__(256) peer_combine_kernel(const __grid_constant__ PeerParams p) {
  __shared__ int s_ok;
  // launched as a programmatic dependent: the next kernel may begin its launch now, and this one waits for the
  // stream's previous kernel (the decode partial) to complete before anything below
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (threadIdx.x == 0) {
    s_ok = 1;
    if (!p.pushed) __threadfence_system();  // the partial (written before this kernel on the stream) ahead of the flags
    for (int r = 0; r < p.R && !p.pushed; ++r)  // (push mode: the decode's last block announced the call)
      if (r != p.rank) {
        uint32_t* f = reinterpret_cast<uint32_t*>(const_cast<float*>(p.bufs[r]) + flags_offset(p.half)) + p.rank;
        st_release_sys(f, p.epoch);
      }
  }
  __syncthreads();
  // thread r waits for peer r's flag (all peers at once, each wait bounded); the block barrier then orders every
  // thread's reads of the partials after the observed flags
  if (int(threadIdx.x) < p.R && int(threadIdx.x) != p.rank) {
    const uint32_t* mine = reinterpret_cast<const uint32_t*>(p.bufs[p.rank] + flags_offset(p.half));
    const int r = threadIdx.x;
    uint64_t t0 = 0;
    for (uint32_t i = 1; int32_t(ld_acquire_sys(mine + r) - p.epoch) < 0; ++i) {
      if ((i & 255u) == 0) {
        const uint64_t now = globaltimer_ns();
        if (t0 == 0) {
          t0 = now;
        } else if (now - t0 > kWaitNs) {
          report_timeout(101);
          s_ok = 0;
          break;
        }
      }
    }
  }
  __syncthreads();
  if (!s_ok) return;
  // one warp a row, as decode::combine_kernel, with rank r's partial at bufs[r] + parity * half (pull mode: read over
  // NVLink) or in this rank's own buffer, slot r (push mode: the peers wrote it here)
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= p.rows) return;
  const int64_t base = int64_t(p.parity) * p.half;
  const int64_t slot = int64_t(p.rows) * (p.D + 1);
  const float* src[XCH_MAX_RANKS];
#pragma unroll
  for (int r = 0; r < XCH_MAX_RANKS; ++r)
    src[r] = r < p.R ? (p.pushed ? p.bufs[p.rank] + base + r * slot : p.bufs[r] + base) : nullptr;
  if (!p.vec)
    merge_row_scalar<T>(p, src, row, lane);
  else if (p.D == 64)
    merge_row<T, 2>(p, src, row, lane);
  else if (p.D == 128)
    merge_row<T, 4>(p, src, row, lane);
  else
    merge_row<T, 8>(p, src, row, lane);
}

}  // namespace xch
}  // namespace lb2
