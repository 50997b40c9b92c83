// QSA indexer block selection (qwen4_exp_vendor.py:271-292, as stream_fast.py's `select` keeps it,
// stream_fast.py:6243-6305): for each query row (b, s), over the pooled block keys p_n (n < n_blocks),
//   score_n = sum_h max(q_h . p_n, 0) / div            (div = sqrt(head_dim), fp32 as the reference's einsum)
//   score_n = -inf when n >= n_complete = (pos_s + 1) // cr   (a block is a candidate only once it is complete)
// and the indices of the k largest scores. The reference takes them with argpartition (unordered, ties unspecified)
// and the decode path sorts them (`tb`, stream_fast.py:6478-6491); here they come out sorted ascending, ties at the
// threshold taken lowest index first, and a row with fewer than k candidates is padded with n_blocks (the
// reference's `where(picked, top, n_blocks)`).
//
// Two kernels: the scores (an HBM stream over the pooled keys, bulk-copied into shared-memory stages, 16 keys a
// warp tile on mma.sync with the heads as columns), then a radix select a row on a cluster of CTAs (four 8-bit passes
// over order-preserving integer keys held in registers, warp-aggregated histogram increments) and an ordered
// compaction that writes the picks in index order.
#pragma once

#include "common.cuh"

namespace lb2 {
namespace qsasel {

struct ScoreParams {
  const __nv_bfloat16* q;       // [B, S, H, D]
  const __nv_bfloat16* pooled;  // [B, ., D]: rows 0 .. n_blocks - 1, batch stride pool_bstride elements
  int64_t pool_bstride;
  float* scores;                // [B * S, n_blocks]
  int B, S, H, n_blocks, cr;
  int ipr;                      // chunks a row: ceil(n_blocks / chunk)
  int64_t items;                // rows * ipr
  int64_t offset;               // row s sits at position offset + s
  float div;
};

constexpr int SC_WARPS = 8;                      // consumer warps
constexpr int SC_THREADS = (SC_WARPS + 1) * 32;  // and one producer warp
constexpr int SC_KEYS = 16 * SC_WARPS;           // keys a chunk: 16 a consumer warp
constexpr int SC_NS = 3;                         // stages
__host__ __device__ constexpr int sc_stage(int D) { return SC_KEYS * D * 2; }  // bytes a stage: one chunk's keys
__host__ __device__ constexpr int sc_smem(int D) { return SC_NS * sc_stage(D) + 2 * SC_NS * 8; }

// D += A B, m16n8k16, bf16 operands, fp32 accumulators (a0..a3 and b0, b1 in the PTX fragment order).
__device__ __forceinline__ void mma_bf16x(float* c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                          uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Persistent CTAs over the items (row, chunk of SC_KEYS keys), each CTA a contiguous range of them. The producer
// warp streams the chunks' keys (contiguous rows of the pooled buffer) into SC_NS shared-memory stages with 1-D bulk
// copies; consumer warp w scores keys 16 w .. 16 w + 15 of a chunk on mma.sync m16n8k16 (bf16 products, fp32 sums)
// with the keys as the 16 rows, the H <= 8 query heads as the 8 columns (heads past H zero) and the head dim as K.
// Lane (g = lane / 4, t = lane % 4) reads rows g and g + 8 16 bytes at a time (elements 32 L + 8 t .. + 8 for
// L < D / 32), so the K order of the MMAs is permuted, the same way for the query fragments: MMA 2 L + u takes, as
// its K pairs (2 t, 2 t + 1) and (2 t + 8, 2 t + 9), elements 32 L + 8 t + 4 u + {0, 1} and + {2, 3}. The sums are
// unchanged. Lane (g, t) ends with keys g and g + 8 against heads 2 t, 2 t + 1: relu, add, then the sum over the
// four lanes of the group. A partial last chunk leaves stale rows in its stage: their rows are computed and dropped.
template <int D>
__global__ void __launch_bounds__(SC_THREADS) score_kernel(const ScoreParams p) {
  constexpr int KL = D / 32;          // 16-byte pieces a lane per key row
  constexpr int STAGE = sc_stage(D);
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + SC_NS * STAGE);
  uint64_t* empty = full + SC_NS;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int64_t j0 = p.items * blockIdx.x / gridDim.x, j1 = p.items * (blockIdx.x + 1) / gridDim.x;
  const int n = int(j1 - j0);
  // the top-k grid may launch now (programmatic dependent launch): it waits for this grid's end before reading
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  if (threadIdx.x == 0) {
    for (int i = 0; i < SC_NS; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], SC_WARPS);
    }
    fence_barrier_init();
  }
  __syncthreads();
  if (warp == SC_WARPS) {  // producer
    if (lane == 0) {
      int j = 0;
      for (; j < n; ++j) {
        const int st = j % SC_NS;
        if (j >= SC_NS && !mbar_wait(&empty[st], ((j / SC_NS) - 1) & 1, 81)) break;
        const int64_t it = j0 + j;
        const int row = int(it / p.ipr), ch = int(it - int64_t(row) * p.ipr);
        const int base = ch * SC_KEYS, nb = min(SC_KEYS, p.n_blocks - base);
        const uint32_t bytes = uint32_t(nb) * D * 2;
        mbar_arrive_expect_tx(&full[st], bytes);
        bulk_g2s(smem + st * STAGE, p.pooled + int64_t(row / p.S) * p.pool_bstride + int64_t(base) * D, bytes,
                 &full[st]);
      }
      // the copies still in flight land before the CTA ends
      for (int i = j > SC_NS ? j - SC_NS : 0; i < j; ++i)
        if (!mbar_wait(&full[i % SC_NS], (i / SC_NS) & 1, 82)) break;
    }
    return;
  }
  int cur_row = -1, n_complete = 0;
  uint4 qb[KL];  // B fragments of the query heads (column g < H), in the permuted K order
  float* out = nullptr;
  for (int j = 0; j < n; ++j) {
    const int st = j % SC_NS;
    const int64_t it = j0 + j;
    const int row = int(it / p.ipr), ch = int(it - int64_t(row) * p.ipr);
    if (row != cur_row) {
      cur_row = row;
      const uint4* qr = reinterpret_cast<const uint4*>(p.q + (int64_t(row) * p.H + g) * D) + t;
#pragma unroll
      for (int l = 0; l < KL; ++l) qb[l] = g < p.H ? qr[4 * l] : make_uint4(0u, 0u, 0u, 0u);
      const int64_t pos = p.offset + (row % p.S);
      const int64_t nc = pos + 1 <= 0 ? 0 : (pos + 1) / p.cr;
      n_complete = nc < p.n_blocks ? int(nc) : p.n_blocks;
      out = p.scores + int64_t(row) * p.n_blocks;
    }
    if (!mbar_wait(&full[st], (j / SC_NS) & 1, 83)) break;
    const int r16 = warp * 16;  // the warp's first key in the chunk
    const uint4* pa = reinterpret_cast<const uint4*>(smem + st * STAGE + (r16 + g) * (D * 2)) + t;
    const uint4* pb = pa + 8 * (D * 2 / 16);  // row g + 8
    uint4 ra[KL], rb[KL];
#pragma unroll
    for (int l = 0; l < KL; ++l) {
      ra[l] = pa[4 * l];
      rb[l] = pb[4 * l];
    }
    __syncwarp();  // the warp's reads of the stage are done
    if (lane == 0) mbar_arrive(&empty[st]);
    float c[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int l = 0; l < KL; ++l) {
      mma_bf16x(c, ra[l].x, rb[l].x, ra[l].y, rb[l].y, qb[l].x, qb[l].y);
      mma_bf16x(c, ra[l].z, rb[l].z, ra[l].w, rb[l].w, qb[l].z, qb[l].w);
    }
    float s0 = fmaxf(c[0], 0.f) + fmaxf(c[1], 0.f);  // key g, heads 2 t and 2 t + 1
    float s1 = fmaxf(c[2], 0.f) + fmaxf(c[3], 0.f);  // key g + 8
#pragma unroll
    for (int o = 1; o < 4; o <<= 1) {
      s0 += __shfl_xor_sync(0xffffffffu, s0, o);
      s1 += __shfl_xor_sync(0xffffffffu, s1, o);
    }
    if (t < 2) {
      const int m = ch * SC_KEYS + r16 + g + 8 * t;
      if (m < p.n_blocks) out[m] = m < n_complete ? (t ? s1 : s0) / p.div : -INFINITY;
    }
  }
}

// Order-preserving integer key of a finite float (larger float, larger key).
__device__ __forceinline__ uint32_t okey(float x) {
  const uint32_t u = __float_as_uint(x);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

constexpr int TK_THREADS = 512;
constexpr int TK_PER = 32;     // most scores a thread holds in registers: up to TK_THREADS * TK_PER a CTA
constexpr int TK_SPAN = 4096;  // scores a CTA of the row's cluster aims for (clusters of 1, 2, 4 or 8 CTAs)
constexpr int TK_CL_MAX = 8;

// Exclusive prefix sum of v over the block's threads (and the total).
__device__ __forceinline__ int block_scan(int v, int* tmp, int& total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) tmp[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int w = lane < TK_THREADS / 32 ? tmp[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    tmp[32 + lane] = w;  // inclusive over warps
  }
  __syncthreads();
  total = tmp[32 + TK_THREADS / 32 - 1];
  const int before = (warp ? tmp[32 + warp - 1] : 0) + x - v;
  __syncthreads();  // tmp reusable
  return before;
}

__device__ __forceinline__ void hist_add(uint32_t* hist, uint32_t bin) {
  // lanes with the same bin add once (the scores crowd into a few bins)
  const uint32_t same = __match_any_sync(__activemask(), bin);
  if ((threadIdx.x & 31) == __ffs(same) - 1) atomicAdd(&hist[bin], uint32_t(__popc(same)));
}

// One row a cluster of CL CTAs (grid (CL, rows)): the k largest finite scores, their indices ascending, padded with
// n_blocks. CTA c of the cluster takes the scores [c span, c span + span) and thread t of it a contiguous piece of
// `per` of those, held in registers (key 0 marks a non-finite score: finite keys are never 0) when per <= TK_PER and
// re-read on every pass otherwise. Each of the four 8-bit radix passes counts the keys that match the digits chosen
// so far into the CTA's histogram; after a cluster barrier every CTA sums the CL histograms through distributed
// shared memory and picks the same digit (double-buffered histograms, so one barrier a pass). The first pass's
// histogram counts every finite score, which gives the number of candidates. Then the CTAs exchange their counts of
// keys above and equal to the threshold and write their picks in index order.
template <int PER>
__global__ void __launch_bounds__(TK_THREADS, 1) topk_kernel(const float* scores, int n_blocks, int k, int32_t* top) {
  __shared__ uint32_t hist[2][256];
  __shared__ uint32_t gh[256];  // the cluster's histogram (CL > 1)
  __shared__ int tmp[64];
  __shared__ int xch[2];  // this CTA's counts of keys above and equal to the threshold, read by the cluster
  __shared__ uint32_t sel_digit;
  __shared__ int sel_rem, s_kk;
  const int CL = int(cluster_size()), rank = int(cluster_rank());
  const int row = blockIdx.y, tid = threadIdx.x, lane = tid & 31;
  const float* sc = scores + int64_t(row) * n_blocks;
  int32_t* out = top + int64_t(row) * k;
  const int span = ((n_blocks + CL - 1) / CL + 3) & ~3;
  const int lo = min(n_blocks, rank * span), hi = min(n_blocks, lo + span);
  const int per = ((span + TK_THREADS - 1) / TK_THREADS + 3) & ~3;
  const bool held = per <= PER;
  const int i0 = min(hi, lo + tid * per), i1 = min(hi, i0 + per);
  asm volatile("griddepcontrol.wait;" ::: "memory");  // the score grid has completed and its writes are visible
  uint32_t keys[PER];
  if (held) {
    // 16-byte loads when every piece starts on a multiple of 4 scores (the scores buffer is 16-byte aligned)
    const bool vec = (n_blocks & 3) == 0;
#pragma unroll
    for (int e = 0; e < PER; e += 4) {
      float x[4];
      if (vec) {
        const float4 v = i0 + e < i1 ? *reinterpret_cast<const float4*>(sc + i0 + e)
                                     : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
        x[0] = v.x, x[1] = v.y, x[2] = v.z, x[3] = v.w;
      } else {
#pragma unroll
        for (int u = 0; u < 4; ++u) x[u] = i0 + e + u < i1 ? sc[i0 + e + u] : -INFINITY;
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) keys[e + u] = isfinite(x[u]) ? okey(x[u]) : 0u;
    }
  }
  for (int i = tid; i < 512; i += TK_THREADS) (&hist[0][0])[i] = 0;
  uint32_t prefix = 0, mask = 0;
  int remaining = 0, kk = 0;  // picks still to place among keys matching prefix; picks in all
  for (int pass = 0; pass < 4; ++pass) {
    const int shift = 24 - 8 * pass;
    uint32_t* h = hist[pass & 1];
    __syncthreads();  // h zeroed
    if (held) {
      // whole warps (the block is whole warps and every thread holds PER keys): no divergence around the match
#pragma unroll
      for (int e = 0; e < PER; ++e) {
        const bool m = keys[e] != 0u && (keys[e] & mask) == prefix;
        if (__any_sync(0xffffffffu, m)) {
          const uint32_t bin = m ? (keys[e] >> shift) & 255u : 256u;
          const uint32_t same = __match_any_sync(0xffffffffu, bin);
          if (m && lane == __ffs(same) - 1) atomicAdd(&h[bin], uint32_t(__popc(same)));
        }
      }
    } else {
      for (int i = lo + tid; i < hi; i += TK_THREADS) {
        const float x = sc[i];
        if (!isfinite(x)) continue;
        const uint32_t key = okey(x);
        if ((key & mask) == prefix) hist_add(h, (key >> shift) & 255u);
      }
    }
    cluster_sync();  // every CTA's histogram complete
    if (CL > 1 && tid < 256) {
      // the cluster's counts of bin tid: the CL remote reads in flight together
      uint32_t c[TK_CL_MAX];
#pragma unroll
      for (int r = 0; r < TK_CL_MAX; ++r) c[r] = r < CL ? ld_cluster_u32(smem_u32(h + tid), r) : 0u;
      uint32_t sum = 0;
#pragma unroll
      for (int r = 0; r < TK_CL_MAX; ++r) sum += c[r];
      gh[tid] = sum;
    }
    if (CL > 1) __syncthreads();
    if (tid < 32) {
      const uint32_t* hs = CL > 1 ? gh : h;
      int cnt[8], tot = 0;  // eight bins a lane from the top
#pragma unroll
      for (int e = 0; e < 8; ++e) tot += cnt[e] = int(hs[255 - (lane * 8 + e)]);
      int incl = tot;  // keys in the bins above and including this lane's eight
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
      }
      const int want = pass == 0 ? min(k, __shfl_sync(0xffffffffu, incl, 31)) : remaining;
      if (pass == 0 && lane == 0) s_kk = want;
      const int above = incl - tot;
      const uint32_t hit = __ballot_sync(0xffffffffu, above < want && incl >= want);
      if (hit != 0u && lane == __ffs(hit) - 1) {
        int acc = above, e = 0;
        for (; e < 7; ++e) {
          if (acc + cnt[e] >= want) break;
          acc += cnt[e];
        }
        sel_digit = uint32_t(255 - (lane * 8 + e));
        sel_rem = want - acc;
      }
    }
    // the other histogram was last read by the cluster before this pass's barrier: clear it for the next pass
    for (int i = tid; i < 256; i += TK_THREADS) hist[(pass + 1) & 1][i] = 0;
    __syncthreads();
    if (pass == 0) kk = s_kk;
    if (kk == 0) break;  // no candidates (the same in every CTA of the cluster)
    prefix |= sel_digit << shift;
    mask |= 255u << shift;
    remaining = sel_rem;
  }
  if (kk > 0) {
    // prefix is the k-th largest key: take every larger key and the first `remaining` equal ones, in index order
    int gt = 0, eq = 0;
    if (held) {
#pragma unroll
      for (int e = 0; e < PER; ++e) {
        gt += keys[e] != 0u && keys[e] > prefix;
        eq += keys[e] != 0u && keys[e] == prefix;
      }
    } else {
      for (int i = i0; i < i1; ++i) {
        const float x = sc[i];
        const uint32_t key = isfinite(x) ? okey(x) : 0u;
        gt += key != 0u && key > prefix;
        eq += key != 0u && key == prefix;
      }
    }
    int eq_cta, gt_cta;
    const int eq_before = block_scan(eq, tmp, eq_cta);
    block_scan(gt, tmp, gt_cta);
    if (tid == 0) xch[0] = gt_cta, xch[1] = eq_cta;
    cluster_sync();
    int base = 0, eq_base = 0;  // picks and equal keys in the cluster's lower CTAs
    for (int r = 0; r < rank; ++r) {
      const int x0 = int(ld_cluster_u32(smem_u32(&xch[0]), r)), x1 = int(ld_cluster_u32(smem_u32(&xch[1]), r));
      base += x0 + max(0, min(x1, remaining - eq_base));
      eq_base += x1;
    }
    const int take_eq = max(0, min(eq, remaining - eq_base - eq_before));
    int total;
    int pos = base + block_scan(gt + take_eq, tmp, total);
    int eq_seen = 0;
    if (held) {
#pragma unroll
      for (int e = 0; e < PER; ++e) {
        const uint32_t key = keys[e];
        if (key != 0u && (key > prefix || (key == prefix && eq_seen++ < take_eq))) out[pos++] = i0 + e;
      }
    } else {
      for (int i = i0; i < i1; ++i) {
        const float x = sc[i];
        const uint32_t key = isfinite(x) ? okey(x) : 0u;
        if (key != 0u && (key > prefix || (key == prefix && eq_seen++ < take_eq))) out[pos++] = i;
      }
    }
  }
  for (int j = kk + rank * TK_THREADS + tid; j < k; j += CL * TK_THREADS) out[j] = n_blocks;
  cluster_sync();  // no CTA leaves while the cluster may still read its shared memory
}

// CTAs a row's cluster: 1, 2, 4 or 8, about TK_SPAN scores each.
inline int topk_cluster(int n_blocks) {
  int cl = 1;
  while (cl < TK_CL_MAX && int64_t(cl) * TK_SPAN < n_blocks) cl *= 2;
  return cl;
}

// Scores a thread of a cluster of cl CTAs takes (the kernel's `per`): topk_kernel<8>, <16> or <TK_PER> holds them.
inline int topk_per(int n_blocks, int cl) {
  const int span = ((n_blocks + cl - 1) / cl + 3) & ~3;
  return ((span + TK_THREADS - 1) / TK_THREADS + 3) & ~3;
}

}  // namespace qsasel
}  // namespace lb2
