// fp32 attention on CUDA cores, for fp32 q / k / v (the reference's CPU-runnable configuration runs in fp32; the
// tensor-core kernels take bf16 / f16). Exact fp32 arithmetic: one warp per (sequence, query head, query row), the
// head dimension spread over the lanes, keys in order with an online softmax (the arithmetic of CpuAttn,
// cpu_ext/cpu_kern.cpp:564-606: scaled q, f32 dot products, running max and sum). Masks none / causal
// (bottom-right) / boolean array; optional sigmoid gate. Throughput is not the point of this path: its shapes are
// small; the bf16 / f16 paths carry the heavy configurations.
#pragma once

#include "common.cuh"

namespace lb2 {
namespace f32attn {

struct Params {
  const float* q;
  const float* k;
  const float* v;
  float* o;
  const float* gate;
  const uint8_t* mask;
  int64_t q_st[3], k_st[3], v_st[3], o_st[3], g_st[3], m_st[2];
  const int32_t* kv_len;  // optional per-sequence key counts (decode calls)
  int B, Hq, Hkv, T, N, G, mask_kind;
  float scale;
};

template <int D>
__global__ void __launch_bounds__(128) attn_f32_kernel(const Params p) {
  constexpr int V = D / 32;
  const int64_t wid = int64_t(blockIdx.x) * 4 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (wid >= int64_t(p.B) * p.Hq * p.T) return;
  const int t = int(wid % p.T);
  const int h = int((wid / p.T) % p.Hq);
  const int b = int(wid / (int64_t(p.T) * p.Hq));
  const int hk = h / p.G;
  const int len = p.kv_len ? min(max(p.kv_len[b], 0), p.N) : p.N;
  const int lim = p.mask_kind == LB2_MASK_CAUSAL ? min(len, len - p.T + t + 1) : len;  // keys [0, lim)
  float qv[V], acc[V];
  const float* qr = p.q + b * p.q_st[0] + int64_t(h) * p.q_st[1] + int64_t(t) * p.q_st[2];
#pragma unroll
  for (int i = 0; i < V; ++i) {
    qv[i] = qr[lane + 32 * i] * p.scale;
    acc[i] = 0.f;
  }
  float m = -INFINITY, l = 0.f;
  const float* kb = p.k + b * p.k_st[0] + int64_t(hk) * p.k_st[1];
  const float* vb = p.v + b * p.v_st[0] + int64_t(hk) * p.v_st[1];
  const uint8_t* mr = p.mask_kind == LB2_MASK_ARRAY ? p.mask + int64_t(t) * p.m_st[0] : nullptr;
  for (int n = 0; n < lim; ++n) {
    if (mr && !mr[int64_t(n) * p.m_st[1]]) continue;
    const float* kr = kb + int64_t(n) * p.k_st[2];
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < V; ++i) s = fmaf(kr[lane + 32 * i], qv[i], s);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const float mn = fmaxf(m, s);
    const float c = expf(m - mn);  // exp(-inf) = 0 on the first key
    const float e = expf(s - mn);
    l = l * c + e;
    m = mn;
    const float* vr = vb + int64_t(n) * p.v_st[2];
#pragma unroll
    for (int i = 0; i < V; ++i) acc[i] = fmaf(vr[lane + 32 * i], e, acc[i] * c);
  }
  const float inv = l > 0.f ? 1.f / l : 0.f;
  float* orow = p.o + b * p.o_st[0] + int64_t(h) * p.o_st[1] + int64_t(t) * p.o_st[2];
  const float* grow = p.gate ? p.gate + b * p.g_st[0] + int64_t(h) * p.g_st[1] + int64_t(t) * p.g_st[2] : nullptr;
#pragma unroll
  for (int i = 0; i < V; ++i) {
    float x = acc[i] * inv;
    if (grow) x = x / (1.f + expf(-grow[lane + 32 * i]));
    orow[lane + 32 * i] = x;
  }
}

}  // namespace f32attn
}  // namespace lb2
