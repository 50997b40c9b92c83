// CPU oracle for the attention / Gated-DeltaNet hot path.
//
// TEST INFRASTRUCTURE ONLY. Nothing in the product path (larder_b200/) links, loads or calls this file; only
// tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs do, as the checker or as the timed CPU arm.
//
// It restates, over raw buffers, the two numerical kernels of the reference's CPU extension:
//   * orc_attn follows CpuAttn (cpu_ext/cpu_kern.cpp:493-659): f32 scores with q pre-scaled, keys in blocks of 32,
//     an online softmax per (query position, q head), and for few rows the keys split into P <= 64 ranges that are
//     merged by log-sum-exp (cpu_kern.cpp:544-546, :607-628). Bottom-right causal: row t of T sees keys
//     0 .. N - T + t (cpu_kern.cpp:553). GQA: q head h reads KV head h / (Hq / Hkv) (cpu_kern.cpp:559).
//   * orc_gdn follows CpuGdn (cpu_kern.cpp:404-485): per (b, v-head) the state is decayed, read by k, written by
//     the delta and read by q, one position at a time. Extended with the two cases the reference's CUDA recurrence
//     also takes (gdn_cuda.py:68-71, :40-57): a per-Dk gate g [B, T, Hv, Dk] and a [B, T] position mask (a masked
//     position writes y = 0 and keeps the state).
//
// Arithmetic order mirrors the reference: dot products accumulate in 16 lanes with fused multiply-adds and are
// summed by the same halving tree as _mm512_reduce_add_ps; the GDN state update is a multiply then an add
// (no contraction; this file is built with -ffp-contract=off); bf16 -> f32 is a shift and f32 -> bf16 rounds to
// nearest even (cpu_kern.cpp:41-55).
//
// One deliberate difference: CpuAttn leaves a fully masked 32-key block's scores at -inf when nothing in the key
// range was visible yet (cpu_kern.cpp:583 `continue`), and its P.V loop then multiplies V by -inf, which turns the
// range's accumulator into inf/NaN. Here a masked key contributes exactly nothing, which is what the reference's
// float64 test oracle (tests/test_cpu_kern.py:141-149) computes.
#include <omp.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <vector>

namespace {

enum DT { F32 = 0, BF16 = 1, F16 = 2 };

inline float bf2f(uint16_t h) {
  uint32_t u = uint32_t(h) << 16;
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

inline uint16_t f2bf(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return uint16_t((u >> 16) | 0x40);
  u += 0x7fffu + ((u >> 16) & 1u);
  return uint16_t(u >> 16);
}

// IEEE half <-> float through GCC's _Float16 (conversions round to nearest even).
inline float h2f(uint16_t h) {
  _Float16 x;
  std::memcpy(&x, &h, 2);
  return float(x);
}

inline uint16_t f2h(float f) {
  const _Float16 x = _Float16(f);
  uint16_t h;
  std::memcpy(&h, &x, 2);
  return h;
}

inline float ld(const void* p, int64_t i, int t) {
  switch (t) {
    case F32: return static_cast<const float*>(p)[i];
    case BF16: return bf2f(static_cast<const uint16_t*>(p)[i]);
    default: return h2f(static_cast<const uint16_t*>(p)[i]);
  }
}

inline void st(void* p, int64_t i, float v, int t) {
  switch (t) {
    case F32: static_cast<float*>(p)[i] = v; break;
    case BF16: static_cast<uint16_t*>(p)[i] = f2bf(v); break;
    default: static_cast<uint16_t*>(p)[i] = f2h(v); break;
  }
}

// _mm512_reduce_add_ps's order: halves (i, i + 8), then (i, i + 4), then (i, i + 2), then the last pair.
inline float hsum16(const float* a) {
  float h8[8], h4[4];
  for (int i = 0; i < 8; ++i) h8[i] = a[i + 8] + a[i];
  for (int i = 0; i < 4; ++i) h4[i] = h8[i + 4] + h8[i];
  const float p0 = h4[0] + h4[2], p1 = h4[1] + h4[3];
  return p0 + p1;
}

struct Part {
  float m, l;
};

}  // namespace

extern "C" {

// Number of OpenMP threads the oracle uses when a call passes threads <= 0.
int orc_default_threads(void) { return omp_get_num_procs(); }

// softmax(scale * q k^T + mask) v. q [B, Hq, T, D], k [B, Hkv, N, D], v [B, Hkv, N, Dv] with element strides for
// the first three axes and a unit last stride; mask (kind 2) a bool [T, N] with strides ms[0], ms[1]; o written
// contiguous [B, Hq, T, Dv]. mask_kind: 0 none, 1 causal (bottom-right), 2 boolean array. Returns 0, or -1 on an
// unsupported shape (as the reference's attn() refuses: G <= 16, D % 16 == 0, D <= 512, Dv % 16 == 0).
int orc_attn(const void* q, const int64_t* qs, int qdt, const void* k, const int64_t* ks, int kdt, const void* v,
             const int64_t* vs, int vdt, const uint8_t* m, const int64_t* ms, void* o, int odt, int B, int Hq, int T,
             int D, int Hkv, int N, int Dv, float scale, int mask_kind, int threads) {
  if (Hkv <= 0 || Hq % Hkv || Hq / Hkv > 16 || D % 16 || D > 512 || Dv % 16 || Dv > 512) return -1;
  if (threads <= 0) threads = omp_get_num_procs();
  const int G = Hq / Hkv;
  const int rows = B * Hkv * T;
  int P = 1;
  if (rows < 2 * threads) P = std::max(1, std::min({(2 * threads + rows - 1) / rows, N / 256, 64}));
  const int span = (N + P - 1) / P;
  std::vector<float> acc(size_t(rows) * P * G * Dv);
  std::vector<Part> parts(size_t(rows) * P * G);
#pragma omp parallel for schedule(dynamic, 1) num_threads(threads)
  for (int task = 0; task < rows * P; ++task) {
    const int p = task % P, row = task / P;
    const int t = row % T, hk = (row / T) % Hkv, b = row / (T * Hkv);
    const int lim = mask_kind == 1 ? std::min(N, N - T + t + 1) : N;
    const int n0 = p * span, n1 = std::min(lim, n0 + span);
    float* ac = acc.data() + (size_t(row) * P + p) * G * Dv;
    Part* pt = parts.data() + (size_t(row) * P + p) * G;
    std::vector<float> qf(size_t(G) * D);
    for (int g = 0; g < G; ++g) {
      const int64_t qo = b * qs[0] + int64_t(hk * G + g) * qs[1] + t * qs[2];
      for (int d = 0; d < D; ++d) qf[size_t(g) * D + d] = ld(q, qo + d, qdt) * scale;
      pt[g] = {-INFINITY, 0.f};
      std::fill(ac + size_t(g) * Dv, ac + size_t(g + 1) * Dv, 0.f);
    }
    constexpr int KB = 32;
    float s[16][KB];
    float kk[512];
    for (int j0 = n0; j0 < n1; j0 += KB) {
      const int nb = std::min(KB, n1 - j0);
      for (int j = 0; j < nb; ++j) {
        const int n = j0 + j;
        const int64_t ko = b * ks[0] + hk * ks[1] + n * ks[2];
        for (int d = 0; d < D; ++d) kk[d] = ld(k, ko + d, kdt);
        const bool keep = mask_kind != 2 || m[t * ms[0] + n * ms[1]];
        for (int g = 0; g < G; ++g) {
          float lane[16] = {0};
          const float* qg = qf.data() + size_t(g) * D;
          for (int d = 0; d < D; d += 16)
            for (int i = 0; i < 16; ++i) lane[i] = std::fma(kk[d + i], qg[d + i], lane[i]);
          s[g][j] = keep ? hsum16(lane) : -INFINITY;
        }
      }
      for (int g = 0; g < G; ++g) {
        float mx_ = pt[g].m;
        for (int j = 0; j < nb; ++j) mx_ = std::max(mx_, s[g][j]);
        if (mx_ == -INFINITY) {
          for (int j = 0; j < nb; ++j) s[g][j] = 0.f;  // nothing visible yet: these keys add nothing
          continue;
        }
        const float c = std::exp(pt[g].m - mx_);
        float l = pt[g].l * c;
        for (int j = 0; j < nb; ++j) {
          s[g][j] = std::exp(s[g][j] - mx_);
          l += s[g][j];
        }
        pt[g] = {mx_, l};
        float* ag = ac + size_t(g) * Dv;
        for (int d = 0; d < Dv; ++d) ag[d] = ag[d] * c;
      }
      for (int j = 0; j < nb; ++j) {
        const int64_t vo = b * vs[0] + hk * vs[1] + int64_t(j0 + j) * vs[2];
        for (int d = 0; d < Dv; ++d) {
          const float vv = ld(v, vo + d, vdt);
          for (int g = 0; g < G; ++g) {
            float* ag = ac + size_t(g) * Dv + d;
            *ag = std::fma(vv, s[g][j], *ag);
          }
        }
      }
    }
  }
#pragma omp parallel for num_threads(threads)
  for (int row = 0; row < rows; ++row) {
    const int t = row % T, hk = (row / T) % Hkv, b = row / (T * Hkv);
    for (int g = 0; g < G; ++g) {
      float mm = -INFINITY;
      for (int p = 0; p < P; ++p) mm = std::max(mm, parts[(size_t(row) * P + p) * G + g].m);
      float l = 0.f, w[64];
      for (int p = 0; p < P; ++p) {
        const Part& pp = parts[(size_t(row) * P + p) * G + g];
        w[p] = pp.m == -INFINITY ? 0.f : std::exp(pp.m - mm);
        l += pp.l * w[p];
      }
      const float inv = l > 0.f ? 1.f / l : 0.f;
      const int64_t oo = ((int64_t(b) * Hq + hk * G + g) * T + t) * Dv;
      for (int d = 0; d < Dv; ++d) {
        float x = 0.f;
        for (int p = 0; p < P; ++p) x += acc[((size_t(row) * P + p) * G + g) * Dv + d] * w[p];
        st(o, oo + d, x * inv, odt);
      }
    }
  }
  return 0;
}

// The gated delta recurrence. q, k [B, T, Hk, Dk] (dtype qdt), v [B, T, Hv, Dv] (vdt), g [B, T, Hv] or, with
// g_vec, [B, T, Hv, Dk] (gdt), beta [B, T, Hv] (bdt), s0 / s [B, Hv, Dv, Dk] f32, y [B, T, Hv, Dv] (ydt), mask
// [B, T] bytes or null; all contiguous. Returns 0, or -1 on an unsupported shape (Dk % 16, Dk > 512, Hv % Hk).
int orc_gdn(const void* q, const void* k, int qdt, const void* v, int vdt, const void* g, int gdt, int g_vec,
            const void* beta, int bdt, const uint8_t* mask, const float* s0, void* y, int ydt, float* s, int B, int T,
            int Hk, int Dk, int Hv, int Dv, int threads) {
  if (Dk % 16 || Dk > 512 || Hk <= 0 || Hv % Hk) return -1;
  if (threads <= 0) threads = omp_get_num_procs();
  const int rf = Hv / Hk;
  const int tasks = B * Hv;
#pragma omp parallel for schedule(dynamic, 1) num_threads(threads)
  for (int bh = 0; bh < tasks; ++bh) {
    const int b = bh / Hv, h = bh % Hv, hk = h / rf;
    float* S = s + size_t(bh) * Dv * Dk;
    std::memcpy(S, s0 + size_t(bh) * Dv * Dk, sizeof(float) * size_t(Dv) * Dk);
    float kq[2][512], gv[512];
    for (int t = 0; t < T; ++t) {
      const int64_t qo = ((int64_t(b) * T + t) * Hk + hk) * Dk;
      const int64_t vo = ((int64_t(b) * T + t) * Hv + h) * Dv;
      const int64_t go = (int64_t(b) * T + t) * Hv + h;
      if (mask && !mask[int64_t(b) * T + t]) {
        for (int i = 0; i < Dv; ++i) st(y, vo + i, 0.f, ydt);
        continue;
      }
      for (int i = 0; i < Dk; ++i) {
        kq[0][i] = ld(k, qo + i, qdt);
        kq[1][i] = ld(q, qo + i, qdt);
      }
      if (g_vec) {
        for (int i = 0; i < Dk; ++i) gv[i] = ld(g, go * Dk + i, gdt);
      } else {
        const float gs = ld(g, go, gdt);
        for (int i = 0; i < Dk; ++i) gv[i] = gs;
      }
      const float bt = ld(beta, go, bdt);
      for (int i = 0; i < Dv; ++i) {
        float* row = S + size_t(i) * Dk;
        float kv[16] = {0};
        for (int j = 0; j < Dk; j += 16)
          for (int l = 0; l < 16; ++l) {
            const float sr = row[j + l] * gv[j + l];
            row[j + l] = sr;
            kv[l] = std::fma(sr, kq[0][j + l], kv[l]);
          }
        const float delta = (ld(v, vo + i, vdt) - hsum16(kv)) * bt;
        float yv[16] = {0};
        for (int j = 0; j < Dk; j += 16)
          for (int l = 0; l < 16; ++l) {
            const float prod = kq[0][j + l] * delta;
            const float sr = row[j + l] + prod;
            row[j + l] = sr;
            yv[l] = std::fma(sr, kq[1][j + l], yv[l]);
          }
        st(y, vo + i, hsum16(yv), ydt);
      }
    }
  }
  return 0;
}

// Dtype conversion helpers for the host side of the tests (round to nearest even, as the kernels' inputs are made).
void orc_f32_to_bf16(const float* x, uint16_t* y, int64_t n) {
  for (int64_t i = 0; i < n; ++i) y[i] = f2bf(x[i]);
}
void orc_f32_to_f16(const float* x, uint16_t* y, int64_t n) {
  for (int64_t i = 0; i < n; ++i) y[i] = f2h(x[i]);
}

}  // extern "C"
