// larder_b200: the C-ABI library. One translation unit (so the device status word is one symbol) that includes
// every kernel header and implements the entry points declared in include/larder_b200.h.
#include <algorithm>
#include <cstring>
#include <initializer_list>
#include <mutex>
#include <string>
#include <type_traits>
#include <utility>

#include "common.cuh"
#include "attn_decode.cuh"
#include "gdn_recurrent.cuh"
#include "attn_prefill.cuh"
#include "attn_prefill2.cuh"
#include "gdn_chunked.cuh"
#include "attn_f32.cuh"
#include "attn_glue.cuh"
#include "qsa_select.cuh"
#include "peer_xch.cuh"
#include "kv_runs.cuh"
#include "attn_tiles.cuh"
#include "gdn_glue.cuh"

namespace lb2 {

static thread_local std::string t_error;

void set_error(const std::string& msg) { t_error = msg; }

int fail(int code, const std::string& msg) {
  t_error = msg;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  t_error = std::string(what) + ": " + cudaGetErrorString(e);
  return LB2_ECUDA;
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(f);
  });
  return fn;
}

int encode_tensor_map(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* base, const uint64_t* dims,
                      const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swizzle) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(LB2_ECUDA, "cuTensorMapEncodeTiled is not available from the driver");
  if (reinterpret_cast<uintptr_t>(base) & 15) return fail(LB2_EINVAL, "TMA base address is not 16-byte aligned");
  for (int i = 0; i < rank - 1; ++i)
    if (strides_bytes[i] % 16) return fail(LB2_EINVAL, "TMA stride is not a multiple of 16 bytes");
  cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  CUresult r = fn(map, dtype, cuuint32_t(rank), const_cast<void*>(base), reinterpret_cast<const cuuint64_t*>(dims),
                  reinterpret_cast<const cuuint64_t*>(strides_bytes), reinterpret_cast<const cuuint32_t*>(box), estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(LB2_EINVAL, "cuTensorMapEncodeTiled failed (code " + std::to_string(r) + ")");
  return LB2_OK;
}

int sm_count(int device) {
  static int cached[64] = {0};
  if (device < 0 || device >= 64) return 148;
  if (!cached[device]) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || n <= 0) n = 148;
    cached[device] = n;
  }
  return cached[device];
}

static size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// ------------------------------------------------------------------------------------------------ decode

namespace decode {

// The combine keeps one weight per partial of a (b, hk) pair in shared memory, so a sequence has at most MAX_PARTS
// splits; a smaller requested split is raised to respect that.
static int min_split(int N) {
  const int per = (N + MAX_PARTS - 1) / MAX_PARTS;
  return (per + BK - 1) / BK * BK;
}

// How a call is scheduled: split = 0 asks for the balanced schedule (equal tile runs, one CTA an SM, never fewer than
// two tiles a CTA at full capacity); split > 0 for split units of that many keys (rounded up to whole tiles).
struct Plan {
  int balanced, split, nsplit, grid;
  int64_t slots;  // partial slots the workspace holds
};

static Plan plan(int B, int Hkv, int N, int D, int split) {
  int dev = 0;
  cudaGetDevice(&dev);
  const int sms = sm_count(dev);
  Plan pl{};
  if (split > 0) {
    pl.balanced = 0;
    pl.split = std::max((split + BK - 1) / BK * BK, min_split(N));
    pl.nsplit = (N + pl.split - 1) / pl.split;
    pl.grid = sms;
    pl.slots = int64_t(B) * Hkv * pl.nsplit;
  } else {
    const int64_t tiles = int64_t(B) * Hkv * ((N + BK - 1) / BK);
    pl.balanced = 1;
    pl.split = 0;
    pl.nsplit = 0;
    pl.grid = int(std::max<int64_t>(1, std::min<int64_t>({int64_t(sms), int64_t(MAX_PARTS), tiles / 2})));
    pl.slots = int64_t(pl.grid) + int64_t(B) * Hkv;
  }
  return pl;
}

static int rows_tiles(int G, int T) { return G * T <= 8 ? 1 : G * T <= 16 ? 2 : 4; }

struct WsLayout {
  size_t ml, o, total;
};

// Item partials, one per (slot, row): (max, sum) pairs, then unnormalised O rows. Every value a call reads was
// written earlier in the same call, so nothing in the workspace needs to start at zero.
static WsLayout ws_layout(int64_t slots, int rows, int D) {
  WsLayout w;
  const size_t parts = size_t(slots) * rows;
  w.ml = 0;
  w.o = align_up(parts * 2 * sizeof(float), 256);
  w.total = w.o + parts * D * sizeof(float);
  return w;
}

template <typename T, int D, int NT>
static int launch_t(const CUtensorMap& qm, const CUtensorMap& km, const CUtensorMap& vm, const Params& p,
                    cudaStream_t st) {
  using C = Cfg<D, NT>;
  auto kern = decode_kernel<T, D, NT>;
  static int attr_dev = -1;
  int dev = 0;
  LB2_CUDA(cudaGetDevice(&dev));
  if (attr_dev != dev) {
    LB2_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES));
    attr_dev = dev;
  }
  cudaLaunchAttribute pdl[1];
  pdl[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  pdl[0].val.programmaticStreamSerializationAllowed = 1;
  {
    // a programmatic dependent of the stream's previous kernel: its launch and shared-memory set-up overlap that
    // kernel's tail (the kernel waits on the grid dependency before its first global read)
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(unsigned(p.grid));
    cfg.blockDim = dim3(C::THREADS);
    cfg.dynamicSmemBytes = C::SMEM_BYTES;
    cfg.stream = st;
    cfg.attrs = pdl;
    cfg.numAttrs = 1;
    LB2_CUDA(cudaLaunchKernelEx(&cfg, kern, qm, km, vm, p));
  }
  {
    // the split combine as a programmatic dependent: its launch overlaps the decode grid's tail
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(unsigned(int64_t(p.B) * p.Hkv));
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    LB2_CUDA(cudaLaunchKernelEx(&cfg, split_combine_kernel<T, D>, p));
  }
  return LB2_OK;
}

// NT: 8-row tiles of folded rows (1, 2 or 4; D = 256 takes at most 2).
template <typename T>
static int launch_d(int D, int NT, const CUtensorMap& qm, const CUtensorMap& km, const CUtensorMap& vm,
                    const Params& p, cudaStream_t st) {
  if (D == 64)
    return NT == 1 ? launch_t<T, 64, 1>(qm, km, vm, p, st)
                   : NT == 2 ? launch_t<T, 64, 2>(qm, km, vm, p, st) : launch_t<T, 64, 4>(qm, km, vm, p, st);
  if (D == 128)
    return NT == 1 ? launch_t<T, 128, 1>(qm, km, vm, p, st)
                   : NT == 2 ? launch_t<T, 128, 2>(qm, km, vm, p, st) : launch_t<T, 128, 4>(qm, km, vm, p, st);
  return NT == 1 ? launch_t<T, 256, 1>(qm, km, vm, p, st) : launch_t<T, 256, 2>(qm, km, vm, p, st);
}

static int kv_map(CUtensorMap* m, const void* base, const int64_t* st, int B, int H, int N, int D, int dtype) {
  const uint64_t dims[4] = {uint64_t(D), uint64_t(N), uint64_t(H), uint64_t(B)};
  const uint64_t strides[3] = {uint64_t(st[2]) * 2, uint64_t(st[1]) * 2, uint64_t(st[0]) * 2};
  const uint32_t box[4] = {64, uint32_t(BK), 1, 1};
  return encode_tensor_map(m, dtype == LB2_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                           4, base, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

static int run(const void* q, const int64_t* q_st, const void* k, const int64_t* k_st, const void* v,
               const int64_t* v_st, void* o, const int64_t* o_st, float* part_o, float* part_lse,
               const int32_t* kv_len, int B, int Hq, int Hkv, int T, int N, int D, int dtype, float scale, int causal,
               int split, void* workspace, size_t workspace_bytes, void* stream, int npush = 0,
               float* const* push_o = nullptr, float* const* push_lse = nullptr, uint32_t* push_count = nullptr,
               uint32_t* const* push_flag = nullptr, uint32_t push_epoch = 0, const int32_t* picks = nullptr,
               int nsel = 0, int cr = 0, int pick_n = 0) {
  LB2_CHECK_ARG(B > 0 && Hq > 0 && Hkv > 0 && T > 0 && N > 0, "decode: empty shape");
  LB2_CHECK_ARG(Hq % Hkv == 0, "decode: Hq must be a multiple of Hkv");
  LB2_CHECK_ARG(D == 64 || D == 128 || D == 256, "decode: head dim must be 64, 128 or 256");
  LB2_CHECK_ARG(dtype == LB2_BF16 || dtype == LB2_F16, "decode: dtype must be bf16 or f16");
  const int G = Hq / Hkv, rows = G * T;
  LB2_CHECK_ARG(rows <= (D == 256 ? 16 : 32), "decode: too many folded rows (G*T) for the split-KV kernel");
  for (int i = 0; i < 3; ++i)
    LB2_CHECK_ARG(q_st[i] % 8 == 0 && k_st[i] % 8 == 0 && v_st[i] % 8 == 0,
                  "decode: q/k/v strides must be multiples of 8 elements");
  LB2_CHECK_ARG((reinterpret_cast<uintptr_t>(q) & 15) == 0, "decode: q must be 16-byte aligned");
  const int NT = rows_tiles(G, T);
  LB2_CHECK_ARG(int64_t(B) * Hkv * ((N + BK - 1) / BK) < (int64_t(1) << 30), "decode: too many key tiles a call");
  const Plan pl = plan(B, Hkv, N, D, split);
  const WsLayout w = ws_layout(pl.slots, rows, D);
  LB2_CHECK_ARG(workspace != nullptr && workspace_bytes >= w.total, "decode: workspace too small");
  LB2_CHECK_ARG((reinterpret_cast<uintptr_t>(workspace) & 255) == 0, "decode: workspace must be 256-byte aligned");
  LB2_CHECK_ARG(B <= MAX_B, "decode: at most 1024 sequences a call");
  CUtensorMap qm, km, vm;
  // (pick mode reads K and V by copies of its own; the maps, over the cache view, go unused)
  int rc = kv_map(&km, k, k_st, B, Hkv, picks ? pick_n : N, D, dtype);
  if (rc) return rc;
  rc = kv_map(&vm, v, v_st, B, Hkv, picks ? pick_n : N, D, dtype);
  if (rc) return rc;
  {  // the folded Q tile of one KV head: a (64, T, G, 1) box of the (D, T, Hq, B) view of q
    const uint64_t dims[4] = {uint64_t(D), uint64_t(T), uint64_t(Hq), uint64_t(B)};
    const uint64_t strides[3] = {uint64_t(q_st[2]) * 2, uint64_t(q_st[1]) * 2, uint64_t(q_st[0]) * 2};
    const uint32_t box[4] = {64, uint32_t(T), uint32_t(G), 1};
    rc = encode_tensor_map(&qm, dtype == LB2_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                           4, q, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  Params p{};
  for (int i = 0; i < 3; ++i) p.o_st[i] = o_st ? o_st[i] : 0;
  p.o = o;
  p.part_o = part_o;
  p.part_lse = part_lse;
  p.emit = part_o != nullptr || npush > 0;
  p.npush = npush;
  for (int i = 0; i < npush; ++i) {
    p.push_o[i] = push_o[i];
    p.push_lse[i] = push_lse[i];
    p.push_flag[i] = push_flag[i];
  }
  p.push_count = push_count;
  p.push_epoch = push_epoch;
  p.kv_len = kv_len;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  p.ws_ml = reinterpret_cast<float*>(ws + w.ml);
  p.ws_o = reinterpret_cast<float*>(ws + w.o);
  p.B = B;
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.T = T;
  p.N = N;
  p.G = G;
  p.rows = rows;
  p.balanced = pl.balanced;
  p.split = pl.split;
  p.nsplit = pl.nsplit;
  p.grid = pl.grid;
  p.causal = causal && T > 1;
  p.scale_log2 = scale * 1.4426950408889634f;
  if (picks) {
    LB2_CHECK_ARG(B == 1 && !causal && kv_len == nullptr, "decode: pick mode takes one sequence, no mask");
    LB2_CHECK_ARG((reinterpret_cast<uintptr_t>(k) & 15) == 0 && (reinterpret_cast<uintptr_t>(v) & 15) == 0,
                  "decode: k / v must be 16-byte aligned");
    p.picks = picks;
    p.nsel = nsel;
    p.cr = cr;
    p.pick_n = pick_n;
    p.pk = static_cast<const uint8_t*>(k);
    p.pv = static_cast<const uint8_t*>(v);
    p.pk_hst = k_st[1] * 2;
    p.pk_pst = k_st[2] * 2;
    p.pv_hst = v_st[1] * 2;
    p.pv_pst = v_st[2] * 2;
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  return dtype == LB2_BF16 ? launch_d<__nv_bfloat16>(D, NT, qm, km, vm, p, st)
                           : launch_d<__half>(D, NT, qm, km, vm, p, st);
}

}  // namespace decode

// ------------------------------------------------------------------------------------------------ prefill

namespace prefill {

template <typename T, int D>
static int launch(const CUtensorMap& qm, const CUtensorMap& km, const CUtensorMap& vm, const Params& p,
                  cudaStream_t st) {
  auto kern = fmha_kernel<T, D>;
  static int attr_dev = -1;
  int dev = 0;
  LB2_CUDA(cudaGetDevice(&dev));
  if (attr_dev != dev) {
    LB2_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg<D>::SMEM_BYTES));
    attr_dev = dev;
  }
  dim3 grid(unsigned(p.B * p.Hq * p.mtiles));
  kern<<<grid, THREADS, Cfg<D>::SMEM_BYTES, st>>>(qm, km, vm, p);
  LB2_CUDA(cudaGetLastError());
  return LB2_OK;
}

static int map4(CUtensorMap* m, const void* base, const int64_t* st, int B, int H, int L, int D, int dtype,
                int box_rows) {
  const uint64_t dims[4] = {uint64_t(D), uint64_t(L), uint64_t(H), uint64_t(B)};
  const uint64_t strides[3] = {uint64_t(st[2]) * 2, uint64_t(st[1]) * 2, uint64_t(st[0]) * 2};
  const uint32_t box[4] = {64, uint32_t(box_rows), 1, 1};
  return encode_tensor_map(m, dtype == LB2_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                           4, base, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

}  // namespace prefill

namespace prefill2 {

// Persistent clusters of two CTAs: as many as fit on the device at once (at most one a 256-row item), each looping
// over its items.
template <typename T, int D>
static int launch(const CUtensorMap& qm, const CUtensorMap& km, const CUtensorMap& vm, const Params& p,
                  cudaStream_t st) {
  auto kern = fmha2_kernel<T, D>;
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(THREADS);
  cfg.dynamicSmemBytes = Cfg<D>::SMEM_BYTES;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  static int attr_dev = -1, max_clusters = 0;
  int dev = 0;
  LB2_CUDA(cudaGetDevice(&dev));
  if (attr_dev != dev) {
    LB2_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg<D>::SMEM_BYTES));
    cfg.gridDim = dim3(2);
    LB2_CUDA(cudaOccupancyMaxActiveClusters(&max_clusters, kern, &cfg));
    if (max_clusters < 1) return fail(LB2_ECUDA, "prefill: no 2-CTA cluster of the pair kernel fits the device");
    attr_dev = dev;
  }
  const int64_t items = int64_t(p.B) * p.Hq * p.mtiles;
  cfg.gridDim = dim3(unsigned(2 * std::min<int64_t>(items, max_clusters)));
  LB2_CUDA(cudaLaunchKernelEx(&cfg, kern, qm, km, vm, p));
  return LB2_OK;
}

}  // namespace prefill2

// ------------------------------------------------------------------------------------------------ fp32 attention

namespace f32attn {

static int run(const void* q, const int64_t* q_st, const void* k, const int64_t* k_st, const void* v,
               const int64_t* v_st, void* o, const int64_t* o_st, const void* gate, const int64_t* g_st,
               const uint8_t* mask, const int64_t* m_st, const int32_t* kv_len, int B, int Hq, int Hkv, int T, int N,
               int D, float scale, int mask_kind, void* stream) {
  LB2_CHECK_ARG(D == 32 || D == 64 || D == 128 || D == 256, "fp32 attention: head dim 32, 64, 128 or 256");
  Params p{};
  p.q = static_cast<const float*>(q);
  p.k = static_cast<const float*>(k);
  p.v = static_cast<const float*>(v);
  p.o = static_cast<float*>(o);
  p.gate = static_cast<const float*>(gate);
  p.mask = mask_kind == LB2_MASK_ARRAY ? mask : nullptr;
  for (int i = 0; i < 3; ++i) {
    p.q_st[i] = q_st[i];
    p.k_st[i] = k_st[i];
    p.v_st[i] = v_st[i];
    p.o_st[i] = o_st[i];
    p.g_st[i] = gate ? g_st[i] : 0;
  }
  p.m_st[0] = p.mask ? m_st[0] : 0;
  p.m_st[1] = p.mask ? m_st[1] : 0;
  p.kv_len = kv_len;
  p.B = B;
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.T = T;
  p.N = N;
  p.G = Hq / Hkv;
  p.mask_kind = mask_kind;
  p.scale = scale;
  const int64_t warps = int64_t(B) * Hq * T;
  dim3 grid(unsigned((warps + 3) / 4));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (D) {
    case 32: attn_f32_kernel<32><<<grid, 128, 0, st>>>(p); break;
    case 64: attn_f32_kernel<64><<<grid, 128, 0, st>>>(p); break;
    case 128: attn_f32_kernel<128><<<grid, 128, 0, st>>>(p); break;
    default: attn_f32_kernel<256><<<grid, 128, 0, st>>>(p); break;
  }
  LB2_CUDA(cudaGetLastError());
  return LB2_OK;
}

}  // namespace f32attn

// ------------------------------------------------------------------------------------------------ allocation-free decode

// The scratch of lb2_attn_decode_noalloc (split partials): a file-scope device array, so that
// the entry point never allocates. Host code must not pass this name to a kernel (in host code it is a host-side
// stand-in); its device address comes from cudaGetSymbolAddress, once per device.
static __device__ __align__(256) uint8_t g_noalloc_scratch[LB2_NOALLOC_SCRATCH_BYTES];

namespace noalloc {

static std::mutex g_mu;
static void* g_addr[64];  // device address of g_noalloc_scratch, per device

// The array's device address on the current device, looked up on the first call there (with that device current).
static int scratch(void** out) {
  int dev = 0;
  LB2_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return fail(LB2_EINVAL, "decode_noalloc: device index out of range");
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_addr[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(g_noalloc_scratch)");
    g_addr[dev] = p;
  }
  *out = g_addr[dev];
  return LB2_OK;
}

}  // namespace noalloc
}  // namespace lb2

using namespace lb2;

extern "C" {

int lb2_abi_version(void) { return 1; }

const char* lb2_error(void) { return t_error.c_str(); }

int lb2_status(void* stream) {
  LB2_CUDA(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)));
  int v = 0, zero = 0;
  LB2_CUDA(cudaMemcpyFromSymbol(&v, g_status, sizeof(int)));
  if (v) LB2_CUDA(cudaMemcpyToSymbol(g_status, &zero, sizeof(int)));
  if (v) set_error("a device wait gave up (where " + std::to_string(v >> 8) + ")");
  return v;
}

size_t lb2_attn_decode_workspace_size(int B, int Hq, int Hkv, int T, int N, int D, int split) {
  if (B <= 0 || Hkv <= 0 || Hq % Hkv || N <= 0 || T <= 0) return 0;
  return decode::ws_layout(decode::plan(B, Hkv, N, D, split).slots, (Hq / Hkv) * T, D).total;
}

int lb2_attn_decode(const void* q, const int64_t* q_st, const void* k, const int64_t* k_st, const void* v,
                    const int64_t* v_st, void* o, const int64_t* o_st, const int32_t* kv_len, int B, int Hq, int Hkv,
                    int T, int N, int D, int dtype, float scale, int causal, int split, void* workspace,
                    size_t workspace_bytes, void* stream) {
  LB2_CHECK_ARG(o != nullptr && o_st != nullptr, "decode: output missing");
  if (dtype == LB2_F32) {  // exact fp32 on CUDA cores; needs no workspace
    LB2_CHECK_ARG(B > 0 && Hq > 0 && Hkv > 0 && T > 0 && N > 0 && Hq % Hkv == 0, "decode: shape");
    return f32attn::run(q, q_st, k, k_st, v, v_st, o, o_st, nullptr, nullptr, nullptr, nullptr, kv_len, B, Hq, Hkv,
                        T, N, D, scale, causal && T > 1 ? LB2_MASK_CAUSAL : LB2_MASK_NONE, stream);
  }
  return decode::run(q, q_st, k, k_st, v, v_st, o, o_st, nullptr, nullptr, kv_len, B, Hq, Hkv, T, N, D, dtype, scale,
                     causal, split, workspace, workspace_bytes, stream);
}

int lb2_attn_decode_partial(const void* q, const int64_t* q_st, const void* k, const int64_t* k_st, const void* v,
                            const int64_t* v_st, float* part_o, float* part_lse, const int32_t* kv_len, int B, int Hq,
                            int Hkv, int T, int N, int D, int dtype, float scale, int split, void* workspace,
                            size_t workspace_bytes, void* stream) {
  LB2_CHECK_ARG(part_o != nullptr && part_lse != nullptr, "decode_partial: outputs missing");
  return decode::run(q, q_st, k, k_st, v, v_st, nullptr, nullptr, part_o, part_lse, kv_len, B, Hq, Hkv, T, N, D,
                     dtype, scale, 0, split, workspace, workspace_bytes, stream);
}

int lb2_attn_decode_noalloc(const void* q, const int64_t* q_st, const void* k, const int64_t* k_st, const void* v,
                            const int64_t* v_st, void* o, const int64_t* o_st, const int32_t* kv_len, int B, int Hq,
                            int Hkv, int T, int N, int D, int dtype, float scale, int causal, int split,
                            void* stream) {
  LB2_CHECK_ARG(o != nullptr && o_st != nullptr, "decode_noalloc: output missing");
  if (dtype == LB2_F32)  // the exact fp32 kernel uses no scratch at all, as in lb2_attn_decode
    return lb2_attn_decode(q, q_st, k, k_st, v, v_st, o, o_st, kv_len, B, Hq, Hkv, T, N, D, dtype, scale, causal,
                           split, nullptr, 0, stream);
  const size_t need = lb2_attn_decode_workspace_size(B, Hq, Hkv, T, N, D, split);
  LB2_CHECK_ARG(need > 0, "decode_noalloc: empty or unsupported shape");
  if (need > LB2_NOALLOC_SCRATCH_BYTES)
    return fail(LB2_EINVAL, "decode_noalloc: this call needs " + std::to_string(need) + " bytes of scratch, more than "
                            "the " + std::to_string(LB2_NOALLOC_SCRATCH_BYTES) + "-byte static array; use a larger "
                            "split or lb2_attn_decode with a caller workspace");
  void* ws = nullptr;
  int rc = noalloc::scratch(&ws);
  if (rc) return rc;
  // The array keeps whatever the last call left; every partial this call reads is written by this call first, so
  // nothing needs clearing.
  return decode::run(q, q_st, k, k_st, v, v_st, o, o_st, nullptr, nullptr, kv_len, B, Hq, Hkv, T, N, D, dtype, scale,
                     causal, split, ws, LB2_NOALLOC_SCRATCH_BYTES, stream);
}

static int combine_partials(const float* part_o, int64_t so, const float* part_lse, int64_t sl, int R, int B, int Hq,
                            int T, int D, void* o, const int64_t* o_st, int dtype, void* stream) {
  LB2_CHECK_ARG(R > 0 && B > 0 && Hq > 0 && T > 0 && D > 0, "combine: empty shape");
  LB2_CHECK_ARG(int64_t(B) * Hq * T < (int64_t(1) << 31), "combine: too many rows");
  const int rows = B * Hq * T;
  const int warps = 8;
  dim3 grid((rows + warps - 1) / warps);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == LB2_BF16)
    decode::combine_kernel<__nv_bfloat16><<<grid, warps * 32, 0, st>>>(part_o, part_lse, R, so, sl, rows, Hq, T, D, o,
                                                                       o_st[0], o_st[1], o_st[2]);
  else if (dtype == LB2_F16)
    decode::combine_kernel<__half><<<grid, warps * 32, 0, st>>>(part_o, part_lse, R, so, sl, rows, Hq, T, D, o,
                                                                o_st[0], o_st[1], o_st[2]);
  else if (dtype == LB2_F32)
    decode::combine_kernel<float><<<grid, warps * 32, 0, st>>>(part_o, part_lse, R, so, sl, rows, Hq, T, D, o,
                                                               o_st[0], o_st[1], o_st[2]);
  else
    return fail(LB2_EINVAL, "combine: dtype");
  LB2_CUDA(cudaGetLastError());
  return LB2_OK;
}

int lb2_attn_combine(const float* part_o, const float* part_lse, int R, int B, int Hq, int T, int D, void* o,
                     const int64_t* o_st, int dtype, void* stream) {
  const int64_t rows = int64_t(B) * Hq * T;
  return combine_partials(part_o, rows * D, part_lse, rows, R, B, Hq, T, D, o, o_st, dtype, stream);
}

int lb2_attn_combine_packed(const float* packed, int R, int B, int Hq, int T, int D, void* o, const int64_t* o_st,
                            int dtype, void* stream) {
  const int64_t rows = int64_t(B) * Hq * T;
  return combine_partials(packed, rows * (D + 1), packed + rows * D, rows * (D + 1), R, B, Hq, T, D, o, o_st, dtype,
                          stream);
}


// ------------------------------------------------------------------------------------------------ host-buffer decode

namespace {

// Per-device state of lb2_attn_decode_host: its two copy streams, the events that order two staging slots, and the
// count of calls (slot = count % 2). Created on a device's first call, kept until exit.
struct HostDecodeState {
  cudaStream_t h2d = nullptr, d2h = nullptr;
  cudaEvent_t h2d_done[2] = {}, dec_done[2] = {}, d2h_done[2] = {};
  uint64_t calls = 0;
  bool ready = false;
};
HostDecodeState g_host_decode[64];
std::mutex g_host_decode_mu;  // guards the lazy creation: two threads' first calls on one device make one set

int host_decode_state(HostDecodeState** out) {
  int dev = 0;
  LB2_CUDA(cudaGetDevice(&dev));
  LB2_CHECK_ARG(dev >= 0 && dev < 64, "decode_host: device index");
  HostDecodeState& s = g_host_decode[dev];
  std::lock_guard<std::mutex> lock(g_host_decode_mu);
  if (!s.ready) {
    LB2_CUDA(cudaStreamCreateWithFlags(&s.h2d, cudaStreamNonBlocking));
    LB2_CUDA(cudaStreamCreateWithFlags(&s.d2h, cudaStreamNonBlocking));
    for (int j = 0; j < 2; ++j)
      for (cudaEvent_t* e : {&s.h2d_done[j], &s.dec_done[j], &s.d2h_done[j]})
        LB2_CUDA(cudaEventCreateWithFlags(e, cudaEventDisableTiming));
    s.ready = true;
  }
  *out = &s;
  return LB2_OK;
}

size_t host_stage_bytes(int B, int Hq, int T, int D, int dtype) {
  const size_t row = size_t(B) * Hq * T * D * (dtype == LB2_F32 ? 4 : 2);
  return (row + 255) / 256 * 256;  // one q or o image, 256-byte aligned
}

}  // namespace

size_t lb2_attn_decode_host_workspace_size(int B, int Hq, int Hkv, int T, int N, int D, int dtype, int split) {
  const size_t dec = lb2_attn_decode_workspace_size(B, Hq, Hkv, T, N, D, split);
  if (dec == 0 || D <= 0) return 0;
  return 4 * host_stage_bytes(B, Hq, T, D, dtype) + dec;
}

int lb2_attn_decode_host(const void* q_host, const void* k, const int64_t* k_st, const void* v, const int64_t* v_st,
                         void* o_host, const int32_t* kv_len, int B, int Hq, int Hkv, int T, int N, int D, int dtype,
                         float scale, int causal, int split, void* workspace, size_t workspace_bytes, void* stream) {
  LB2_CHECK_ARG(q_host && o_host, "decode_host: host buffers missing");
  LB2_CHECK_ARG(B > 0 && Hq > 0 && T > 0 && D > 0, "decode_host: shape");
  const size_t need = lb2_attn_decode_host_workspace_size(B, Hq, Hkv, T, N, D, dtype, split);
  LB2_CHECK_ARG(need > 0 && workspace_bytes >= need && (reinterpret_cast<uintptr_t>(workspace) & 255) == 0,
                "decode_host: workspace too small or not 256-byte aligned");
  HostDecodeState* s = nullptr;
  if (const int rc = host_decode_state(&s)) return rc;
  const size_t stage = host_stage_bytes(B, Hq, T, D, dtype);
  const size_t bytes = size_t(B) * Hq * T * D * (dtype == LB2_F32 ? 4 : 2);
  const int j = int(s->calls & 1);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  void* q_dev = ws + j * stage;
  void* o_dev = ws + (2 + j) * stage;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // q in on the copy stream, once this slot's o of two calls back is out (which followed that call's decode, so its
  // q in this slot has been read too)
  LB2_CUDA(cudaStreamWaitEvent(s->h2d, s->d2h_done[j], 0));
  LB2_CUDA(cudaMemcpyAsync(q_dev, q_host, bytes, cudaMemcpyHostToDevice, s->h2d));
  LB2_CUDA(cudaEventRecord(s->h2d_done[j], s->h2d));
  // the decode on the caller's stream once q is in: one wait, which also orders it after the slot's o of two calls
  // back has left (each wait on another stream's event costs the caller's stream device time)
  LB2_CUDA(cudaStreamWaitEvent(st, s->h2d_done[j], 0));
  const int64_t qs[3] = {int64_t(Hq) * T * D, int64_t(T) * D, D};
  if (const int rc = lb2_attn_decode(q_dev, qs, k, k_st, v, v_st, o_dev, qs, kv_len, B, Hq, Hkv, T, N, D, dtype, scale,
                                     causal, split, ws + 4 * stage, workspace_bytes - 4 * stage, stream))
    return rc;
  LB2_CUDA(cudaEventRecord(s->dec_done[j], st));
  // o out on the other copy stream
  LB2_CUDA(cudaStreamWaitEvent(s->d2h, s->dec_done[j], 0));
  LB2_CUDA(cudaMemcpyAsync(o_host, o_dev, bytes, cudaMemcpyDeviceToHost, s->d2h));
  LB2_CUDA(cudaEventRecord(s->d2h_done[j], s->d2h));
  ++s->calls;
  return LB2_OK;
}

int lb2_attn_decode_host_drain(void* stream) {
  HostDecodeState* s = nullptr;
  if (const int rc = host_decode_state(&s)) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  for (int j = 0; j < 2; ++j) LB2_CUDA(cudaStreamWaitEvent(st, s->d2h_done[j], 0));
  return LB2_OK;
}

// ------------------------------------------------------------------------------------------------ peer exchange

size_t lb2_xch_bytes(int B, int Hq, int T, int D) {
  if (B <= 0 || Hq <= 0 || T <= 0 || D <= 0) return 0;
  const int64_t half = int64_t(B) * Hq * T * (D + 1);
  return size_t(xch::flags_offset(half) * 4 + xch::XCH_MAX_RANKS * 4);
}

int lb2_xch_alloc(size_t bytes, void** ptr) {
  LB2_CHECK_ARG(ptr && bytes > 0, "xch_alloc: size");
  *ptr = nullptr;
  LB2_CUDA(cudaMalloc(ptr, bytes));
  const cudaError_t e = cudaMemset(*ptr, 0, bytes);  // flags start at 0: no call published yet
  if (e != cudaSuccess) {
    cudaFree(*ptr);
    *ptr = nullptr;
    return cuda_fail(e, "cudaMemset(exchange buffer)");
  }
  return LB2_OK;
}

int lb2_xch_free(void* ptr) {
  if (ptr) LB2_CUDA(cudaFree(ptr));
  return LB2_OK;
}

int lb2_xch_handle(void* ptr, void* handle) {
  LB2_CHECK_ARG(ptr && handle, "xch_handle: null pointer");
  cudaIpcMemHandle_t h;
  LB2_CUDA(cudaIpcGetMemHandle(&h, ptr));
  std::memcpy(handle, &h, sizeof(h));
  return LB2_OK;
}

int lb2_xch_open(const void* handle, void** ptr) {
  LB2_CHECK_ARG(ptr && handle, "xch_open: null pointer");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  *ptr = nullptr;
  LB2_CUDA(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
  return LB2_OK;
}

int lb2_xch_close(void* ptr) {
  if (ptr) LB2_CUDA(cudaIpcCloseMemHandle(ptr));
  return LB2_OK;
}

}  // extern "C"

namespace {

// The peer merge as a programmatic dependent of the decode partial before it (its launch overlaps that grid's tail;
// the kernel waits on the grid dependency first).
int xch_combine_launch(const xch::PeerParams& p, int dtype, void* stream) {
  const int warps = 8;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned((p.rows + warps - 1) / warps));
  cfg.blockDim = dim3(warps * 32);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (dtype == LB2_BF16)
    LB2_CUDA(cudaLaunchKernelEx(&cfg, xch::peer_combine_kernel<__nv_bfloat16>, p));
  else if (dtype == LB2_F16)
    LB2_CUDA(cudaLaunchKernelEx(&cfg, xch::peer_combine_kernel<__half>, p));
  else if (dtype == LB2_F32)
    LB2_CUDA(cudaLaunchKernelEx(&cfg, xch::peer_combine_kernel<float>, p));
  else
    return fail(LB2_EINVAL, "combine_peers: dtype");
  return LB2_OK;
}

}  // namespace

extern "C" {

int lb2_attn_combine_peers(const uint64_t* bufs, int R, int rank, uint32_t epoch, int B, int Hq, int T, int D, void* o,
                           const int64_t* o_st, int dtype, void* stream) {
  LB2_CHECK_ARG(R >= 1 && R <= xch::XCH_MAX_RANKS && rank >= 0 && rank < R, "combine_peers: 1 to 8 ranks");
  LB2_CHECK_ARG(B > 0 && Hq > 0 && T > 0 && D > 0 && int64_t(B) * Hq * T < (int64_t(1) << 31), "combine_peers: shape");
  LB2_CHECK_ARG(epoch > 0, "combine_peers: calls count from 1");
  xch::PeerParams p{};
  for (int r = 0; r < R; ++r) {
    LB2_CHECK_ARG(bufs[r] != 0, "combine_peers: a rank's buffer is missing");
    p.bufs[r] = reinterpret_cast<const float*>(bufs[r]);
  }
  p.R = R;
  p.rank = rank;
  p.parity = int(epoch & 1u);
  p.epoch = epoch;
  p.rows = B * Hq * T;
  p.half = int64_t(p.rows) * (D + 1);
  p.vec = p.rows % 4 == 0 && (D == 64 || D == 128 || D == 256);
  for (int r = 0; r < R; ++r) p.vec = p.vec && (bufs[r] & 15) == 0;
  p.Hq = Hq;
  p.Tq = T;
  p.D = D;
  p.o = o;
  p.o0 = o_st[0];
  p.o1 = o_st[1];
  p.o2 = o_st[2];
  return xch_combine_launch(p, dtype, stream);
}

size_t lb2_xch_push_bytes(int R, int B, int Hq, int T, int D) {
  if (R < 1 || R > xch::XCH_MAX_RANKS || B <= 0 || Hq <= 0 || T <= 0 || D <= 0) return 0;
  const int64_t half = int64_t(R) * B * Hq * T * (D + 1);
  return size_t(xch::flags_offset(half) * 4 + xch::XCH_MAX_RANKS * 4 + 16);  // flags, then the rank's block count
}

int lb2_attn_decode_push(const void* q, const int64_t* q_st, const void* k, const int64_t* k_st, const void* v,
                         const int64_t* v_st, const int32_t* kv_len, int B, int Hq, int Hkv, int T, int N, int D,
                         int dtype, float scale, int split, void* workspace, size_t workspace_bytes,
                         const uint64_t* bufs, int R, int rank, uint32_t epoch, void* stream) {
  LB2_CHECK_ARG(R >= 1 && R <= xch::XCH_MAX_RANKS && rank >= 0 && rank < R, "decode_push: 1 to 8 ranks");
  LB2_CHECK_ARG(epoch > 0, "decode_push: calls count from 1");
  const int64_t rows = int64_t(B) * Hq * T, slot = rows * (D + 1), half = R * slot;
  float* po[xch::XCH_MAX_RANKS];
  float* pl[xch::XCH_MAX_RANKS];
  uint32_t* flag[xch::XCH_MAX_RANKS];
  for (int r = 0; r < R; ++r) {
    LB2_CHECK_ARG(bufs[r] != 0 && (bufs[r] & 15) == 0, "decode_push: a rank's buffer is missing or misaligned");
    po[r] = reinterpret_cast<float*>(bufs[r]) + int64_t(epoch & 1u) * half + rank * slot;
    pl[r] = po[r] + rows * D;
    flag[r] = reinterpret_cast<uint32_t*>(reinterpret_cast<float*>(bufs[r]) + xch::flags_offset(half)) + rank;
  }
  uint32_t* count = reinterpret_cast<uint32_t*>(reinterpret_cast<float*>(bufs[rank]) + xch::flags_offset(half)) +
                    xch::XCH_MAX_RANKS;
  return decode::run(q, q_st, k, k_st, v, v_st, nullptr, nullptr, nullptr, nullptr, kv_len, B, Hq, Hkv, T, N, D, dtype,
                     scale, 0, split, workspace, workspace_bytes, stream, R, po, pl, count, flag, epoch);
}

int lb2_attn_combine_pushed(const uint64_t* bufs, int R, int rank, uint32_t epoch, int B, int Hq, int T, int D, void* o,
                            const int64_t* o_st, int dtype, void* stream) {
  LB2_CHECK_ARG(R >= 1 && R <= xch::XCH_MAX_RANKS && rank >= 0 && rank < R, "combine_pushed: 1 to 8 ranks");
  LB2_CHECK_ARG(B > 0 && Hq > 0 && T > 0 && D > 0 && int64_t(B) * Hq * T < (int64_t(1) << 31),
                "combine_pushed: shape");
  LB2_CHECK_ARG(epoch > 0, "combine_pushed: calls count from 1");
  xch::PeerParams p{};
  for (int r = 0; r < R; ++r) {
    LB2_CHECK_ARG(bufs[r] != 0, "combine_pushed: a rank's buffer is missing");
    p.bufs[r] = reinterpret_cast<const float*>(bufs[r]);
  }
  p.R = R;
  p.rank = rank;
  p.parity = int(epoch & 1u);
  p.epoch = epoch;
  p.rows = B * Hq * T;
  p.half = int64_t(R) * p.rows * (D + 1);
  p.pushed = 1;
  p.vec = p.rows % 4 == 0 && (D == 64 || D == 128 || D == 256) && (bufs[rank] & 15) == 0;
  p.Hq = Hq;
  p.Tq = T;
  p.D = D;
  p.o = o;
  p.o0 = o_st[0];
  p.o1 = o_st[1];
  p.o2 = o_st[2];
  return xch_combine_launch(p, dtype, stream);
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // extern "C"

namespace {

// The prefill on the kernel its shape takes: CTA pairs for head dims 128 / 256 over more than one row tile, else the
// single-CTA kernel. `tiled`: the array mask's kept-tile lists are built in `ws` first and the kernel reads only
// those tiles.
bool prefill_pair(int D, int T) { return (D == 128 || D == 256) && T > prefill::BM; }
int prefill_rows(int D, int T) { return prefill_pair(D, T) ? 2 * prefill::BM : prefill::BM; }
int prefill_bn(int D, int T) {
  return prefill_pair(D, T) ? prefill2::Cfg<256>::BN : D == 256 ? prefill::Cfg<256>::BN
                                                     : D == 128 ? prefill::Cfg<128>::BN : prefill::Cfg<64>::BN;
}
size_t tiles_bytes(int T, int N, int D) {
  const int64_t nrb = (T + prefill_rows(D, T) - 1) / prefill_rows(D, T), nkt = (N + prefill_bn(D, T) - 1) /
                                                                              prefill_bn(D, T);
  return size_t((nrb * nkt + 255) / 256 * 256 + nrb * nkt * 4 + nrb * 4 + 256);
}

int prefill_run(const void* q, const int64_t* q_st, const void* k, const int64_t* k_st, const void* v,
                const int64_t* v_st, void* o, const int64_t* o_st, const void* gate, const int64_t* g_st,
                const uint8_t* mask, const int64_t* m_st, int B, int Hq, int Hkv, int T, int N, int D, int dtype,
                float scale, int mask_kind, bool tiled, void* ws, size_t ws_bytes, void* stream) {
  LB2_CHECK_ARG(B > 0 && Hq > 0 && Hkv > 0 && T > 0 && N > 0, "prefill: empty shape");
  LB2_CHECK_ARG(Hq % Hkv == 0, "prefill: Hq must be a multiple of Hkv");
  if (dtype == LB2_F32)  // exact fp32 on CUDA cores (the tensor-core kernel takes 16-bit operands)
    return f32attn::run(q, q_st, k, k_st, v, v_st, o, o_st, gate, g_st, mask, m_st, nullptr, B, Hq, Hkv, T, N, D,
                        scale, mask_kind, stream);
  LB2_CHECK_ARG(D == 64 || D == 128 || D == 256, "prefill: head dim must be 64, 128 or 256");
  LB2_CHECK_ARG(dtype == LB2_BF16 || dtype == LB2_F16, "prefill: dtype must be bf16 or f16");
  LB2_CHECK_ARG(mask_kind >= LB2_MASK_NONE && mask_kind <= LB2_MASK_ARRAY, "prefill: mask kind");
  LB2_CHECK_ARG(mask_kind != LB2_MASK_ARRAY || (mask != nullptr && m_st != nullptr), "prefill: array mask missing");
  for (int i = 0; i < 3; ++i) {
    LB2_CHECK_ARG(q_st[i] % 8 == 0 && k_st[i] % 8 == 0 && v_st[i] % 8 == 0 && o_st[i] % 8 == 0,
                  "prefill: strides must be multiples of 8 elements");
    LB2_CHECK_ARG(!gate || g_st[i] % 8 == 0, "prefill: gate strides must be multiples of 8 elements");
  }
  LB2_CHECK_ARG(aligned16(q) && aligned16(k) && aligned16(v) && aligned16(o) && (!gate || aligned16(gate)),
                "prefill: tensors must be 16-byte aligned");
  // Head dims 128 and 256 over more than one row tile run on CTA pairs (each CTA loads half of every K and V tile).
  const bool pair = (D == 128 || D == 256) && T > prefill::BM;
  static_assert(prefill2::Cfg<128>::HN == prefill2::Cfg<256>::HN && prefill2::Cfg<128>::BN == prefill2::Cfg<256>::BN,
                "one K / V box height for both pair head dims");
  CUtensorMap qm, km, vm;
  const int BN = D == 256 ? prefill::Cfg<256>::BN : prefill::Cfg<128>::BN;
  int rc = prefill::map4(&qm, q, q_st, B, Hq, T, D, dtype, prefill::BM);
  if (!rc) rc = prefill::map4(&km, k, k_st, B, Hkv, N, D, dtype, pair ? prefill2::Cfg<256>::HN : BN);
  if (!rc) rc = prefill::map4(&vm, v, v_st, B, Hkv, N, D, dtype, pair ? prefill2::Cfg<256>::BN : BN);
  if (rc) return rc;
  prefill::Params p{};
  p.o = o;
  p.gate = gate;
  for (int i = 0; i < 3; ++i) {
    p.o_st[i] = o_st[i];
    p.g_st[i] = gate ? g_st[i] : 0;
  }
  p.mask = mask_kind == LB2_MASK_ARRAY ? mask : nullptr;
  p.m_st[0] = p.mask ? m_st[0] : 0;
  p.m_st[1] = p.mask ? m_st[1] : 0;
  p.B = B;
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.T = T;
  p.N = N;
  p.G = Hq / Hkv;
  p.mask_kind = mask_kind;
  p.mtiles = pair ? (T + 2 * prefill::BM - 1) / (2 * prefill::BM) : (T + prefill::BM - 1) / prefill::BM;
  p.scale_log2 = scale * 1.4426950408889634f;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (tiled && p.mask) {
    LB2_CHECK_ARG(ws != nullptr && ws_bytes >= tiles_bytes(T, N, D) && (reinterpret_cast<uintptr_t>(ws) & 15) == 0,
                  "prefill_tiled: workspace too small or not 16-byte aligned");
    const int RB = prefill_rows(D, T), TBN = prefill_bn(D, T);
    const int nrb = (T + RB - 1) / RB, nkt = (N + TBN - 1) / TBN;
    uint8_t* flags = static_cast<uint8_t*>(ws);
    int32_t* list = reinterpret_cast<int32_t*>(flags + (int64_t(nrb) * nkt + 255) / 256 * 256);
    int32_t* count = list + int64_t(nrb) * nkt;
    const int vec = m_st[1] == 1 && m_st[0] % 16 == 0 && TBN % 16 == 0 && (reinterpret_cast<uintptr_t>(mask) & 15) == 0;
    tiles::flag_kernel<<<dim3(unsigned(nkt), unsigned(nrb)), 256, 0, st>>>(mask, m_st[0], m_st[1], T, N, RB, TBN,
                                                                             nkt, flags, vec);
    tiles::compact_kernel<<<unsigned((nrb + 3) / 4), 128, 0, st>>>(flags, nrb, nkt, list, count);
    LB2_CUDA(cudaGetLastError());
    p.tl = list;
    p.tn = count;
    p.tl_ld = nkt;
  }
  if (pair) {
    if (D == 128)
      return dtype == LB2_BF16 ? prefill2::launch<__nv_bfloat16, 128>(qm, km, vm, p, st)
                               : prefill2::launch<__half, 128>(qm, km, vm, p, st);
    return dtype == LB2_BF16 ? prefill2::launch<__nv_bfloat16, 256>(qm, km, vm, p, st)
                             : prefill2::launch<__half, 256>(qm, km, vm, p, st);
  }
  if (dtype == LB2_BF16) {
    if (D == 64) return prefill::launch<__nv_bfloat16, 64>(qm, km, vm, p, st);
    if (D == 128) return prefill::launch<__nv_bfloat16, 128>(qm, km, vm, p, st);
    return prefill::launch<__nv_bfloat16, 256>(qm, km, vm, p, st);
  }
  if (D == 64) return prefill::launch<__half, 64>(qm, km, vm, p, st);
  if (D == 128) return prefill::launch<__half, 128>(qm, km, vm, p, st);
  return prefill::launch<__half, 256>(qm, km, vm, p, st);
}

}  // namespace

extern "C" {

int lb2_attn_prefill(const void* q, const int64_t* q_st, const void* k, const int64_t* k_st, const void* v,
                     const int64_t* v_st, void* o, const int64_t* o_st, const void* gate, const int64_t* g_st,
                     const uint8_t* mask, const int64_t* m_st, int B, int Hq, int Hkv, int T, int N, int D, int dtype,
                     float scale, int mask_kind, void* stream) {
  return prefill_run(q, q_st, k, k_st, v, v_st, o, o_st, gate, g_st, mask, m_st, B, Hq, Hkv, T, N, D, dtype, scale,
                     mask_kind, false, nullptr, 0, stream);
}

size_t lb2_attn_prefill_tiled_workspace_size(int T, int N, int D) {
  if (T <= 0 || N <= 0) return 0;
  return tiles_bytes(T, N, D);
}

int lb2_attn_prefill_tiled(const void* q, const int64_t* q_st, const void* k, const int64_t* k_st, const void* v,
                           const int64_t* v_st, void* o, const int64_t* o_st, const void* gate, const int64_t* g_st,
                           const uint8_t* mask, const int64_t* m_st, int B, int Hq, int Hkv, int T, int N, int D,
                           int dtype, float scale, void* workspace, size_t workspace_bytes, void* stream) {
  LB2_CHECK_ARG(mask != nullptr && m_st != nullptr, "prefill_tiled: an array mask is required");
  return prefill_run(q, q_st, k, k_st, v, v_st, o, o_st, gate, g_st, mask, m_st, B, Hq, Hkv, T, N, D, dtype, scale,
                     LB2_MASK_ARRAY, true, workspace, workspace_bytes, stream);
}

size_t lb2_gdn_chunked_workspace_size(int B, int T, int Hk, int Hv, int Dk, int Dv) {
  (void)Hk;
  if (B <= 0 || T < 0 || Hv <= 0 || Dk != gdnchunk::DK || Dv != gdnchunk::DV) return 0;
  const int64_t nchunks = (int64_t(T) + gdnchunk::C - 1) / gdnchunk::C;
  return size_t(int64_t(B) * Hv * nchunks * gdnchunk::UNIT_BYTES) + 256;
}

int lb2_gdn_chunked(const void* q, const void* k, int qdt, const void* v, int vdt, const void* g, int gdt,
                    const void* beta, int bdt, const float* state_in, float* state_out, void* y, int B, int T, int Hk,
                    int Dk, int Hv, int Dv, void* workspace, size_t workspace_bytes, void* stream) {
  LB2_CHECK_ARG(B > 0 && T >= 0 && Hk > 0 && Hv > 0, "gdn_chunked: empty shape");
  LB2_CHECK_ARG(Hv % Hk == 0, "gdn_chunked: Hv must be a multiple of Hk");
  LB2_CHECK_ARG(Dk == gdnchunk::DK && Dv == gdnchunk::DV, "gdn_chunked: Dk = Dv = 128 only");
  LB2_CHECK_ARG(qdt == LB2_BF16 || qdt == LB2_F16, "gdn_chunked: q/k must be bf16 or f16");
  for (int dt : {vdt, gdt, bdt}) LB2_CHECK_ARG(dt >= LB2_F32 && dt <= LB2_F16, "gdn_chunked: dtype");
  LB2_CHECK_ARG(vdt == qdt, "gdn_chunked: v must share q's dtype (y is written in it)");
  LB2_CHECK_ARG(aligned16(q) && aligned16(k) && aligned16(v) && aligned16(workspace),
                "gdn_chunked: q, k, v and workspace 16-byte aligned");
  LB2_CHECK_ARG(workspace_bytes >= lb2_gdn_chunked_workspace_size(B, T, Hk, Hv, Dk, Dv), "gdn_chunked: workspace too small");
  LB2_CHECK_ARG(((uintptr_t(state_in) | uintptr_t(state_out)) & 7) == 0, "gdn_chunked: states 8-byte aligned");
  gdnchunk::Params p{q, k, v, g, beta, qdt, vdt, gdt, bdt, state_in, state_out, y, B, T, Hk, Hv,
                     (T + gdnchunk::C - 1) / gdnchunk::C, static_cast<float*>(workspace)};
  // Q and K tiles of the scan: [B, T, Hk, Dk] contiguous, 64-column boxes of 64 positions (rows past T read as 0)
  CUtensorMap qm, km, vm;
  std::memset(&qm, 0, sizeof(qm));
  std::memset(&km, 0, sizeof(km));
  std::memset(&vm, 0, sizeof(vm));
  if (T > 0) {
    const int64_t qk_st[3] = {int64_t(T) * Hk * Dk, Dk, int64_t(Hk) * Dk};
    const int64_t v_st[3] = {int64_t(T) * Hv * Dv, Dv, int64_t(Hv) * Dv};
    int rc = prefill::map4(&qm, q, qk_st, B, Hk, T, Dk, qdt, gdnchunk::C);
    if (!rc) rc = prefill::map4(&km, k, qk_st, B, Hk, T, Dk, qdt, gdnchunk::C);
    if (!rc) rc = prefill::map4(&vm, v, v_st, B, Hv, T, Dv, vdt, gdnchunk::C);
    if (rc) return rc;
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  static int attr_dev = -1;
  int dev = 0;
  LB2_CUDA(cudaGetDevice(&dev));
  if (attr_dev != dev) {
    LB2_CUDA(cudaFuncSetAttribute(gdnchunk::prep_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  gdnchunk::PrepSmem::BYTES));
    LB2_CUDA(cudaFuncSetAttribute(gdnchunk::prep_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  gdnchunk::PrepSmem::BYTES));
    LB2_CUDA(cudaFuncSetAttribute(gdnchunk::scan_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  gdnchunk::TcSmem::BYTES));
    LB2_CUDA(cudaFuncSetAttribute(gdnchunk::scan_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  gdnchunk::TcSmem::BYTES));
    attr_dev = dev;
  }
  const dim3 gp(unsigned(p.nchunks), unsigned(Hv), unsigned(B)), gs(gdnchunk::DV / gdnchunk::DVB, Hv, B);
  if (qdt == LB2_BF16) {
    if (p.nchunks > 0)
      gdnchunk::prep_kernel<__nv_bfloat16><<<gp, 128, gdnchunk::PrepSmem::BYTES, st>>>(qm, km, vm, p);
    gdnchunk::scan_kernel<__nv_bfloat16><<<gs, gdnchunk::TC_THREADS, gdnchunk::TcSmem::BYTES, st>>>(qm, km, p);
  } else {
    if (p.nchunks > 0) gdnchunk::prep_kernel<__half><<<gp, 128, gdnchunk::PrepSmem::BYTES, st>>>(qm, km, vm, p);
    gdnchunk::scan_kernel<__half><<<gs, gdnchunk::TC_THREADS, gdnchunk::TcSmem::BYTES, st>>>(qm, km, p);
  }
  LB2_CUDA(cudaGetLastError());
  return LB2_OK;
}

int lb2_gdn_recurrent(const void* q, const void* k, int qdt, const void* v, int vdt, const void* g, int gdt,
                      int g_vec, const void* beta, int bdt, const uint8_t* mask, const float* state_in,
                      float* state_out, void* y, int B, int T, int Hk, int Dk, int Hv, int Dv, void* stream) {
  LB2_CHECK_ARG(B > 0 && T >= 0 && Hk > 0 && Hv > 0 && Dv > 0, "gdn: empty shape");
  LB2_CHECK_ARG(Hv % Hk == 0, "gdn: Hv must be a multiple of Hk");
  LB2_CHECK_ARG(Dk == 32 || Dk == 64 || Dk == 128 || Dk == 256, "gdn: Dk must be 32, 64, 128 or 256");
  for (int dt : {qdt, vdt, gdt, bdt}) LB2_CHECK_ARG(dt >= LB2_F32 && dt <= LB2_F16, "gdn: dtype");
  gdnrec::Params p{q, k, v, g, beta, mask, state_in, state_out, y, qdt, vdt, gdt, bdt, g_vec, B, T, Hk, Dk, Hv, Dv};
  LB2_CHECK_ARG(Dv % 4 == 0, "gdn: Dv must be a multiple of 4");
  {  // q / k rows are read as 8-byte (Dk = 128) or 16-byte (Dk = 256) vectors
    const uintptr_t need = Dk == 256 ? 15 : Dk == 128 ? 7 : 0;
    LB2_CHECK_ARG(((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k)) & need) == 0,
                  "gdn: q and k must be 8-byte aligned (16-byte at Dk = 256)");
  }
  LB2_CHECK_ARG((reinterpret_cast<uintptr_t>(state_in) & 15) == 0 && (reinterpret_cast<uintptr_t>(state_out) & 15) == 0,
                "gdn: state buffers must be 16-byte aligned");
  const int warps = 4;
  // value rows a warp: four for a decode step (more state in flight; eight measured 2 % slower at Dk = 128), one for
  // longer passes (more warps)
  const int R = T > 1 ? 1 : 4;
  LB2_CHECK_ARG(int64_t(B) * Hv < 65536, "gdn: at most 65535 (sequence, head) pairs a call");
  dim3 grid(unsigned((Dv / R + warps - 1) / warps), unsigned(B * Hv));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
#define LB2_GDN_LAUNCH(QT)                                                                           \
  if (R == 1) {                                                                                      \
    switch (Dk) {                                                                                    \
      case 32: gdnrec::recurrent_kernel<QT, 1, 1><<<grid, warps * 32, 0, st>>>(p); break;            \
      case 64: gdnrec::recurrent_kernel<QT, 2, 1><<<grid, warps * 32, 0, st>>>(p); break;            \
      case 128: gdnrec::recurrent_kernel<QT, 4, 1><<<grid, warps * 32, 0, st>>>(p); break;           \
      default: gdnrec::recurrent_kernel<QT, 8, 1><<<grid, warps * 32, 0, st>>>(p); break;            \
    }                                                                                                \
  } else {                                                                                           \
    switch (Dk) {                                                                                    \
      case 32: gdnrec::recurrent_kernel<QT, 1, 4><<<grid, warps * 32, 0, st>>>(p); break;            \
      case 64: gdnrec::recurrent_kernel<QT, 2, 4><<<grid, warps * 32, 0, st>>>(p); break;            \
      case 128: gdnrec::recurrent_kernel<QT, 4, 4><<<grid, warps * 32, 0, st>>>(p); break;           \
      default: gdnrec::recurrent_kernel<QT, 8, 4><<<grid, warps * 32, 0, st>>>(p); break;            \
    }                                                                                                \
  }
  if (qdt == LB2_BF16) {
    LB2_GDN_LAUNCH(__nv_bfloat16)
  } else if (qdt == LB2_F16) {
    LB2_GDN_LAUNCH(__half)
  } else {
    LB2_GDN_LAUNCH(float)
  }
#undef LB2_GDN_LAUNCH
  LB2_CUDA(cudaGetLastError());
  return LB2_OK;
}

// ------------------------------------------------------------------------------------------------ gathers

}  // extern "C"

namespace {

// How a run-gather moves data: 16-byte units when every base is 16-byte aligned, rows are contiguous and every
// stride is a whole number of units; else one element a unit (raw bits).
struct RunUnits {
  bool vec;
  int esz, per;  // element bytes; elements a unit
};

// views: (strides, count) pairs, each the element strides of one view with the dim stride last.
RunUnits run_units(int dtype, int D, std::initializer_list<const void*> bases,
                   std::initializer_list<std::pair<const int64_t*, int>> views) {
  RunUnits u{true, dtype == LB2_F32 ? 4 : 2, 0};
  const int per = 16 / u.esz;
  if ((int64_t(D) * u.esz) % 16) u.vec = false;
  for (const void* b : bases)
    if (reinterpret_cast<uintptr_t>(b) & 15) u.vec = false;
  for (const auto& v : views) {
    const int64_t* st = v.first;
    if (st[v.second - 1] != 1) u.vec = false;
    for (int i = 0; i + 1 < v.second; ++i)
      if (st[i] % per) u.vec = false;
  }
  u.per = u.vec ? per : 1;
  return u;
}

template <typename U>
kvr::Rows<U> rows_of(const void* base, int64_t hs, int64_t rs, int64_t ds, int per) {
  return kvr::Rows<U>{static_cast<const U*>(base), hs / per, rs / per, per > 1 ? 1 : ds};
}

// Calls f with a value of the unit type: uint4 for 16-byte units, else the element's raw-bits type.
template <typename F>
int with_units(const RunUnits& u, F&& f) {
  if (u.vec) return f(uint4{});
  if (u.esz == 4) return f(0u);
  return f(static_cast<unsigned short>(0));
}

}  // namespace

extern "C" {

int lb2_kv_gather_picks(const void* k, const int64_t* k_st, const void* v, const int64_t* v_st, const int32_t* tb,
                        int nsel, int cr, int n, void* kg, void* vg, int Hk, int D, int dtype, void* stream) {
  LB2_CHECK_ARG(nsel >= 0 && cr > 0 && n >= 0 && Hk > 0 && D > 0, "kv_gather_picks: shape");
  LB2_CHECK_ARG(dtype >= LB2_F32 && dtype <= LB2_F16, "kv_gather_picks: dtype");
  const int m = nsel * cr + n - n / cr * cr;
  if (m == 0) return LB2_OK;
  const RunUnits ru = run_units(dtype, D, {k, v, kg, vg}, {{k_st, 3}, {v_st, 3}});
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const dim3 grid(unsigned(nsel + 1), 2);
  return with_units(ru, [&](auto unit) {
    using U = decltype(unit);
    kvr::view_runs_kernel<U><<<grid, kvr::RUN_THREADS, 0, st>>>(
        rows_of<U>(k, k_st[0], k_st[1], k_st[2], ru.per), rows_of<U>(v, v_st[0], v_st[1], v_st[2], ru.per), tb, nsel,
        cr, n, static_cast<U*>(kg), static_cast<U*>(vg), Hk, D / ru.per);
    LB2_CUDA(cudaGetLastError());
    return LB2_OK;
  });
}

size_t lb2_qsa_decode_workspace_size(int nsel, int cr, int n, int Hq, int Hk, int D) {
  if (nsel < 0 || cr <= 0 || n < 0 || Hq <= 0 || Hk <= 0 || Hq % Hk) return 0;
  const int m = nsel * cr + n - n / cr * cr;
  return m > 0 ? lb2_attn_decode_workspace_size(1, Hq, Hk, 1, m, D, 0) : 0;
}

int lb2_qsa_decode(const void* q, const int64_t* q_st, const void* k, const int64_t* k_st, const void* v,
                   const int64_t* v_st, void* o, const int64_t* o_st, const int32_t* tb, int nsel, int cr, int n, int Hq,
                   int Hk, int D, int dtype, float scale, void* workspace, size_t workspace_bytes, void* stream) {
  LB2_CHECK_ARG(nsel >= 0 && cr > 0 && n >= 0 && Hq > 0 && Hk > 0, "qsa_decode: shape");
  LB2_CHECK_ARG(nsel == 0 || tb != nullptr, "qsa_decode: picks missing");
  const int m = nsel * cr + n - n / cr * cr;
  LB2_CHECK_ARG(m > 0, "qsa_decode: no key to attend to");
  return decode::run(q, q_st, k, k_st, v, v_st, o, o_st, nullptr, nullptr, nullptr, 1, Hq, Hk, 1, m, D, dtype, scale,
                     0, 0, workspace, workspace_bytes, stream, 0, nullptr, nullptr, nullptr, nullptr, 0, tb, nsel, cr,
                     n);
}

int lb2_kvh_put(const uint64_t* table, const void* k, const int64_t* k_st, const void* v, const int64_t* v_st,
                int64_t pos0, int s, int Hk, int D, int dtype, int logc, void* stream) {
  LB2_CHECK_ARG(s >= 0 && pos0 >= 0 && Hk > 0 && D > 0 && logc > 0 && logc < 31, "kvh_put: shape");
  LB2_CHECK_ARG(dtype >= LB2_F32 && dtype <= LB2_F16, "kvh_put: dtype");
  if (s == 0) return LB2_OK;
  const RunUnits ru = run_units(dtype, D, {k, v}, {{k_st, 3}, {v_st, 3}});
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const dim3 grid(unsigned((s + 31) / 32), 2);
  return with_units(ru, [&](auto unit) {
    using U = decltype(unit);
    kvr::home_put_kernel<U><<<grid, kvr::RUN_THREADS, 0, st>>>(
        table, rows_of<U>(k, k_st[0], k_st[1], k_st[2], ru.per), rows_of<U>(v, v_st[0], v_st[1], v_st[2], ru.per),
        pos0, s, Hk, D / ru.per, logc);
    LB2_CUDA(cudaGetLastError());
    return LB2_OK;
  });
}

int lb2_kvh_gather(const uint64_t* table, const int32_t* tb, int nsel, int cr, int n, void* kg, void* vg, int Hk,
                   int D, int dtype, int logc, void* stream) {
  LB2_CHECK_ARG(nsel >= 0 && cr > 0 && n >= 0 && Hk > 0 && D > 0 && logc > 0 && logc < 31, "kvh_gather: shape");
  LB2_CHECK_ARG(dtype >= LB2_F32 && dtype <= LB2_F16, "kvh_gather: dtype");
  LB2_CHECK_ARG((int64_t(1) << logc) % cr == 0, "kvh_gather: the block size must divide the chunk size");
  const int m = nsel * cr + n - n / cr * cr;
  if (m == 0) return LB2_OK;
  const RunUnits ru = run_units(dtype, D, {kg, vg}, {});
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const dim3 grid(unsigned(nsel + 1), 2);
  return with_units(ru, [&](auto unit) {
    using U = decltype(unit);
    kvr::home_runs_kernel<U><<<grid, kvr::RUN_THREADS, 0, st>>>(table, tb, nsel, cr, n, static_cast<U*>(kg),
                                                                static_cast<U*>(vg), Hk, D / ru.per, logc);
    LB2_CUDA(cudaGetLastError());
    return LB2_OK;
  });
}

int lb2_kvh_lru_plan(const int32_t* tb, int nsel, int32_t* slot_of, int max_blocks, int32_t* block_of, int32_t* stamp,
                     int32_t* ref, int32_t* meta, int ns, int32_t* sl, void* stream) {
  LB2_CHECK_ARG(nsel >= 1 && nsel <= kvr::LRU_MAX_NSEL, "kvh_lru_plan: 1 to 1024 picks a token");
  const int nt = (nsel + 31) / 32 * 32;
  LB2_CHECK_ARG(ns >= nt, "kvh_lru_plan: the pool needs at least ceil32(nsel) slots");
  LB2_CHECK_ARG(max_blocks >= 1, "kvh_lru_plan: max_blocks");
  LB2_CHECK_ARG(tb && slot_of && block_of && stamp && ref && meta && sl, "kvh_lru_plan: null pointer");
  kvr::lru_plan_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(tb, nsel, slot_of, max_blocks, block_of, stamp,
                                                                        ref, meta, ns, sl);
  LB2_CUDA(cudaGetLastError());
  return LB2_OK;
}

int lb2_kvh_lru_gather(const uint64_t* table, void* pool, int ns, const int32_t* tb, const int32_t* sl, int nsel, int cr,
                       int n, const void* kn, const int64_t* kn_st, const void* vn, const int64_t* vn_st, void* kg,
                       void* vg, int Hk, int D, int dtype, int logc, void* stream) {
  LB2_CHECK_ARG(nsel >= 0 && cr > 0 && n >= 1 && ns >= 1 && Hk > 0 && D > 0 && logc > 0 && logc < 31,
                "kvh_lru_gather: shape");
  LB2_CHECK_ARG(dtype >= LB2_F32 && dtype <= LB2_F16, "kvh_lru_gather: dtype");
  LB2_CHECK_ARG((int64_t(1) << logc) % cr == 0, "kvh_lru_gather: the block size must divide the chunk size");
  const RunUnits ru = run_units(dtype, D, {pool, kn, vn, kg, vg}, {{kn_st, 2}, {vn_st, 2}});
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const dim3 grid(unsigned(nsel + 1), 2);
  return with_units(ru, [&](auto unit) {
    using U = decltype(unit);
    kvr::lru_runs_kernel<U><<<grid, kvr::RUN_THREADS, 0, st>>>(
        table, static_cast<U*>(pool), ns, tb, sl, nsel, cr, n, rows_of<U>(kn, kn_st[0], 0, kn_st[1], ru.per),
        rows_of<U>(vn, vn_st[0], 0, vn_st[1], ru.per), static_cast<U*>(kg), static_cast<U*>(vg), Hk, D / ru.per,
        logc);
    LB2_CUDA(cudaGetLastError());
    return LB2_OK;
  });
}

int lb2_kvh_lru_inval(int32_t* slot_of, int32_t* block_of, int32_t* ref, int ns, int lim, void* stream) {
  LB2_CHECK_ARG(ns >= 1 && lim >= 0, "kvh_lru_inval: shape");
  kvr::lru_trim_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(slot_of, block_of, ref, ns, lim);
  LB2_CUDA(cudaGetLastError());
  return LB2_OK;
}

// ------------------------------------------------------------------------------------------------ GDN glue

int lb2_gdn_step_glue(const void* conv, const void* a, const void* b, const float* A_log, const float* dt_bias,
                      const float* state_in, float* state_out, void* y, int NR, int Hk, int Dk, int Hv, int Dv,
                      int dtype, float sq, float sk, float eps, void* stream) {
  LB2_CHECK_ARG(NR >= 0 && Hk > 0 && Hv > 0 && Dv > 0 && Hv % Hk == 0, "gdn_step_glue: shape");
  LB2_CHECK_ARG(Dk == 64 || Dk == 128, "gdn_step_glue: Dk must be 64 or 128");
  LB2_CHECK_ARG(dtype == LB2_BF16 || dtype == LB2_F16, "gdn_step_glue: dtype must be bf16 or f16");
  gdnrec::GlueParams p{conv, a, b, A_log, dt_bias, state_in, state_out, y, NR, Hk, Hv, Dv, sq, sk, eps};
  if (NR == 0) return LB2_OK;
  // value rows a warp: four (more blocks for one sequence's heads: one token 6.4-6.5 us with step_glue and norm_gate
  // at 32 heads of 128 x 128, 6.8 with eight rows a warp, 6.3-6.5 with two)
  const int R = Dv % 4 == 0 ? 4 : Dv % 2 == 0 ? 2 : 1;
  const dim3 grid(unsigned((Dv / R + 3) / 4), unsigned(Hv));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  auto launch = [&](auto t_tag, auto npt_tag) {
    using T = decltype(t_tag);
    constexpr int NPT = decltype(npt_tag)::value;
    switch (R) {
      case 8: gdnrec::glue_step_kernel<T, NPT, 8><<<grid, 128, 0, st>>>(p); break;
      case 4: gdnrec::glue_step_kernel<T, NPT, 4><<<grid, 128, 0, st>>>(p); break;
      case 2: gdnrec::glue_step_kernel<T, NPT, 2><<<grid, 128, 0, st>>>(p); break;
      default: gdnrec::glue_step_kernel<T, NPT, 1><<<grid, 128, 0, st>>>(p); break;
    }
  };
  using N4 = std::integral_constant<int, 4>;
  using N2 = std::integral_constant<int, 2>;
  if (dtype == LB2_BF16) {
    if (Dk == 128) launch(__nv_bfloat16{}, N4{});
    else launch(__nv_bfloat16{}, N2{});
  } else {
    if (Dk == 128) launch(__half{}, N4{});
    else launch(__half{}, N2{});
  }
  LB2_CUDA(cudaGetLastError());
  return LB2_OK;
}

int lb2_gdn_norm_gate(const void* x, const void* z, const void* w, void* out, int64_t R, int D, int dtype, float eps,
                      void* stream) {
  LB2_CHECK_ARG(R >= 0 && D > 0, "gdn_norm_gate: shape");
  LB2_CHECK_ARG(dtype >= LB2_F32 && dtype <= LB2_F16, "gdn_norm_gate: dtype");
  if (R == 0) return LB2_OK;
  dim3 grid(unsigned((R + 3) / 4));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == LB2_BF16)
    glue::norm_gate_kernel<__nv_bfloat16><<<grid, 128, 0, st>>>(
        static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(z),
        static_cast<const __nv_bfloat16*>(w), static_cast<__nv_bfloat16*>(out), R, D, eps);
  else if (dtype == LB2_F16)
    glue::norm_gate_kernel<__half><<<grid, 128, 0, st>>>(static_cast<const __half*>(x), static_cast<const __half*>(z),
                                                          static_cast<const __half*>(w), static_cast<__half*>(out), R,
                                                          D, eps);
  else
    glue::norm_gate_kernel<float><<<grid, 128, 0, st>>>(static_cast<const float*>(x), static_cast<const float*>(z),
                                                        static_cast<const float*>(w), static_cast<float*>(out), R, D,
                                                        eps);
  LB2_CUDA(cudaGetLastError());
  return LB2_OK;
}

int lb2_attn_qk_norm_rope(const void* qg, const void* kr, const void* q_norm_w, const void* k_norm_w, float eps,
                          const void* cos, const void* sin, int cs_dtype, void* q, void* k, int B, int S, int NQ,
                          int NK, int D, int R, int dtype, void* stream) {
  LB2_CHECK_ARG(B >= 0 && S >= 0 && NQ > 0 && NK > 0, "qk_norm_rope: shape");
  LB2_CHECK_ARG(dtype == LB2_BF16, "qk_norm_rope: bf16 rows only (the reference's path)");
  LB2_CHECK_ARG(cs_dtype >= LB2_F32 && cs_dtype <= LB2_F16, "qk_norm_rope: cos / sin dtype");
  LB2_CHECK_ARG(D == 128 || D == 256 || D == 512, "qk_norm_rope: head dim 128, 256 or 512");
  LB2_CHECK_ARG(R >= 0 && R <= D && R % 2 == 0, "qk_norm_rope: rope dims must be even and at most the head dim");
  for (const void* ptr : {qg, kr, q_norm_w, k_norm_w, static_cast<const void*>(q), static_cast<const void*>(k)})
    LB2_CHECK_ARG(aligned16(ptr), "qk_norm_rope: rows and weights 16-byte aligned");
  const int64_t items = int64_t(B) * S * (NQ + NK);
  if (items == 0) return LB2_OK;
  LB2_CHECK_ARG(R == 0 || (cos && sin), "qk_norm_rope: cos / sin missing");
  LB2_CHECK_ARG(int64_t(B) * S < (int64_t(1) << 31), "qk_norm_rope: too many rows");
  aglue::QkParams p{static_cast<const __nv_bfloat16*>(qg), static_cast<const __nv_bfloat16*>(kr),
                    static_cast<const __nv_bfloat16*>(q_norm_w), static_cast<const __nv_bfloat16*>(k_norm_w), cos, sin,
                    cs_dtype, eps, static_cast<__nv_bfloat16*>(q), static_cast<__nv_bfloat16*>(k), B, S, NQ, NK, R};
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // the pair-strided form for rope widths 0, 32, 64 and 128
  const int mode = R == 0 ? 0 : (R == 32 || R == 64) ? 1 : R == 128 ? 2 : -1;
  if (mode >= 0) {
    const dim3 g1(unsigned((int64_t(B) * S + aglue::QROWS - 1) / aglue::QROWS),
                  unsigned((NQ + NK + aglue::WARPS - 1) / aglue::WARPS));
    LB2_CHECK_ARG(g1.y < 65536, "qk_norm_rope: too many heads");
#define LB2_QK_PAIR_T(DD, MM)                                                                    \
  if (cs_dtype == LB2_F32)                                                                       \
    aglue::qk_rope_pair_kernel<DD, MM, float><<<g1, aglue::WARPS * 32, 0, st>>>(p);              \
  else if (cs_dtype == LB2_BF16)                                                                 \
    aglue::qk_rope_pair_kernel<DD, MM, __nv_bfloat16><<<g1, aglue::WARPS * 32, 0, st>>>(p);      \
  else                                                                                           \
    aglue::qk_rope_pair_kernel<DD, MM, __half><<<g1, aglue::WARPS * 32, 0, st>>>(p)
#define LB2_QK_PAIR(DD)                                                               \
  if (mode == 0)                                                                      \
    aglue::qk_rope_pair_kernel<DD, 0, float><<<g1, aglue::WARPS * 32, 0, st>>>(p);    \
  else if (mode == 1) {                                                               \
    LB2_QK_PAIR_T(DD, 1);                                                             \
  } else {                                                                            \
    LB2_QK_PAIR_T(DD, 2);                                                             \
  }
    if (D == 128) {
      LB2_QK_PAIR(128);
    } else if (D == 256) {
      LB2_QK_PAIR(256);
    } else {
      LB2_QK_PAIR(512);
    }
#undef LB2_QK_PAIR
#undef LB2_QK_PAIR_T
    LB2_CUDA(cudaGetLastError());
    return LB2_OK;
  }
  const dim3 grid(unsigned((int64_t(B) * S + aglue::ROWS - 1) / aglue::ROWS),
                  unsigned((NQ + NK + aglue::WARPS - 1) / aglue::WARPS));
  LB2_CHECK_ARG(grid.y < 65536, "qk_norm_rope: too many heads");
  if (D == 128)
    aglue::qk_norm_rope_kernel<128><<<grid, aglue::WARPS * 32, 0, st>>>(p);
  else if (D == 256)
    aglue::qk_norm_rope_kernel<256><<<grid, aglue::WARPS * 32, 0, st>>>(p);
  else
    aglue::qk_norm_rope_kernel<512><<<grid, aglue::WARPS * 32, 0, st>>>(p);
  LB2_CUDA(cudaGetLastError());
  return LB2_OK;
}

int lb2_attn_out_gate(const void* o, const void* qg, void* out, int64_t rows, int NQ, int D, int dtype, void* stream) {
  LB2_CHECK_ARG(rows >= 0 && NQ > 0, "out_gate: shape");
  LB2_CHECK_ARG(dtype == LB2_BF16, "out_gate: bf16 rows only (the reference's path)");
  LB2_CHECK_ARG(D == 128 || D == 256 || D == 512, "out_gate: head dim 128, 256 or 512");
  LB2_CHECK_ARG(aligned16(o) && aligned16(qg) && aligned16(out), "out_gate: rows 16-byte aligned");
  const int64_t items = rows * NQ;
  if (items == 0) return LB2_OK;
  LB2_CHECK_ARG(rows < (int64_t(1) << 31), "out_gate: too many rows");
  aglue::GateParams p{static_cast<const __nv_bfloat16*>(o), static_cast<const __nv_bfloat16*>(qg),
                      static_cast<__nv_bfloat16*>(out), rows, NQ};
  const dim3 grid(unsigned(rows), unsigned((NQ + aglue::WARPS - 1) / aglue::WARPS));
  LB2_CHECK_ARG(grid.y < 65536, "out_gate: too many heads");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (D == 128)
    aglue::out_gate_kernel<128><<<grid, aglue::WARPS * 32, 0, st>>>(p);
  else if (D == 256)
    aglue::out_gate_kernel<256><<<grid, aglue::WARPS * 32, 0, st>>>(p);
  else
    aglue::out_gate_kernel<512><<<grid, aglue::WARPS * 32, 0, st>>>(p);
  LB2_CUDA(cudaGetLastError());
  return LB2_OK;
}

size_t lb2_qsa_select_workspace_size(int B, int S, int n_blocks) {
  if (B < 0 || S < 0 || n_blocks < 0) return 0;
  return size_t(int64_t(B) * S * n_blocks * int64_t(sizeof(float))) + 256;
}

int lb2_qsa_select(const void* q, const void* pooled, int64_t pool_bstride, int B, int S, int H, int D, int n_blocks,
                   int64_t offset, int cr, int k, float div, void* workspace, size_t workspace_bytes, int32_t* top,
                   void* stream) {
  LB2_CHECK_ARG(B >= 0 && S >= 0 && n_blocks >= 0 && k >= 0, "qsa_select: shape");
  LB2_CHECK_ARG(H >= 1 && H <= 8, "qsa_select: 1 to 8 indexer heads");
  LB2_CHECK_ARG(D == 64 || D == 128, "qsa_select: indexer head dim 64 or 128");
  LB2_CHECK_ARG(cr >= 1 && div > 0.f, "qsa_select: compress ratio and divisor must be positive");
  LB2_CHECK_ARG(int64_t(B) * S < 65536, "qsa_select: at most 65535 query rows a call");
  LB2_CHECK_ARG(pool_bstride >= int64_t(n_blocks) * D, "qsa_select: pooled rows overlap across the batch");
  LB2_CHECK_ARG(aligned16(pooled) && aligned16(q) && pool_bstride % 8 == 0, "qsa_select: q and pooled keys 16-byte aligned");
  LB2_CHECK_ARG(workspace_bytes >= lb2_qsa_select_workspace_size(B, S, n_blocks) && aligned16(workspace),
                "qsa_select: workspace too small or misaligned");
  const int rows = B * S;
  if (rows == 0 || k == 0) return LB2_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  float* scores = static_cast<float*>(workspace);
  if (n_blocks > 0) {
    const int ipr = (n_blocks + qsasel::SC_KEYS - 1) / qsasel::SC_KEYS;
    qsasel::ScoreParams p{static_cast<const __nv_bfloat16*>(q), static_cast<const __nv_bfloat16*>(pooled),
                          pool_bstride, scores, B, S, H, n_blocks, cr, ipr, int64_t(rows) * ipr, offset, div};
    auto kern = D == 128 ? qsasel::score_kernel<128> : qsasel::score_kernel<64>;
    const int smem = D == 128 ? qsasel::sc_smem(128) : qsasel::sc_smem(64);
    // persistent: as many CTAs as are resident at once (cached per device and head dim)
    static int res_dev[2] = {-1, -1}, resident[2] = {0, 0};
    const int di = D == 128 ? 1 : 0;
    int dev = 0;
    LB2_CUDA(cudaGetDevice(&dev));
    if (res_dev[di] != dev) {
      int sms = 0, per_sm = 0;
      LB2_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
      LB2_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
      LB2_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, qsasel::SC_THREADS, smem));
      if (per_sm < 1) return fail(LB2_ECUDA, "qsa_select: the score kernel does not fit an SM");
      resident[di] = sms * per_sm;
      res_dev[di] = dev;
    }
    const int64_t grid = std::min<int64_t>(p.items, resident[di]);
    kern<<<static_cast<unsigned>(grid), qsasel::SC_THREADS, smem, st>>>(p);
    LB2_CUDA(cudaGetLastError());
  }
  // A cluster of CTAs a row: the size topk_cluster picks for the row length, halved while the rows' clusters would
  // not all be resident at once and the halves still hold their scores in registers.
  auto topk_for = [](int per) {
    return per <= 8 ? qsasel::topk_kernel<8> : per <= 16 ? qsasel::topk_kernel<16> : qsasel::topk_kernel<qsasel::TK_PER>;
  };
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(qsasel::TK_THREADS);
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // overlaps the score grid's tail
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  int cl = qsasel::topk_cluster(n_blocks);
  static int fit_dev = -1, fit[4][3];  // resident clusters of (size 1, 2, 4, 8) x (topk_kernel<8>, <16>, <32>)
  int dev = 0;
  LB2_CUDA(cudaGetDevice(&dev));
  if (fit_dev != dev) {
    for (int a = 0; a < 4; ++a)
      for (int b = 0; b < 3; ++b) {
        attr[0].val.clusterDim.x = 1u << a;
        cfg.gridDim = dim3(1u << a);
        cfg.numAttrs = 1;
        LB2_CUDA(cudaOccupancyMaxActiveClusters(&fit[a][b], topk_for(8 << b), &cfg));
      }
    fit_dev = dev;
  }
  auto fits = [&](int c) {
    const int per = qsasel::topk_per(n_blocks, c);
    const int a = c == 1 ? 0 : c == 2 ? 1 : c == 4 ? 2 : 3, b = per <= 8 ? 0 : per <= 16 ? 1 : 2;
    return rows <= fit[a][b];
  };
  while (cl > 1 && !fits(cl) && qsasel::topk_per(n_blocks, cl / 2) <= qsasel::TK_PER) cl /= 2;
  attr[0].val.clusterDim.x = static_cast<unsigned>(cl);
  cfg.gridDim = dim3(static_cast<unsigned>(cl), static_cast<unsigned>(rows));
  cfg.numAttrs = 2;
  LB2_CUDA(cudaLaunchKernelEx(&cfg, topk_for(qsasel::topk_per(n_blocks, cl)), static_cast<const float*>(scores),
                              n_blocks, k, top));
  return LB2_OK;
}

}  // extern "C"
