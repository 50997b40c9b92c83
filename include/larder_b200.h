/* larder_b200: B200 (sm_100a) kernels for Larder's attention / Gated-DeltaNet hot path, behind a plain C ABI.
 *
 * Every entry point takes raw device pointers, element strides (int64, in elements of the tensor's own dtype),
 * shapes, dtype codes and a cudaStream_t passed as void*. Launches are asynchronous on that stream; the return
 * value is a status code (LB2_OK or an error), and lb2_error() gives the calling thread's last message. The caller
 * owns every buffer: outputs and workspaces are allocated by the caller (the Python layer uses torch) and the
 * library never allocates or frees device memory on these paths. Device-side waits are time-bounded; a wait that
 * gives up records itself in a device status word read (and cleared) by lb2_status().
 *
 * Reference interfaces each entry replaces are cited per function (paths within IamCooller/larder).
 */
#ifndef LARDER_B200_H
#define LARDER_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* dtype codes (cpu_ext/cpu_kern.cpp:32's DT enum, same values) */
#define LB2_F32 0
#define LB2_BF16 1
#define LB2_F16 2

/* attention mask kinds (cpu_ext/cpu_kern.cpp:634: 0 none, 1 causal bottom-right, 2 boolean [T, N] array) */
#define LB2_MASK_NONE 0
#define LB2_MASK_CAUSAL 1
#define LB2_MASK_ARRAY 2

/* status codes */
#define LB2_OK 0
#define LB2_EINVAL 1   /* unsupported shape, dtype, stride or alignment */
#define LB2_ECUDA 2    /* a CUDA runtime call or launch failed */
#define LB2_ETIMEOUT 3 /* a bounded device wait gave up (lb2_status) */

/* Version of this ABI; bumped on any signature change. */
int lb2_abi_version(void);

/* The calling thread's last error message ("" when none). Mirrors native/moe_pipe_cuda.cpp:1658-1690's
 * mpc_error(): one message slot, entry points return a status. */
const char* lb2_error(void);

/* Synchronises `stream`, then returns and clears the current device's status word: LB2_OK, or, for the first event
 * since the last call, LB2_ETIMEOUT | (where << 8) when a device wait gave up, LB2_EINVAL | (where << 8) when a
 * kernel skipped an out-of-range index it was given (the KV home's LRU entry points). */
int lb2_status(void* stream);

/* ------------------------------------------------------------------------------------------------------------
 * Prefill / multi-row attention (tcgen05 tensor cores, TMEM accumulators, TMA-staged tiles).
 *
 * o = softmax(scale * q k^T + mask) v, optionally times sigmoid(gate).
 *   q    [B, Hq, T, D]   strides q_st[0..2] for B, H, T; unit stride on D
 *   k, v [B, Hkv, N, D]  strides k_st / v_st; unit stride on D (K/V may be slices of a longer cache buffer)
 *   o    [B, Hq, T, D]   strides o_st
 *   gate [B, Hq, T, D]   strides g_st, or NULL (the gated-attention epilogue of qwen4_exp_vendor.py:397-401:
 *                        out * sigmoid(gate), gate being [B, T, Hq * D] seen through these strides)
 *   mask uint8 [T, N]    strides m_st[0..1], only for LB2_MASK_ARRAY
 * Causal is bottom-right: row t sees keys 0 .. N - T + t. GQA: q head h reads KV head h / (Hq / Hkv).
 * dtype LB2_BF16 or LB2_F16 for q, k, v, o, gate alike; D in {64, 128, 256}; row strides multiples of 8 elements
 * and every base 16-byte aligned (TMA). dtype LB2_F32 (the reference's CPU-runnable fp32 configuration) runs an
 * exact fp32 CUDA-core kernel instead (D in {32, 64, 128, 256}, any strides with a unit last stride).
 * Replaces: the patched scaled_dot_product_attention's prefill route (chunkattn.py:451-537) and each chunk of
 * chunkattn.chunked (chunkattn.py:359-423), qsa_tiles.chunked's array-masked chunk (qsa_tiles.py:266-292), and
 * the stock mx.fast.scaled_dot_product_attention they call (chunkattn.py:419-420). */
int lb2_attn_prefill(const void* q, const int64_t* q_st, const void* k, const int64_t* k_st, const void* v,
                     const int64_t* v_st, void* o, const int64_t* o_st, const void* gate, const int64_t* g_st,
                     const uint8_t* mask, const int64_t* m_st, int B, int Hq, int Hkv, int T, int N, int D, int dtype,
                     float scale, int mask_kind, void* stream);

/* The same prefill for an array mask, with tile skipping: the mask's kept tiles are listed first (for each block of
 * query rows the kernel takes together -- 256 rows on CTA pairs, else 128 -- the key tiles holding a key one of its
 * rows keeps), and the kernel reads only those tiles' K / V and issues only their products. Same result as
 * lb2_attn_prefill with LB2_MASK_ARRAY (every element is still masked as given); the work falls with the mask's
 * tile density. workspace: lb2_attn_prefill_tiled_workspace_size(T, N, D) bytes, 16-byte aligned, any contents.
 * Replaces: qsa_tiles.chunked / tile_chunk (qsa_tiles.py:216-292), which run each 16-row group's products over only
 * the 16-key tiles it keeps. */
size_t lb2_attn_prefill_tiled_workspace_size(int T, int N, int D);
int lb2_attn_prefill_tiled(const void* q, const int64_t* q_st, const void* k, const int64_t* k_st, const void* v,
                           const int64_t* v_st, void* o, const int64_t* o_st, const void* gate, const int64_t* g_st,
                           const uint8_t* mask, const int64_t* m_st, int B, int Hq, int Hkv, int T, int N, int D,
                           int dtype, float scale, void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------------------------------------------
 * Split-KV decode attention (few query rows over a long KV cache; HBM-bandwidth bound).
 *
 * The G*T query rows that share a KV head are folded into one tile (foldattn.py:230-259). A persistent kernel
 * (one CTA an SM) computes fp32 partials (o, max, sum) with an online softmax over key ranges, and a second kernel
 * merges the partials of each (b, kv head) by log-sum-exp (foldattn.py:188-211, cpu_kern.cpp:607-628) and writes o.
 * split = 0: balanced schedule -- the call's 64-key tiles are cut into equal runs, one a CTA, whatever the
 * per-sequence lengths; split > 0: key ranges of `split` keys (rounded up to a multiple of 64, and raised so that a
 * sequence has at most 512 of them) dealt to the CTAs round-robin.
 *   q [B, Hq, T, D], k/v [B, Hkv, N, D] (N = capacity), o [B, Hq, T, D]: strides as in lb2_attn_prefill
 *   kv_len int32 [B] device array of per-sequence key counts (<= N), or NULL for N everywhere
 *   causal: 1 for bottom-right causal over each sequence's own length (T >= 2 verify rows), else 0
 *   workspace: lb2_attn_decode_workspace_size() bytes, 256-byte aligned, any contents (a call writes every
 *   partial it reads). Calls that share a workspace must be ordered on one stream.
 * Limits: G*T <= 32 for D <= 128, G*T <= 16 for D = 256; dtype LB2_BF16 or LB2_F16; D in {64, 128, 256}.
 * dtype LB2_F32 runs the exact fp32 CUDA-core kernel (no workspace used).
 * Replaces: decode SDPA (chunkattn.gqa_sdpa + _gqa_route, chunkattn.py:638-657, :679-696; stream_fast.py's
 * _sdpa_parts / two-pass vector SDPA, :5952-6098), foldattn.fold (foldattn.py:230-259) and the stock decode SDPA
 * attn_cuda calls (stream_fast.py:6439). */
size_t lb2_attn_decode_workspace_size(int B, int Hq, int Hkv, int T, int N, int D, int split);
int lb2_attn_decode(const void* q, const int64_t* q_st, const void* k, const int64_t* k_st, const void* v,
                    const int64_t* v_st, void* o, const int64_t* o_st, const int32_t* kv_len, int B, int Hq, int Hkv,
                    int T, int N, int D, int dtype, float scale, int causal, int split, void* workspace,
                    size_t workspace_bytes, void* stream);

/* The same decode for a caller whose queries and outputs live in host memory (q_host, o_host: contiguous
 * [B, Hq, T, D] of dtype, pinned for the copies to overlap): the call copies q in, decodes on `stream` and copies o
 * out, and returns at once. The copies run on two streams of the library's own (one pair per device, made at the
 * device's first call), through two staging slots in the workspace (lb2_attn_decode_host_workspace_size bytes,
 * 256-byte aligned) used by alternate calls, so that a call's copies overlap the kernels of the calls either side.
 * o_host of every call issued so far is complete once lb2_attn_decode_host_drain(stream) has been called and the
 * stream has reached that point. One caller stream per device at a time (the slots and events are shared). The
 * reference's decode takes arrays wherever MLX keeps them; this is its host-buffer form (stream_fast.py:6411-6441's
 * attn_cuda for a caller that holds q and reads o on the host). */
size_t lb2_attn_decode_host_workspace_size(int B, int Hq, int Hkv, int T, int N, int D, int dtype, int split);
int lb2_attn_decode_host(const void* q_host, const void* k, const int64_t* k_st, const void* v, const int64_t* v_st,
                         void* o_host, const int32_t* kv_len, int B, int Hq, int Hkv, int T, int N, int D, int dtype,
                         float scale, int causal, int split, void* workspace, size_t workspace_bytes, void* stream);
int lb2_attn_decode_host_drain(void* stream);

/* The same decode over this rank's KV range only, emitting the range's normalised partial output and its
 * log-sum-exp instead of the final o: part_o fp32 [B, Hq, T, D] contiguous, part_lse fp32 [B, Hq, T] (natural
 * log; -inf for a row with no visible key). For KV-range shards across GPUs merged by lb2_attn_combine.
 * kv_len / workspace as lb2_attn_decode. Every query row sees every key of the range (decode rows: the range
 * lies wholly before the query position). */
int lb2_attn_decode_partial(const void* q, const int64_t* q_st, const void* k, const int64_t* k_st, const void* v,
                            const int64_t* v_st, float* part_o, float* part_lse, const int32_t* kv_len, int B, int Hq,
                            int Hkv, int T, int N, int D, int dtype, float scale, int split, void* workspace,
                            size_t workspace_bytes, void* stream);

/* Allocation-free variant of lb2_attn_decode, for callers that cannot call cudaMalloc: an engine whose device
 * memory is owned and budgeted by its own allocator (every byte counted against a memory budget, so a library-side
 * allocation would break the budget), or a caller on a latency-critical path where cudaMalloc's implicit device
 * synchronisation is not acceptable. This entry has no counterpart in the reference (whose decode runs inside MLX's
 * allocator); it exists for such callers of this library.
 * Arguments and results as lb2_attn_decode, without the workspace (dtype LB2_F32 runs the exact fp32 kernel, which
 * needs no scratch, exactly as lb2_attn_decode does): the bf16 / f16 split partials live in a
 * file-scope device array of LB2_NOALLOC_SCRATCH_BYTES (8 MiB) that every GPU loading this library holds until the
 * process exits. A call whose workspace (lb2_attn_decode_workspace_size) exceeds that size returns LB2_EINVAL;
 * choose a larger `split` or use lb2_attn_decode. The first call on a device looks up the array's device address
 * (cudaGetSymbolAddress, with that device current); make that first call before any stream capture. It calls no
 * cudaMalloc / cudaFree. All calls share the one array, which keeps the last call's contents (harmless: a call
 * writes every partial it reads before reading it); calls that overlap on the GPU (different streams, or different
 * host threads on one device) race on it and must be ordered by the caller. */
#define LB2_NOALLOC_SCRATCH_BYTES (8u << 20)
int lb2_attn_decode_noalloc(const void* q, const int64_t* q_st, const void* k, const int64_t* k_st, const void* v,
                            const int64_t* v_st, void* o, const int64_t* o_st, const int32_t* kv_len, int B, int Hq,
                            int Hkv, int T, int N, int D, int dtype, float scale, int causal, int split,
                            void* stream);

/* Merges R partials: o[row] = sum_r w_r part_o[r][row] / sum_r w_r, w_r = exp(part_lse[r][row] - max_r lse),
 * rows = B * Hq * T (row-major [B, Hq, T]), o [B, Hq, T, D] with strides o_st in dtype. An all -inf row gives 0.
 * Replaces the LSE merge of foldattn_merge (foldattn.py:188-211) / cpu_kern.cpp:607-628, across ranks. */
int lb2_attn_combine(const float* part_o, const float* part_lse, int R, int B, int Hq, int T, int D, void* o,
                     const int64_t* o_st, int dtype, void* stream);

/* lb2_attn_combine over the buffer an all-gather of packed partials produces: for each of the R ranks, its o rows
 * (rows * D floats) then its lse values (rows floats), the ranks' blocks back to back (rows * (D + 1) floats
 * each). A rank packs its partial in place (lb2_attn_decode_partial into the two parts of one buffer), so the
 * exchange is one all-gather and the merge reads the gathered buffer as it lands, with no copy between. Same
 * merge and reference as lb2_attn_combine. */
int lb2_attn_combine_packed(const float* packed, int R, int B, int Hq, int T, int D, void* o, const int64_t* o_st,
                            int dtype, void* stream);

/* The same exchange over NVLink peer memory instead of a collective (no counterpart in the reference, which is
 * single-GPU: this is the B200 form of the KV-range merge, foldattn.py:188-211 across GPUs). Each rank allocates one
 * exchange buffer (lb2_xch_alloc of lb2_xch_bytes(B, Hq, T, D) bytes, zeroed), exports it (lb2_xch_handle: 64
 * bytes to send to the other ranks) and maps every peer's (lb2_xch_open; lb2_xch_close / lb2_xch_free at the end).
 * Call e = 1, 2, ... of a rank: lb2_attn_decode_partial writes its partial into half e % 2 of its own buffer
 * (part_o at float offset (e % 2) * B Hq T (D + 1), part_lse right after the o rows), then lb2_attn_combine_peers
 * (bufs: host array of the R buffers as mapped in this process, its own at `rank`) publishes e to every peer, waits
 * for every peer's e (bounded: 2 s, then lb2_status reports LB2_ETIMEOUT and o is not written) and merges the R
 * partials read in place over NVLink into o [B, Hq, T, D] (strides o_st). Every rank makes the same calls in the
 * same order; R <= 8 (one NVSwitch node). */
size_t lb2_xch_bytes(int B, int Hq, int T, int D);
int lb2_xch_alloc(size_t bytes, void** ptr);
int lb2_xch_free(void* ptr);
int lb2_xch_handle(void* ptr, void* handle);
int lb2_xch_open(const void* handle, void** ptr);
int lb2_xch_close(void* ptr);
int lb2_attn_combine_peers(const uint64_t* bufs, int R, int rank, uint32_t epoch, int B, int Hq, int T, int D, void* o,
                           const int64_t* o_st, int dtype, void* stream);

/* The same exchange in push form (no counterpart in the reference either): every rank's buffer holds all R partials
 * (lb2_xch_push_bytes(R, B, Hq, T, D) bytes, from lb2_xch_alloc, shared as above). Call e = 1, 2, ... of a rank:
 * lb2_attn_decode_push computes this rank's range partial (o rows in bf16, lse in fp32) and its epilogue stores it
 * straight into slot `rank` of
 * half e % 2 of EVERY rank's buffer (bufs: the R buffers as mapped here; peer stores over NVLink, fenced at system
 * scope); its last block to finish announces e to every rank. lb2_attn_combine_pushed then waits (bounded, 2 s) for
 * every peer's e and merges the R slots of its OWN buffer, so the merge reads local memory only. kv_len / workspace /
 * split as lb2_attn_decode_partial; every call of an exchange has the same shape. */
size_t lb2_xch_push_bytes(int R, int B, int Hq, int T, int D);
int lb2_attn_decode_push(const void* q, const int64_t* q_st, const void* k, const int64_t* k_st, const void* v,
                         const int64_t* v_st, const int32_t* kv_len, int B, int Hq, int Hkv, int T, int N, int D,
                         int dtype, float scale, int split, void* workspace, size_t workspace_bytes,
                         const uint64_t* bufs, int R, int rank, uint32_t epoch, void* stream);
int lb2_attn_combine_pushed(const uint64_t* bufs, int R, int rank, uint32_t epoch, int B, int Hq, int T, int D, void* o,
                            const int64_t* o_st, int dtype, void* stream);

/* ------------------------------------------------------------------------------------------------------------
 * Gated-DeltaNet recurrence, one position at a time (decode steps, short verify passes).
 *
 * For each (b, v head hv, value row dv), over t: s <- s * g_t; kv = s . k_t; delta = (v_t[dv] - kv) * beta_t;
 * s <- s + k_t * delta; y_t[dv] = s . q_t (gdn_cuda.py:18-66). v head hv reads k head hv / (Hv / Hk).
 *   q, k [B, T, Hk, Dk] (qdt), v [B, T, Hv, Dv] (vdt), g [B, T, Hv] or, with g_vec, [B, T, Hv, Dk] (gdt),
 *   beta [B, T, Hv] (bdt), state_in / state_out fp32 [B, Hv, Dv, Dk] (may alias), y [B, T, Hv, Dv] (qdt),
 *   mask uint8 [B, T] or NULL (a masked position writes y = 0 and keeps the state). All contiguous.
 * Dk in {32, 64, 128, 256}; dtypes LB2_F32 / LB2_BF16 / LB2_F16.
 * Replaces: gdn_cuda.recurrence (gdn_cuda.py:88-99) and, with the gating done by the caller, the patched
 * gated_delta_update (gdn_cuda.py:336-353). */
int lb2_gdn_recurrent(const void* q, const void* k, int qdt, const void* v, int vdt, const void* g, int gdt,
                      int g_vec, const void* beta, int bdt, const uint8_t* mask, const float* state_in,
                      float* state_out, void* y, int B, int T, int Hk, int Dk, int Hv, int Dv, void* stream);

/* ------------------------------------------------------------------------------------------------------------
 * Gated-DeltaNet chunked prefill: the same recurrence and result as lb2_gdn_recurrent, computed in chunks of 64
 * positions (intra-chunk products on tensor cores, the chunk's triangular system solved in fp32, the state
 * carried chunk to chunk). Scalar gate only (g [B, T, Hv]), no mask; Dk = Dv = 128; q/k/v bf16 or f16, g f32,
 * beta in q's dtype or f32. workspace: lb2_gdn_chunked_workspace_size() bytes.
 * Replaces: gdn_cuda.recurrence's prefill calls (one launch for all T, gdn_cuda.py:88-99) via the patched
 * gated_delta_update (gdn_cuda.py:336-353). */
size_t lb2_gdn_chunked_workspace_size(int B, int T, int Hk, int Hv, int Dk, int Dv);
int lb2_gdn_chunked(const void* q, const void* k, int qdt, const void* v, int vdt, const void* g, int gdt,
                    const void* beta, int bdt, const float* state_in, float* state_out, void* y, int B, int T, int Hk,
                    int Dk, int Hv, int Dv, void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------------------------------------------
 * QSA decode over picked KV blocks and the paged KV home.
 *
 * Gathers the rows the reference's QSA decode attends to: the sorted picked blocks tb (int32 [nsel], block size cr)
 * and the sequence's trailing partial block; row r < nsel*cr is position tb[r/cr]*cr + r%cr, row r >= nsel*cr is
 * position own0 + r - nsel*cr with own0 = n/cr*cr, m = nsel*cr + n - own0 rows. kg / vg [Hk, m, D] contiguous.
 * k / v: [Hk, n, D] views (one sequence) with strides k_st / v_st (head, position, dim). A picked block reaching
 * outside [0, n) is not read: its rows come back as zeros and lb2_status reports LB2_EINVAL.
 * Replaces: stream_fast._qsa_gather (stream_fast.py:6448-6491); attn_cuda then runs the decode over kg / vg
 * (stream_fast.py:6411-6441), here lb2_attn_decode. */
int lb2_kv_gather_picks(const void* k, const int64_t* k_st, const void* v, const int64_t* v_st, const int32_t* tb,
                        int nsel, int cr, int n, void* kg, void* vg, int Hk, int D, int dtype, void* stream);

/* The QSA decode step with the gather inside the decode: one query row q [1, Hq, 1, D] (strides q_st: batch, head,
 * row) attends to the rows lb2_kv_gather_picks would gather from the [Hk, n, D] views k / v (strides k_st / v_st,
 * multiples of 8 elements, bases 16-byte aligned), read straight from the views by the split-KV decode kernel's
 * threads; o [1, Hq, 1, D] (strides o_st). The result is bit-equal to gather + lb2_attn_decode (split = 0). bf16 / f16,
 * D = 64, 128 or 256; the workspace (256-byte aligned) as lb2_qsa_decode_workspace_size says. A pick reaching
 * outside [0, n) reads row 0 and lb2_status reports LB2_EINVAL.
 * Replaces: stream_fast._qsa_gather + attn_cuda's attention (stream_fast.py:6411-6491). */
size_t lb2_qsa_decode_workspace_size(int nsel, int cr, int n, int Hq, int Hk, int D);
int lb2_qsa_decode(const void* q, const int64_t* q_st, const void* k, const int64_t* k_st, const void* v,
                   const int64_t* v_st, void* o, const int64_t* o_st, const int32_t* tb, int nsel, int cr, int n, int Hq,
                   int Hk, int D, int dtype, float scale, void* workspace, size_t workspace_bytes, void* stream);

/* The paged home: positions in chunks of 2^logc, each chunk [K/V][Hk][2^logc][D] contiguous, chunk addresses in a
 * uint64 device table (device memory or pinned, GPU-mapped host memory; each chunk 16-byte aligned, 2^logc a
 * multiple of cr). put writes s new positions pos0.. of
 * k / v [Hk, s, D] (strides) into the home; gather reads the picked rows (as lb2_kv_gather_picks) from it, with
 * cache-bypassing loads. Replaces: kv_host's layout and its put / gather kernels (kv_host.py:17-18, :36-41,
 * :64-291, decode :612-648); the VRAM LRU in front of it follows. */
int lb2_kvh_put(const uint64_t* table, const void* k, const int64_t* k_st, const void* v, const int64_t* v_st,
                int64_t pos0, int s, int Hk, int D, int dtype, int logc, void* stream);
int lb2_kvh_gather(const uint64_t* table, const int32_t* tb, int nsel, int cr, int n, void* kg, void* vg, int Hk,
                   int D, int dtype, int logc, void* stream);

/* The VRAM LRU in front of the home: a pool of ns slots in device memory, slot x holding one picked block's cr
 * positions [K/V][Hk][cr][D] (pool [ns, 2, Hk, cr, D], the home's dtype), and its int32 device state, owned by the
 * caller: slot_of [max_blocks] (-1 at first), block_of [ns] (-1), stamp [ns] (-1), ref [ns] (0), meta [4] (0:
 * CLOCK hand, token count, hits, misses).
 * plan: one token's picks tb [nsel] (distinct, sorted, 1 <= nsel <= 1024, ns >= ceil32(nsel)) -> sl [nsel]: the
 *   hit's slot, -2 - victim for a miss that takes the CLOCK victim, -1 for a miss read from the home uncached.
 *   Replaces kv_host's plan kernel (kv_host.py:116-185).
 * gather: with sl, the token's QSA rows as lb2_kvh_gather gives them for a sequence of n positions (the new one
 *   included), read from the pool on a hit and from the home otherwise (a miss with a victim fills the victim's
 *   slot), and the new position's row kn / vn [Hk, D] (strides head, dim) written into the home at n - 1 and used
 *   wherever position n - 1 is gathered. Replaces kv_host's gather kernel (kv_host.py:187-257).
 * inval: slots holding a block >= lim drop it (before positions from lim * cr on are rewritten). Replaces kv_host's
 *   inval kernel (kv_host.py:259-276).
 * Out-of-range picks or slots are skipped (zeros in their rows) and reported through lb2_status. */
int lb2_kvh_lru_plan(const int32_t* tb, int nsel, int32_t* slot_of, int max_blocks, int32_t* block_of, int32_t* stamp,
                     int32_t* ref, int32_t* meta, int ns, int32_t* sl, void* stream);
int lb2_kvh_lru_gather(const uint64_t* table, void* pool, int ns, const int32_t* tb, const int32_t* sl, int nsel, int cr,
                       int n, const void* kn, const int64_t* kn_st, const void* vn, const int64_t* vn_st, void* kg,
                       void* vg, int Hk, int D, int dtype, int logc, void* stream);
int lb2_kvh_lru_inval(int32_t* slot_of, int32_t* block_of, int32_t* ref, int ns, int lim, void* stream);

/* ------------------------------------------------------------------------------------------------------------
 * Gated-DeltaNet decode-row glue.
 *
 * step_glue: NR positions of one sequence from the conv output before silu, conv [NR, 2 Hk Dk + Hv Dv] (dtype), a / b
 * [NR, Hv] (dtype), A_log / dt_bias [Hv] fp32, state [Hv, Dv, Dk] fp32 (in / out may alias) -> y [NR, Hv, Dv]
 * (dtype): silu, q / k RMSNorm (eps) scaled by sq / sk (the 16-bit-rounded Dk^-1 and Dk^-0.5), sigmoid(b),
 * compute_g and one recurrence step a position. Dk in {64, 128}. Replaces gdn_cuda.step_glue (gdn_cuda.py:118-198,
 * :235-254).
 * norm_gate: out = silu(z) * (w * rms_norm(x)), rows of D elements. Replaces gdn_cuda.norm_gate
 * (gdn_cuda.py:200-222, :257-268). */
int lb2_gdn_step_glue(const void* conv, const void* a, const void* b, const float* A_log, const float* dt_bias,
                      const float* state_in, float* state_out, void* y, int NR, int Hk, int Dk, int Hv, int Dv,
                      int dtype, float sq, float sk, float eps, void* stream);
int lb2_gdn_norm_gate(const void* x, const void* z, const void* w, void* out, int64_t R, int D, int dtype, float eps,
                      void* stream);

/* ------------------------------------------------------------------------------------------------------------
 * The attention layer's glue on either side of the SDPA (bf16 rows).
 *
 * q / k RMSNorm + rotate-half RoPE: for each row (b, s) and each of the NQ query and NK key heads, x = the head's D
 * values (query head h: columns [2hD, 2hD + D) of q_proj's output qg [B, S, NQ * 2D], whose other half is the output
 * gate; key head h: columns [hD, hD + D) of k_proj's output kr [B, S, NK * D]):
 *   inv = 1 / sqrt(sum(x^2) / D + eps) (fp32), o_j = bf16(w_j * bf16(x_j * inv)),
 *   j < R: r_j = bf16(bf16(o_j * bf16(cos_j)) + bf16(rot_j * bf16(sin_j))), rot_j = -o_{j+R/2} (j < R/2) else
 *   o_{j-R/2}; j >= R: r_j = o_j,
 * into q [B, NQ, S, D] and k [B, NK, S, D]. cos / sin [S, R] contiguous, cs_dtype LB2_F32 / BF16 / F16; norm weights
 * [D] bf16. D in {128, 256, 512}, R even and <= D. Rows, outputs and weights 16-byte aligned, contiguous.
 * Replaces: the qk kernel of layer_glue.py:241-286 as attn_step calls it (layer_glue.py:592-597). */
int lb2_attn_qk_norm_rope(const void* qg, const void* kr, const void* q_norm_w, const void* k_norm_w, float eps,
                          const void* cos, const void* sin, int cs_dtype, void* q, void* k, int B, int S, int NQ,
                          int NK, int D, int R, int dtype, void* stream);

/* Output gate: out[r, hD + j] = bf16(o[r, hD + j] * bf16(sigmoid(qg[r, 2hD + D + j]))) over `rows` rows of NQ heads
 * (o, out [rows, NQ * D], qg [rows, NQ * 2D], bf16, contiguous, 16-byte aligned; out may be o).
 * Replaces: the agate kernel of layer_glue.py:288-296 (attn_step, layer_glue.py:614-617), whose sigmoid is a
 * table of bf16(sigmoid(x)) for every bf16 pattern x. */
int lb2_attn_out_gate(const void* o, const void* qg, void* out, int64_t rows, int NQ, int D, int dtype, void* stream);

/* ------------------------------------------------------------------------------------------------------------
 * QSA indexer block selection: the top-k part of the indexer (qwen4_exp_vendor.py:271-292, stream_fast.py's
 * `select`, :6243-6305), given its normalised and rotated q [B, S, H, D] and pooled block keys [B, ., D] (bf16,
 * batch stride pool_bstride elements, rows 0 .. n_blocks - 1 used). For each row (b, s) at position offset + s:
 *   score_n = sum_h max(q_h . pooled_n, 0) / div (fp32; the reference divides by sqrt(head_dim)),
 *   -inf for n >= (offset + s + 1) / cr (blocks not yet complete),
 * and top [B, S, k] int32: the indices of the k largest finite scores in ascending order (the order `tb` takes in
 * stream_fast.py:6478-6491), ties at the threshold lowest index first (the reference's argpartition leaves ties
 * unspecified), padded with n_blocks where fewer than k blocks are candidates (the reference's
 * where(picked, top, n_blocks)). The workspace (lb2_qsa_select_workspace_size) holds each row's scores after the
 * call, [B * S, n_blocks] fp32. H <= 8, D in {64, 128}, B * S < 65536. */
size_t lb2_qsa_select_workspace_size(int B, int S, int n_blocks);
int lb2_qsa_select(const void* q, const void* pooled, int64_t pool_bstride, int B, int S, int H, int D, int n_blocks,
                   int64_t offset, int cr, int k, float div, void* workspace, size_t workspace_bytes, int32_t* top,
                   void* stream);

#ifdef __cplusplus
}
#endif

#endif /* LARDER_B200_H */
