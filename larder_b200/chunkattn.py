"""Chunked / wide-cut causal prefill attention and the patched scaled_dot_product_attention, on B200.

The drop-in for the reference's chunkattn.py surface: `chunked`, `install`, `calibrate`, `prefill_attn_slope`,
`layout` and `_wrap` keep their names, arguments and meaning (chunkattn.py:250-304, :318-423, :428-537,
:1087-1176); the computation is this package's CUDA kernels.

What changes on B200: the prefill kernel (lb2_attn_prefill, tcgen05 tensor cores with TMEM accumulators) is a
fused flash-style kernel, so no [Hq, T, N] score buffer ever exists and query-row chunking is a scheduling choice,
not a memory bound. The reference cuts the rows only to bound MLX's score buffer (chunkattn.py:359-405: "same
result as" one causal SDPA); `chunked()` here runs all T rows as ONE launch, whose row tiles are ordered heaviest
first across the whole pass, so no chunk leaves its own partial last wave. Each row still reads the keys its causal
horizon allows, in the same 64-key tiles and the same order as a chunk-by-chunk cut would, so the result is the
same. `_bounds` and `_cut` keep the reference's arithmetic for callers that use them to size things.
Few-row calls (decode, verify passes) go to the split-KV decode kernel instead (lb2_attn_decode).

There is no stock fallback: an unsupported call (attention sinks, a quantised cache, an additive mask, fp32 on the
tensor-core path) raises instead of silently running another implementation.
"""
import torch

from . import ops

LOOPED = 4096     # the reference's softmax switch (chunkattn.py:307); kept for _cut's arithmetic
KEY_ALIGN = 64    # the reference's cut alignment (chunkattn.py:311)
ROW_CANDIDATES = (5, 8, 16, 32, 64, 128, 256)

# (Hq, Hkv, D) -> (per_key_bytes, min_rows, key_floor), as the reference's table; calibrate() fills it.
layout = {}
# The kernel entry array-masked prefills take: None for ops.attn_prefill (looked up at each call), or
# ops.attn_prefill_tiled (tile skipping) once qsa_tiles.install has rebound it (the reference's qsa_tiles.install
# rebinds `chunked` the same way).
array_prefill = None


def _cut(nk, n, floor):
    """Keys a chunk whose last row sees `nk` of `n` takes under the reference's rounding (chunkattn.py:318-322):
    at least `floor` when n reaches it, rounded up to KEY_ALIGN, at most n."""
    if n >= floor:
        nk = max(nk, floor)
    return min(n, -(-nk // KEY_ALIGN) * KEY_ALIGN)


def _bounds(T, rows, min_rows):
    """Chunk edges over T rows: `rows` apart, a last chunk under min_rows folded into the one before
    (chunkattn.py:350-356)."""
    rows = max(rows, min_rows)
    bounds = list(range(0, T, rows)) + [T]
    if len(bounds) > 2 and bounds[-1] - bounds[-2] < min_rows:
        bounds.pop(-2)
    return bounds


def chunked(q, k, v, scale, rows, min_rows, floor=0, mask=None, fused=False, gate=None):
    """Causal SDPA of q's T rows, the last T of k/v's N positions (row r sees keys 0 .. N - T + r), the result of
    the reference's row-chunked pass (chunkattn.py:359-423) in one launch. `rows`, `min_rows` and `floor` are the
    reference's chunking knobs (kept for its signature; here they change no result and no work). `mask`: a bool
    [..., T, N] array instead of the causal rule. `fused` is accepted for the reference's signature (the kernel is
    fused). `gate` ([B, Hq, T, D] view, optional): the output is multiplied by sigmoid(gate) inside the kernel.
    Returns [B, Hq, T, D] in q's dtype."""
    B, Hq, T, D = q.shape
    N = k.shape[2]
    out = torch.empty((B, Hq, T, D), dtype=q.dtype, device=q.device)
    if mask is None:
        return ops.attn_prefill(q, k, v, scale, "causal", gate=gate, out=out)
    return (array_prefill or ops.attn_prefill)(q, k, v, scale, mask.reshape(T, N), gate=gate, out=out)


def _arr_mask(mask, T, N):
    """A boolean [1?, 1?, T, N] mask, the one array mask the kernels take (chunkattn.py:431-434)."""
    return (isinstance(mask, torch.Tensor) and mask.dtype == torch.bool and mask.dim() >= 2
            and tuple(mask.shape[-2:]) == (T, N) and all(d == 1 for d in mask.shape[:-2]))


def attend(queries, keys, values, scale, mask=None):
    """One attention call routed to the kernel that fits it: few query rows with no mask or the causal rule go to
    the split-KV decode kernel, everything else to the tensor-core prefill kernel."""
    B, Hq, T, D = queries.shape
    Hkv, N = keys.shape[1], keys.shape[2]
    if Hq % Hkv:
        raise ValueError("attention: Hq must be a multiple of Hkv")
    causal = isinstance(mask, str) and mask == "causal"
    if isinstance(mask, str) and not causal:
        raise ValueError(f"attention: unsupported mask {mask!r}")
    if mask is not None and not causal and not _arr_mask(mask, T, N):
        raise ValueError("attention: only 'causal' or a boolean [..., T, N] mask with leading dims of 1")
    few = (Hq // Hkv) * T <= ops.decode_rows_limit(D)
    if few and (mask is None or causal):
        return ops.attn_decode(queries, keys, values, scale, causal=causal and T > 1)
    if mask is not None and not causal:
        return (array_prefill or ops.attn_prefill)(queries, keys, values, scale, mask)
    return ops.attn_prefill(queries, keys, values, scale, mask)


def _wrap(stock):
    """The patched module-level scaled_dot_product_attention (chunkattn.py:451-537's signature). `stock` is kept as
    the `.stock` marker the reference's patchers share; it is never called (no fallback)."""

    def scaled_dot_product_attention(queries, keys, values, cache, scale, mask, sinks=None):
        if sinks is not None:
            raise NotImplementedError("scaled_dot_product_attention: attention sinks are not on this path")
        if hasattr(cache, "bits"):
            raise NotImplementedError("scaled_dot_product_attention: quantised KV caches are not on this path")
        return attend(queries, keys, values, scale, mask)

    scaled_dot_product_attention.stock = stock
    scaled_dot_product_attention.chunkattn = True
    return scaled_dot_product_attention


def calibrate(shapes, dtype=torch.bfloat16, verbose=False):
    """{(Hq, Hkv, D): (per_key_bytes, min_rows, key_floor)} for every shape the kernels take. The fused kernel
    holds no per-(row, key) buffer (per_key_bytes 0), is exact at any chunk width (min_rows 1) and needs no key
    floor (0); shapes outside the kernels' envelope (D not in {64, 128, 256}, Hq % Hkv) are left out, as the
    reference leaves shapes it cannot serve (chunkattn.py:1087-1122)."""
    out = {}
    for hq, hkv, d in sorted(shapes):
        if hq % hkv or d not in (64, 128, 256) or dtype not in (torch.bfloat16, torch.float16):
            if verbose:
                print(f"  chunkattn {hq}/{hkv}x{d}: outside the kernels' envelope")
            continue
        out[(hq, hkv, d)] = (0.0, 1, 0)
    return out


def prefill_attn_slope(model=None, dtype=None, sdpa_rows=0):
    """Bytes one layer's prefill attention holds per (row, key), per row and per key: all zero, since the fused
    kernel materialises no scores -- the reference's answer for a fused shape (chunkattn.py:250-304)."""
    return (0.0, 0.0, 0.0, 0.0, 0)


def _heads(m):
    if hasattr(m, "n_heads") and hasattr(m, "n_kv_heads"):
        return m.n_heads, m.n_kv_heads
    if hasattr(m, "num_attention_heads") and hasattr(m, "num_key_value_heads"):
        return m.num_attention_heads, m.num_key_value_heads
    return None


def _attention_modules(model):
    """The python modules whose attention calls the shared sdpa helper and the (Hq, Hkv, D) of every attention
    layer found (chunkattn.py's _attention_modules: module attributes looked up at call time)."""
    import sys
    mods, shapes = set(), set()
    modules = model.modules() if hasattr(model, "modules") else [model]
    for m in modules:
        mod = sys.modules.get(type(m).__module__)
        if mod is not None and hasattr(mod, "scaled_dot_product_attention"):
            mods.add(mod)
        heads = _heads(m)
        if heads is not None and hasattr(m, "scale"):
            shapes.add((heads[0], heads[1], round(m.scale ** -2)))
    return mods, shapes


def install(model, table=None, verbose=False):
    """Rebind `scaled_dot_product_attention` in the modules of the model's attention layers to this package's
    kernels (chunkattn.py:1132-1176), composing with another patcher's wrapper by testing this module's own
    `.chunkattn` marker. Returns the installed table."""
    global layout
    mods, shapes = _attention_modules(model)
    if table is None:
        table = calibrate(shapes, verbose=verbose)
    for mod in mods:
        if not hasattr(mod.scaled_dot_product_attention, "chunkattn"):
            mod.scaled_dot_product_attention = _wrap(mod.scaled_dot_product_attention)
    layout = table
    return table
