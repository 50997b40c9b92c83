"""Folded GQA multi-row attention on B200: the drop-in for the reference's foldattn.py surface (`fold`, `install`,
`layout`, foldattn.py:230-259, :268-402).

fold(q, k, v, scale, chunks): causal (bottom-right) GQA attention of q [B, Hq, T, D] against k, v [B, Hkv, N, D],
the last T of the N positions being q's own. As in the reference, the G*T query rows that share a KV head are folded
into one tile so each K/V element is read once per call, and the keys are split into `chunks` ranges whose fp32
partials are merged by log-sum-exp. Here that is the split-KV decode kernel (lb2_attn_decode, causal), with the
chunk count turned into a split length (a multiple of 64 keys).
"""
import torch

from . import ops
from .chunkattn import _heads

MAX_ROWS = 8           # the reference's verify-pass envelope (foldattn.py:19)
CHUNKS = (4, 8, 16, 32)

# (Hq, Hkv, D, T, floor(log2 N)) -> chunks, as the reference's routing table.
layout = {}


def fold(q, k, v, scale, chunks):
    """Causal GQA attention of few query rows over a long KV cache, the keys split into `chunks` ranges."""
    N = k.shape[2]
    per = -(-N // max(1, int(chunks)))   # keys a chunk
    split = max(64, -(-per // 64) * 64)  # rounded up to whole 64-key tiles
    return ops.attn_decode(q, k, v, scale, causal=True, split=split)


def _route(q, k, cache, mask, sinks):
    T = q.shape[2]
    if (T < 2 or T > MAX_ROWS or sinks is not None or hasattr(cache, "bits") or not isinstance(mask, str)
            or mask != "causal" or q.dtype not in (torch.bfloat16, torch.float16) or k.dtype != q.dtype
            or q.shape[1] % k.shape[1] or (q.shape[1] // k.shape[1]) * T > ops.decode_rows_limit(q.shape[3])):
        return None
    return layout.get((q.shape[1], k.shape[1], q.shape[3], T, k.shape[2].bit_length() - 1), 16)


def _wrap(stock):
    """The patched scaled_dot_product_attention for verify passes; calls outside fold's envelope go to `stock`,
    which is another wrapper of this package (chunkattn's), never a CPU path."""
    def scaled_dot_product_attention(queries, keys, values, cache, scale, mask, sinks=None):
        chunks = _route(queries, keys, cache, mask, sinks)
        if chunks is None:
            return stock(queries, keys, values, cache=cache, scale=scale, mask=mask, sinks=sinks)
        return fold(queries, keys, values, scale, chunks)

    scaled_dot_product_attention.stock = stock
    scaled_dot_product_attention.foldattn = True
    return scaled_dot_product_attention


def calibrate(shapes, layers=1, dtype=torch.bfloat16, rows=range(2, MAX_ROWS + 1), buckets=range(4, 16)):
    """{(Hq, Hkv, D, T, log2 N): chunks}: every (T, bucket) the folded kernel takes, with about one split a 1024
    keys (at least 4, at most 32 chunks)."""
    out = {}
    for hq, hkv, d in sorted(shapes):
        for T in rows:
            if hq % hkv or (hq // hkv) * T > ops.decode_rows_limit(d):
                continue
            for b in buckets:
                out[(hq, hkv, d, T, b)] = min(32, max(4, (1 << b) // 1024))
    return out


def install(model, table=None, verbose=False):
    """Route the model's multi-row causal attention through fold (foldattn.py:372-402), composing with chunkattn's
    wrapper by testing this module's own `.foldattn` marker."""
    global layout
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
    if table is None:
        table = calibrate(shapes)
    for mod in mods:
        if not hasattr(mod.scaled_dot_product_attention, "foldattn"):
            mod.scaled_dot_product_attention = _wrap(mod.scaled_dot_product_attention)
    layout = table
    return table
