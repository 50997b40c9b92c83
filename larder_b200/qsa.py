"""QSA decode over picked KV blocks on B200: the drop-in for stream_fast.py's `_qsa_gather` and the attention of
`attn_cuda` (stream_fast.py:6411-6491).

The reference's Flash-Next decode (B = 1, T = 1) attends only to the blocks its indexer picked -- sorted block ids
`tb` (int32) of `cr` positions each -- plus the sequence's trailing partial block. `qsa_gather` copies exactly those
rows, in that order, out of the cache views (a bit-exact gather); `qsa_attend` runs the split-KV decode kernel over
them, as attn_cuda runs SDPA over the gathered rows.
"""
import torch

from . import ops


def qsa_gather(k, v, tb, cr):
    """K and V [1, Hk, m, D] of the sorted picked blocks tb and the trailing partial block of the cache views k, v
    [1, Hk, n, D] (stream_fast.py:6481-6491)."""
    return ops.kv_gather_picks(k, v, tb.to(torch.int32), cr)


def qsa_attend(q, k, v, tb, cr, scale):
    """attn_cuda's attention for one decode row: q [1, Hq, 1, D] over the picks of k, v [1, Hk, n, D]."""
    kg, vg = qsa_gather(k, v, tb, cr)
    return ops.attn_decode(q, kg, vg, scale)
