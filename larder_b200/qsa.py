"""QSA decode over picked KV blocks on B200: the indexer's block selection (the top-k of stream_fast.py's `select`,
:6243-6305, qwen4_exp_vendor.py:271-292), and the drop-in for stream_fast.py's `_qsa_gather` and the attention of
`attn_cuda` (stream_fast.py:6411-6491).

The reference's Flash-Next decode (B = 1, T = 1) attends only to the blocks its indexer picked -- sorted block ids
`tb` (int32) of `cr` positions each -- plus the sequence's trailing partial block. `qsa_gather` copies exactly those
rows, in that order, out of the cache views (a bit-exact gather); `qsa_attend` runs the split-KV decode kernel over
them, as attn_cuda runs SDPA over the gathered rows.
"""
import math

import torch

from . import ops
from ._lib import check, lib


def qsa_select(q, pooled, offset, cr, k, n_blocks=None, div=None, scores_out=False):
    """The indexer's block picks for query rows q [B, S, H, D] (already q_layernorm'd and rotated, as
    qwen4_exp_vendor.py:279-281 leaves them) over pooled block keys [B, >= n_blocks, D] (k_layernorm'd and rotated,
    :267-273), the rows at positions offset .. offset + S - 1: score_n = sum_h relu(q_h . pooled_n) / div (div =
    sqrt(D) as the reference), blocks not yet complete at a row ((pos + 1) // cr <= n) excluded, the k best.
    Returns top int32 [B, S, k] in ascending order (ties lowest index first), padded with n_blocks where a row has
    fewer than k candidate blocks; with scores_out, also the fp32 scores [B, S, n_blocks] (-inf for excluded blocks).
    """
    ops._cuda(q, pooled)
    if q.dtype != torch.bfloat16 or pooled.dtype != torch.bfloat16:
        raise ValueError("qsa_select: bf16 q and pooled keys (the indexer's dtype)")
    B, S, H, D = q.shape
    n_blocks = pooled.shape[1] if n_blocks is None else int(n_blocks)
    if pooled.shape[0] != B or pooled.shape[2] != D or n_blocks > pooled.shape[1]:
        raise ValueError("qsa_select: pooled must be [B, >= n_blocks, D] matching q")
    if pooled.stride(2) != 1 or pooled.stride(1) != D:
        raise ValueError("qsa_select: pooled rows must be contiguous")
    q = q.contiguous()
    div = math.sqrt(D) if div is None else float(div)
    top = torch.empty((B, S, k), dtype=torch.int32, device=q.device)
    ws = ops.workspace(q.device, lib().lb2_qsa_select_workspace_size(B, S, n_blocks), "qsa_select")
    rc = lib().lb2_qsa_select(ops._ptr(q), ops._ptr(pooled), pooled.stride(0), B, S, H, D, n_blocks, int(offset),
                              int(cr), int(k), div, ops._ptr(ws), ws.numel(), ops._ptr(top), ops._stream(q))
    check(rc, "qsa_select")
    if scores_out:
        scores = ws[:B * S * n_blocks * 4].view(torch.float32).view(B, S, n_blocks).clone()
        return top, scores
    return top


def qsa_gather(k, v, tb, cr):
    """K and V [1, Hk, m, D] of the sorted picked blocks tb and the trailing partial block of the cache views k, v
    [1, Hk, n, D] (stream_fast.py:6481-6491)."""
    return ops.kv_gather_picks(k, v, tb.to(torch.int32), cr)


def qsa_attend(q, k, v, tb, cr, scale):
    """attn_cuda's attention for one decode row: q [1, Hq, 1, D] over the picks of k, v [1, Hk, n, D]: the gather
    kernel, then the split-KV decode over the gathered rows. (ops.qsa_decode reads the picks in place inside the
    decode kernel, bit-equal; at Flash-Next's decode shapes it is the slower of the two, 16.1 against 14.6 us.)"""
    kg, vg = qsa_gather(k, v, tb, cr)
    return ops.attn_decode(q, kg, vg, scale)
