"""The attention layer's glue around the SDPA, as layer_glue.attn_step (layer_glue.py:578-619) runs it: q / k RMSNorm
and rotate-half RoPE in one kernel before the cache update and the SDPA, and the output gate after it. The model
around them (projections, the indexer, the cache object) is the caller's; these are the two kernels attn_step calls
(`_kern(("qk",))`, layer_glue.py:592-597, and `_kern(("agate",))`, :614-617), on CUDA tensors. bf16 only, as the
reference's path (attn_eligible, layer_glue.py:571-576, admits bf16 norm weights only).
"""
import torch

from . import ops
from ._lib import check, lib


def attn_eligible(head_dim, q_norm_weight, k_norm_weight, rope_dims):
    """The shapes the kernels take: head dim 128, 256 or 512, bf16 [head_dim] norm weights, an even rope width no
    wider than the head (the reference's own checks: layer_glue.py:571-576, :590-591)."""
    return (head_dim in (128, 256, 512) and rope_dims % 2 == 0 and 0 <= rope_dims <= head_dim
            and all(w.dtype == torch.bfloat16 and tuple(w.shape) == (head_dim,) for w in (q_norm_weight, k_norm_weight)))


def qk_norm_rope(qg, kr, q_norm_weight, k_norm_weight, eps, cos, sin, n_heads, n_kv_heads):
    """q, k = the reference's qk kernel (layer_glue.py:241-286):

    qg [B, S, n_heads * 2 D] is q_proj's output (each head's D query values, then its D gate values), kr
    [B, S, n_kv_heads * D] k_proj's; each head row is RMS-normalised (fp32 sum of squares, bf16 roundings as the
    reference), scaled by its norm weight and rotated over its first R = cos.shape[-1] dims (rotate-half RoPE with
    cos / sin [S, R] of the rows' positions). Returns q [B, n_heads, S, D] and k [B, n_kv_heads, S, D], the layout
    the cache update and the SDPA take."""
    ops._cuda(qg, kr, q_norm_weight, k_norm_weight, cos, sin)
    if qg.dtype != torch.bfloat16 or kr.dtype != torch.bfloat16:
        raise ValueError("qk_norm_rope: bf16 rows only")
    B, S = qg.shape[0], qg.shape[1]
    D = qg.shape[-1] // (2 * n_heads)
    if qg.shape[-1] != 2 * n_heads * D or kr.shape[:2] != qg.shape[:2] or kr.shape[-1] != n_kv_heads * D:
        raise ValueError("qk_norm_rope: qg must be [B, S, n_heads * 2D] and kr [B, S, n_kv_heads * D]")
    R = cos.shape[-1]
    if cos.numel() != S * R or sin.numel() != S * R or sin.shape[-1] != R or cos.dtype != sin.dtype:
        raise ValueError("qk_norm_rope: cos / sin must both be [S, R] of one dtype")
    cos, sin = cos.reshape(S, R), sin.reshape(S, R)
    if not attn_eligible(D, q_norm_weight, k_norm_weight, R):
        raise ValueError(f"qk_norm_rope: head dim {D} with rope dims {R} and these norm weights is not supported")
    qg, kr, cos, sin = qg.contiguous(), kr.contiguous(), cos.contiguous(), sin.contiguous()
    q = torch.empty((B, n_heads, S, D), dtype=torch.bfloat16, device=qg.device)
    k = torch.empty((B, n_kv_heads, S, D), dtype=torch.bfloat16, device=qg.device)
    rc = lib().lb2_attn_qk_norm_rope(ops._ptr(qg), ops._ptr(kr), ops._ptr(q_norm_weight.contiguous()),
                                     ops._ptr(k_norm_weight.contiguous()), float(eps), ops._ptr(cos), ops._ptr(sin),
                                     ops.dtype_code(cos), ops._ptr(q), ops._ptr(k), B, S, n_heads, n_kv_heads, D, R,
                                     ops.dtype_code(qg), ops._stream(qg))
    check(rc, "qk_norm_rope")
    return q, k


def out_gate(out, qg, n_heads, result=None):
    """The reference's agate kernel (layer_glue.py:288-296): out [B, S, n_heads * D] (the SDPA's output, heads
    interleaved per row) times the bf16 sigmoid of each head's gate half of qg [B, S, n_heads * 2D], rounded to bf16.
    `result` (default a new tensor) may be `out` itself."""
    ops._cuda(out, qg)
    if out.dtype != torch.bfloat16 or qg.dtype != torch.bfloat16:
        raise ValueError("out_gate: bf16 rows only")
    D = out.shape[-1] // n_heads
    rows = out.numel() // (n_heads * D)
    if out.shape[-1] != n_heads * D or qg.shape[-1] != 2 * n_heads * D or qg.numel() != 2 * out.numel():
        raise ValueError("out_gate: out must be [..., n_heads * D] and qg [..., n_heads * 2D] over the same rows")
    if not (out.is_contiguous() and qg.is_contiguous()):
        raise ValueError("out_gate: out and qg must be contiguous")
    if result is None:
        result = torch.empty_like(out)
    elif result.shape != out.shape or result.dtype != out.dtype or not result.is_contiguous():
        raise ValueError("out_gate: result must match out")
    rc = lib().lb2_attn_out_gate(ops._ptr(out), ops._ptr(qg), ops._ptr(result), rows, n_heads, D, ops.dtype_code(out),
                                 ops._stream(out))
    check(rc, "out_gate")
    return result


__all__ = ["attn_eligible", "qk_norm_rope", "out_gate"]
