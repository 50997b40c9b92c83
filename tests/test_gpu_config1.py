"""BASELINE configs[0] on the GPU: the CPU-runnable single attention layer (Qwen1.5-MoE-A2.7B shape), fp32.
Batch 1, 16 query = 16 KV heads x 128, q/k/v ~ N(0,1) from a seed, scale 1/sqrt(128): a 512-token causal prefill
in chunks of 128 (chunk c: rows 128c .. 128c + 127 over keys 0 .. 128(c+1) - 1), then one decode token whose own K/V
is appended first (mlx_lm's update_and_fetch precedes the SDPA, qwen4_exp_vendor.py:377-378), so it attends over 513
keys. Compared elementwise with the reference's fp32 bar (|got - ref| <= 1e-5 max|ref|, tests/test_cpu_kern.py:167)
against the float64 reference, and with the f32 oracle."""
import numpy as np
import pytest
import torch

import checks
import oracle
from larder_b200 import chunkattn, ops

pytestmark = pytest.mark.gpu


def test_config1_fp32_prefill_chunks_then_decode():
    rng = np.random.default_rng(0)
    H, D, T = 16, 128, 512
    x = rng.normal(0, 1, (3, 1, H, T + 1, D)).astype(np.float32)
    q, k, v = (torch.from_numpy(a).cuda() for a in x)
    scale = D ** -0.5
    outs = []
    for c in range(4):
        r0, r1 = 128 * c, 128 * (c + 1)
        outs.append(ops.attn_prefill(q[:, :, r0:r1], k[:, :, :r1], v[:, :, :r1], scale, "causal"))
    pre = torch.cat(outs, dim=2).cpu().numpy()
    ref = oracle.attn_ref64(x[0][:, :, :T], x[1][:, :, :T], x[2][:, :, :T], scale, oracle.causal_mask(T, T))
    checks.attn_close(pre, ref, oracle.F32, "prefill chunks")
    # the chunked drop-in gives the same
    pre2 = chunkattn.chunked(q[:, :, :T], k[:, :, :T], v[:, :, :T], scale, 128, 128).cpu().numpy()
    checks.attn_close(pre2, ref, oracle.F32, "chunkattn.chunked")
    # decode token 513 over all 513 keys (its own K/V appended first)
    dec = ops.attn_decode(q[:, :, T:T + 1], k, v, scale).cpu().numpy()
    ref_d = oracle.attn_ref64(x[0][:, :, T:T + 1], x[1], x[2], scale)
    checks.attn_close(dec, ref_d, oracle.F32, "decode")
    orc = oracle.attn(x[0][:, :, T:T + 1], x[1], x[2], scale, oracle.F32)
    assert np.abs(dec - orc).max() <= 1e-5 * np.abs(orc).max()
