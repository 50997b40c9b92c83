"""The drop-in modules on the GPU, against the CPU oracle: chunkattn.chunked (the 2048-row wide cut, scaled down),
the patched scaled_dot_product_attention for decode and prefill calls, foldattn.fold for verify rows, and
gdn_cuda.gated_delta_update with its gating. Bar: max-abs 2e-2 and cosine >= 0.9999 of the f32 oracle."""
import numpy as np
import pytest
import torch

import checks
import oracle
from gpu_util import f32, to_np
from larder_b200 import chunkattn, foldattn, gdn_cuda, ops

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _status_clean():
    yield
    assert ops.status() == 0, "a device wait gave up"


def oref(q, k, v, scale, kind=oracle.MASK_NONE, mask=None):
    dt = oracle.BF16 if q.dtype == torch.bfloat16 else oracle.F16
    m = None if mask is None else mask.cpu().numpy()
    return oracle.attn(to_np(q), to_np(k), to_np(v), scale, dt, kind, m, out_dt=oracle.F32)


def rnd(g, *shape):
    return torch.randn(*shape, generator=g).to(torch.bfloat16).cuda()


def test_chunked_wide_cut_equals_whole_causal():
    """The layer-major wide cut (stream_fast.py:7285, LM_W) at a quarter scale: T = N = 2048 in 512-row chunks, 16/2
    heads x 256, with the sigmoid gate fused; equal to the oracle and bit-equal to one whole causal call."""
    g = torch.Generator().manual_seed(71)
    B, Hq, Hkv, D, T = 1, 16, 2, 256, 2048
    q = rnd(g, B, T, Hq, D).transpose(1, 2)
    k, v = rnd(g, B, Hkv, T, D), rnd(g, B, Hkv, T, D)
    gate = rnd(g, B, T, Hq * D).view(B, T, Hq, D).transpose(1, 2)
    out = f32(chunkattn.chunked(q, k, v, D ** -0.5, 512, 128, gate=gate))
    ref = oref(q, k, v, D ** -0.5, oracle.MASK_CAUSAL) * (1 / (1 + np.exp(-f32(gate))))
    checks.grading_close(out, ref, what="wide cut")
    whole = f32(ops.attn_prefill(q, k, v, D ** -0.5, "causal", gate=gate))
    assert np.array_equal(out, whole)


def test_chunked_array_mask():
    g = torch.Generator().manual_seed(72)
    B, Hq, Hkv, D, T, N = 1, 8, 2, 128, 300, 900
    q, k, v = rnd(g, B, Hq, T, D), rnd(g, B, Hkv, N, D), rnd(g, B, Hkv, N, D)
    causal = torch.arange(T)[:, None] + N - T >= torch.arange(N)[None, :]
    keep = torch.rand(T, N, generator=g) < 0.5
    keep[:, 0] = True
    m = (causal & keep).cuda()
    out = f32(chunkattn.chunked(q, k, v, D ** -0.5, 128, 128, mask=m[None, None]))
    checks.grading_close(out, oref(q, k, v, D ** -0.5, oracle.MASK_ARRAY, m), what="array-masked chunks")


def test_patched_sdpa_decode_and_prefill():
    g = torch.Generator().manual_seed(73)
    f = chunkattn._wrap(stock=None)
    q1, k, v = rnd(g, 2, 32, 1, 128), rnd(g, 2, 4, 3000, 128), rnd(g, 2, 4, 3000, 128)
    checks.grading_close(f32(f(q1, k, v, None, 128 ** -0.5, None)), oref(q1, k, v, 128 ** -0.5), what="decode")
    q2 = rnd(g, 2, 32, 200, 128)
    checks.grading_close(f32(f(q2, k, v, None, 128 ** -0.5, "causal")),
                         oref(q2, k, v, 128 ** -0.5, oracle.MASK_CAUSAL), what="prefill")


@pytest.mark.parametrize("T,chunks", [(2, 4), (5, 16), (8, 32)])
def test_fold_verify_rows(T, chunks):
    """foldattn.fold: tests/test_foldattn.py's shape family (32/8 x 128, N not a tile multiple, K/V slices)."""
    g = torch.Generator().manual_seed(80 + T)
    B, Hq, Hkv, D, N = 2, 16, 4, 128, 4100
    q = rnd(g, B, Hq, T, D)
    kb, vb = rnd(g, B, Hkv, N + 200, D), rnd(g, B, Hkv, N + 200, D)
    k, v = kb[:, :, :N], vb[:, :, :N]
    out = f32(foldattn.fold(q, k, v, D ** -0.5, chunks))
    checks.grading_close(out, oref(q, k, v, D ** -0.5, oracle.MASK_CAUSAL), what=f"fold T={T}")


def test_gated_delta_update_with_gating():
    """gated_delta_update's own gating (sigmoid beta, compute_g), 35B head shapes, a decode-length pass."""
    g = torch.Generator().manual_seed(90)
    B, T, Hk, Hv, D = 2, 17, 4, 8, 128
    q = torch.nn.functional.normalize(torch.randn(B, T, Hk, D, generator=g), dim=-1).to(torch.bfloat16)
    k = torch.nn.functional.normalize(torch.randn(B, T, Hk, D, generator=g), dim=-1).to(torch.bfloat16)
    v = torch.randn(B, T, Hv, D, generator=g).to(torch.bfloat16)
    a = torch.randn(B, T, Hv, generator=g).to(torch.bfloat16)
    b = torch.randn(B, T, Hv, generator=g).to(torch.bfloat16)
    A_log = torch.randn(Hv, generator=g) * 0.5
    dt_bias = torch.randn(Hv, generator=g) * 0.5
    y, s = gdn_cuda.gated_delta_update(q.cuda(), k.cuda(), v.cuda(), a.cuda(), b.cuda(), A_log.cuda(),
                                       dt_bias.cuda())
    beta = torch.sigmoid(b.float())
    gg = gdn_cuda.compute_g(A_log, a, dt_bias)
    yr, sr = oracle.gdn(to_np(q), to_np(k), to_np(v), gg.numpy(), beta.numpy(),
                        np.zeros((B, Hv, D, D), np.float32), oracle.BF16, g_dt=oracle.F32, b_dt=oracle.F32)
    checks.grading_close(f32(y), oracle.to_f32(yr, oracle.BF16), what="y")
    assert np.abs(s.cpu().numpy() - sr).max() <= 1e-3 * np.abs(sr).max()
