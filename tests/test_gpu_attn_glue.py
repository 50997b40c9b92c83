"""The attention layer's glue on the GPU (layer_glue.py:241-296, attn_step :578-619): q / k RMSNorm + rotate-half
RoPE and the output gate, against the CPU restatement of the reference's kernels with its bf16 rounding points.

The bar is the reference's own for its 16-bit CUDA paths (test_qsa_cuda.py:144, :163-164): at least 99 % of the
outputs bit-equal and none more than one bf16 step away (the sums of squares run in different fp32 orders), widened
by the first-order effect of the one rounding such an order can flip: bf16(x inv) one step off becomes w steps of
o = bf16(w bf16(x inv)) (two steps where w > 1), and a rotated column r = bf16(bf16(o c) + bf16(rot s)) takes |c|, |s|
times its inputs' allowance plus one step of the larger term (the terms can nearly cancel)."""
import numpy as np
import pytest
import torch

import oracle
from gpu_util import to_np, to_torch
from larder_b200 import layer_glue, ops

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _status_clean():
    yield
    assert ops.status() == 0, "a device wait gave up"


def rope_tables(S, R, offset=0, base=10000.0):
    """cos / sin [S, R] of positions offset .. offset + S - 1 (rotate-half layout: both halves repeat the angles)."""
    pos = np.arange(offset, offset + S, dtype=np.float64)[:, None]
    ang = pos * base ** (-np.arange(R // 2) * 2.0 / R)[None]
    ang = np.concatenate([ang, ang], axis=1)
    return np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)


def bf16_step(x):
    """One bf16 step (ulp) at the magnitude of fp32 values x (the smallest normal step at 0)."""
    e = np.floor(np.log2(np.maximum(np.abs(np.asarray(x, np.float64)), 2.0 ** -126)))
    return 2.0 ** (e - 7)


def assert_bf16_close(got, ref, extra=None):
    """got / ref bf16 bit patterns: >= 99 % equal, every other one a single bf16 step away (plus `extra`, an
    elementwise allowance of ref's shape, where given)."""
    g, r = got.astype(np.int32).ravel(), ref.astype(np.int32).ravel()
    same = g == r
    assert same.mean() >= 0.99, f"only {same.mean():.4f} bit-equal"
    gf, rf = oracle.bf16_to_f32(got).ravel(), oracle.bf16_to_f32(ref).ravel()
    step = np.abs(oracle.bf16_to_f32((r & 0xFFFF).astype(np.uint16) ^ 1) - rf)  # one ulp at ref's magnitude
    tol = step * 1.0001 + 1e-30 + (0 if extra is None else np.asarray(extra, np.float64).ravel())
    assert np.all(np.abs(gf - rf) <= tol), float(np.max(np.abs(gf - rf) - tol))


def glue_allowance(o_bits, w_bits, cs, sn, R):
    """The allowance beyond one step of the result for one flipped rounding of bf16(x inv): o_bits [B, H, S, D] are
    the normalised rows before RoPE (the oracle with no rotated dims), w_bits [D] the norm weight, cs / sn [S, R] as
    the kernel rounds them."""
    o = oracle.bf16_to_f32(o_bits).astype(np.float64)
    w = np.abs(oracle.bf16_to_f32(w_bits).astype(np.float64))
    dn = w * bf16_step(o / np.where(w > 0, w, 1))  # one step of x inv, times the weight
    extra = dn.copy()
    if R:
        c, s_ = np.abs(cs[None, None].astype(np.float64)), np.abs(sn[None, None].astype(np.float64))
        rot = np.concatenate([o[..., R // 2:R], o[..., :R // 2]], axis=-1)
        do = bf16_step(o) + dn
        drot = np.concatenate([do[..., R // 2:R], do[..., :R // 2]], axis=-1)
        extra[..., :R] = (bf16_step(np.maximum(np.abs(o[..., :R]) * c, np.abs(rot[..., :R]) * s_))
                          + c * do[..., :R] + s_ * drot[..., :R])
    return extra


def inputs(B, S, NQ, NK, D, R, seed, offset=0):
    rng = np.random.default_rng(seed)
    qg = oracle.f32_to_bf16(rng.standard_normal((B, S, NQ * 2 * D)).astype(np.float32) * 3)
    kr = oracle.f32_to_bf16(rng.standard_normal((B, S, NK * D)).astype(np.float32) * 3)
    qw = oracle.f32_to_bf16((1 + 0.2 * rng.standard_normal(D)).astype(np.float32))
    kw = oracle.f32_to_bf16((1 + 0.2 * rng.standard_normal(D)).astype(np.float32))
    cs, sn = rope_tables(S, R, offset)
    return qg, kr, qw, kw, cs, sn


@pytest.mark.parametrize("B, S, NQ, NK, D, R, cs_dt", [
    (1, 1, 16, 2, 256, 64, oracle.F32),     # a decode row of configs[2]'s model (partial rope, a quarter)
    (2, 37, 16, 2, 256, 64, oracle.BF16),   # prefill rows, batch of two, bf16 tables
    (1, 5, 32, 4, 128, 128, oracle.F32),    # configs[4]'s heads, full rope
    (1, 3, 4, 1, 512, 0, oracle.F32),       # no rope
    (1, 6, 4, 2, 128, 32, oracle.F32),      # a quarter of 128 rotated (the partner eight lanes away)
    (1, 3, 4, 2, 512, 128, oracle.BF16),    # 128 of 512 rotated (the partner in the lane's other column pair)
    (1, 4, 8, 2, 256, 24, oracle.F32),      # a width that is not a multiple of 16: RoPE through shared memory
    (1, 7, 8, 2, 256, 64, oracle.F16),      # f16 tables
    (1, 3, 4, 2, 128, 24, oracle.F16),      # f16 tables through shared memory
])
def test_qk_norm_rope_matches_oracle(B, S, NQ, NK, D, R, cs_dt):
    qg, kr, qw, kw, cs, sn = inputs(B, S, NQ, NK, D, R, seed=B * 100 + S, offset=4093)
    # the tables as the kernel reads them (each use rounds a table value to bf16, in the oracle too)
    if cs_dt == oracle.BF16:
        cs, sn = oracle.bf16_to_f32(oracle.f32_to_bf16(cs)), oracle.bf16_to_f32(oracle.f32_to_bf16(sn))
    elif cs_dt == oracle.F16:
        cs, sn = cs.astype(np.float16).astype(np.float32), sn.astype(np.float16).astype(np.float32)
    rq, rk = oracle.qk_norm_rope(qg, kr, qw, kw, 1e-6, cs, sn, NQ, NK)
    nq, nk = oracle.qk_norm_rope(qg, kr, qw, kw, 1e-6, np.zeros((S, 0), np.float32), np.zeros((S, 0), np.float32),
                                 NQ, NK)
    cb, sb = oracle.bf16_to_f32(oracle.f32_to_bf16(cs)), oracle.bf16_to_f32(oracle.f32_to_bf16(sn))
    dt = {oracle.BF16: torch.bfloat16, oracle.F16: torch.float16}.get(cs_dt, torch.float32)
    q, k = layer_glue.qk_norm_rope(to_torch(qg, oracle.BF16), to_torch(kr, oracle.BF16), to_torch(qw, oracle.BF16),
                                   to_torch(kw, oracle.BF16), 1e-6, torch.from_numpy(cs).to(dt).cuda(),
                                   torch.from_numpy(sn).to(dt).cuda(), NQ, NK)
    assert tuple(q.shape) == (B, NQ, S, D) and tuple(k.shape) == (B, NK, S, D)
    assert_bf16_close(to_np(q), rq, glue_allowance(nq, qw, cb, sb, R))
    assert_bf16_close(to_np(k), rk, glue_allowance(nk, kw, cb, sb, R))


def test_qk_norm_rope_empty_and_rejects():
    qg, kr, qw, kw, cs, sn = inputs(1, 0, 4, 1, 128, 64, seed=3)
    t = lambda a: to_torch(a, oracle.BF16)
    q, k = layer_glue.qk_norm_rope(t(qg), t(kr), t(qw), t(kw), 1e-6, torch.from_numpy(cs).cuda(),
                                   torch.from_numpy(sn).cuda(), 4, 1)
    assert q.shape == (1, 4, 0, 128) and k.shape == (1, 1, 0, 128)
    qg, kr, qw, kw, cs, sn = inputs(1, 2, 4, 1, 128, 64, seed=4)
    with pytest.raises(ValueError):  # odd rope width
        layer_glue.qk_norm_rope(t(qg), t(kr), t(qw), t(kw), 1e-6, torch.from_numpy(cs[:, :63]).cuda(),
                                torch.from_numpy(sn[:, :63]).cuda(), 4, 1)
    with pytest.raises(ValueError):  # fp16 rows: the reference's path is bf16
        layer_glue.qk_norm_rope(t(qg).half(), t(kr).half(), t(qw), t(kw), 1e-6, torch.from_numpy(cs).cuda(),
                                torch.from_numpy(sn).cuda(), 4, 1)


@pytest.mark.parametrize("rows, NQ, D", [(1, 16, 256), (4099, 16, 256), (33, 32, 128)])
def test_out_gate_matches_oracle_and_in_place(rows, NQ, D):
    rng = np.random.default_rng(rows)
    o = oracle.f32_to_bf16(rng.standard_normal((rows, NQ * D)).astype(np.float32))
    qg = oracle.f32_to_bf16((rng.standard_normal((rows, NQ * 2 * D)) * 4).astype(np.float32))
    ref = oracle.out_gate(o, qg, NQ)
    ot, qt = to_torch(o, oracle.BF16), to_torch(qg, oracle.BF16)
    got = layer_glue.out_gate(ot, qt, NQ)
    assert_bf16_close(to_np(got), ref)
    layer_glue.out_gate(ot, qt, NQ, result=ot)  # in place
    assert np.array_equal(to_np(ot), to_np(got))
