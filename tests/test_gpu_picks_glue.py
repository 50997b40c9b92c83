"""QSA picks, the paged KV home and the GDN decode glue on the GPU.

Gathers are byte work: bit-exact against torch indexing of the same positions (stream_fast.py:6448-6491's row
order: picked blocks in sorted order, then the trailing partial block). Attention over the picks is checked against
the CPU oracle over the same rows and against an array-masked pass over the whole cache (the reference's Metal path
is bit-equal to that masked SDPA). The glue kernels are checked against fp32 compositions of the reference's
operations with its 16-bit rounding points (gdn_cuda.py:118-268)."""
import numpy as np
import pytest
import torch

import checks
import oracle
from gpu_util import f32, to_np
from larder_b200 import gdn_cuda, kv_host, ops, qsa

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _status_clean():
    yield
    assert ops.status() == 0, "a device wait gave up"


def picks(n, cr, nsel, gen):
    nb = n // cr
    tb = torch.randperm(nb, generator=gen)[:nsel].sort().values.to(torch.int32)
    own0 = n // cr * cr
    pos = torch.cat([(tb[:, None].long() * cr + torch.arange(cr)).reshape(-1), torch.arange(own0, n)])
    return tb, pos


def test_qsa_gather_bit_exact_and_attend():
    """Flash-Next decode shapes: 24/2 heads x 256, CR = 4, 512 picked blocks, a capacity-padded cache."""
    g = torch.Generator().manual_seed(21)
    Hq, Hk, D, cr, nsel, n, cap = 24, 2, 256, 4, 512, 10003, 10240
    kb = torch.randn(1, Hk, cap, D, generator=g).to(torch.bfloat16).cuda()
    vb = torch.randn(1, Hk, cap, D, generator=g).to(torch.bfloat16).cuda()
    k, v = kb[:, :, :n], vb[:, :, :n]
    tb, pos = picks(n, cr, nsel, g)
    kg, vg = qsa.qsa_gather(k, v, tb.cuda(), cr)
    assert torch.equal(kg, k[:, :, pos.cuda()]) and torch.equal(vg, v[:, :, pos.cuda()])
    q = torch.randn(1, Hq, 1, D, generator=g).to(torch.bfloat16).cuda()
    out = f32(qsa.qsa_attend(q, k, v, tb.cuda(), cr, D ** -0.5))
    ref = oracle.attn(to_np(q), to_np(kg), to_np(vg), D ** -0.5, oracle.BF16, out_dt=oracle.F32)
    checks.grading_close(out, ref, what="picks")
    m = torch.zeros(1, n, dtype=torch.bool)
    m[0, pos] = True
    full = f32(ops.attn_prefill(q, k, v, D ** -0.5, m.cuda()))
    checks.grading_close(out, full, what="picks vs masked pass")


@pytest.mark.parametrize("Hq, Hk, D, cr, nsel, n, cap", [
    (24, 2, 256, 4, 512, 10003, 10240),   # Flash-Next's decode shapes, a capacity-padded cache
    (24, 2, 256, 8, 300, 4099, 4352),     # CR 8, a 3-row tail
    (16, 2, 128, 1, 700, 2048, 2048),     # CR 1 (picked single rows), no tail
    (8, 1, 64, 3, 50, 1001, 1024),        # a block size that does not divide the 64-key tile
    (32, 4, 128, 16, 1, 40, 64),          # one pick and a tail: less than one tile
])
def test_qsa_decode_in_place_equals_gather_then_decode(Hq, Hk, D, cr, nsel, n, cap):
    """The decode kernel reading the picked rows in place (the CTA's copies) is bit-equal to the gather kernel
    followed by the same decode over the gathered rows; and both match the oracle over those rows."""
    g = torch.Generator().manual_seed(30 + cr + D)
    kb = torch.randn(1, Hk, cap, D, generator=g).to(torch.bfloat16).cuda()
    vb = torch.randn(1, Hk, cap, D, generator=g).to(torch.bfloat16).cuda()
    k, v = kb[:, :, :n], vb[:, :, :n]
    tb, pos = picks(n, cr, nsel, g)
    q = torch.randn(1, Hq, 1, D, generator=g).to(torch.bfloat16).cuda()
    kg, vg = qsa.qsa_gather(k, v, tb.cuda(), cr)
    two_step = ops.attn_decode(q, kg, vg, D ** -0.5)
    fused = ops.qsa_decode(q, k, v, tb.cuda(), cr, D ** -0.5)
    assert torch.equal(fused, two_step)
    if nsel <= 64:
        ref = oracle.attn(to_np(q), to_np(kg), to_np(vg), D ** -0.5, oracle.BF16, out_dt=oracle.F32)
        checks.grading_close(f32(fused), ref, what="picks in place")


def test_qsa_decode_in_place_reports_an_out_of_range_pick():
    """A pick past the view's end is not read (the kernel takes row 0 in its place) and lb2_status reports LB2_EINVAL
    from the pick-mode producer (where 98); the other rows attend as usual, so the output stays finite."""
    g = torch.Generator().manual_seed(44)
    Hq, Hk, D, cr, n = 8, 2, 128, 4, 400
    k = torch.randn(1, Hk, n, D, generator=g).to(torch.bfloat16).cuda()
    v = torch.randn(1, Hk, n, D, generator=g).to(torch.bfloat16).cuda()
    q = torch.randn(1, Hq, 1, D, generator=g).to(torch.bfloat16).cuda()
    tb = torch.tensor([0, 5, n // cr], dtype=torch.int32).cuda()  # block n // cr starts at row n: outside
    out = ops.qsa_decode(q, k, v, tb, cr, D ** -0.5)
    assert ops.status() == (98 << 8) | 1
    assert torch.isfinite(out.float()).all()


@pytest.mark.parametrize("host", [False, True])
def test_kv_home_put_gather_decode(host):
    """Rows appended in three puts across a chunk boundary (4096), then the picks gathered from the home equal the
    same picks of a contiguous cache; one decode row through Home.decode against the oracle."""
    g = torch.Generator().manual_seed(22 + host)
    Hq, Hk, D, cr, nsel = 16, 2, 128, 4, 300
    home = kv_host.Home(Hk, D, torch.bfloat16, "cuda", host=host)
    parts = [torch.randn(2, 1, Hk, s, D, generator=g).to(torch.bfloat16).cuda() for s in (3000, 2000, 1)]
    for kv in parts:
        home.put(kv[0], kv[1])
    k = torch.cat([p[0] for p in parts], dim=2)
    v = torch.cat([p[1] for p in parts], dim=2)
    n = k.shape[2]
    assert home.n == n == 5001 and len(home.chunks) == 2
    tb, pos = picks(n, cr, nsel, g)
    kg, vg = home.gather(tb.cuda(), cr)
    assert torch.equal(kg, k[:, :, pos.cuda()]) and torch.equal(vg, v[:, :, pos.cuda()])
    q = torch.randn(1, Hq, 1, D, generator=g).to(torch.bfloat16).cuda()
    k1 = torch.randn(1, Hk, 1, D, generator=g).to(torch.bfloat16).cuda()
    v1 = torch.randn(1, Hk, 1, D, generator=g).to(torch.bfloat16).cuda()
    out = f32(home.decode(q, k1, v1, tb.cuda(), cr, D ** -0.5))
    k2, v2 = torch.cat([k, k1], 2), torch.cat([v, v1], 2)
    pos2 = torch.cat([(tb[:, None].long() * cr + torch.arange(cr)).reshape(-1), torch.arange((n + 1) // cr * cr, n + 1)])
    ref = oracle.attn(to_np(q), to_np(k2[:, :, pos2.cuda()]), to_np(v2[:, :, pos2.cuda()]), D ** -0.5, oracle.BF16,
                      out_dt=oracle.F32)
    checks.grading_close(out, ref, what="home decode")


def _silu_bf16(x):
    sg = torch.sigmoid(x.float()).to(torch.bfloat16)
    return (x.float() * sg.float()).to(torch.bfloat16)


def test_step_glue_matches_composition():
    """qwen3_5's decode row from the conv output: silu, q/k RMSNorm (eps 1e-6 / Dk) and scales Dk^-1 / Dk^-0.5,
    sigmoid(b), compute_g, recurrence -- 3 positions, 16/32 heads x 128, from a random state."""
    g = torch.Generator().manual_seed(31)
    NR, Hk, Hv, Dk, Dv = 3, 16, 32, 128, 128
    CD = 2 * Hk * Dk + Hv * Dv
    conv = torch.randn(1, NR, CD, generator=g).to(torch.bfloat16)
    a = torch.randn(1, NR, Hv, generator=g).to(torch.bfloat16)
    b = torch.randn(1, NR, Hv, generator=g).to(torch.bfloat16)
    A_log = torch.randn(Hv, generator=g) * 0.5
    dt_bias = torch.randn(Hv, generator=g) * 0.5
    s0 = torch.randn(1, Hv, Dv, Dk, generator=g) * 0.1
    y, s = gdn_cuda.step_glue(conv.cuda(), a.cuda(), b.cuda(), A_log.cuda(), dt_bias.cuda(), s0.cuda(), Hk, Dk, Hv, Dv)
    # fp32 composition with the same rounding points
    sv = _silu_bf16(conv[0])                                                 # [NR, CD]
    qr = sv[:, :Hk * Dk].float().reshape(NR, Hk, Dk)
    kr = sv[:, Hk * Dk:2 * Hk * Dk].float().reshape(NR, Hk, Dk)
    eps = 1e-6 / Dk
    qn = (qr * torch.rsqrt((qr * qr).mean(-1, keepdim=True) + eps)).to(torch.bfloat16)
    kn = (kr * torch.rsqrt((kr * kr).mean(-1, keepdim=True) + eps)).to(torch.bfloat16)
    sq = torch.tensor(Dk ** -1.0, dtype=torch.bfloat16).float()
    sk = torch.tensor(Dk ** -0.5, dtype=torch.bfloat16).float()
    qf = (qn.float() * sq).to(torch.bfloat16)
    kf = (kn.float() * sk).to(torch.bfloat16)
    vf = _silu_bf16(conv[0, :, 2 * Hk * Dk:]).reshape(NR, Hv, Dv)
    beta = torch.sigmoid(b[0].float()).to(torch.bfloat16)
    gg = gdn_cuda.compute_g(A_log, a[0], dt_bias)
    yr, sr = oracle.gdn(to_np(qf[None]), to_np(kf[None]), to_np(vf[None]), gg[None].numpy(), to_np(beta[None]),
                        s0.numpy(), oracle.BF16, g_dt=oracle.F32, b_dt=oracle.BF16)
    checks.grading_close(f32(y), oracle.to_f32(yr, oracle.BF16), what="glue y")
    assert np.abs(s.cpu().numpy() - sr).max() <= 1e-3 * np.abs(sr).max()


def test_norm_gate_matches_formula():
    g = torch.Generator().manual_seed(32)
    R, D = 96, 128
    x = torch.randn(R, D, generator=g).to(torch.bfloat16)
    z = torch.randn(R, D, generator=g).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(D, generator=g)).to(torch.bfloat16)
    out = f32(gdn_cuda.norm_gate(x.cuda(), z.cuda(), w.cuda(), 1e-6))
    xf = x.float()
    n = (w.float() * (xf * torch.rsqrt((xf * xf).mean(-1, keepdim=True) + 1e-6)).to(torch.bfloat16).float())
    n = n.to(torch.bfloat16).float()
    ref = (torch.nn.functional.silu(z.float()) * n).numpy()
    checks.grading_close(out, ref, what="norm_gate")
