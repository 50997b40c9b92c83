"""GPU parity of the Gated-DeltaNet kernels against the CPU oracle (CpuGdn's arithmetic, extended with the
vector gate and mask of the reference's CUDA recurrence) and the golden vectors of tests/test_gdn_cuda.py's cases.
Bars: y within max-abs 2e-2 and cosine >= 0.9999 of the f32 oracle; state within 1e-2 relative (the build's
grading bars); plus the reference test's own property that a masked position writes y = 0."""
import numpy as np
import pytest
import torch

import cases
import checks
import oracle
from gpu_util import f32, to_torch
from larder_b200 import ops

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _status_clean():
    yield
    assert ops.status() == 0, "a device wait gave up"


def run_case(c, fn):
    dt = c["dt"]
    q, k, v = (to_torch(c[n], dt) for n in ("q", "k", "v"))
    g = to_torch(c["g"], c["g_dt"])
    beta = to_torch(c["beta"], c["b_dt"])
    state = torch.from_numpy(c["state"]).cuda()
    mask = None if c["mask"] is None else torch.from_numpy(c["mask"]).cuda()
    y, s = fn(q, k, v, g, beta, state, mask)
    yr, sr = oracle.gdn(c["q"], c["k"], c["v"], c["g"], c["beta"], c["state"], dt, g_dt=c["g_dt"], b_dt=c["b_dt"],
                        mask=c["mask"])
    return f32(y), s.cpu().numpy(), oracle.to_f32(yr, dt), sr


@pytest.mark.parametrize("i", range(len(cases.GDN_CUDA_CASES)))
def test_recurrent_reference_cases(i):
    c = cases.gdn_cuda_case(i)
    y, s, yr, sr = run_case(c, lambda q, k, v, g, b, s, m: ops.gdn_recurrent(q, k, v, g, b, s, m))
    checks.grading_close(y, yr, what=f"case {i} y")
    assert np.abs(s - sr).max() <= 1e-4 * np.abs(sr).max() + 1e-6, f"case {i} state"
    checks.golden_close(s, f"gdncuda{i}.s", 1e-4, what="state vs golden")
    if c["mask"] is not None:
        assert not y[~c["mask"]].any(), "a masked position wrote y"


def test_recurrent_cpu_case():
    c = cases.gdn_cpu_case()
    y, s, yr, sr = run_case(c, lambda q, k, v, g, b, s, m: ops.gdn_recurrent(q, k, v, g, b, s, m))
    checks.grading_close(y, yr, what="y")
    checks.golden_close(s, "gdncpu.s", 1e-4, what="state vs golden")


def test_recurrent_decode_batch16_config4():
    """Config 4's decode: 64 recurrent steps at B=16 (Hk 16, Hv 32, 128 x 128) from a random state, one call a step,
    the state carried in place; checked after the 64 steps."""
    gen = torch.Generator().manual_seed(4)
    B, Hk, Hv, D, steps = 16, 16, 32, 128, 64
    q = torch.nn.functional.normalize(torch.randn(B, steps, Hk, D, generator=gen), dim=-1).to(torch.bfloat16)
    k = torch.nn.functional.normalize(torch.randn(B, steps, Hk, D, generator=gen), dim=-1).to(torch.bfloat16)
    v = torch.randn(B, steps, Hv, D, generator=gen).to(torch.bfloat16)
    beta = torch.sigmoid(torch.randn(B, steps, Hv, generator=gen)).to(torch.bfloat16)
    g = torch.exp(-torch.nn.functional.softplus(torch.randn(B, steps, Hv, generator=gen)))
    s0 = torch.randn(B, Hv, D, D, generator=gen) * 0.1
    s = s0.cuda()
    ys = []
    for t in range(steps):
        y, s = ops.gdn_recurrent(q[:, t:t + 1].cuda(), k[:, t:t + 1].cuda(), v[:, t:t + 1].cuda(),
                                 g[:, t:t + 1].cuda(), beta[:, t:t + 1].cuda(), s)
        ys.append(f32(y))
    from gpu_util import to_np
    yr, sr = oracle.gdn(to_np(q), to_np(k), to_np(v), g.numpy(), to_np(beta), s0.numpy(), oracle.BF16,
                        g_dt=oracle.F32, b_dt=oracle.BF16)
    checks.grading_close(np.concatenate(ys, axis=1), oracle.to_f32(yr, oracle.BF16), what="y")
    rel = np.abs(s.cpu().numpy() - sr).max() / np.abs(sr).max()
    assert rel <= 1e-2, rel
