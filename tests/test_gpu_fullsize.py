"""Parity at the timed configurations' full sizes, on one GPU, against the CPU oracle (the bar of the other GPU tests:
max-abs 2e-2 and cosine >= 0.9999 of the f32 oracle).

  * the 8192-row wide cut exactly as bench.py times it -- 2048-row chunks over keys 0 .. 2048(c + 1),
    16q/2kv x 256, bf16, the sigmoid gate fused, through chunkattn.chunked -- against the oracle one chunk at a time
    (the reference's loop, chunkattn.py:359-423) times sigmoid(gate);
  * configs[4]'s prefill share: two of its 8192-token causal sequences (32q/4kv x 128) in one launch, as one rank's
    share runs;
  * configs[4]'s decode arithmetic on one GPU: B = 64 over a 32768-key cache cut into eight 4096-key ranges, one
    lb2_attn_decode_partial call a range into the packed [o rows | lse] layout the all-gather moves, merged by
    lb2_attn_combine_packed -- against the oracle over each whole sequence.
"""
import numpy as np
import pytest
import torch

import checks
import oracle
from gpu_util import to_np
from larder_b200 import chunkattn, ops

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _status_clean():
    yield
    assert ops.status() == 0, "a device wait gave up"


def _bf16(g, *shape, dev="cuda"):
    return torch.randn(*shape, generator=g, device=dev, dtype=torch.float32).to(torch.bfloat16)


def test_config3_wide_cut_full_size():
    dev = torch.device("cuda", torch.cuda.current_device())
    g = torch.Generator(device=dev).manual_seed(3000)  # bench.py's configs[2] inputs
    B, Hq, Hkv, D, T, W = 1, 16, 2, 256, 8192, 2048
    q = _bf16(g, B, T, Hq, D, dev=dev)
    k = _bf16(g, B, Hkv, T, D, dev=dev)
    v = _bf16(g, B, Hkv, T, D, dev=dev)
    gate = _bf16(g, B, T, Hq * D, dev=dev)
    qv, gv = q.transpose(1, 2), gate.view(B, T, Hq, D).transpose(1, 2)
    out = chunkattn.chunked(qv, k, v, D ** -0.5, W, W, gate=gv).float().cpu().numpy()
    kn, vn = to_np(k), to_np(v)
    sig = 1.0 / (1.0 + np.exp(-gv.float().cpu().numpy().astype(np.float64)))
    ref = np.empty(out.shape, np.float64)
    for c in range(T // W):
        r0, r1 = c * W, (c + 1) * W
        ref[:, :, r0:r1] = oracle.attn(to_np(qv[:, :, r0:r1]), kn[:, :, :r1], vn[:, :, :r1], D ** -0.5, oracle.BF16,
                                       oracle.MASK_CAUSAL, out_dt=oracle.F32) * sig[:, :, r0:r1]
    checks.grading_close(out, ref, what="configs[2] wide cut, 8192 rows")


def test_config5_prefill_share_full_size():
    dev = torch.device("cuda", torch.cuda.current_device())
    g = torch.Generator(device=dev).manual_seed(5000)  # bench.py's configs[4] prefill inputs (rank 0)
    S, Hq, Hkv, D, T = 2, 32, 4, 128, 8192
    q = _bf16(g, S, T, Hq, D, dev=dev).transpose(1, 2)
    k = _bf16(g, S, Hkv, T, D, dev=dev)
    v = _bf16(g, S, Hkv, T, D, dev=dev)
    out = ops.attn_prefill(q, k, v, D ** -0.5, "causal").float().cpu().numpy()
    ref = oracle.attn(to_np(q), to_np(k), to_np(v), D ** -0.5, oracle.BF16, oracle.MASK_CAUSAL, out_dt=oracle.F32)
    checks.grading_close(out, ref, what="configs[4] prefill, 2 x 8192 causal, 32q/4kv x 128")


def test_config5_decode_ranges_merged_full_size():
    dev = torch.device("cuda", torch.cuda.current_device())
    g = torch.Generator(device=dev).manual_seed(77)
    B, Hq, Hkv, D, N, R = 64, 32, 4, 128, 32768, 8
    q = _bf16(g, B, Hq, 1, D, dev=dev)
    k = _bf16(g, B, Hkv, N, D, dev=dev)
    v = _bf16(g, B, Hkv, N, D, dev=dev)
    rows = B * Hq
    gathered = torch.empty(R, rows * (D + 1), dtype=torch.float32, device=dev)
    for r in range(R):  # rank r's partial, packed as it would enter the all-gather
        s0, s1 = r * N // R, (r + 1) * N // R
        ops.attn_decode_partial(q, k[:, :, s0:s1], v[:, :, s0:s1], D ** -0.5,
                                out=(gathered[r, :rows * D].view(B, Hq, 1, D), gathered[r, rows * D:].view(B, Hq, 1)))
    out = ops.attn_combine_packed(gathered, R, B, Hq, 1, D, torch.bfloat16).float().cpu().numpy()
    qn, kn, vn = to_np(q), to_np(k), to_np(v)
    del k, v
    ref = np.empty(out.shape, np.float32)
    for b in range(B):
        ref[b:b + 1] = oracle.attn(qn[b:b + 1], kn[b:b + 1], vn[b:b + 1], D ** -0.5, oracle.BF16, out_dt=oracle.F32)
    checks.grading_close(out, ref, what="configs[4] decode, 64 x 32768 keys in 8 merged ranges")
