"""The allocation-free decode entry point, lb2_attn_decode_noalloc, called through the C ABI.

Some callers cannot call cudaMalloc: an engine whose device memory belongs to its own budgeted allocator, or a
latency-critical caller that cannot take cudaMalloc's implicit device synchronisation. For them the library keeps the
split-KV decode's scratch in a static device array and takes no workspace argument. These tests check that its output
matches the workspace entry point (lb2_attn_decode) and the CPU oracle within the bar the other GPU tests use, on two
calls in a row with different inputs and lengths (the array keeps the previous call's contents, so stale partials
would show), under both schedules (balanced, whose partial slots follow from the ragged lengths, and fixed splits);
that fp32 calls, which need no scratch, run as lb2_attn_decode runs them; and that a call needing more scratch than
the array holds is refused with an error instead of running.

This file is named so that pytest collects it last; it passes alone in a fresh process and after the other tests.
"""
import ctypes
import os
import re

import numpy as np
import pytest
import torch

import checks
import oracle
from gpu_util import to_np
from larder_b200 import _lib, ops

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _scratch_bytes():
    """LB2_NOALLOC_SCRATCH_BYTES as include/larder_b200.h defines it."""
    text = open(os.path.join(ROOT, "include", "larder_b200.h")).read()
    m = re.search(r"#define\s+LB2_NOALLOC_SCRATCH_BYTES\s+\((\d+)u\s*<<\s*(\d+)\)", text)
    assert m, "LB2_NOALLOC_SCRATCH_BYTES not found in the header"
    return int(m.group(1)) << int(m.group(2))


def _call_noalloc(q, k, v, out, kv_len, scale, split=0, dtype=_lib.BF16):
    L = _lib.lib()
    return L.lb2_attn_decode_noalloc(
        ctypes.c_void_p(q.data_ptr()), _lib.i64(*q.stride()[:3]), ctypes.c_void_p(k.data_ptr()),
        _lib.i64(*k.stride()[:3]), ctypes.c_void_p(v.data_ptr()), _lib.i64(*v.stride()[:3]),
        ctypes.c_void_p(out.data_ptr()), _lib.i64(*out.stride()[:3]),
        ctypes.c_void_p(0 if kv_len is None else kv_len.data_ptr()), q.shape[0], q.shape[1], k.shape[1], q.shape[2],
        k.shape[2], q.shape[3], dtype, ctypes.c_float(scale), 0, int(split),
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))


def _inputs(seed, dtype=torch.bfloat16, B=16, cap=8192):
    g = torch.Generator().manual_seed(seed)
    Hq, Hkv, D = 32, 4, 128
    q = torch.randn(B, Hq, 1, D, generator=g).to(dtype).cuda()
    k = torch.randn(B, Hkv, cap, D, generator=g).to(dtype).cuda()
    v = torch.randn(B, Hkv, cap, D, generator=g).to(dtype).cuda()
    lens = torch.randint(cap // 8, cap + 1, (B,), generator=g).to(torch.int32).cuda()
    return q, k, v, lens


@pytest.mark.parametrize("split", [0, 2048])
def test_noalloc_matches_workspace_entry_and_oracle_on_two_calls(split):
    scale = 128 ** -0.5
    L = _lib.lib()
    need = L.lb2_attn_decode_workspace_size(16, 32, 4, 1, 8192, 128, split)
    assert 0 < need <= _scratch_bytes()
    for seed in (101 + split, 202 + split):  # different inputs and lengths each call
        q, k, v, lens = _inputs(seed)
        out = torch.empty_like(q)
        rc = _call_noalloc(q, k, v, out, lens, scale, split)
        assert rc == 0, L.lb2_error().decode()
        ref = ops.attn_decode(q, k, v, scale, kv_len=lens, split=split)
        torch.cuda.synchronize()
        got = out.float().cpu().numpy()
        checks.grading_close(got, ref.float().cpu().numpy(), what=f"split {split} seed {seed} vs lb2_attn_decode")
        for b, n in enumerate(lens.tolist()):
            orc = oracle.attn(to_np(q[b:b + 1]), to_np(k[b:b + 1, :, :n]), to_np(v[b:b + 1, :, :n]), scale,
                              oracle.BF16, out_dt=oracle.F32)
            checks.grading_close(got[b:b + 1], orc, what=f"split {split} seed {seed} sequence {b} vs the oracle")
        assert ops.status() == 0, "a device wait gave up"


def test_noalloc_fp32_runs_like_the_workspace_entry():
    """fp32 runs the exact CUDA-core kernel, which needs no scratch: same result as lb2_attn_decode, bit for bit."""
    q, k, v, lens = _inputs(404, torch.float32, B=2, cap=1000)
    out = torch.empty_like(q)
    rc = _call_noalloc(q, k, v, out, lens, 128 ** -0.5, dtype=_lib.F32)
    assert rc == 0, _lib.lib().lb2_error().decode()
    ref = ops.attn_decode(q, k, v, 128 ** -0.5, kv_len=lens)
    torch.cuda.synchronize()
    assert torch.equal(out, ref)
    assert ops.status() == 0


def test_noalloc_refuses_more_scratch_than_it_holds():
    q, k, v, lens = _inputs(303)
    out = torch.zeros_like(q)
    need = _lib.lib().lb2_attn_decode_workspace_size(16, 32, 4, 1, 8192, 128, 64)
    assert need > _scratch_bytes()  # 64-key splits need more than the array holds
    rc = _call_noalloc(q, k, v, out, lens, 128 ** -0.5, split=64)
    assert rc == _lib.EINVAL
    assert b"static array" in _lib.lib().lb2_error()
    torch.cuda.synchronize()
    assert np.all(out.float().cpu().numpy() == 0), "a refused call must not write its output"
