"""The allocation-free decode entry point, lb2_attn_decode_noalloc, called through the C ABI.

Some callers cannot call cudaMalloc: an engine whose device memory belongs to its own budgeted allocator, or a
latency-critical caller that cannot take cudaMalloc's implicit device synchronisation. For them the library keeps the
split-KV decode's scratch in a static device array and takes no workspace argument. These tests check that its output
matches the workspace entry point (lb2_attn_decode) within the bar the other GPU tests use, on two calls in a row with
different inputs (the array keeps the previous call's contents, so stale partials or counters would show), and that a
call needing more scratch than the array holds is refused with an error instead of running.

This file is named so that pytest collects it last; it passes alone in a fresh process and after the other tests.
"""
import ctypes

import numpy as np
import pytest
import torch

import checks
from larder_b200 import _lib, ops

pytestmark = pytest.mark.gpu


def _call_noalloc(q, k, v, out, kv_len, scale, split=0):
    L = _lib.lib()
    return L.lb2_attn_decode_noalloc(
        ctypes.c_void_p(q.data_ptr()), _lib.i64(*q.stride()[:3]), ctypes.c_void_p(k.data_ptr()),
        _lib.i64(*k.stride()[:3]), ctypes.c_void_p(v.data_ptr()), _lib.i64(*v.stride()[:3]),
        ctypes.c_void_p(out.data_ptr()), _lib.i64(*out.stride()[:3]),
        ctypes.c_void_p(0 if kv_len is None else kv_len.data_ptr()), q.shape[0], q.shape[1], k.shape[1], q.shape[2],
        k.shape[2], q.shape[3], _lib.BF16, ctypes.c_float(scale), 0, int(split),
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))


def _inputs(seed):
    g = torch.Generator().manual_seed(seed)
    B, Hq, Hkv, D, cap = 16, 32, 4, 128, 8192
    q = torch.randn(B, Hq, 1, D, generator=g).to(torch.bfloat16).cuda()
    k = torch.randn(B, Hkv, cap, D, generator=g).to(torch.bfloat16).cuda()
    v = torch.randn(B, Hkv, cap, D, generator=g).to(torch.bfloat16).cuda()
    lens = torch.randint(1024, cap + 1, (B,), generator=g).to(torch.int32).cuda()
    return q, k, v, lens


def test_noalloc_matches_workspace_entry_on_two_calls():
    scale = 128 ** -0.5
    split = 2048  # this batch's scratch then fits the static array
    L = _lib.lib()
    need = L.lb2_attn_decode_workspace_size(16, 32, 4, 1, 8192, 128, split)
    assert 0 < need <= _lib_scratch_bytes()
    for seed in (101, 202):
        q, k, v, lens = _inputs(seed)
        out = torch.empty_like(q)
        rc = _call_noalloc(q, k, v, out, lens, scale, split)
        assert rc == 0, L.lb2_error().decode()
        ref = ops.attn_decode(q, k, v, scale, kv_len=lens, split=split)
        torch.cuda.synchronize()
        checks.grading_close(out.float().cpu().numpy(), ref.float().cpu().numpy(), what=f"seed {seed}")
        assert ops.status() == 0, "a device wait gave up"


def test_noalloc_refuses_more_scratch_than_it_holds():
    q, k, v, lens = _inputs(303)
    out = torch.zeros_like(q)
    rc = _call_noalloc(q, k, v, out, lens, 128 ** -0.5, split=64)  # 64-key splits need far more than 8 MiB
    assert rc == _lib.EINVAL
    assert b"static array" in _lib.lib().lb2_error()
    torch.cuda.synchronize()
    assert np.all(out.float().cpu().numpy() == 0), "a refused call must not write its output"


def _lib_scratch_bytes():
    return 8 << 20  # LB2_NOALLOC_SCRATCH_BYTES in include/larder_b200.h
