"""The exchange merges of the KV-range-sharded decode on ONE GPU: R ranks' partials laid out in local exchange buffers
exactly as the peers would leave them (pull form: a buffer a rank; push form: one buffer holding all R slots, the o
rows in bf16), every peer's flag already at the call's epoch, so the kernels find their inputs and merge without
waiting. Checked against a float64 log-sum-exp merge of the same partials (foldattn.py:188-211's merge), on the
vector path (rows a multiple of 4) and the scalar one."""
import ctypes

import numpy as np
import pytest
import torch

import oracle
from larder_b200 import _lib, ops

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _status_clean():
    yield
    assert ops.status() == 0, "a device wait gave up"


def partials(R, rows, D, seed):
    rng = np.random.default_rng(seed)
    o = oracle.bf16_to_f32(oracle.f32_to_bf16(rng.standard_normal((R, rows, D)).astype(np.float32)))
    lse = (rng.standard_normal((R, rows)) * 3).astype(np.float32)
    return o, lse


def merge64(o, lse):
    w = np.exp(lse.astype(np.float64) - lse.max(0, keepdims=True))
    return (w[..., None] * o).sum(0) / w.sum(0)[..., None]


def i64(*v):
    return (ctypes.c_int64 * len(v))(*v)


def ptrs(*t):
    return (ctypes.c_uint64 * len(t))(*[x.data_ptr() for x in t])


@pytest.mark.parametrize("R, B, Hq, D", [(8, 4, 8, 128), (4, 2, 16, 256), (3, 1, 3, 128), (2, 5, 4, 64)])
def test_push_merge_of_local_slots(R, B, Hq, D):
    L = _lib.lib()
    rows, epoch, rank = B * Hq, 1, R - 1
    o, lse = partials(R, rows, D, seed=R * 100 + D)
    nbytes = L.lb2_xch_push_bytes(R, B, Hq, 1, D)
    buf = torch.zeros(nbytes // 4 + 4, dtype=torch.float32, device="cuda")
    half, slot = R * rows * (D + 1), rows * (D + 1)
    for r in range(R):  # slot r of half epoch % 2: the o rows as bf16, then the lse after rows * D floats
        s0 = (epoch & 1) * half + r * slot
        bits = torch.from_numpy(oracle.f32_to_bf16(o[r]).reshape(-1).view(np.int16))
        buf[s0:s0 + rows * D // 2] = bits.cuda().view(torch.float32)
        buf[s0 + rows * D:s0 + rows * D + rows] = torch.from_numpy(lse[r]).cuda()
    flags = buf[2 * half:2 * half + 8].view(torch.int32)
    flags[:R] = epoch  # every peer's partial of this call has landed
    out = torch.empty(B, Hq, 1, D, dtype=torch.bfloat16, device="cuda")
    rc = L.lb2_attn_combine_pushed(ptrs(*[buf] * R), R, rank, epoch, B, Hq, 1, D, ctypes.c_void_p(out.data_ptr()),
                                   i64(*out.stride()[:3]), _lib.BF16, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0
    ref = merge64(o, lse).reshape(B, Hq, 1, D)
    got = out.float().cpu().numpy()
    assert np.abs(got - ref).max() <= 2 ** -8 * np.abs(ref).max() + 1e-6


@pytest.mark.parametrize("R, B, Hq, D", [(8, 4, 8, 128), (3, 1, 3, 128)])
def test_pull_merge_of_local_buffers(R, B, Hq, D):
    L = _lib.lib()
    rows, epoch, rank = B * Hq, 1, 0
    o, lse = partials(R, rows, D, seed=R * 10 + D + 1)
    nbytes = L.lb2_xch_bytes(B, Hq, 1, D)
    half = rows * (D + 1)
    bufs = []
    for r in range(R):  # rank r's own buffer: its partial in half epoch % 2 (fp32 o rows, then the lse)
        b = torch.zeros(nbytes // 4 + 4, dtype=torch.float32, device="cuda")
        s0 = (epoch & 1) * half
        b[s0:s0 + rows * D] = torch.from_numpy(o[r].reshape(-1)).cuda()
        b[s0 + rows * D:s0 + rows * D + rows] = torch.from_numpy(lse[r]).cuda()
        bufs.append(b)
    bufs[rank][2 * half:2 * half + 8].view(torch.int32)[:R] = epoch
    out = torch.empty(B, Hq, 1, D, dtype=torch.bfloat16, device="cuda")
    rc = L.lb2_attn_combine_peers(ptrs(*bufs), R, rank, epoch, B, Hq, 1, D, ctypes.c_void_p(out.data_ptr()),
                                  i64(*out.stride()[:3]), _lib.BF16, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0
    ref = merge64(o, lse).reshape(B, Hq, 1, D)
    assert np.abs(out.float().cpu().numpy() - ref).max() <= 2 ** -8 * np.abs(ref).max() + 1e-6
