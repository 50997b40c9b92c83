"""Decode with q and o in host memory (lb2_attn_decode_host): calls in a row, their copies overlapping on the
library's streams, each output equal bit for bit to the device-buffer decode of the same q (the same kernel runs
on a staged copy of it). Pinned and pageable host tensors."""
import pytest
import torch

from larder_b200 import ops

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _status_clean():
    yield
    assert ops.status() == 0, "a device wait gave up"


@pytest.mark.parametrize("pinned", [True, False])
def test_decode_host_equals_device_decode(pinned):
    g = torch.Generator().manual_seed(41 + pinned)
    B, Hq, Hkv, D, N = 4, 32, 4, 128, 3000
    k = torch.randn(B, Hkv, N, D, generator=g).to(torch.bfloat16).cuda()
    v = torch.randn(B, Hkv, N, D, generator=g).to(torch.bfloat16).cuda()
    kv_len = torch.tensor([3000, 1, 1777, 2048], dtype=torch.int32).cuda()
    qs = [torch.randn(B, Hq, 1, D, generator=g).to(torch.bfloat16) for _ in range(5)]
    if pinned:
        qs = [q.pin_memory() for q in qs]
    outs = [torch.empty(B, Hq, 1, D, dtype=torch.bfloat16) for _ in qs]
    if pinned:
        outs = [o.pin_memory() for o in outs]
    for q, o in zip(qs, outs):  # issued back to back, nothing waited for in between
        ops.attn_decode_host(q, k, v, D ** -0.5, o, kv_len=kv_len)
    ops.attn_decode_host_drain()
    torch.cuda.synchronize()
    for i, (q, o) in enumerate(zip(qs, outs)):
        ref = ops.attn_decode(q.cuda(), k, v, D ** -0.5, kv_len=kv_len).cpu()
        assert torch.equal(o, ref), f"call {i}"
