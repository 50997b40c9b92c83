"""The multi-GPU path on real GPUs (NCCL), as spawned child processes, one per GPU; skipped when the box has fewer
than 2 GPUs. KV-range-sharded decode (partials + all-gather + log-sum-exp combine) against one whole-cache decode,
and sequence-sharded prefill against the oracle. NVLS stays off (NCCL_NVLS_ENABLE=0); no rank leaves mid-step."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu
WORLD = 2


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, port, rq):
    import datetime
    import torch.distributed as dist
    from larder_b200 import ops, sharded
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=WORLD, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        g = torch.Generator().manual_seed(9)
        B, Hq, Hkv, D, N = 8, 32, 4, 128, 8192
        q = torch.randn(B, Hq, 1, D, generator=g).to(torch.bfloat16).to(dev)
        k = torch.randn(B, Hkv, N, D, generator=g).to(torch.bfloat16).to(dev)
        v = torch.randn(B, Hkv, N, D, generator=g).to(torch.bfloat16).to(dev)
        s0, s1 = sharded.kv_range(N, rank, WORLD)
        o = sharded.kv_sharded_decode(q, k[:, :, s0:s1], v[:, :, s0:s1], D ** -0.5)
        whole = ops.attn_decode(q, k, v, D ** -0.5)
        err = (o.float() - whole.float()).abs().max().item()
        st = ops.status(rank)
        rq.put((rank, err, st))
    finally:
        torch.cuda.synchronize(dev)
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < WORLD, reason="needs 2 GPUs")
def test_kv_sharded_decode_nccl_equals_whole():
    ctx = mp.get_context("spawn")
    rq = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, port, rq)) for r in range(WORLD)]
    for p in procs:
        p.start()
    res = [rq.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, err, st in res:
        assert st == 0 and err <= 2e-2, (rank, err, st)


def _peer_worker(rank, port, rq, push=False):
    import datetime
    import torch.distributed as dist
    from larder_b200 import ops, sharded
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=WORLD, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    xch = None
    try:
        g = torch.Generator().manual_seed(19)
        B, Hq, Hkv, D, N = 8, 32, 4, 128, 8192
        k = torch.randn(B, Hkv, N, D, generator=g).to(torch.bfloat16).to(dev)
        v = torch.randn(B, Hkv, N, D, generator=g).to(torch.bfloat16).to(dev)
        s0, s1 = sharded.kv_range(N, rank, WORLD)
        xch = sharded.PeerExchange(B, Hq, 1, D, push=push)
        err, same = 0.0, True
        for _ in range(5):  # both halves of the exchange buffer, each reused
            q = torch.randn(B, Hq, 1, D, generator=g).to(torch.bfloat16).to(dev)
            o = xch.decode(q, k[:, :, s0:s1], v[:, :, s0:s1], D ** -0.5)
            whole = ops.attn_decode(q, k, v, D ** -0.5)
            err = max(err, (o.float() - whole.float()).abs().max().item())
            same &= torch.equal(o, sharded.kv_sharded_decode(q, k[:, :, s0:s1], v[:, :, s0:s1], D ** -0.5))
        st = ops.status(rank)
        rq.put((rank, err, same, st))
    finally:
        torch.cuda.synchronize(dev)
        if xch is not None:
            xch.close()
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < WORLD, reason="needs 2 GPUs")
def test_kv_sharded_decode_peer_memory_equals_whole_and_nccl():
    """The exchange over NVLink peer memory (PeerExchange): five calls in a row, each equal to one decode over the
    whole cache (grading tolerance) and bit-equal to the NCCL path (same partials, same merge order)."""
    ctx = mp.get_context("spawn")
    rq = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_peer_worker, args=(r, port, rq)) for r in range(WORLD)]
    for p in procs:
        p.start()
    res = [rq.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, err, same, st in res:
        assert st == 0 and err <= 2e-2 and same, (rank, err, same, st)


@pytest.mark.skipif(torch.cuda.device_count() < WORLD, reason="needs 2 GPUs")
def test_kv_sharded_decode_push_equals_whole_and_nccl():
    """The push form (each rank's decode stores its partial, o rows in bf16, into every rank's buffer; the merge reads
    local memory): five calls in a row, equal to one whole-cache decode and to the NCCL path within the bar."""
    ctx = mp.get_context("spawn")
    rq = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_peer_worker, args=(r, port, rq, True)) for r in range(WORLD)]
    for p in procs:
        p.start()
    res = [rq.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, err, same, st in res:
        assert st == 0 and err <= 2e-2, (rank, err, same, st)


def test_sequence_sharded_prefill_matches_oracle():
    """The prefill share of each of 2 ranks (run here one after the other on one GPU: the share is independent work)."""
    import checks
    import oracle
    from gpu_util import f32, to_np
    from larder_b200 import sharded
    g = torch.Generator().manual_seed(11)
    B, Hq, Hkv, D, T = 4, 8, 2, 128, 384
    q = torch.randn(B, Hq, T, D, generator=g).to(torch.bfloat16).cuda()
    k = torch.randn(B, Hkv, T, D, generator=g).to(torch.bfloat16).cuda()
    v = torch.randn(B, Hkv, T, D, generator=g).to(torch.bfloat16).cuda()
    out = np.zeros((B, Hq, T, D), np.float32)
    for r in range(2):
        s0, s1, o = sharded.sharded_prefill(q, k, v, D ** -0.5, rank=r, world=2)
        out[s0:s1] = f32(o)
    ref = oracle.attn(to_np(q), to_np(k), to_np(v), D ** -0.5, oracle.BF16, oracle.MASK_CAUSAL, out_dt=oracle.F32)
    checks.grading_close(out, ref)
