"""The multi-GPU choreography on CPU ranks (torch.distributed gloo, world size 2): sequence and KV-range
partitioning, and the KV-sharded decode's pack / all-gather / log-sum-exp merge -- with the CPU oracle planted as the
per-range partial and the merge (test-only checkers), so that the exchange itself is what is tested. A rank that
fails is seen by the other as an error within the process group's timeout (no hang)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from larder_b200 import sharded


def test_sequence_and_kv_ranges_cover_exactly():
    for n, w in ((64, 8), (10, 4), (3, 4), (32768, 8)):
        spans = [sharded.sequence_shard(n, r, w) for r in range(w)]
        assert spans[0][0] == 0 and spans[-1][1] == n
        assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
        assert max(s1 - s0 for s0, s1 in spans) - min(s1 - s0 for s0, s1 in spans) <= 1
    assert sharded.kv_range(32768, 3, 8) == (12288, 16384)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _oracle_partial(q, k, v, scale, kv_len, part_o, part_lse):
    """Per-range normalised output and natural-log LSE, from the f64 reference (test checker), into the packed
    buffer's two parts."""
    qn, kn, vn = (t.double().numpy() for t in (q, k, v))
    G = qn.shape[1] // kn.shape[1]
    kr, vr = np.repeat(kn, G, 1), np.repeat(vn, G, 1)
    s = scale * qn @ np.swapaxes(kr, -1, -2)
    m = s.max(-1, keepdims=True)
    p = np.exp(s - m)
    lse = (m + np.log(p.sum(-1, keepdims=True)))[..., 0]
    o = (p / p.sum(-1, keepdims=True)) @ vr
    part_o.copy_(torch.from_numpy(o).float())
    part_lse.copy_(torch.from_numpy(lse).float())


def _torch_combine(gathered, shape, dtype):
    B, Hq, T, D = shape
    world, rows = gathered.shape[0], B * Hq * T
    po = gathered[:, :rows * D].reshape(world, B, Hq, T, D)
    pl = gathered[:, rows * D:].reshape(world, B, Hq, T)
    w = torch.softmax(pl, dim=0)
    return (w[..., None] * po).sum(0).to(dtype)


def _worker(rank, world, port, q, k, v, scale, result_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=__import__("datetime").timedelta(seconds=30))
    try:
        s0, s1 = sharded.kv_range(k.shape[2], rank, world)
        o = sharded.kv_sharded_decode(q, k[:, :, s0:s1], v[:, :, s0:s1], scale, partial_fn=_oracle_partial,
                                      combine_fn=_torch_combine, out_dtype=torch.float32)
        result_q.put((rank, o.numpy()))
    finally:
        dist.destroy_process_group()


def test_kv_sharded_decode_two_gloo_ranks_equals_whole():
    g = torch.Generator().manual_seed(5)
    B, Hq, Hkv, D, N = 2, 8, 2, 64, 300
    q = torch.randn(B, Hq, 1, D, generator=g)
    k = torch.randn(B, Hkv, N, D, generator=g)
    v = torch.randn(B, Hkv, N, D, generator=g)
    ctx = mp.get_context("spawn")
    rq = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q, k, v, D ** -0.5, rq)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(rq.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    ref = oracle.attn_ref64(q.numpy(), k.numpy(), v.numpy(), D ** -0.5)
    for r in range(2):
        assert np.abs(res[r] - ref).max() < 1e-5


def _dying_worker(rank, world, port, result_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=__import__("datetime").timedelta(seconds=5))
    if rank == 1:
        os._exit(3)  # a rank that leaves between steps, nothing in flight
    try:
        t = torch.zeros(4)
        dist.all_reduce(t)
        result_q.put((rank, "no error"))
    except Exception as e:  # the survivor learns of it as an error, within the timeout
        result_q.put((rank, type(e).__name__))


def test_dead_rank_is_an_error_not_a_hang():
    ctx = mp.get_context("spawn")
    rq = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dying_worker, args=(r, 2, port, rq)) for r in range(2)]
    for p in procs:
        p.start()
    rank, what = rq.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
    assert rank == 0 and what != "no error"


class _FakeXchLib:
    """The exchange's CUDA calls stood in for on CPU ranks: allocation, 64-byte handles and mappings as plain
    numbers, every call recorded; the open of `fail_rank` fails."""

    def __init__(self, rank, fail_rank):
        self.rank, self.fail_rank, self.calls = rank, fail_rank, []

    def lb2_xch_bytes(self, B, Hq, T, D):
        return 2 * B * Hq * T * (D + 1) * 4 + 32

    def lb2_xch_alloc(self, nbytes, pptr):
        pptr._obj.value = 0x10000 * (self.rank + 1)
        self.calls.append(("alloc", nbytes))
        return 0

    def lb2_xch_handle(self, ptr, buf):
        import ctypes
        ctypes.memmove(buf, (b"H%d" % self.rank).ljust(64, b"\0"), 64)
        return 0

    def lb2_xch_open(self, hbuf, pptr):
        if self.rank == self.fail_rank:
            return 1
        peer = int(hbuf.raw[1:2])
        pptr._obj.value = 0x900000 + peer
        self.calls.append(("open", peer))
        return 0

    def lb2_xch_close(self, p):
        self.calls.append(("close", p.value))
        return 0

    def lb2_xch_free(self, p):
        self.calls.append(("free", p.value))
        return 0

    def lb2_error(self):
        return b"mapping refused"


def _xch_worker(rank, world, port, fail_rank, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        fake = _FakeXchLib(rank, fail_rank)
        sharded.lib = lambda: fake
        try:
            xch = sharded.PeerExchange(2, 4, 1, 8)
        except RuntimeError as e:
            q.put((rank, "raised", str(e), fake.calls))
            return
        bufs = list(xch.bufs)
        xch.close()
        q.put((rank, "ok", bufs, fake.calls))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("fail_rank", [-1, 1])
def test_peer_exchange_setup_all_or_nothing(fail_rank):
    """PeerExchange on two CPU ranks with the CUDA calls faked: each rank maps the other's buffer and keeps its own
    at its rank; close unmaps the peer before freeing its own. When one rank cannot map, both raise (neither goes on
    to a step the other left), and each releases what it had set up."""
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_xch_worker, args=(r, world, port, fail_rank, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, status, info, calls in res:
        base = 0x10000 * (rank + 1)
        if fail_rank < 0:
            assert status == "ok"
            assert info[rank] == base and info[1 - rank] == 0x900000 + (1 - rank)
            assert calls[-2:] == [("close", 0x900000 + (1 - rank)), ("free", base)]
        else:
            assert status == "raised" and "could not map" in info
            assert calls[-1] == ("free", base)
            assert (("close", 0x900000 + (1 - rank)) in calls) == (rank != fail_rank)



def _split_worker(rank, world, port, q, k, v, scale, result_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=__import__("datetime").timedelta(seconds=30))
    try:
        s0, s1 = sharded.kv_range(k.shape[2], rank, world)

        def merge(po, pl, dtype):
            w = torch.softmax(pl, dim=0)
            return (w[..., None] * po).sum(0).to(dtype)
        o = sharded.kv_sharded_decode_split(q, k[:, :, s0:s1], v[:, :, s0:s1], scale, partial_fn=_oracle_partial,
                                            merge_fn=merge, out_dtype=torch.float32)
        result_q.put((rank, o.numpy()))
    finally:
        dist.destroy_process_group()


def test_split_merge_two_gloo_ranks_equals_whole():
    """The split merge's plumbing (all-to-all of the partials, each rank merging B / R sequences, all-gather of the
    merged rows) on two CPU ranks, the f64 partial and a torch merge in place of the CUDA kernels."""
    g = torch.Generator().manual_seed(6)
    B, Hq, Hkv, D, N = 4, 4, 2, 64, 200
    q = torch.randn(B, Hq, 1, D, generator=g)
    k = torch.randn(B, Hkv, N, D, generator=g)
    v = torch.randn(B, Hkv, N, D, generator=g)
    ctx = mp.get_context("spawn")
    rq = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_split_worker, args=(r, 2, port, q, k, v, D ** -0.5, rq)) for r in range(2)]
    for p in procs:
        p.start()
    res = [rq.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    ref = oracle.attn_ref64(q.numpy(), k.numpy(), v.numpy(), D ** -0.5)
    for rank, o in res:
        assert np.abs(o - ref).max() < 1e-4, rank
