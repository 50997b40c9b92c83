"""Multi-GPU layer: one process per GPU, torch.distributed (NCCL over NVLink / NVSwitch) for the plumbing.

The reference is single-process and single-GPU (no collective exists in it); the hot path partitions two ways:

  * prefill by independent sequences: rank r of R takes its contiguous share of the batch and runs the prefill
    kernel on it locally -- no exchange at all (weak scaling). `sequence_shard` gives the share.
  * long-context decode by KV range: each sequence's KV cache is cut into R contiguous ranges, one per rank,
    resident on that rank. Each rank computes its range's normalised partial output and log-sum-exp
    (lb2_attn_decode_partial, written straight into a packed [o rows | lse] buffer), the ranks exchange them with one
    all-gather of that buffer (about B * Hq * T * (D + 1) * 4 bytes a rank), and every rank merges the gathered
    blocks in place with the log-sum-exp combine kernel (lb2_attn_combine_packed): o = sum_r exp(lse_r - lse*) o_r / sum_r exp(lse_r - lse*), the merge of foldattn_merge
    (foldattn.py:188-211) and cpu_kern.cpp:607-628 taken across GPUs.

`PeerExchange` is the same decode without a collective on the data path: each rank's partial lands in its own
exchange buffer, shared with the other ranks through CUDA IPC, and lb2_attn_combine_peers merges all ranks' partials
read in place over NVLink, after a flag each rank publishes into every peer's buffer (bounded waits).

`partial_fn(q, k, v, scale, kv_len, part_o, part_lse)` fills a rank's partial into the two parts of its packed buffer
and `combine_fn(gathered [world, rows * (D + 1)], (B, Hq, T, D), dtype)` merges the gathered blocks in place; both
default to this package's CUDA entry points (lb2_attn_decode_partial, lb2_attn_combine_packed). Tests on CPU ranks
(gloo) pass the CPU oracle instead, as the checker of the exchange itself.
"""
import ctypes
import datetime

import torch
import torch.distributed as dist

from . import ops
from ._lib import check, i64, lib


def init(backend="nccl", timeout_s=60, device=None):
    """Initialise the process group from the torchrun environment with a short timeout, so that ranks waiting on a
    rank that died end with an error instead of waiting for good. Returns (rank, world)."""
    if not dist.is_initialized():
        kw = {"timeout": datetime.timedelta(seconds=timeout_s)}
        if backend == "nccl" and device is not None:
            kw["device_id"] = device
        dist.init_process_group(backend, **kw)
    return dist.get_rank(), dist.get_world_size()


def sequence_shard(n_seq, rank, world):
    """[start, stop) of the sequences rank `rank` of `world` prefills: contiguous blocks, the first n_seq % world
    ranks one longer."""
    base, extra = divmod(n_seq, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def kv_range(n_keys, rank, world):
    """[start, stop) of the keys of a sequence rank `rank` holds: contiguous ranges (config 5's 8 x 4096 of 32768)."""
    return sequence_shard(n_keys, rank, world)


def _cuda_partial(q, k, v, scale, kv_len, part_o, part_lse):
    ops.attn_decode_partial(q, k, v, scale, kv_len=kv_len, out=(part_o, part_lse))


def _cuda_combine(gathered, shape, dtype):
    B, Hq, T, D = shape
    return ops.attn_combine_packed(gathered, gathered.shape[0], B, Hq, T, D, dtype)


def kv_sharded_decode(q, k_local, v_local, scale, kv_len_local=None, group=None, partial_fn=None, combine_fn=None,
                      out_dtype=None):
    """Decode attention over a KV cache whose key range is split across the ranks of `group`.

    q [B, Hq, T, D] (the same on every rank), k_local / v_local [B, Hkv, n_local, D] this rank's contiguous range,
    kv_len_local int32 [B] (keys of the range each sequence fills, or None). Every query row must see every key of
    every range (decode rows lie after the whole cache). Returns o [B, Hq, T, D] on every rank."""
    partial_fn = partial_fn or _cuda_partial
    combine_fn = combine_fn or _cuda_combine
    world = dist.get_world_size(group)
    B, Hq, T, D = q.shape
    rows = B * Hq * T
    # the partial lands packed in one buffer, [o rows | lse], the all-gather's input as it stands
    packed = torch.empty(rows * (D + 1), dtype=torch.float32, device=q.device)
    partial_fn(q, k_local, v_local, scale, kv_len_local, packed[:rows * D].view(B, Hq, T, D),
               packed[rows * D:].view(B, Hq, T))
    gathered = torch.empty(world * rows * (D + 1), dtype=torch.float32, device=q.device)
    dist.all_gather_into_tensor(gathered, packed, group=group)
    return combine_fn(gathered.view(world, rows * (D + 1)), (B, Hq, T, D), out_dtype or q.dtype)


def _cuda_merge(part_o, part_lse, dtype):
    return ops.attn_combine(part_o, part_lse, dtype)


def kv_sharded_decode_split(q, k_local, v_local, scale, kv_len_local=None, group=None, partial_fn=None,
                            merge_fn=None, out_dtype=None):
    """kv_sharded_decode with the merge split by sequences instead of repeated on every rank: rank r merges only the
    sequences [r B / R, (r + 1) B / R) (the same log-sum-exp merge), then the merged rows are all-gathered. The
    exchange is an all-to-all of the partials (each rank receives 1/R of every peer's partial: about
    B Hq T (D + 1) 4 (R - 1) / R bytes, against (R - 1) times the whole partial for the all-gather) and an all-gather
    of the output rows in q's dtype. B must be a multiple of the group's size. `partial_fn` as kv_sharded_decode's;
    `merge_fn(part_o [R, B / R, Hq, T, D], part_lse [R, B / R, Hq, T], dtype)` defaults to lb2_attn_combine."""
    partial_fn = partial_fn or _cuda_partial
    merge_fn = merge_fn or _cuda_merge
    world = dist.get_world_size(group)
    B, Hq, T, D = q.shape
    if B % world:
        raise ValueError("kv_sharded_decode_split: the batch must be a multiple of the ranks")
    rows = B * Hq * T
    part_o = torch.empty(rows * D, dtype=torch.float32, device=q.device)
    part_lse = torch.empty(rows, dtype=torch.float32, device=q.device)
    partial_fn(q, k_local, v_local, scale, kv_len_local, part_o.view(B, Hq, T, D), part_lse.view(B, Hq, T))
    got_o = torch.empty_like(part_o)
    got_lse = torch.empty_like(part_lse)
    dist.all_to_all_single(got_o, part_o, group=group)      # block r of each rank: the sequences rank r merges
    dist.all_to_all_single(got_lse, part_lse, group=group)
    b = B // world
    mine = merge_fn(got_o.view(world, b, Hq, T, D), got_lse.view(world, b, Hq, T), out_dtype or q.dtype)
    o = torch.empty((B, Hq, T, D), dtype=mine.dtype, device=q.device)
    dist.all_gather_into_tensor(o, mine, group=group)
    return o


def sharded_prefill(q, k, v, scale, mask="causal", gate=None, rank=None, world=None):
    """Prefill of a batch of independent sequences, this rank's share only: q [B, Hq, T, D], k / v [B, Hkv, N, D]
    (the whole batch's views; only this rank's rows are read). Returns (start, stop, o_local)."""
    rank = dist.get_rank() if rank is None else rank
    world = dist.get_world_size() if world is None else world
    s0, s1 = sequence_shard(q.shape[0], rank, world)
    g = None if gate is None else gate[s0:s1]
    return s0, s1, ops.attn_prefill(q[s0:s1], k[s0:s1], v[s0:s1], scale, mask, gate=g)


class PeerExchange:
    """KV-range-sharded decode over NVLink peer memory for one decode shape (B, Hq, T, D) on the ranks of `group`
    (at most 8, one GPU each, all on one NVSwitch node). Every rank builds it with the same shape, calls `decode` the
    same number of times in the same order, and calls `close` at the end (all ranks)."""

    def __init__(self, B, Hq, T, D, group=None, push=False):
        """push=True: every rank's partial is stored straight into every rank's buffer by its decode kernel
        (lb2_attn_decode_push) and the merge reads only local memory (lb2_attn_combine_pushed); else each rank
        keeps its partial and the merge reads the peers' over NVLink (lb2_attn_combine_peers)."""
        self.group = group
        self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        if self.world > 8:
            raise ValueError("PeerExchange: at most 8 ranks")
        self.shape = (B, Hq, T, D)
        self.push = push
        self.rows = B * Hq * T
        self.half = self.rows * (D + 1)
        L = lib()
        ptr = ctypes.c_void_p()
        nbytes = L.lb2_xch_push_bytes(self.world, B, Hq, T, D) if push else L.lb2_xch_bytes(B, Hq, T, D)
        check(L.lb2_xch_alloc(nbytes, ctypes.byref(ptr)), "xch_alloc")
        self.base = ptr.value
        handle = ctypes.create_string_buffer(64)
        check(L.lb2_xch_handle(ctypes.c_void_p(self.base), handle), "xch_handle")
        handles = [None] * self.world
        dist.all_gather_object(handles, handle.raw, group=group)
        self.opened, bufs, err = [], [], ""
        for r, h in enumerate(handles):
            if r == self.rank:
                bufs.append(self.base)
                continue
            p = ctypes.c_void_p()
            rc = L.lb2_xch_open(ctypes.create_string_buffer(h, 64), ctypes.byref(p))
            if rc:
                err = L.lb2_error().decode()
                break
            self.opened.append(p.value)
            bufs.append(p.value)
        # every rank mapped every peer, or all give up together (none goes on to a step the others left)
        dev = torch.device("cpu") if dist.get_backend(group) == "gloo" else \
            torch.device("cuda", torch.cuda.current_device())
        ok = torch.tensor([0 if err else 1], dtype=torch.int32, device=dev)
        dist.all_reduce(ok, op=dist.ReduceOp.MIN, group=group)
        if not int(ok.item()):
            for p in self.opened:
                L.lb2_xch_close(ctypes.c_void_p(p))
            L.lb2_xch_free(ctypes.c_void_p(self.base))
            self.base, self.opened = None, []
            raise RuntimeError(f"PeerExchange: a rank could not map its peers' buffers ({err or 'another rank'})")
        self.bufs = (ctypes.c_uint64 * self.world)(*bufs)
        self.epoch = 0

    def decode(self, q, k_local, v_local, scale, kv_len_local=None, out_dtype=None):
        """As kv_sharded_decode: o [B, Hq, T, D] on every rank, from this rank's key range k_local / v_local."""
        B, Hq, T, D = q.shape
        if (B, Hq, T, D) != self.shape:
            raise ValueError(f"PeerExchange: built for {self.shape}, called with {(B, Hq, T, D)}")
        self.epoch += 1
        o = torch.empty((B, Hq, T, D), dtype=out_dtype or q.dtype, device=q.device)
        if self.push:
            ops.decode_push(q, k_local, v_local, scale, kv_len_local, 0, self.bufs, self.world, self.rank, self.epoch)
            rc = lib().lb2_attn_combine_pushed(self.bufs, self.world, self.rank, self.epoch, B, Hq, T, D,
                                               ops._ptr(o), i64(*o.stride()[:3]), ops.dtype_code(o), ops._stream(o))
            check(rc, "attn_combine_pushed")
            return o
        o_ptr = self.base + (self.epoch & 1) * self.half * 4
        ops.decode_partial_into(q, k_local, v_local, scale, kv_len_local, 0, o_ptr, o_ptr + self.rows * D * 4)
        rc = lib().lb2_attn_combine_peers(self.bufs, self.world, self.rank, self.epoch, B, Hq, T, D, ops._ptr(o),
                                          i64(*o.stride()[:3]), ops.dtype_code(o), ops._stream(o))
        check(rc, "attn_combine_peers")
        return o

    def close(self):
        """Unmap the peers' buffers and free this rank's, once every rank's kernels are done with them."""
        if self.base is None:
            return
        if torch.cuda.is_available():
            torch.cuda.synchronize()
        dist.barrier(group=self.group)
        for p in self.opened:
            check(lib().lb2_xch_close(ctypes.c_void_p(p)), "xch_close")
        dist.barrier(group=self.group)
        check(lib().lb2_xch_free(ctypes.c_void_p(self.base)), "xch_free")
        self.base, self.opened = None, []
