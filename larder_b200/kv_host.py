"""The paged KV home on B200: the drop-in for kv_host.py's storage layout and its put / gather path
(kv_host.py:17-18, :36-41, :388-416, :612-648).

A `Home` keeps one cache's K and V in chunks of 2^LOGC (4096) positions, each chunk [K/V][Hk][4096][D] contiguous,
with a uint64 table of chunk addresses on the device (at most MAXC = 128 chunks: 524,288 positions). Chunks live
in device memory, or in pinned host memory that the GPU reads through its mapped address (the reference's
`MOE_KV_HOST` mode, where the card's memory goes to other uses). `put` appends rows (lb2_kvh_put); `decode` gathers a
QSA decode's picks from the home (lb2_kvh_gather, cache-bypassing loads) and runs the split-KV decode over them, as
the reference's `_AttnCache.decode` + `attn_cuda` do.

With `lru=True` a Home keeps the reference's VRAM LRU of picked blocks in front of it (kv_host.py:116-291,
:612-643, :748-775): a device pool of `lru_slots(nsel)` blocks. Each decode plans the token's picks by CLOCK
(lb2_kvh_lru_plan), then gathers them from the pool on a hit and from the home otherwise, filling the victims
(lb2_kvh_lru_gather, which also writes the new row into the home). `trim` drops the pool's blocks at or past the cut
(lb2_kvh_lru_inval).
"""
import torch

from . import ops

LOGC = 12     # positions a chunk, as a power of two
MAXC = 128    # chunks a home at most
LRU_MULT = 4  # pool blocks a layer, in multiples of the picks a token (the reference's MOE_KV_LRU default)
STATS = {"put": 0, "gathered": 0}


def lru_slots(nsel):
    """Pool blocks for nsel picks a token: LRU_MULT top-ks, at least one plan block's threads (kv_host.py:456-458)."""
    return max(LRU_MULT * nsel, (nsel + 31) // 32 * 32)


class Lru:
    """The pool [slots, 2, Hk, cr, D] and its int32 state on the device (kv_host.py:748-761): slot_of per block
    (-1), block_of, stamp (-1) and ref per slot, meta = (CLOCK hand, tokens, hits, misses)."""

    def __init__(self, hk, d, dtype, device, nsel, cr):
        self.nsel, self.cr = nsel, cr
        self.slots = lru_slots(nsel)
        i32 = dict(dtype=torch.int32, device=device)
        self.pool = torch.zeros((self.slots, 2, hk, cr, d), dtype=dtype, device=device)
        self.slot_of = torch.full(((MAXC << LOGC) // cr,), -1, **i32)
        self.block_of = torch.full((self.slots,), -1, **i32)
        self.stamp = torch.full((self.slots,), -1, **i32)
        self.ref = torch.zeros(self.slots, **i32)
        self.meta = torch.zeros(4, **i32)

    @property
    def nbytes(self):
        return sum(t.numel() * t.element_size() for t in (self.pool, self.slot_of, self.block_of, self.stamp,
                                                          self.ref, self.meta))


class Home:
    def __init__(self, hk, d, dtype, device, host=False, lru=False):
        self.hk, self.d, self.dtype = hk, d, dtype
        self.device = torch.device(device)
        self.host = host
        self.use_lru = lru
        self.lru = None
        self.chunks = []
        self.table = torch.zeros(MAXC, dtype=torch.int64, device=self.device)
        self.n = 0

    def _chunk(self):
        shape = (2, self.hk, 1 << LOGC, self.d)
        if self.host:
            return torch.empty(shape, dtype=self.dtype, pin_memory=True)  # pinned; mapped into the GPU's space
        return torch.empty(shape, dtype=self.dtype, device=self.device)

    def grow(self, n):
        """Room for n positions; False past MAXC chunks."""
        need = (n + (1 << LOGC) - 1) >> LOGC
        if need > MAXC:
            return False
        while len(self.chunks) < need:
            c = self._chunk()
            self.chunks.append(c)
            self.table[len(self.chunks) - 1] = c.data_ptr()
        return True

    def put(self, k, v):
        """Append k / v [1, Hk, s, D] as the next s positions."""
        s = k.shape[-2]
        if not self.grow(self.n + s):
            raise ValueError("kv_host: the home is full")
        ops.kvh_put(self.table, k, v, self.n, LOGC)
        self.n += s
        STATS["put"] += s

    def gather(self, tb, cr):
        """The picked rows (sorted blocks tb of cr positions, then the trailing partial block) from the home."""
        STATS["gathered"] += 1
        return ops.kvh_gather(self.table, tb.to(torch.int32), cr, self.n, self.hk, self.d, self.dtype, LOGC,
                              self.device)

    def decode_rows(self, k, v, tb, cr):
        """Append this position's k / v [1, Hk, 1, D] and return the picks' rows kg, vg [1, Hk, m, D]: through the
        LRU when the home has one (kv_host.py:612-643), else put + gather."""
        if not self.use_lru:
            self.put(k, v)
            return self.gather(tb, cr)
        tb = tb.reshape(-1).to(torch.int32)
        n = self.n + 1
        if not self.grow(n):
            raise ValueError("kv_host: the home is full")
        if self.lru is None or self.lru.nsel != tb.numel() or self.lru.cr != cr:
            self.lru = Lru(self.hk, self.d, self.dtype, self.device, tb.numel(), cr)
        sl = ops.kvh_lru_plan(tb, self.lru)
        kg, vg = ops.kvh_lru_gather(self.table, self.lru, tb, sl, cr, n, k, v, LOGC)
        self.n = n
        STATS["put"] += 1
        STATS["gathered"] += 1
        return kg, vg

    def decode(self, q, k, v, tb, cr, scale):
        """One decode row: append this position's k / v, then attend to the picks (kv_host.py:612-648's contract)."""
        kg, vg = self.decode_rows(k, v, tb, cr)
        return ops.attn_decode(q, kg, vg, scale)

    def trim(self, n):
        """Keep the first n positions; the LRU drops every block that holds one past them."""
        self.n = min(self.n, n)
        if self.lru is not None:
            ops.kvh_lru_inval(self.lru, self.n // self.lru.cr)


def report(homes=()):
    """Counters; with `homes`, the LRU hits and misses summed over their pools (one device read)."""
    out = dict(STATS)
    pools = [h.lru for h in homes if h.lru is not None]
    if pools:
        hm = torch.stack([p.meta[2:4] for p in pools]).sum(0).tolist()
        out.update(hits=hm[0], misses=hm[1], lru_blocks=max(p.slots for p in pools))
    return out
