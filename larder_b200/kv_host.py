"""The paged KV home on B200: the drop-in for kv_host.py's storage layout and its put / gather path
(kv_host.py:17-18, :36-41, :388-416, :612-648).

A `Home` keeps one cache's K and V in chunks of 2^LOGC (4096) positions, each chunk [K/V][Hk][4096][D] contiguous,
with a uint64 table of chunk addresses on the device (at most MAXC = 128 chunks: 524,288 positions). Chunks live
in device memory, or in pinned host memory that the GPU reads through its mapped address (the reference's
`MOE_KV_HOST` mode, where the card's memory goes to other uses). `put` appends rows (lb2_kvh_put); `decode` gathers a
QSA decode's picks from the home (lb2_kvh_gather, cache-bypassing loads) and runs the split-KV decode over them, as
the reference's `_AttnCache.decode` + `attn_cuda` do. The reference's VRAM LRU of picked blocks is not built: picks
are read straight from the home.
"""
import torch

from . import ops

LOGC = 12     # positions a chunk, as a power of two
MAXC = 128    # chunks a home at most
STATS = {"put": 0, "gathered": 0}


class Home:
    def __init__(self, hk, d, dtype, device, host=False):
        self.hk, self.d, self.dtype = hk, d, dtype
        self.device = torch.device(device)
        self.host = host
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

    def decode(self, q, k, v, tb, cr, scale):
        """One decode row: append this position's k / v, then attend to the picks (kv_host.py:612-648's contract)."""
        self.put(k, v)
        kg, vg = self.gather(tb, cr)
        return ops.attn_decode(q, kg, vg, scale)


def report():
    return dict(STATS)
