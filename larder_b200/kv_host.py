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

`make_class(base)` and `install(q4, switch, nsel, cr, hk, d, dtype)` are the reference's drop-in surface
(kv_host.py:516-799): the caller's attention cache class (mlx_lm's KVCache contract: `keys`, `values`, `offset`,
`step`, `update_and_fetch(keys, values)`) gets a subclass that behaves as the base below H positions and keeps its
K / V in a Home from there on, with `decode(k, v, tb, cr)` for a QSA decode row through the LRU.
"""
import os
import weakref

import torch

from . import ops

LOGC = 12     # positions a chunk, as a power of two
MAXC = 128    # chunks a home at most
LRU_MULT = 4  # pool blocks a layer, in multiples of the picks a token (the reference's MOE_KV_LRU default)
STATS = {"put": 0, "gathered": 0, "staged": 0}
H = 1 << 62   # positions from which a cache of the installed class keeps its K / V in a Home (install sets it)
NSEL = CR = None
HOST = True   # homes in pinned host memory (the reference's mode); LB2_KV_HOME=device keeps them in device memory
CLS = BASE = None
ROW_BYTES = 0
_HOMED = weakref.WeakSet()


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


def report(homes=None):
    """Counters; the LRU hits and misses summed over the pools of `homes` (default: the homes of every cache of the
    installed class alive now), one device read."""
    out = dict(STATS)
    if homes is None:
        homes = [c.home for c in list(_HOMED) if c.home is not None]
    out["homed"] = len(homes)
    pools = [h.lru for h in homes if h.lru is not None]
    if pools:
        hm = torch.stack([p.meta[2:4] for p in pools]).sum(0).tolist()
        out.update(hits=hm[0], misses=hm[1], lru_blocks=max(p.slots for p in pools))
    return out


# --------------------------------------------------------------------------------- the cache class


def _stage(home, n):
    """K and V [1, Hk, n, D] holding the home's positions 0 .. n - 1 (one gather of whole chunks plus the tail)."""
    if n == 0:
        z = torch.empty((1, home.hk, 0, home.d), dtype=home.dtype, device=home.device)
        return z, z.clone()
    full = torch.arange(n >> LOGC, dtype=torch.int32, device=home.device)
    STATS["staged"] += n
    return ops.kvh_gather(home.table, full, 1 << LOGC, n, home.hk, home.d, home.dtype, LOGC, home.device)


def make_class(base):
    """The caller's attention cache class with the home (kv_host.py:516-773): below H positions it is `base`
    itself (its own buffer and growth); a pass that takes it to H or past moves its rows into a Home and keeps them
    there, every later pass appending to the home. `update_and_fetch` then returns views of a staged copy of the
    rows (kept while passes follow one another, re-staged after a trim), and `decode(k, v, tb, cr)` takes one QSA
    decode row: the row is appended and the picks come back through the LRU, without staging anything."""

    class _AttnCache(base):
        __doc__ = base.__doc__
        _k = _v = None
        _off = 0
        home = None
        scratch = None  # (k, v) staged rows 0 .. offset - 1 of a homed cache

        @property
        def keys(self):
            return self._k if self.home is None else self._staged()[0]

        @keys.setter
        def keys(self, a):
            self._leave()
            self._k = a

        @property
        def values(self):
            return self._v if self.home is None else self._staged()[1]

        @values.setter
        def values(self, a):
            self._leave()
            self._v = a

        @property
        def offset(self):
            return self._off

        @offset.setter
        def offset(self, n):
            # positions given back are rewritten later: the home and its LRU forget them now
            if self.home is not None and n < self._off:
                self.home.trim(n)
                self.scratch = None
            self._off = n

        @property
        def kv_host(self):
            return self.home is not None

        @property
        def nbytes(self):
            if self.home is None:
                return super().nbytes
            sc = 0 if self.scratch is None else sum(t.numel() * t.element_size() for t in self.scratch)
            return sc + (0 if self.home.lru is None else self.home.lru.nbytes)

        def empty(self):
            return self.home is None and self._k is None

        def update_and_fetch(self, keys, values):
            s = keys.shape[2]
            if self.home is None:
                if self._off + s < H or not self._enter(keys):
                    return super().update_and_fetch(keys, values)
            prev = self._off
            if self.home.n != prev:
                self.home.trim(prev)
            self.home.put(keys, values)
            sc = self.scratch
            if sc is not None and sc[0].shape[2] == prev:
                sc = (torch.cat([sc[0], keys], dim=2), torch.cat([sc[1], values], dim=2))
            else:
                sc = _stage(self.home, prev + s)
            self.scratch = sc
            self._off = prev + s
            return sc

        def decode(self, k, v, tb, cr):
            """One decode row on the sorted picks tb (stream_fast.py's attn_cuda pass, kv_host.py:612-648): the
            row k / v [1, Hk, 1, D] appended, then (kg, vg) [1, Hk, m, D] as _qsa_gather gives them over the cache
            with the row. None while the cache is under H: the caller takes its flag-off path."""
            if self.home is None:
                if self._off + 1 < H or not self._enter(k):
                    return None
            if self.home.n != self._off:
                self.home.trim(self._off)
            self.scratch = None
            kg, vg = self.home.decode_rows(k, v, tb, cr)
            self._off += 1
            return kg, vg

        def _enter(self, keys):
            """Into a Home, the rows held so far copied there; False keeps the cache as the base (B > 1)."""
            if keys.shape[0] != 1:
                return False
            home = Home(keys.shape[1], keys.shape[3], keys.dtype, keys.device, host=HOST and keys.is_cuda,
                        lru=NSEL is not None)
            if self._k is not None and self._off:
                home.put(self._k[:, :, :self._off], self._v[:, :, :self._off])
            self._k = self._v = None
            self.home = home
            _HOMED.add(self)
            return True

        def _leave(self):
            self.home = None
            self.scratch = None
            _HOMED.discard(self)

        def _staged(self):
            if self.scratch is None or self.scratch[0].shape[2] != self._off:
                self.scratch = _stage(self.home, self._off)
            return self.scratch

    _AttnCache.__qualname__ = base.__qualname__
    _AttnCache.__name__ = base.__name__
    return _AttnCache


def install(q4, switch, nsel, cr, hk, d, dtype):
    """Put the homed cache in place of `q4._AttnCache` (the model module's attention cache class) for every cache
    made from now on, homed from max(switch, twice the positions the LRU holds) (kv_host.py:776-799). Returns whether
    it is on: False for more than 1024 picks a token (the plan kernel's limit). MOE_KV_HOST_FROM overrides the line
    (the reference's switch); LB2_KV_HOME=device keeps homes in device memory instead of pinned host memory."""
    global H, NSEL, CR, CLS, BASE, ROW_BYTES, HOST
    if CLS is not None:
        return True
    if nsel > 1024:
        return False
    BASE = q4._AttnCache
    CLS = q4._AttnCache = make_class(BASE)
    ROW_BYTES = 2 * hk * d * torch.empty((), dtype=dtype).element_size()
    NSEL, CR = nsel, cr
    H = max(int(switch), 2 * lru_slots(nsel) * cr)
    if os.environ.get("MOE_KV_HOST_FROM"):
        H = int(os.environ["MOE_KV_HOST_FROM"])
    HOST = os.environ.get("LB2_KV_HOME", "host") != "device"
    return True


def uninstall(q4):
    """Put the base class back (tests, and callers that switch the mode off)."""
    global CLS, BASE, H, NSEL, CR
    if CLS is not None and q4._AttnCache is CLS:
        q4._AttnCache = BASE
    CLS = BASE = NSEL = CR = None
    H = 1 << 62
