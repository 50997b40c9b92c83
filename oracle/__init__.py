"""CPU oracle for the attention / Gated-DeltaNet hot path -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs import this package, and only as the checker
(or as the timed CPU arm). The product package larder_b200 never imports it and has no CPU path.

Two layers:
  * liboracle.so (oracle.cpp): a C++ restatement of the reference's CPU kernels CpuAttn and CpuGdn
    (cpu_ext/cpu_kern.cpp:404-485, :493-659), OpenMP-threaded over all host cores, f32 arithmetic in the
    reference's order. This is the f32 oracle the GPU kernels are graded against and the timed CPU baseline.
  * attn_ref64 / gdn_ref64: float64 numpy restatements of the reference tests' own oracles
    (tests/test_cpu_kern.py:141-149 for attention, tests/test_gdn_cuda.py:29-45 for the recurrence), used to pin
    liboracle.so against the reference's tolerances (tests/test_cpu_kern.py:25, :129-133, :167-169).

Arrays are numpy. bf16 has no numpy dtype, so bf16 data travels as uint16 bit patterns (`BF16` marks them);
helpers convert with round-to-nearest-even as the reference does (cpu_kern.cpp:48-55).
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")

F32, BF16, F16 = 0, 1, 2
MASK_NONE, MASK_CAUSAL, MASK_ARRAY = 0, 1, 2

_lib = None


def build(force=False):
    """Compile liboracle.so with oracle/Makefile (g++ + OpenMP)."""
    if force or not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < os.path.getmtime(
            os.path.join(HERE, "oracle.cpp")):
        subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        p, i, f, i64p = ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.POINTER(ctypes.c_int64)
        L.orc_attn.argtypes = [p, i64p, i, p, i64p, i, p, i64p, i, p, i64p, p, i, i, i, i, i, i, i, i, f, i, i]
        L.orc_attn.restype = i
        L.orc_gdn.argtypes = [p, p, i, p, i, p, i, i, p, i, p, p, p, i, p, i, i, i, i, i, i, i]
        L.orc_gdn.restype = i
        L.orc_default_threads.restype = i
        _lib = L
    return _lib


def default_threads():
    """Threads the oracle uses by default: every host core it can see (the reference uses physical cores,
    cpu_kernels.py:14-22, :91)."""
    return int(lib().orc_default_threads())


# ---------------------------------------------------------------------------------------------- dtype helpers

def f32_to_bf16(x):
    """float32 array -> uint16 bf16 bit patterns, round to nearest even (NaN kept quiet)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    return np.where(nan, ((u >> 16) | 0x40).astype(np.uint16), r)


def bf16_to_f32(h):
    return (np.asarray(h, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def to_f32(a, dt):
    if dt == F32:
        return np.asarray(a, dtype=np.float32)
    if dt == BF16:
        return bf16_to_f32(a)
    return np.asarray(a).view(np.float16).astype(np.float32)


def from_f32(x, dt):
    """float32 -> the storage of dtype code dt (uint16 bits for bf16 and f16)."""
    if dt == F32:
        return np.ascontiguousarray(x, dtype=np.float32)
    if dt == BF16:
        return f32_to_bf16(x)
    return np.ascontiguousarray(x, dtype=np.float32).astype(np.float16).view(np.uint16)


def _ptr(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def _strides(a, n=3):
    """Element strides of the first n axes of a numpy array."""
    return (ctypes.c_int64 * n)(*[s // a.itemsize for s in a.strides[:n]])


# ---------------------------------------------------------------------------------------------- f32 oracle

def attn(q, k, v, scale, dt, mask_kind=MASK_NONE, mask=None, out_dt=None, threads=0):
    """softmax(scale q k^T + mask) v through liboracle.so (CpuAttn's arithmetic).

    q [B, Hq, T, D], k [B, Hkv, N, D], v [B, Hkv, N, Dv] numpy arrays in storage dtype `dt` (uint16 bits for
    bf16/f16); any strides with a unit last stride (slices of a longer cache buffer are fine). mask: bool [T, N]
    (kind 2). Returns [B, Hq, T, Dv] in storage dtype out_dt (default dt)."""
    out_dt = dt if out_dt is None else out_dt
    for a in (q, k, v):
        assert a.strides[-1] == a.itemsize, "last axis must have unit stride"
    B, Hq, T, D = q.shape
    Hkv, N, Dv = k.shape[1], k.shape[2], v.shape[3]
    o = np.zeros((B, Hq, T, Dv), dtype=np.float32 if out_dt == F32 else np.uint16)
    m8 = None
    ms = (ctypes.c_int64 * 2)(0, 0)
    if mask_kind == MASK_ARRAY:
        m8 = np.ascontiguousarray(mask, dtype=np.uint8).reshape(T, N)
        ms = (ctypes.c_int64 * 2)(N, 1)
    rc = lib().orc_attn(_ptr(q), _strides(q), dt, _ptr(k), _strides(k), dt, _ptr(v), _strides(v), dt, _ptr(m8), ms,
                        _ptr(o), out_dt, B, Hq, T, D, Hkv, N, Dv, float(scale), int(mask_kind), int(threads))
    if rc != 0:
        raise ValueError(f"oracle attn: unsupported shape {q.shape} {k.shape}")
    return o


def gdn(q, k, v, g, beta, state, dt, v_dt=None, g_dt=F32, b_dt=None, mask=None, threads=0):
    """The gated delta recurrence through liboracle.so (CpuGdn's arithmetic): returns (y, state_out).

    q, k [B, T, Hk, Dk] and v [B, T, Hv, Dv] in storage dtypes dt / v_dt; g [B, T, Hv] or [B, T, Hv, Dk] (g_dt);
    beta [B, T, Hv] (b_dt); state [B, Hv, Dv, Dk] float32; mask [B, T] bool or None. y comes back in dt."""
    v_dt = dt if v_dt is None else v_dt
    b_dt = dt if b_dt is None else b_dt
    q, k, v, g, beta = (np.ascontiguousarray(a) for a in (q, k, v, g, beta))
    state = np.ascontiguousarray(state, dtype=np.float32)
    B, T, Hk, Dk = q.shape
    Hv, Dv = v.shape[2], v.shape[3]
    y = np.zeros((B, T, Hv, Dv), dtype=np.float32 if dt == F32 else np.uint16)
    s = np.zeros_like(state)
    m8 = None if mask is None else np.ascontiguousarray(mask, dtype=np.uint8)
    rc = lib().orc_gdn(_ptr(q), _ptr(k), dt, _ptr(v), v_dt, _ptr(g), g_dt, int(g.ndim == 4), _ptr(beta), b_dt,
                       _ptr(m8), _ptr(state), _ptr(y), dt, _ptr(s), B, T, Hk, Dk, Hv, Dv, int(threads))
    if rc != 0:
        raise ValueError(f"oracle gdn: unsupported shape {q.shape} {v.shape}")
    return y, s


# ---------------------------------------------------------------------------------------------- float64 references

def attn_ref64(q, k, v, scale, mask=None):
    """tests/test_cpu_kern.py:141-149 in float64: q, k, v float arrays, mask bool [T, N] or None."""
    q, k, v = (np.asarray(a, dtype=np.float64) for a in (q, k, v))
    G = q.shape[1] // k.shape[1]
    k, v = np.repeat(k, G, 1), np.repeat(v, G, 1)
    s = scale * q @ np.swapaxes(k, -1, -2)
    if mask is not None:
        s = np.where(mask, s, -np.inf)
    mx = s.max(-1, keepdims=True)
    p = np.exp(s - np.where(np.isfinite(mx), mx, 0.0))
    den = p.sum(-1, keepdims=True)
    return (p / np.where(den > 0, den, 1.0)) @ v


def causal_mask(T, N):
    """Bottom-right causal: row t sees keys 0 .. N - T + t (tests/test_cpu_kern.py:159)."""
    return np.arange(T)[:, None] + N - T >= np.arange(N)[None, :]


def gdn_ref64(q, k, v, g, beta, state, mask=None):
    """tests/test_gdn_cuda.py:29-45 in float64: masked steps skipped (y = 0, state kept)."""
    q, k, v, g, beta, s = (np.asarray(x, dtype=np.float64) for x in (q, k, v, g, beta, state))
    B, T, Hk, Dk = q.shape
    r = v.shape[2] // Hk
    q, k = np.repeat(q, r, axis=2), np.repeat(k, r, axis=2)
    m = np.ones((B, T), bool) if mask is None else np.asarray(mask, bool)
    ys = np.zeros(v.shape)
    for t in range(T):
        gt = g[:, t]
        sn = s * (gt[..., None, None] if gt.ndim == 2 else gt[..., None, :])
        kv = (sn * k[:, t, :, None, :]).sum(-1)
        sn = sn + k[:, t, :, None, :] * ((v[:, t] - kv) * beta[:, t, :, None])[..., None]
        y = (sn * q[:, t, :, None, :]).sum(-1)
        s = np.where(m[:, t, None, None, None], sn, s)
        ys[:, t] = np.where(m[:, t, None, None], y, 0.0)
    return ys, s


# ---------------------------------------------------------------------------------------------- seeded inputs

def rms_norm(x, eps=1e-6):
    """mx.fast.rms_norm(x, None, eps) over the last axis, float32."""
    x = np.asarray(x, dtype=np.float32)
    return x / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + np.float32(eps))


def softplus(x):
    x = np.asarray(x, dtype=np.float64)
    return np.where(x > 20, x, np.log1p(np.exp(np.minimum(x, 20))))


def compute_g(A_log, a, dt_bias):
    """mlx_lm's compute_g, g = exp(-exp(A_log) * softplus(a + dt_bias)) (spelled out in gdn_cuda.py:146-149)."""
    return np.exp(-np.exp(np.asarray(A_log, np.float64)) * softplus(np.asarray(a, np.float64) +
                                                                      np.asarray(dt_bias, np.float64))).astype(np.float32)


def sigmoid(x):
    return (1.0 / (1.0 + np.exp(-np.asarray(x, dtype=np.float64)))).astype(np.float32)


# ---------------------------------------------------------------------------------------------- attention glue

def _bf(x):
    """float32 values rounded to bf16 (nearest even), kept as float32."""
    return bf16_to_f32(f32_to_bf16(np.asarray(x, dtype=np.float32)))


def qk_norm_rope(qg, kr, qw, kw, eps, cs, sn, NQ, NK):
    """The reference's qk kernel (layer_glue.py:241-286) restated on the CPU, bf16 as uint16 bits.

    qg [B, S, NQ * 2D] (each query head's D values, then its D gate values), kr [B, S, NK * D], qw / kw [D];
    cs / sn [S, R] float32 (the kernel casts them to bf16). For each head row x: inv = 1 / sqrt(sum(x^2) / D + eps),
    o = bf16(w * bf16(x * inv)); on the first R dims r = bf16(bf16(o * bf16(cos)) + bf16(rot * bf16(sin))) with
    rot = (-o[R/2:R], o[:R/2]). Returns q [B, NQ, S, D] and k [B, NK, S, D] bf16 bits. The sum of squares runs in
    float64 here, the reference's in an fp32 tree: where x * inv sits on a bf16 rounding boundary the two can
    differ by one bf16 step."""
    qg, kr = np.asarray(qg, np.uint16), np.asarray(kr, np.uint16)
    B, S = qg.shape[:2]
    D = qg.shape[-1] // (2 * NQ)
    cs, sn = np.asarray(cs, np.float32).reshape(S, -1), np.asarray(sn, np.float32).reshape(S, -1)
    R = cs.shape[-1]
    c, s_ = _bf(cs)[None, :, None, :], _bf(sn)[None, :, None, :]

    def rows(x, w):
        ms = (x.astype(np.float64) ** 2).sum(-1, keepdims=True) / D
        inv = (np.float32(1) / np.sqrt((ms.astype(np.float32) + np.float32(eps)).astype(np.float32))).astype(np.float32)
        o = _bf(bf16_to_f32(w) * _bf(x * inv))
        if R:
            rot = np.concatenate([-o[..., R // 2:R], o[..., :R // 2]], axis=-1)
            o = o.copy()
            o[..., :R] = _bf(_bf(o[..., :R] * c) + _bf(rot * s_))
        return np.ascontiguousarray(o.transpose(0, 2, 1, 3))

    xq = bf16_to_f32(qg).reshape(B, S, NQ, 2 * D)[..., :D]
    xk = bf16_to_f32(kr).reshape(B, S, NK, D)
    return f32_to_bf16(rows(xq, qw)), f32_to_bf16(rows(xk, kw))


def out_gate(o, qg, NQ):
    """The reference's agate kernel (layer_glue.py:288-296) restated: out = bf16(o * bf16(sigmoid(gate))), gate the
    second half of each head's 2D columns of qg; o [..., NQ * D], qg [..., NQ * 2D], bf16 bits."""
    o, qg = np.asarray(o, np.uint16), np.asarray(qg, np.uint16)
    D = o.shape[-1] // NQ
    g = bf16_to_f32(qg).reshape(-1, NQ, 2 * D)[..., D:]
    sig = _bf(sigmoid(g))
    return f32_to_bf16(bf16_to_f32(o).reshape(-1, NQ, D) * sig).reshape(o.shape)


# ---------------------------------------------------------------------------------------------- QSA block selection

def qsa_select(q, pooled, offset, cr, k, div):
    """The indexer's scores and top-k (qwen4_exp_vendor.py:271-292) in float64, bf16 inputs as uint16 bits: q
    [B, S, H, D], pooled [B, n_blocks, D]. Returns (top [B, S, k] int ascending, ties lowest index first, padded
    with n_blocks; scores [B, S, n_blocks] float64 with -inf for blocks not yet complete)."""
    qf = bf16_to_f32(q).astype(np.float64)
    pf = bf16_to_f32(pooled).astype(np.float64)
    B, S, H, D = qf.shape
    nb = pf.shape[1]
    sc = np.maximum(np.einsum("bshd,bnd->bsnh", qf, pf), 0).sum(-1) / div
    n_complete = np.maximum(offset + np.arange(S) + 1, 0) // cr
    sc = np.where(np.arange(nb)[None, None, :] < n_complete[None, :, None], sc, -np.inf)
    top = np.full((B, S, k), nb, dtype=np.int64)
    for b in range(B):
        for s in range(S):
            fin = np.isfinite(sc[b, s])
            kk = min(k, int(fin.sum()))
            order = np.argsort(-sc[b, s], kind="stable")[:kk]
            top[b, s, :kk] = np.sort(order)
    return top, sc


# ---------------------------------------------------------------------------------------------- KV home's VRAM LRU

def lru_plan(tb, slot_of, block_of, stamp, ref, meta, ns):
    """One token's plan of the reference's LRU (kv_host.py:116-185), restated over its rounds; the int32 state arrays
    are updated in place. Returns sl [nsel]: the hit's slot, -2 - victim, or -1.

    Hits take this token's stamp t = meta[1] + 1 and their reference bit. Each round looks at NT = ceil32(nsel)
    consecutive slots from hand + scanned: a slot is protected when stamped t, eligible when not protected and its
    bit is clear. Eligible slots are taken in order while victims are still needed; if the round supplies the last
    victim it ends there (cut = that slot's place), else it covers all NT slots; unprotected, non-eligible slots up to
    the cut lose their bit. The scan stops when every miss has a victim or after 2 ns + NT slots. The i-th miss (in
    pick order) takes the i-th victim, evicting the victim's block."""
    tb = np.asarray(tb, np.int64)
    nsel = tb.size
    nt = (nsel + 31) // 32 * 32
    t = int(meta[1]) + 1
    s = slot_of[tb].astype(np.int64)
    hit = s >= 0
    stamp[s[hit]] = t
    ref[s[hit]] = 1
    miss = ~hit
    M = int(miss.sum())
    hand, found, scanned = int(meta[0]), 0, 0
    victims = []
    lanes = np.arange(nt)
    while found < M and scanned < 2 * ns + nt:
        xs = (hand + scanned + lanes) % ns
        prot = stamp[xs] == t
        elig = ~prot & (ref[xs] == 0)
        need = M - found
        idx = np.flatnonzero(elig)
        take = min(idx.size, need)
        cut = int(idx[take - 1]) if take == need else nt - 1
        chosen = xs[idx[:take]]
        victims.extend(int(x) for x in chosen)
        stamp[chosen] = t
        passed = (lanes <= cut) & ~prot & ~elig
        ref[xs[passed]] = 0
        found += take
        scanned += cut + 1
    sl = np.full(nsel, -1, np.int32)
    r = 0
    for j in range(nsel):
        if hit[j]:
            sl[j] = s[j]
            continue
        if r < found:
            x = victims[r]
            old = int(block_of[x])
            if old >= 0:
                slot_of[old] = -1
            block_of[x] = tb[j]
            slot_of[tb[j]] = x
            ref[x] = 0
            sl[j] = -2 - x
        r += 1
    meta[0] = (hand + scanned) % ns
    meta[1] = t
    meta[2] += nsel - M
    meta[3] += M
    return sl


def lru_gather(k, v, pool, tb, sl, cr, n):
    """The token's rows through the LRU (kv_host.py:187-257): k / v [Hk, >= n, D] hold the sequence's positions
    (n - 1 the new one), pool [ns, 2, Hk, cr, D] is updated in place (a miss with a victim fills it). Row r < nsel cr
    is position tb[r / cr] cr + r % cr, from the pool on a hit (sl >= 0), else from k / v; then the trailing partial
    block. Returns kg, vg [Hk, m, D]."""
    tb = np.asarray(tb, np.int64)
    nsel = tb.size
    own0 = n // cr * cr
    m = nsel * cr + n - own0
    Hk, D = k.shape[0], k.shape[2]
    out = [np.zeros((Hk, m, D), k.dtype), np.zeros((Hk, m, D), k.dtype)]
    for r in range(m):
        slot = vic = -1
        if r >= nsel * cr:
            pos = own0 + r - nsel * cr
        else:
            pos = int(tb[r // cr]) * cr + r % cr
            c = int(sl[r // cr])
            slot = c if c >= 0 else -1
            vic = -2 - c if c <= -2 else -1
        for kv, src in enumerate((k, v)):
            x = pool[slot, kv, :, r % cr] if (slot >= 0 and pos != n - 1) else src[:, pos]
            out[kv][:, r] = x
            if vic >= 0:
                pool[vic, kv, :, r % cr] = x
    return out[0], out[1]


def lru_inval(slot_of, block_of, ref, lim):
    """Slots holding a block >= lim drop it (kv_host.py:259-276), in place."""
    for x in range(block_of.size):
        b = int(block_of[x])
        if b >= 0 and b >= lim:
            slot_of[b] = -1
            block_of[x] = -1
            ref[x] = 0
