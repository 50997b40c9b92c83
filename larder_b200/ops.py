"""torch-facing wrappers of the C-ABI entry points: shape/dtype/stride checks, output and workspace allocation,
the caller's current CUDA stream. Every function here runs a CUDA kernel of liblarder_b200; none has a CPU path.

Tensors follow the reference's layouts (mlx_lm's): attention q [B, Hq, T, D] (often a transposed view of
[B, T, Hq, D]), k / v [B, Hkv, N, D] (often slices of a capacity-padded cache buffer); Gated-DeltaNet q / k
[B, T, Hk, Dk], v [B, T, Hv, Dv], state [B, Hv, Dv, Dk] fp32.
"""
import ctypes

import torch

from . import _lib
from ._lib import check, i64, lib

_DT = {torch.float32: _lib.F32, torch.bfloat16: _lib.BF16, torch.float16: _lib.F16}
_WS = {}  # (device index, tag) -> uint8 workspace, grown on demand


def dtype_code(t):
    try:
        return _DT[t.dtype]
    except KeyError:
        raise ValueError(f"unsupported dtype {t.dtype}") from None


def _cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("larder_b200 runs on CUDA tensors only (no CPU path)")


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _stream(t):
    """The caller's current CUDA stream on t's device, as the cudaStream_t handle (an int) the C ABI takes."""
    if _raw_stream is not None:
        return _raw_stream(t.device.index)
    return torch.cuda.current_stream(t.device).cuda_stream


def _ptr(t):
    """A tensor's device address as the C ABI's void* (None for NULL); the argtypes convert plain ints."""
    return None if t is None else t.data_ptr()


def _unit_last(t, name):
    if t.stride(-1) != 1:
        raise ValueError(f"{name}: the last axis must have unit stride")


def workspace(device, nbytes, tag):
    """A 256-byte aligned uint8 buffer of at least nbytes on device, kept per (device, tag) and reused by later
    calls on the same stream."""
    key = (device.index if device.index is not None else torch.cuda.current_device(), tag)
    ws = _WS.get(key)
    if ws is None or ws.numel() < nbytes:
        buf = torch.zeros(max(int(nbytes), 256) + 256, dtype=torch.uint8, device=device)
        ws = buf[(-buf.data_ptr()) % 256:]
        _WS[key] = ws
    return ws


def status(device=None):
    """Synchronise the current stream and return (and clear) the library's device status word (0 = ok)."""
    dev = torch.device("cuda", torch.cuda.current_device() if device is None else device)
    return lib().lb2_status(ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream))


# ---------------------------------------------------------------------------------------------------- attention

def attn_prefill(q, k, v, scale, mask=None, gate=None, out=None):
    """softmax(scale q k^T + mask) v [* sigmoid(gate)] on tcgen05 tensor cores.

    mask: None, "causal" (bottom-right) or a bool tensor broadcastable from [T, N] (leading dims of 1)."""
    _cuda(q, k, v, gate)
    for t, n in ((q, "q"), (k, "k"), (v, "v")):
        _unit_last(t, n)
    B, Hq, T, D = q.shape
    Hkv, N = k.shape[1], k.shape[2]
    if k.dtype != q.dtype or v.dtype != q.dtype:
        raise ValueError("q, k, v must share a dtype")
    if v.shape[-1] != D:
        raise ValueError("v's head dim must equal q's")
    if out is None:
        out = torch.empty((B, Hq, T, D), dtype=q.dtype, device=q.device)
    kind, m, mst = _lib.MASK_NONE, None, i64(0, 0)
    if isinstance(mask, str):
        if mask != "causal":
            raise ValueError(f"unsupported mask {mask!r}")
        kind = _lib.MASK_CAUSAL
    elif mask is not None:
        if mask.dtype != torch.bool or tuple(mask.shape[-2:]) != (T, N) or any(d != 1 for d in mask.shape[:-2]):
            raise ValueError("array masks must be bool [..., T, N] with leading dims of 1")
        m = mask.reshape(T, N).view(torch.uint8)  # (bool and uint8 share a byte layout: no copy, strides kept)
        kind, mst = _lib.MASK_ARRAY, i64(m.stride(0), m.stride(1))
    gst = i64(0, 0, 0)
    if gate is not None:
        if gate.shape != (B, Hq, T, D) or gate.dtype != q.dtype:
            raise ValueError("gate must be [B, Hq, T, D] in q's dtype")
        _unit_last(gate, "gate")
        gst = i64(*gate.stride()[:3])
    rc = lib().lb2_attn_prefill(_ptr(q), i64(*q.stride()[:3]), _ptr(k), i64(*k.stride()[:3]), _ptr(v),
                                i64(*v.stride()[:3]), _ptr(out), i64(*out.stride()[:3]), _ptr(gate), gst,
                                _ptr(m), mst, B, Hq, Hkv, T, N, D, dtype_code(q), float(scale), kind, _stream(q))
    check(rc, "attn_prefill")
    return out


def attn_prefill_tiled(q, k, v, scale, mask, gate=None, out=None):
    """attn_prefill with a bool array mask [..., T, N] and tile skipping: only the key tiles that some row of a row
    block keeps are read and multiplied (lb2_attn_prefill_tiled). Same result as attn_prefill(..., mask)."""
    _cuda(q, k, v, gate, mask)
    for t, n in ((q, "q"), (k, "k"), (v, "v")):
        _unit_last(t, n)
    B, Hq, T, D = q.shape
    Hkv, N = k.shape[1], k.shape[2]
    if k.dtype != q.dtype or v.dtype != q.dtype:
        raise ValueError("q, k, v must share a dtype")
    if mask.dtype != torch.bool or tuple(mask.shape[-2:]) != (T, N) or any(d != 1 for d in mask.shape[:-2]):
        raise ValueError("array masks must be bool [..., T, N] with leading dims of 1")
    m = mask.reshape(T, N).view(torch.uint8)  # (no copy, strides kept)
    if out is None:
        out = torch.empty((B, Hq, T, D), dtype=q.dtype, device=q.device)
    gst = i64(0, 0, 0)
    if gate is not None:
        if gate.shape != (B, Hq, T, D) or gate.dtype != q.dtype:
            raise ValueError("gate must be [B, Hq, T, D] in q's dtype")
        _unit_last(gate, "gate")
        gst = i64(*gate.stride()[:3])
    ws = workspace(q.device, lib().lb2_attn_prefill_tiled_workspace_size(T, N, D), "prefill_tiled")
    rc = lib().lb2_attn_prefill_tiled(_ptr(q), i64(*q.stride()[:3]), _ptr(k), i64(*k.stride()[:3]), _ptr(v),
                                      i64(*v.stride()[:3]), _ptr(out), i64(*out.stride()[:3]), _ptr(gate), gst,
                                      _ptr(m), i64(m.stride(0), m.stride(1)), B, Hq, Hkv, T, N, D, dtype_code(q),
                                      float(scale), _ptr(ws), ws.numel(), _stream(q))
    check(rc, "attn_prefill_tiled")
    return out


def decode_rows_limit(D):
    """Folded rows (G*T) the split-KV decode kernel takes at head dim D."""
    return 16 if D == 256 else 32


_DECODE_WS = {}  # (B, Hq, Hkv, T, N, D, split, device index) -> workspace bytes (the plan depends on the SM count)


def _decode_ws_bytes(B, Hq, Hkv, T, N, D, split, dev):
    key = (B, Hq, Hkv, T, N, D, split, dev)
    n = _DECODE_WS.get(key)
    if n is None:
        n = _DECODE_WS[key] = lib().lb2_attn_decode_workspace_size(B, Hq, Hkv, T, N, D, split)
    return n


def attn_decode(q, k, v, scale, causal=False, kv_len=None, split=0, out=None):
    """Split-KV decode attention: q [B, Hq, T, D] with few rows over k / v [B, Hkv, N, D]; kv_len int32 [B]
    (on the device) gives each sequence's key count, else all N."""
    _cuda(q, k, v, kv_len)
    for t, n in ((q, "q"), (k, "k"), (v, "v")):
        _unit_last(t, n)
    B, Hq, T, D = q.shape
    Hkv, N = k.shape[1], k.shape[2]
    if out is None:
        out = torch.empty((B, Hq, T, D), dtype=q.dtype, device=q.device)
    ws = workspace(q.device, _decode_ws_bytes(B, Hq, Hkv, T, N, D, split, q.device.index), "decode")
    if kv_len is not None and (kv_len.dtype != torch.int32 or kv_len.numel() != B):
        raise ValueError("kv_len must be int32 [B]")
    rc = lib().lb2_attn_decode(_ptr(q), i64(*q.stride()[:3]), _ptr(k), i64(*k.stride()[:3]), _ptr(v),
                               i64(*v.stride()[:3]), _ptr(out), i64(*out.stride()[:3]), _ptr(kv_len), B, Hq, Hkv, T,
                               N, D, dtype_code(q), float(scale), int(bool(causal)), int(split), _ptr(ws), ws.numel(),
                               _stream(q))
    check(rc, "attn_decode")
    return out


def attn_decode_host(q_host, k, v, scale, o_host, causal=False, kv_len=None, split=0):
    """attn_decode for q and o in host memory (contiguous CPU tensors [B, Hq, T, D], pinned for the copies to
    overlap): copies q in, decodes on the current stream, copies o out, without waiting. o_host (of this call and
    the ones before) is complete after attn_decode_host_drain() and a synchronisation of the stream."""
    _cuda(k, v, kv_len)
    for t, n in ((q_host, "q_host"), (o_host, "o_host")):
        if t.is_cuda or not t.is_contiguous():
            raise ValueError(f"attn_decode_host: {n} must be a contiguous host tensor")
    if q_host.shape != o_host.shape or q_host.dtype != o_host.dtype or q_host.dtype != k.dtype:
        raise ValueError("attn_decode_host: q_host, o_host and the cache must share shape / dtype")
    B, Hq, T, D = q_host.shape
    Hkv, N = k.shape[1], k.shape[2]
    if kv_len is not None and (kv_len.dtype != torch.int32 or kv_len.numel() != B):
        raise ValueError("kv_len must be int32 [B]")
    L = lib()
    need = L.lb2_attn_decode_host_workspace_size(B, Hq, Hkv, T, N, D, dtype_code(k), int(split))
    cur = _WS.get((k.device.index if k.device.index is not None else torch.cuda.current_device(), "decode_host"))
    if cur is not None and cur.numel() < need:  # copies still in flight may use the old buffer: let them finish
        attn_decode_host_drain(k.device.index)
        torch.cuda.synchronize(k.device)
    ws = workspace(k.device, need, "decode_host")
    rc = L.lb2_attn_decode_host(q_host.data_ptr(), _ptr(k), i64(*k.stride()[:3]), _ptr(v), i64(*v.stride()[:3]),
                                o_host.data_ptr(), _ptr(kv_len), B, Hq, Hkv, T, N, D, dtype_code(k), float(scale),
                                int(bool(causal)), int(split), _ptr(ws), ws.numel(), _stream(k))
    check(rc, "attn_decode_host")
    return o_host


def attn_decode_host_drain(device=None):
    """Order the current stream after every outstanding attn_decode_host copy out."""
    dev = torch.device("cuda", torch.cuda.current_device() if device is None else device)
    check(lib().lb2_attn_decode_host_drain(ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)),
          "attn_decode_host_drain")


def attn_decode_partial(q, k, v, scale, kv_len=None, split=0, out=None):
    """This KV range's normalised partial output (fp32 [B, Hq, T, D]) and log-sum-exp (fp32 [B, Hq, T]); `out`, a
    pair of contiguous fp32 tensors of those shapes (for instance the two parts of one packed exchange buffer),
    receives them when given."""
    _cuda(q, k, v, kv_len)
    B, Hq, T, D = q.shape
    Hkv, N = k.shape[1], k.shape[2]
    if out is None:
        part_o = torch.empty((B, Hq, T, D), dtype=torch.float32, device=q.device)
        part_lse = torch.empty((B, Hq, T), dtype=torch.float32, device=q.device)
    else:
        part_o, part_lse = out
        for t, shp in ((part_o, (B, Hq, T, D)), (part_lse, (B, Hq, T))):
            if t.dtype != torch.float32 or tuple(t.shape) != shp or not t.is_contiguous() or t.device != q.device:
                raise ValueError(f"attn_decode_partial: out must be contiguous fp32 {shp} on q's device")
    decode_partial_into(q, k, v, scale, kv_len, split, _ptr(part_o), _ptr(part_lse))
    return part_o, part_lse


def decode_partial_into(q, k, v, scale, kv_len, split, part_o_ptr, part_lse_ptr):
    """attn_decode_partial into raw device addresses (contiguous fp32 [B, Hq, T, D] and [B, Hq, T]): the halves of
    a peer-exchange buffer, which no tensor wraps."""
    B, Hq, T, D = q.shape
    Hkv, N = k.shape[1], k.shape[2]
    ws = workspace(q.device, _decode_ws_bytes(B, Hq, Hkv, T, N, D, split, q.device.index), "decode_partial")
    rc = lib().lb2_attn_decode_partial(_ptr(q), i64(*q.stride()[:3]), _ptr(k), i64(*k.stride()[:3]), _ptr(v),
                                       i64(*v.stride()[:3]), part_o_ptr, part_lse_ptr, _ptr(kv_len), B, Hq, Hkv,
                                       T, N, D, dtype_code(q), float(scale), int(split), _ptr(ws), ws.numel(),
                                       _stream(q))
    check(rc, "attn_decode_partial")


def decode_push(q, k, v, scale, kv_len, split, bufs, R, rank, epoch):
    """This rank's KV-range partial stored into slot `rank` of half epoch % 2 of every rank's push-exchange buffer
    (bufs: a ctypes uint64 array of the R buffers as mapped here), lb2_attn_decode_push."""
    B, Hq, T, D = q.shape
    Hkv, N = k.shape[1], k.shape[2]
    ws = workspace(q.device, _decode_ws_bytes(B, Hq, Hkv, T, N, D, split, q.device.index), "decode_partial")
    rc = lib().lb2_attn_decode_push(_ptr(q), i64(*q.stride()[:3]), _ptr(k), i64(*k.stride()[:3]), _ptr(v),
                                    i64(*v.stride()[:3]), _ptr(kv_len), B, Hq, Hkv, T, N, D, dtype_code(q),
                                    float(scale), int(split), _ptr(ws), ws.numel(), bufs, int(R), int(rank),
                                    int(epoch), _stream(q))
    check(rc, "attn_decode_push")


def attn_combine(part_o, part_lse, dtype, out=None):
    """Merge R partials part_o [R, B, Hq, T, D], part_lse [R, B, Hq, T] (fp32) by log-sum-exp."""
    _cuda(part_o, part_lse)
    R, B, Hq, T, D = part_o.shape
    part_o, part_lse = part_o.contiguous(), part_lse.contiguous()
    if out is None:
        out = torch.empty((B, Hq, T, D), dtype=dtype, device=part_o.device)
    rc = lib().lb2_attn_combine(_ptr(part_o), _ptr(part_lse), R, B, Hq, T, D, _ptr(out), i64(*out.stride()[:3]),
                                dtype_code(out), _stream(part_o))
    check(rc, "attn_combine")
    return out


def attn_combine_packed(gathered, R, B, Hq, T, D, dtype, out=None):
    """Merge R partials from an all-gathered packed buffer: R blocks of [o rows (B Hq T D) | lse (B Hq T)] fp32."""
    _cuda(gathered)
    if gathered.dtype != torch.float32 or not gathered.is_contiguous() or gathered.numel() != R * B * Hq * T * (D + 1):
        raise ValueError("attn_combine_packed: gathered must be contiguous fp32 of R * B * Hq * T * (D + 1) values")
    if out is None:
        out = torch.empty((B, Hq, T, D), dtype=dtype, device=gathered.device)
    rc = lib().lb2_attn_combine_packed(_ptr(gathered), R, B, Hq, T, D, _ptr(out), i64(*out.stride()[:3]),
                                       dtype_code(out), _stream(gathered))
    check(rc, "attn_combine_packed")
    return out


# ---------------------------------------------------------------------------------------------------- GDN

def _gdn_common(q, k, v, g, beta, state):
    _cuda(q, k, v, g, beta, state)
    B, T, Hk, Dk = q.shape
    Hv, Dv = v.shape[2], v.shape[3]
    if k.shape != q.shape or k.dtype != q.dtype:
        raise ValueError("q and k must share shape and dtype")
    if state is None:
        state = torch.zeros((B, Hv, Dv, Dk), dtype=torch.float32, device=q.device)
    if state.dtype != torch.float32 or tuple(state.shape) != (B, Hv, Dv, Dk):
        raise ValueError("state must be fp32 [B, Hv, Dv, Dk]")
    q, k, v, g, beta, state = (t.contiguous() for t in (q, k, v, g, beta, state))
    return q, k, v, g, beta, state, (B, T, Hk, Dk, Hv, Dv)


def gdn_recurrent(q, k, v, g, beta, state=None, mask=None, state_out=None):
    """The gated delta recurrence position by position: returns (y [B, T, Hv, Dv] in q's dtype, new state). The new
    state goes to `state_out` when given (fp32, the state's shape, contiguous, not the input state itself)."""
    q, k, v, g, beta, state, (B, T, Hk, Dk, Hv, Dv) = _gdn_common(q, k, v, g, beta, state)
    y = torch.empty((B, T, Hv, Dv), dtype=q.dtype, device=q.device)
    if state_out is None:
        s_out = torch.empty_like(state)
    else:
        if (state_out.shape != state.shape or state_out.dtype != torch.float32 or not state_out.is_contiguous()
                or state_out.data_ptr() == state.data_ptr()):
            raise ValueError("gdn_recurrent: state_out must be a separate contiguous fp32 tensor of the state's shape")
        s_out = state_out
    m = None
    if mask is not None:
        m = mask.reshape(B, T).to(torch.uint8).contiguous()
    rc = lib().lb2_gdn_recurrent(_ptr(q), _ptr(k), dtype_code(q), _ptr(v), dtype_code(v), _ptr(g), dtype_code(g),
                                 int(g.dim() == 4), _ptr(beta), dtype_code(beta), _ptr(m), _ptr(state), _ptr(s_out),
                                 _ptr(y), B, T, Hk, Dk, Hv, Dv, _stream(q))
    check(rc, "gdn_recurrent")
    return y, s_out


def gdn_chunked_supported(q, v, g, mask):
    return (mask is None and g.dim() == 3 and q.shape[-1] == 128 and v.shape[-1] == 128
            and q.dtype in (torch.bfloat16, torch.float16))


def gdn_chunked(q, k, v, g, beta, state=None):
    """The same recurrence in chunks of 64 positions on tensor cores (scalar gate, no mask, Dk = Dv = 128)."""
    q, k, v, g, beta, state, (B, T, Hk, Dk, Hv, Dv) = _gdn_common(q, k, v, g, beta, state)
    y = torch.empty((B, T, Hv, Dv), dtype=q.dtype, device=q.device)
    s_out = torch.empty_like(state)
    nbytes = lib().lb2_gdn_chunked_workspace_size(B, T, Hk, Hv, Dk, Dv)
    ws = workspace(q.device, nbytes, "gdn_chunked")
    rc = lib().lb2_gdn_chunked(_ptr(q), _ptr(k), dtype_code(q), _ptr(v), dtype_code(v), _ptr(g), dtype_code(g),
                               _ptr(beta), dtype_code(beta), _ptr(state), _ptr(s_out), _ptr(y), B, T, Hk, Dk, Hv, Dv,
                               _ptr(ws), ws.numel(), _stream(q))
    check(rc, "gdn_chunked")
    return y, s_out


# ---------------------------------------------------------------------------------------------------- gathers

def kv_gather_picks(k, v, tb, cr, n=None):
    """Rows of one sequence's k / v [Hk, n, D] (or [1, Hk, n, D]) that QSA decode attends to: the sorted picked
    blocks tb (int32, block size cr) and the trailing partial block. Returns kg, vg [1, Hk, m, D]."""
    _cuda(k, v, tb)
    if k.dim() == 4:
        k, v = k[0], v[0]
    Hk, N, D = k.shape
    n = N if n is None else int(n)
    tb = tb.reshape(-1)
    if tb.dtype != torch.int32:
        raise ValueError("tb must be int32")
    nsel = tb.numel()
    m = nsel * cr + n - n // cr * cr
    kg = torch.empty((1, Hk, m, D), dtype=k.dtype, device=k.device)
    vg = torch.empty_like(kg)
    rc = lib().lb2_kv_gather_picks(_ptr(k), i64(*k.stride()), _ptr(v), i64(*v.stride()), _ptr(tb), nsel, int(cr), n,
                                   _ptr(kg), _ptr(vg), Hk, D, dtype_code(k), _stream(k))
    check(rc, "kv_gather_picks")
    return kg, vg


def qsa_decode(q, k, v, tb, cr, scale, n=None, out=None):
    """One QSA decode row with the gather inside the decode kernel: q [1, Hq, 1, D] attends to the rows of k / v
    [Hk, n, D] (or [1, Hk, n, D]) that kv_gather_picks(k, v, tb, cr) would return, read in place. Bit-equal to
    attn_decode over kv_gather_picks' output."""
    _cuda(q, k, v, tb)
    if k.dim() == 4:
        k, v = k[0], v[0]
    for t, nm in ((q, "q"), (k, "k"), (v, "v")):
        _unit_last(t, nm)
    Hk, N, D = k.shape
    n = N if n is None else int(n)
    tb = tb.reshape(-1)
    if tb.dtype != torch.int32:
        raise ValueError("tb must be int32")
    _, Hq, T, _ = q.shape
    if q.shape[0] != 1 or T != 1:
        raise ValueError("qsa_decode: one query row [1, Hq, 1, D]")
    if out is None:
        out = torch.empty_like(q)
    nsel = tb.numel()
    L = lib()
    ws = workspace(q.device, L.lb2_qsa_decode_workspace_size(nsel, int(cr), n, Hq, Hk, D), "decode")
    # (the views as [1, Hk, n, D]: a batch stride of Hk heads, for the tensor maps the kernel is given)
    rc = L.lb2_qsa_decode(_ptr(q), i64(*q.stride()[:3]), _ptr(k), i64(Hk * k.stride(0), *k.stride()[:2]), _ptr(v),
                          i64(Hk * v.stride(0), *v.stride()[:2]), _ptr(out), i64(*out.stride()[:3]), _ptr(tb), nsel,
                          int(cr), n, Hq, Hk, D, dtype_code(q), float(scale), _ptr(ws), ws.numel(), _stream(q))
    check(rc, "qsa_decode")
    return out


def kvh_put(table, k, v, pos0, logc):
    """Write k / v [Hk, s, D] (or [1, Hk, s, D]) as positions pos0 .. pos0 + s - 1 of the paged home `table`."""
    _cuda(table, k, v)
    if k.dim() == 4:
        k, v = k[0], v[0]
    Hk, s, D = k.shape
    rc = lib().lb2_kvh_put(_ptr(table), _ptr(k), i64(*k.stride()), _ptr(v), i64(*v.stride()), int(pos0), s, Hk, D,
                           dtype_code(k), int(logc), _stream(k))
    check(rc, "kvh_put")


def kvh_gather(table, tb, cr, n, Hk, D, dtype, logc, device):
    """The QSA picks of a sequence of n positions read from the paged home: kg, vg [1, Hk, m, D]."""
    tb = tb.reshape(-1)
    nsel = tb.numel()
    m = nsel * cr + n - n // cr * cr
    kg = torch.empty((1, Hk, m, D), dtype=dtype, device=device)
    vg = torch.empty_like(kg)
    rc = lib().lb2_kvh_gather(_ptr(table), _ptr(tb), nsel, int(cr), int(n), _ptr(kg), _ptr(vg), Hk, D,
                              dtype_code(kg), int(logc), _stream(kg))
    check(rc, "kvh_gather")
    return kg, vg


def kvh_lru_plan(tb, lru):
    """One token's plan over the LRU state `lru` (a kv_host.Lru): sl [nsel] int32 on the device, the state updated in
    place (see lb2_kvh_lru_plan)."""
    tb = tb.reshape(-1)
    _cuda(tb, lru.slot_of)
    if tb.dtype != torch.int32:
        raise ValueError("kvh_lru_plan: tb must be int32")
    sl = torch.empty(tb.numel(), dtype=torch.int32, device=tb.device)
    rc = lib().lb2_kvh_lru_plan(_ptr(tb), tb.numel(), _ptr(lru.slot_of), lru.slot_of.numel(), _ptr(lru.block_of),
                                _ptr(lru.stamp), _ptr(lru.ref), _ptr(lru.meta), lru.slots, _ptr(sl), _stream(tb))
    check(rc, "kvh_lru_plan")
    return sl


def kvh_lru_gather(table, lru, tb, sl, cr, n, kn, vn, logc):
    """The token's QSA rows kg, vg [1, Hk, m, D] of a sequence of n positions through the LRU (pool hits, home
    misses filling their victims), and the new row kn / vn ([Hk, D], [1, Hk, 1, D] ...) written into the home at
    n - 1 (see lb2_kvh_lru_gather)."""
    tb = tb.reshape(-1)
    Hk, D = lru.pool.shape[2], lru.pool.shape[4]
    kn, vn = kn.reshape(Hk, D), vn.reshape(Hk, D)
    _cuda(table, tb, sl, kn, vn)
    if kn.dtype != lru.pool.dtype or vn.dtype != lru.pool.dtype:
        raise ValueError("kvh_lru_gather: the new row must have the pool's dtype")
    nsel = tb.numel()
    m = nsel * cr + n - n // cr * cr
    kg = torch.empty((1, Hk, m, D), dtype=kn.dtype, device=kn.device)
    vg = torch.empty_like(kg)
    rc = lib().lb2_kvh_lru_gather(_ptr(table), _ptr(lru.pool), lru.slots, _ptr(tb), _ptr(sl), nsel, int(cr), int(n),
                                  _ptr(kn), i64(*kn.stride()), _ptr(vn), i64(*vn.stride()), _ptr(kg), _ptr(vg), Hk, D,
                                  dtype_code(kg), int(logc), _stream(kg))
    check(rc, "kvh_lru_gather")
    return kg, vg


def kvh_lru_inval(lru, lim):
    """Slots of the LRU holding a block >= lim drop it."""
    rc = lib().lb2_kvh_lru_inval(_ptr(lru.slot_of), _ptr(lru.block_of), _ptr(lru.ref), lru.slots, int(lim),
                                 _stream(lru.slot_of))
    check(rc, "kvh_lru_inval")


# ---------------------------------------------------------------------------------------------------- GDN glue

def _rounded(x, dtype):
    """A Python float rounded to `dtype` (the scalar an op on that dtype applies)."""
    return float(torch.tensor(float(x), dtype=dtype).item())


def gdn_step_glue(conv, a, b, A_log, dt_bias, state, Hk, Dk, Hv, Dv):
    """Fused GDN decode rows (silu, q/k RMSNorm and scales, sigmoid(b), compute_g, recurrence) for B = 1."""
    _cuda(conv, a, b, A_log, dt_bias, state)
    NR = conv.shape[-2]
    conv, a, b = conv.reshape(NR, -1).contiguous(), a.reshape(NR, Hv).contiguous(), b.reshape(NR, Hv).contiguous()
    A_log, dt_bias = A_log.float().contiguous(), dt_bias.float().contiguous()
    state = state.contiguous()
    y = torch.empty((1, NR, Hv, Dv), dtype=conv.dtype, device=conv.device)
    s_out = torch.empty_like(state)
    inv = Dk ** -0.5
    rc = lib().lb2_gdn_step_glue(_ptr(conv), _ptr(a), _ptr(b), _ptr(A_log), _ptr(dt_bias), _ptr(state), _ptr(s_out),
                                 _ptr(y), NR, Hk, Dk, Hv, Dv, dtype_code(conv), _rounded(inv * inv, conv.dtype),
                                 _rounded(inv, conv.dtype), float(1e-6 * inv * inv), _stream(conv))
    check(rc, "gdn_step_glue")
    return y, s_out


def gdn_norm_gate(x, z, weight, eps):
    """silu(z) * (weight * rms_norm(x)) over the last axis."""
    _cuda(x, z, weight)
    D = x.shape[-1]
    xc, zc = x.contiguous(), z.contiguous()
    out = torch.empty_like(xc)
    rc = lib().lb2_gdn_norm_gate(_ptr(xc), _ptr(zc), _ptr(weight.contiguous()), _ptr(out), xc.numel() // D, D,
                                 dtype_code(xc), float(eps), _stream(xc))
    check(rc, "gdn_norm_gate")
    return out
