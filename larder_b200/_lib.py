"""Loader for liblarder_b200.so, the C-ABI library of this package's CUDA kernels.

There is no CPU or PyTorch fallback anywhere in larder_b200: if the library is missing, or the tensors are not on a
CUDA device, calls raise. The library is built in-tree by larder_b200.build (nvcc, sm_100a) so that it travels with
the repository.
"""
import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liblarder_b200.so")

F32, BF16, F16 = 0, 1, 2
MASK_NONE, MASK_CAUSAL, MASK_ARRAY = 0, 1, 2
OK, EINVAL, ECUDA, ETIMEOUT = 0, 1, 2, 3

# Every symbol include/larder_b200.h declares, with its ctypes signature.
_p, _i, _f, _sz = ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_size_t
_i64p = ctypes.POINTER(ctypes.c_int64)
SIGNATURES = {
    "lb2_abi_version": ([], _i),
    "lb2_error": ([], ctypes.c_char_p),
    "lb2_status": ([_p], _i),
    "lb2_attn_prefill": ([_p, _i64p, _p, _i64p, _p, _i64p, _p, _i64p, _p, _i64p, _p, _i64p,
                          _i, _i, _i, _i, _i, _i, _i, _f, _i, _p], _i),
    "lb2_attn_prefill_tiled_workspace_size": ([_i, _i, _i], _sz),
    "lb2_attn_prefill_tiled": ([_p, _i64p, _p, _i64p, _p, _i64p, _p, _i64p, _p, _i64p, _p, _i64p,
                                _i, _i, _i, _i, _i, _i, _i, _f, _p, _sz, _p], _i),
    "lb2_attn_decode_workspace_size": ([_i, _i, _i, _i, _i, _i, _i], _sz),
    "lb2_attn_decode": ([_p, _i64p, _p, _i64p, _p, _i64p, _p, _i64p, _p, _i, _i, _i, _i, _i, _i, _i, _f, _i, _i,
                         _p, _sz, _p], _i),
    "lb2_attn_decode_partial": ([_p, _i64p, _p, _i64p, _p, _i64p, _p, _p, _p, _i, _i, _i, _i, _i, _i, _i, _f, _i,
                                 _p, _sz, _p], _i),
    "lb2_attn_decode_noalloc": ([_p, _i64p, _p, _i64p, _p, _i64p, _p, _i64p, _p, _i, _i, _i, _i, _i, _i, _i, _f, _i,
                                 _i, _p], _i),
    "lb2_attn_combine": ([_p, _p, _i, _i, _i, _i, _i, _p, _i64p, _i, _p], _i),
    "lb2_attn_combine_packed": ([_p, _i, _i, _i, _i, _i, _p, _i64p, _i, _p], _i),
    "lb2_gdn_recurrent": ([_p, _p, _i, _p, _i, _p, _i, _i, _p, _i, _p, _p, _p, _p, _i, _i, _i, _i, _i, _i, _p], _i),
    "lb2_gdn_chunked_workspace_size": ([_i, _i, _i, _i, _i, _i], _sz),
    "lb2_gdn_chunked": ([_p, _p, _i, _p, _i, _p, _i, _p, _i, _p, _p, _p, _i, _i, _i, _i, _i, _i, _p, _sz, _p], _i),
    "lb2_kv_gather_picks": ([_p, _i64p, _p, _i64p, _p, _i, _i, _i, _p, _p, _i, _i, _i, _p], _i),
    "lb2_qsa_decode_workspace_size": ([_i, _i, _i, _i, _i, _i], _sz),
    "lb2_qsa_decode": ([_p, _i64p, _p, _i64p, _p, _i64p, _p, _i64p, _p, _i, _i, _i, _i, _i, _i, _i, _f, _p, _sz, _p],
                       _i),
    "lb2_kvh_put": ([_p, _p, _i64p, _p, _i64p, ctypes.c_int64, _i, _i, _i, _i, _i, _p], _i),
    "lb2_kvh_gather": ([_p, _p, _i, _i, _i, _p, _p, _i, _i, _i, _i, _p], _i),
    "lb2_attn_decode_host_workspace_size": ([_i, _i, _i, _i, _i, _i, _i, _i], _sz),
    "lb2_attn_decode_host": ([_p, _p, _i64p, _p, _i64p, _p, _p, _i, _i, _i, _i, _i, _i, _i, _f, _i, _i, _p, _sz, _p],
                             _i),
    "lb2_attn_decode_host_drain": ([_p], _i),
    "lb2_xch_bytes": ([_i, _i, _i, _i], _sz),
    "lb2_xch_alloc": ([_sz, ctypes.POINTER(ctypes.c_void_p)], _i),
    "lb2_xch_free": ([_p], _i),
    "lb2_xch_handle": ([_p, _p], _i),
    "lb2_xch_open": ([_p, ctypes.POINTER(ctypes.c_void_p)], _i),
    "lb2_xch_close": ([_p], _i),
    "lb2_attn_combine_peers": ([_p, _i, _i, ctypes.c_uint32, _i, _i, _i, _i, _p, _i64p, _i, _p], _i),
    "lb2_xch_push_bytes": ([_i, _i, _i, _i, _i], _sz),
    "lb2_attn_decode_push": ([_p, _i64p, _p, _i64p, _p, _i64p, _p, _i, _i, _i, _i, _i, _i, _i, _f, _i, _p, _sz, _p,
                              _i, _i, ctypes.c_uint32, _p], _i),
    "lb2_attn_combine_pushed": ([_p, _i, _i, ctypes.c_uint32, _i, _i, _i, _i, _p, _i64p, _i, _p], _i),
    "lb2_kvh_lru_plan": ([_p, _i, _p, _i, _p, _p, _p, _p, _i, _p, _p], _i),
    "lb2_kvh_lru_gather": ([_p, _p, _i, _p, _p, _i, _i, _i, _p, _i64p, _p, _i64p, _p, _p, _i, _i, _i, _i, _p], _i),
    "lb2_kvh_lru_inval": ([_p, _p, _p, _i, _i, _p], _i),
    "lb2_gdn_step_glue": ([_p, _p, _p, _p, _p, _p, _p, _p, _i, _i, _i, _i, _i, _i, _f, _f, _f, _p], _i),
    "lb2_gdn_norm_gate": ([_p, _p, _p, _p, ctypes.c_int64, _i, _i, _f, _p], _i),
    "lb2_attn_qk_norm_rope": ([_p, _p, _p, _p, _f, _p, _p, _i, _p, _p, _i, _i, _i, _i, _i, _i, _i, _p], _i),
    "lb2_attn_out_gate": ([_p, _p, _p, ctypes.c_int64, _i, _i, _i, _p], _i),
    "lb2_qsa_select_workspace_size": ([_i, _i, _i], _sz),
    "lb2_qsa_select": ([_p, _p, ctypes.c_int64, _i, _i, _i, _i, _i, ctypes.c_int64, _i, _i, _f, _p, _sz, _p, _p],
                       _i),
}

_lib = None


class LarderError(RuntimeError):
    """A CUDA-side failure reported by liblarder_b200 (launch error or a device wait that gave up)."""


def lib():
    """The loaded library; raises ImportError when it was not built (no fallback exists)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: build it with `python -m larder_b200.build` "
                              "(larder_b200 has no CPU or PyTorch fallback)")
        L = ctypes.CDLL(LIB_PATH)
        for name, (args, res) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = res
        _lib = L
    return _lib


def check(rc, what):
    if rc == OK:
        return
    msg = lib().lb2_error().decode(errors="replace")
    if rc == EINVAL:
        raise ValueError(f"{what}: {msg}")
    raise LarderError(f"{what}: {msg} (status {rc})")


_I64N = [ctypes.c_int64 * n for n in range(5)]
_I64_CACHE = {}  # value tuple -> array: strides repeat from call to call, and the library only reads them


def i64(*vals):
    """An int64 array argument (strides, shapes) from Python ints. The library reads it during the call only."""
    a = _I64_CACHE.get(vals)
    if a is None:
        a = _I64N[len(vals)](*vals) if len(vals) < 5 else (ctypes.c_int64 * len(vals))(*vals)
        if len(_I64_CACHE) < 4096:
            _I64_CACHE[vals] = a
    return a
