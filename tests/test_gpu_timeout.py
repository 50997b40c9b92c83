"""A bounded device wait that runs out, on one GPU, without faulting or hanging it.

lb2_attn_combine_peers waits for every peer's call number in its own exchange buffer. Here rank 0 of R = 2 is given
two exchange buffers of this process: its own, and a stand-in "peer" that never runs a call, so the flag it waits for
is never set. The wait must give up after its 2 s bound, report LB2_ETIMEOUT (where = 101) through lb2_status, and
leave the output unwritten; the context stays usable (a decode afterwards runs and reports 0).
"""
import ctypes
import time

import pytest
import torch

from larder_b200 import _lib, ops

pytestmark = pytest.mark.gpu


def test_combine_peers_wait_runs_out_and_reports():
    L = _lib.lib()
    B, Hq, T, D = 1, 8, 1, 128  # 8 rows: one block, one bounded wait
    nbytes = L.lb2_xch_bytes(B, Hq, T, D)
    bufs = []
    try:
        for _ in range(2):
            p = ctypes.c_void_p()
            assert L.lb2_xch_alloc(nbytes, ctypes.byref(p)) == 0, L.lb2_error()
            bufs.append(p.value)
        o = torch.full((B, Hq, T, D), 7.0, dtype=torch.bfloat16, device="cuda")
        arr = (ctypes.c_uint64 * 2)(*bufs)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        rc = L.lb2_attn_combine_peers(arr, 2, 0, 1, B, Hq, T, D, ctypes.c_void_p(o.data_ptr()),
                                      _lib.i64(*o.stride()[:3]), _lib.BF16,
                                      ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
        assert rc == 0, L.lb2_error()
        st = ops.status()
        waited = time.perf_counter() - t0
        assert st & 0xFF == _lib.ETIMEOUT and st >> 8 == 101, st
        assert 1.5 <= waited <= 30, waited
        assert torch.all(o == 7.0), "a combine whose wait gave up must not write o"
        assert ops.status() == 0, "lb2_status clears the word it reported"
        # the context is still usable
        q = torch.randn(1, 8, 1, 128, device="cuda").to(torch.bfloat16)
        k = torch.randn(1, 2, 256, 128, device="cuda").to(torch.bfloat16)
        ops.attn_decode(q, k, k, 128 ** -0.5)
        assert ops.status() == 0
    finally:
        torch.cuda.synchronize()
        for p in bufs:
            L.lb2_xch_free(ctypes.c_void_p(p))
