"""The reference's installer surface on the GPU: kv_host.make_class / install (kv_host.py:516-799) and
gdn_cuda.install_glue (gdn_cuda.py:271-315), each against what the caller's own lines give.

  * A cache of the installed class crosses the home line inside a prefill pass: every pass returns exactly the rows
    the base cache returns (byte work: bit-exact), decode rows through the LRU return exactly the QSA rows gathered
    from those rows (picked blocks then the tail, stream_fast.py:6448-6491), and a trim followed by new passes
    rewrites positions as the base does. Device and pinned-host homes.
  * A GatedDeltaNet layer patched by install_glue gives, for decode rows, the layer's own output within the grading
    bar, and the same recurrent state and conv state.
"""
import types

import pytest
import torch

import checks
from dropin_models import ArraysCache, GatedDeltaNet, KVCache
from larder_b200 import gdn_cuda, kv_host, ops

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _status_clean():
    yield
    assert ops.status() == 0, "a device wait gave up"


def _picks(n, cr, nsel, g):
    tb = torch.randperm(n // cr, generator=g)[:nsel].sort().values.to(torch.int32)
    pos = torch.cat([(tb[:, None].long() * cr + torch.arange(cr)).reshape(-1), torch.arange(n // cr * cr, n)])
    return tb, pos


@pytest.mark.parametrize("home", ["device", "host"])
def test_homed_cache_matches_its_base(home, monkeypatch):
    monkeypatch.delenv("MOE_KV_HOST_FROM", raising=False)
    monkeypatch.setenv("LB2_KV_HOME", home)
    q4 = types.SimpleNamespace(_AttnCache=KVCache)
    Hk, D, nsel, cr = 2, 128, 16, 4
    try:
        assert kv_host.install(q4, 256, nsel, cr, Hk, D, torch.bfloat16)
        assert kv_host.H == 512  # twice the LRU's 64 blocks of 4 positions
        c, ref = q4._AttnCache(), KVCache()
        g = torch.Generator().manual_seed(7)

        def rows(s):
            return (torch.randn(1, Hk, s, D, generator=g).to(torch.bfloat16).cuda(),
                    torch.randn(1, Hk, s, D, generator=g).to(torch.bfloat16).cuda())
        for s in (200, 200, 200, 37):  # the third pass crosses 512
            k, v = rows(s)
            a, b = c.update_and_fetch(k, v), ref.update_and_fetch(k, v)
            assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1]), s
        assert c.kv_host and c.offset == ref.offset == 637
        for _ in range(6):  # decode rows through the LRU (picks kept from token to token as the reference's test)
            k, v = rows(1)
            kb, vb = ref.update_and_fetch(k, v)
            tb, pos = _picks(ref.offset, cr, nsel, g)
            kg, vg = c.decode(k, v, tb.cuda(), cr)
            assert torch.equal(kg, kb[:, :, pos.cuda()]) and torch.equal(vg, vb[:, :, pos.cuda()])
        assert torch.equal(c.keys, ref.keys[:, :, :ref.offset])  # the staged view
        # a trim (offset given back), then a pass rewriting those positions
        c.offset = ref.offset = 600
        k, v = rows(20)
        a, b = c.update_and_fetch(k, v), ref.update_and_fetch(k, v)
        assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])
        k, v = rows(1)
        kb, vb = ref.update_and_fetch(k, v)
        tb, pos = _picks(ref.offset, cr, nsel, g)
        kg, vg = c.decode(k, v, tb.cuda(), cr)
        assert torch.equal(kg, kb[:, :, pos.cuda()]) and torch.equal(vg, vb[:, :, pos.cuda()])
        rep = kv_host.report()
        assert rep["homed"] >= 1 and rep["hits"] + rep["misses"] == 7 * nsel
    finally:
        kv_host.uninstall(q4)


def test_install_glue_decode_rows_match_the_layer():
    Hk, Hv, Dk, Dv, hidden = 4, 8, 128, 128, 256
    cls = type("GDN", (GatedDeltaNet,), {})
    own = GatedDeltaNet(Hk, Hv, Dk, Dv, hidden, seed=3)
    fused = cls(Hk, Hv, Dk, Dv, hidden, seed=3)
    gdn_cuda.install_glue(rows=2, cls=cls)
    g = torch.Generator().manual_seed(4)
    s0 = (torch.randn(1, Hv, Dv, Dk, generator=g) * 0.1).cuda()
    ca, cb = ArraysCache(s0.clone()), ArraysCache(s0.clone())
    for S in (1, 1, 2):
        x = torch.randn(1, S, hidden, generator=g).to(torch.bfloat16).cuda()
        ya, yb = own(x, None, ca), fused(x, None, cb)
        checks.grading_close(yb.float().cpu().numpy(), ya.float().cpu().numpy(), what=f"S={S}")
        assert torch.equal(ca[0], cb[0])  # conv state: the same rows kept
        assert (ca[1] - cb[1]).abs().max().item() <= 1e-3 * ca[1].abs().max().item()
    assert ca.advanced == cb.advanced == 4
