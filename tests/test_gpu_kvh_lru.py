"""The KV home's VRAM LRU on the GPU (kv_host.py:116-291, :612-643): integer and byte work, so bit-exact.

* The plan and inval kernels replay the golden sequences made by the reference's own emulations of them
  (tests/golden/make_kvh_lru.py): every step's slots and every state array equal.
* Home(lru=True) over decode steps (picks partly kept from the previous token, the block the new row completes
  picked at times, a trim midway, a chunk boundary crossed): each step's gathered rows equal the oracle's (plan +
  gather over a CPU mirror of the home and the pool) and the rows of the whole cache at the picked positions; the
  pool and its state equal the mirror's at the end.
* Picks out of range are skipped with zero rows and reported in the status word, without touching memory.
* Flash-Next's decode shapes (24/2 x 256, CR 4, 512 picks) through Home.decode, attention against the oracle."""
import types

import numpy as np
import pytest
import torch

import oracle
from larder_b200 import kv_host, ops

pytestmark = pytest.mark.gpu

from test_oracle_lru import cases, fresh  # noqa: E402  (the golden sequences)


@pytest.fixture(autouse=True)
def _status_clean():
    yield
    assert ops.status() == 0, "a device wait gave up or an index was out of range"


def u16(t):
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def device_state(so, bo, st, rf, mt):
    dev = [torch.from_numpy(a.copy()).cuda() for a in (so, bo, st, rf, mt)]
    return types.SimpleNamespace(slot_of=dev[0], block_of=dev[1], stamp=dev[2], ref=dev[3], meta=dev[4],
                                 slots=bo.size)


@pytest.mark.parametrize("c", [0, 1])
def test_plan_and_inval_replay_reference_emulation(c):
    g = cases()[c]
    lru = device_state(*fresh(g))
    for i in range(int(g["steps"])):
        if g["op"][i][0] == 1:
            ops.kvh_lru_inval(lru, int(g["op"][i][1]))
        else:
            sl = ops.kvh_lru_plan(torch.from_numpy(g["tb"][i]).cuda(), lru)
            assert np.array_equal(sl.cpu().numpy(), g["sl"][i]), f"step {i}: slots"
        for name, t in (("so", lru.slot_of), ("bo", lru.block_of), ("st", lru.stamp), ("rf", lru.ref),
                        ("mt", lru.meta)):
            assert np.array_equal(t.cpu().numpy(), g[name][i]), f"step {i}: {name}"


@pytest.mark.parametrize("host", [False, True])
def test_home_lru_decode_rows_match_oracle(host):
    rng = np.random.default_rng(31 + host)
    gen = torch.Generator().manual_seed(31 + host)
    Hk, D, cr, nsel, n0, steps, trim_at = 2, 128, 4, 48, 4070, 60, 30
    rows = torch.randn(2, Hk, n0 + steps, D, generator=gen).to(torch.bfloat16)
    home = kv_host.Home(Hk, D, torch.bfloat16, "cuda", host=host, lru=True)
    home.put(rows[0, None, :, :n0].cuda(), rows[1, None, :, :n0].cuda())
    kc, vc = u16(rows[0, :, :n0]), u16(rows[1, :, :n0])  # the mirror of the home, [Hk, n, D]
    ns = kv_host.lru_slots(nsel)
    pool = np.zeros((ns, 2, Hk, cr, D), np.uint16)
    so = np.full((kv_host.MAXC << kv_host.LOGC) // cr, -1, np.int32)
    bo, st, rf, mt = np.full(ns, -1, np.int32), np.full(ns, -1, np.int32), np.zeros(ns, np.int32), np.zeros(4, np.int32)
    n, prev, newest = n0, [], 0
    for step in range(steps):
        if step == trim_at:  # positions from the cut on are rewritten by the next steps
            n -= 9
            home.trim(n)
            oracle.lru_inval(so, bo, rf, n // cr)
            kc, vc = kc[:, :n], vc[:, :n]
        k1, v1 = rows[0, :, n0 + step], rows[1, :, n0 + step]
        kc = np.concatenate([kc, u16(k1)[:, None]], 1)
        vc = np.concatenate([vc, u16(v1)[:, None]], 1)
        n += 1
        nb = n // cr
        keep = {b for b in prev if b < nb and rng.random() < 0.6}
        if n % cr == 0 and rng.random() < 0.5:
            keep.add(nb - 1)  # the block the new row completes
            newest += 1
        rest = np.setdiff1d(np.arange(nb), sorted(keep))
        tb = np.sort(np.concatenate([sorted(keep), rng.choice(rest, nsel - len(keep), replace=False)])).astype(np.int32)
        prev = list(tb)
        kg, vg = home.decode_rows(k1[None, :, None].cuda(), v1[None, :, None].cuda(), torch.from_numpy(tb).cuda(), cr)
        sl = oracle.lru_plan(tb, so, bo, st, rf, mt, ns)
        ko, vo = oracle.lru_gather(kc, vc, pool, tb, sl, cr, n)
        assert np.array_equal(u16(kg[0]), ko) and np.array_equal(u16(vg[0]), vo), f"step {step}: gathered rows"
        pos = np.concatenate([(tb[:, None].astype(np.int64) * cr + np.arange(cr)).reshape(-1), np.arange(nb * cr, n)])
        assert np.array_equal(ko, kc[:, pos]) and np.array_equal(vo, vc[:, pos]), f"step {step}: rows of the cache"
    lru = home.lru
    for name, a, t in (("slot_of", so, lru.slot_of), ("block_of", bo, lru.block_of), ("stamp", st, lru.stamp),
                       ("ref", rf, lru.ref), ("meta", mt, lru.meta)):
        assert np.array_equal(t.cpu().numpy(), a), name
    assert np.array_equal(u16(lru.pool), pool), "pool"
    rep = kv_host.report([home])
    assert rep["hits"] > 0 and rep["misses"] > ns and rep["hits"] + rep["misses"] == nsel * steps, rep
    assert newest > 0 and home.n == n


def test_out_of_range_pick_is_skipped_and_reported():
    Hk, D, cr, nsel = 2, 64, 4, 32
    home = kv_host.Home(Hk, D, torch.bfloat16, "cuda", lru=True)
    kv = torch.randn(2, 1, Hk, 400, D).to(torch.bfloat16).cuda()
    home.put(kv[0], kv[1])
    k1, v1 = torch.randn(2, 1, Hk, 1, D).to(torch.bfloat16).cuda()
    tb = torch.arange(nsel, dtype=torch.int32)
    tb[-1] = (kv_host.MAXC << kv_host.LOGC) // cr  # one past the last block the state can hold
    kg, vg = home.decode_rows(k1, v1, tb.cuda(), cr)
    assert ops.status() == (91 << 8) | 1  # LB2_EINVAL from the plan, the first report
    assert not kg[0, :, (nsel - 1) * cr:nsel * cr].any() and not vg[0, :, (nsel - 1) * cr:nsel * cr].any()
    assert torch.equal(kg[0, :, :4], kv[0, 0, :, :4]), "the valid picks are unaffected"


def test_home_lru_flash_next_shapes():
    """Flash-Next's decode through Home(lru=True).decode: 24/2 heads x 256, CR 4, 512 picks (a plan block of 512
    threads over 2048 slots). Three tokens, the second keeping most of the first's picks (hits); each token's
    attention over its picks against the oracle over the same rows of the whole cache."""
    import checks
    from gpu_util import f32, to_np
    g = torch.Generator().manual_seed(43)
    rng = np.random.default_rng(43)
    Hq, Hk, D, cr, nsel, n0 = 24, 2, 256, 4, 512, 12000
    rows = torch.randn(2, 1, Hk, n0 + 3, D, generator=g).to(torch.bfloat16).cuda()
    home = kv_host.Home(Hk, D, torch.bfloat16, "cuda", lru=True)
    home.put(rows[0, :, :, :n0], rows[1, :, :, :n0])
    prev = None
    for step in range(3):
        n = n0 + step + 1
        nb = n // cr
        if step == 1:
            keep = rng.choice(prev, 400, replace=False)
            rest = np.setdiff1d(np.arange(nb), keep)
            tb = np.sort(np.concatenate([keep, rng.choice(rest, nsel - 400, replace=False)]))
        else:
            tb = np.sort(rng.choice(nb, nsel, replace=False))
        prev = tb
        q = torch.randn(1, Hq, 1, D, generator=g).to(torch.bfloat16).cuda()
        k1, v1 = rows[0, :, :, n - 1:n], rows[1, :, :, n - 1:n]
        out = f32(home.decode(q, k1, v1, torch.from_numpy(tb.astype(np.int32)).cuda(), cr, D ** -0.5))
        pos = np.concatenate([(tb[:, None] * cr + np.arange(cr)).reshape(-1), np.arange(nb * cr, n)])
        pos_t = torch.from_numpy(pos).cuda()
        ref = oracle.attn(to_np(q), to_np(rows[0, :, :, :n][:, :, pos_t]), to_np(rows[1, :, :, :n][:, :, pos_t]),
                          D ** -0.5, oracle.BF16, out_dt=oracle.F32)
        checks.grading_close(out, ref, what=f"token {step}")
    rep = kv_host.report([home])
    assert rep["hits"] >= 400 and rep["hits"] + rep["misses"] == 3 * nsel, rep
