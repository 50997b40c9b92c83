"""The KV home's LRU oracle (oracle.lru_plan / lru_inval) pinned against golden vectors made by the reference's own
NumPy emulations of its plan and inval kernels (tests/test_kv_host_emu.py:110-163, :207-215, run by
tests/golden/make_kvh_lru.py): every step's slots and every state array equal. A mistake planted in the oracle's
input (the CLOCK hand one slot on) is caught."""
import os

import numpy as np
import pytest

import oracle

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "kvh_lru.npz")


def cases():
    z = np.load(GOLD)
    out = []
    for c in range(2):
        g = {k[len(f"c{c}_"):]: z[k] for k in z.files if k.startswith(f"c{c}_")}
        out.append(g)
    return out


def fresh(g):
    ns, mb = int(g["ns"]), int(g["max_blocks"])
    return (np.full(mb, -1, np.int32), np.full(ns, -1, np.int32), np.full(ns, -1, np.int32), np.zeros(ns, np.int32),
            np.zeros(4, np.int32))


def replay(g, so, bo, st, rf, mt):
    """Runs the golden sequence on the oracle; the first step (and what) that differs, or None."""
    ns = int(g["ns"])
    for i in range(int(g["steps"])):
        if g["op"][i][0] == 1:
            oracle.lru_inval(so, bo, rf, int(g["op"][i][1]))
        else:
            sl = oracle.lru_plan(g["tb"][i], so, bo, st, rf, mt, ns)
            if not np.array_equal(sl, g["sl"][i]):
                return i, "sl"
        for name, a in (("so", so), ("bo", bo), ("st", st), ("rf", rf), ("mt", mt)):
            if not np.array_equal(a, g[name][i]):
                return i, name
    return None


@pytest.mark.parametrize("c", [0, 1])
def test_lru_oracle_matches_reference_emulation(c):
    g = cases()[c]
    assert replay(g, *fresh(g)) is None
    # the sequences exercise what the plan decides: hits, misses, evictions and trims
    mt = g["mt"][-1]
    assert mt[2] > 0 and mt[3] > int(g["ns"]) and (g["op"][:, 0] == 1).any()


def test_lru_oracle_planted_mistake_is_caught():
    g = cases()[0]
    so, bo, st, rf, mt = fresh(g)
    mt[0] = 1  # the hand one slot on
    assert replay(g, so, bo, st, rf, mt) is not None
