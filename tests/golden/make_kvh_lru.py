"""Generates tests/golden/kvh_lru.npz: golden vectors for the KV home's LRU plan and invalidation.

The reference pins its LRU kernels in tests/test_kv_host_emu.py with NumPy transliterations of them (`emu_plan`,
`emu_inval`, test_kv_host_emu.py:110-163, :207-215). That file imports MLX at module level, which this machine lacks,
so this script takes only those two functions (and their helper `inplace`) from its source with `ast`, runs them on
NumPy arrays, and records every step of two seeded decode sequences: the picks (kept from the previous token with
probability 0.6, as the reference test's `decode` does, test_kv_host_emu.py:336-347), the occasional trim, and
the LRU state after each step.

Run once, with REFERENCE naming a checkout of the reference repository; the fixture is committed:
    REFERENCE=<checkout of IamCooller/larder> python tests/golden/make_kvh_lru.py
"""
import ast
import os
import sys

import numpy as np

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "kvh_lru.npz")


class _Mx:
    """The two MLX names the emulations use, over NumPy."""
    int32 = np.int32

    @staticmethod
    def array(a, dtype=None):
        return np.asarray(a, dtype=dtype)

    @staticmethod
    def eval(*_):
        pass


def load_emulations(ref):
    src = open(os.path.join(ref, "tests", "test_kv_host_emu.py")).read()
    tree = ast.parse(src)
    keep = [n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name in ("inplace", "emu_plan", "emu_inval")]
    assert len(keep) == 3, "the reference's emulations moved"
    ns = {"np": np, "mx": _Mx}
    exec(compile(ast.Module(body=keep, type_ignores=[]), "test_kv_host_emu.py", "exec"), ns)
    return ns["emu_plan"], ns["emu_inval"]


def sequence(plan, inval, rng, nsel, cr, ns, max_blocks, steps, n0):
    nt = (nsel + 31) // 32 * 32
    so = np.full(max_blocks, -1, np.int32)
    bo = np.full(ns, -1, np.int32)
    st = np.full(ns, -1, np.int32)
    rf = np.zeros(ns, np.int32)
    mt = np.zeros(4, np.int32)
    rec = {"nsel": nsel, "cr": cr, "ns": ns, "max_blocks": max_blocks, "steps": steps}
    hist = {k: [] for k in ("op", "tb", "sl", "so", "bo", "st", "rf", "mt")}
    n, prev = n0, []
    for i in range(steps):
        tb = sl = np.zeros(nsel, np.int32)
        if i % 17 == 16:  # a trim: positions from lim * cr on are rewritten
            n = max(nsel * cr + cr, n - int(rng.integers(1, 6 * cr)))
            lim = n // cr
            inval([so, bo, rf, np.zeros(lim + 1), None], [("NS", ns)])
            op = (1, lim)
        else:
            n += 1
            nb = n // cr
            keep = {b for b in prev if b < nb and rng.random() < 0.6}
            rest = np.setdiff1d(np.arange(nb), sorted(keep))
            tb = np.sort(np.concatenate([sorted(keep), rng.choice(rest, nsel - len(keep), replace=False)]))
            tb = tb.astype(np.int32)
            (sl,) = plan([tb, so, bo, st, rf, mt, None], [("NSEL", nsel), ("NS", ns), ("NT", nt)])
            prev = list(tb)
            op = (0, 0)
        for name, a in (("op", np.array(op)), ("tb", tb), ("sl", sl), ("so", so), ("bo", bo), ("st", st), ("rf", rf),
                        ("mt", mt)):
            hist[name].append(np.asarray(a, np.int32).copy())
    rec.update({k: np.stack(v) for k, v in hist.items()})  # [steps, ...] each
    return rec


def main():
    ref = os.environ.get("REFERENCE")
    if not ref:
        sys.exit("set REFERENCE to a checkout of the reference repository (its tests/ are read and executed)")
    plan, inval = load_emulations(ref)
    rng = np.random.default_rng(2024)
    cases = [
        sequence(plan, inval, rng, nsel=16, cr=4, ns=32, max_blocks=160, steps=70, n0=200),   # the reference test's
        sequence(plan, inval, rng, nsel=40, cr=4, ns=64, max_blocks=160, steps=70, n0=400),  # NT 64, ns = NT
    ]
    flat = {}
    for c, rec in enumerate(cases):
        for key, val in rec.items():
            flat[f"c{c}_{key}"] = np.asarray(val)
    np.savez_compressed(OUT, **flat)
    print(f"wrote {OUT}: {len(cases)} sequences")


if __name__ == "__main__":
    sys.exit(main())
