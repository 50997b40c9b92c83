#!/usr/bin/env python3
"""Writes tests/golden/golden.npz: the expected outputs of the reference tests' float64 oracles on the reference
tests' own seeded inputs (tests/golden/cases.py says which tests and draws).

    python tests/golden/make_golden.py

Per case it stores a digest of the regenerated inputs (so a numpy whose generator drifts is caught, not silently
compared against other inputs) and the float64 result rounded to float32; arrays above cases.MAX_FULL elements are
stored as their projection onto cases.projection(last axis) instead. Nothing here runs the product kernels.
"""
import os
import sys

import numpy as np

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
import cases  # noqa: E402
import oracle  # noqa: E402  (cases put the repo root on sys.path)

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden.npz")


def compact(name, a, store):
    a = np.asarray(a, dtype=np.float64)
    if a.size > cases.MAX_FULL:
        store[name + ".proj"] = (a @ cases.projection(a.shape[-1])).astype(np.float32)
        store[name + ".maxabs"] = np.array(np.abs(a).max())
    else:
        store[name] = a.astype(np.float32)


def main():
    store = {}
    for c in cases.attn_cases():
        i = c["case"]
        store[f"attn{i}.digest"] = np.array(cases.digest(c["q"], c["kc"], c["vc"], c["rnd"]))
        q, k, v = (cases.to64(c[n], c["dt"]) for n in ("q", "k", "v"))
        for kind, m in (("none", None), ("causal", oracle.causal_mask(c["T"], c["N"])), ("array", c["rnd"])):
            compact(f"attn{i}.{kind}", oracle.attn_ref64(q, k, v, c["scale"], m), store)
    c = cases.gdn_cpu_case()
    store["gdncpu.digest"] = np.array(cases.digest(c["q"], c["k"], c["v"], c["g"], c["beta"], c["state"]))
    y, s = oracle.gdn_ref64(cases.to64(c["q"], c["dt"]), cases.to64(c["k"], c["dt"]), cases.to64(c["v"], c["dt"]),
                            c["g"], cases.to64(c["beta"], c["b_dt"]), c["state"])
    compact("gdncpu.y", y, store)
    compact("gdncpu.s", s, store)
    for i in range(len(cases.GDN_CUDA_CASES)):
        c = cases.gdn_cuda_case(i)
        store[f"gdncuda{i}.digest"] = np.array(cases.digest(c["q"], c["k"], c["v"], c["g"], c["beta"], c["state"],
                                                            c["mask"]))
        y, s = oracle.gdn_ref64(cases.to64(c["q"], c["dt"]), cases.to64(c["k"], c["dt"]),
                                cases.to64(c["v"], c["dt"]), c["g"], cases.to64(c["beta"], c["b_dt"]), c["state"],
                                c["mask"])
        compact(f"gdncuda{i}.y", y, store)
        compact(f"gdncuda{i}.s", s, store)
    np.savez_compressed(OUT, **store)
    print(f"wrote {OUT}: {len(store)} arrays, {os.path.getsize(OUT) / 1e3:.0f} KB")


if __name__ == "__main__":
    main()
