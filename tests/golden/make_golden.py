#!/usr/bin/env python3
"""Writes tests/golden/golden.npz: the expected outputs of the reference tests' own float64 oracles, executed from
the reference's source, on the reference tests' own seeded inputs (tests/golden/cases.py regenerates the draws).

    REFERENCE=<checkout of IamCooller/larder> python tests/golden/make_golden.py

The reference's test files import MLX at module level, which this machine lacks, so the oracles are taken out of
their source with `ast` and executed over NumPy (their only MLX use is `x.astype(mx.float32)` on the inputs, which a
one-name shim serves):
  * attention: the nested `ref(q, k, v, scale, mask)` of `test_attn` (tests/test_cpu_kern.py:141-149);
  * GDN, CPU kernel: the float64 loop of `test_gdn` from `Y = np.zeros(...)` to its end (tests/test_cpu_kern.py:121-128);
  * GDN, CUDA kernel: the module-level `ref(q, k, v, g, beta, state, mask)` (tests/test_gdn_cuda.py:29-45).
The sha256 of each source file is stored beside the vectors (`source.*`), so a later regeneration against another
reference revision shows in the fixture's diff.

Per case it stores a digest of the regenerated inputs (so a numpy whose generator drifts is caught, not silently
compared against other inputs) and the float64 result rounded to float32; arrays above cases.MAX_FULL elements are
stored as their projection onto cases.projection(last axis) instead. Nothing here runs the product kernels.
"""
import ast
import hashlib
import os
import sys

import numpy as np

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
import cases  # noqa: E402
import oracle  # noqa: E402  (cases put the repo root on sys.path)

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden.npz")


class _Mx:
    """The one MLX name the reference's float64 oracles touch: `a.astype(mx.float32)` on their inputs."""
    float32 = np.float32


def _source(ref, rel):
    path = os.path.join(ref, rel)
    src = open(path).read()
    return src, ast.parse(src), hashlib.sha256(src.encode()).hexdigest()


def _function(body, name):
    hits = [n for n in body if isinstance(n, ast.FunctionDef) and n.name == name]
    assert len(hits) == 1, f"{name} not found once in the reference source (the tests moved?)"
    return hits[0]


def load_reference_oracles(ref):
    """Returns (attn_ref, gdn_cpu_loop, gdn_cuda_ref, sources) taken from the reference's test files."""
    src_a, tree_a, sha_a = _source(ref, os.path.join("tests", "test_cpu_kern.py"))
    src_g, tree_g, sha_g = _source(ref, os.path.join("tests", "test_gdn_cuda.py"))

    ns_attn = {"np": np, "mx": _Mx}
    inner = _function(_function(tree_a.body, "test_attn").body, "ref")
    exec(compile(ast.Module(body=[inner], type_ignores=[]), "test_cpu_kern.py", "exec"), ns_attn)

    body = _function(tree_a.body, "test_gdn").body
    start = [i for i, n in enumerate(body) if isinstance(n, ast.Assign) and getattr(n.targets[0], "id", "") == "Y"]
    assert len(start) == 1 and isinstance(body[start[0] + 1], ast.For), "test_gdn's float64 loop moved"
    loop = compile(ast.Module(body=body[start[0]:start[0] + 2], type_ignores=[]), "test_cpu_kern.py", "exec")

    def gdn_cpu_loop(Q, K, V, G, Bt, S, B, T, Hk, Hv, D):
        ns = {"np": np, "Q": Q, "K": K, "V": V, "G": G, "Bt": Bt, "S": S.copy(), "B": B, "T": T, "Hk": Hk, "Hv": Hv,
              "D": D}
        exec(loop, ns)
        return ns["Y"], ns["S"]

    ns_gdn = {"np": np, "mx": _Mx}
    exec(compile(ast.Module(body=[_function(tree_g.body, "ref")], type_ignores=[]), "test_gdn_cuda.py", "exec"),
         ns_gdn)
    sources = {"source.test_cpu_kern.sha256": sha_a, "source.test_gdn_cuda.sha256": sha_g}
    return ns_attn["ref"], gdn_cpu_loop, ns_gdn["ref"], sources


def compact(name, a, store):
    a = np.asarray(a, dtype=np.float64)
    if a.size > cases.MAX_FULL:
        store[name + ".proj"] = (a @ cases.projection(a.shape[-1])).astype(np.float32)
        store[name + ".maxabs"] = np.array(np.abs(a).max())
    else:
        store[name] = a.astype(np.float32)


def main():
    ref = os.environ.get("REFERENCE")
    if not ref:
        sys.exit("set REFERENCE to a checkout of the reference repository (its tests/ are read and executed)")
    attn_ref, gdn_cpu_loop, gdn_cuda_ref, sources = load_reference_oracles(ref)
    store = {k: np.array(v) for k, v in sources.items()}
    store["source.functions"] = np.array("tests/test_cpu_kern.py:test_attn.ref, tests/test_cpu_kern.py:test_gdn "
                                         "(float64 loop), tests/test_gdn_cuda.py:ref")
    for c in cases.attn_cases():
        i = c["case"]
        store[f"attn{i}.digest"] = np.array(cases.digest(c["q"], c["kc"], c["vc"], c["rnd"]))
        q, k, v = (oracle.to_f32(c[n], c["dt"]) for n in ("q", "k", "v"))
        for kind, m in (("none", None), ("causal", oracle.causal_mask(c["T"], c["N"])), ("array", c["rnd"])):
            compact(f"attn{i}.{kind}", attn_ref(q, k, v, c["scale"], m), store)
    c = cases.gdn_cpu_case()
    store["gdncpu.digest"] = np.array(cases.digest(c["q"], c["k"], c["v"], c["g"], c["beta"], c["state"]))
    B, T, Hk, D = c["q"].shape
    Hv = c["v"].shape[2]
    y, s = gdn_cpu_loop(cases.to64(c["q"], c["dt"]), cases.to64(c["k"], c["dt"]), cases.to64(c["v"], c["dt"]),
                        c["g"].astype(np.float64), cases.to64(c["beta"], c["b_dt"]), c["state"].astype(np.float64),
                        B, T, Hk, Hv, D)
    compact("gdncpu.y", y, store)
    compact("gdncpu.s", s, store)
    for i in range(len(cases.GDN_CUDA_CASES)):
        c = cases.gdn_cuda_case(i)
        store[f"gdncuda{i}.digest"] = np.array(cases.digest(c["q"], c["k"], c["v"], c["g"], c["beta"], c["state"],
                                                            c["mask"]))
        y, s = gdn_cuda_ref(oracle.to_f32(c["q"], c["dt"]), oracle.to_f32(c["k"], c["dt"]),
                            oracle.to_f32(c["v"], c["dt"]), c["g"], oracle.to_f32(c["beta"], c["b_dt"]), c["state"],
                            c["mask"])
        compact(f"gdncuda{i}.y", y, store)
        compact(f"gdncuda{i}.s", s, store)
    np.savez_compressed(OUT, **store)
    print(f"wrote {OUT}: {len(store)} arrays, {os.path.getsize(OUT) / 1e3:.0f} KB")


if __name__ == "__main__":
    main()
