"""Tolerance checks shared by the CPU and GPU tests.

The reference's own bars (tests/test_cpu_kern.py:25, :129-133, :167-169):
  attention  |got - ref| <= ulp(dtype) * |ref| + 1e-5 * max|ref|, ulp = 2^-8 (bf16), 2^-11 (f16), 0 (f32)
  GDN        state: max|got - ref| / max|ref| < 1e-5; y: |got - ref| <= 2^-8 |ref| + 1e-5 max|ref|
The build's grading bars (the north star): bf16 outputs within max-abs 2e-2 and cosine >= 0.9999 of the f32
reference, GDN recurrent state within 1e-2 relative after 8k tokens.
"""
import numpy as np

import cases
import oracle

ULP = {oracle.F32: 0.0, oracle.BF16: 2.0 ** -8, oracle.F16: 2.0 ** -11}
GOLDEN = None


def golden():
    global GOLDEN
    if GOLDEN is None:
        import os
        GOLDEN = np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "golden.npz"))
    return GOLDEN


def attn_close(got, ref, dt, what=""):
    """The reference's attention bar, elementwise; got / ref float arrays."""
    got, ref = np.asarray(got, np.float64), np.asarray(ref, np.float64)
    tol = ULP[dt] * np.abs(ref) + 1e-5 * np.abs(ref).max()
    worst = float((np.abs(got - ref) - tol).max())
    assert worst <= 0, f"{what}: beyond the reference tolerance by {worst:.3g}"


def golden_close(got, name, rel, abs_scale=None, ulp=0.0, what=""):
    """Compare got (float array) with golden entry `name`: full arrays elementwise with
    ulp * |ref| + rel * max|ref|; projected entries through the same projection, the bound summed over |R|."""
    g = golden()
    got = np.asarray(got, np.float64)
    if name in g.files:
        ref = g[name].astype(np.float64)
        tol = ulp * np.abs(ref) + rel * np.abs(ref).max()
        worst = float((np.abs(got - ref) - tol).max())
        assert worst <= 0, f"{what} {name}: off by {worst:.3g} beyond tolerance"
        return
    R = cases.projection(got.shape[-1])
    proj = got @ R
    ref = g[name + ".proj"].astype(np.float64)
    maxabs = float(g[name + ".maxabs"])
    # |sum_i (got_i - ref_i) R_ij| <= sum_i |R_ij| (ulp |ref_i| + rel maxabs) <= sum_i |R_ij| (ulp + rel) maxabs,
    # plus float32 storage rounding of the projection itself
    bound = np.abs(R).sum(0) * (ulp + rel) * maxabs + 1e-6 * np.abs(ref) + 1e-7 * maxabs
    worst = float((np.abs(proj - ref) - bound).max())
    assert worst <= 0, f"{what} {name}: projection off by {worst:.3g} beyond tolerance"


def grading_close(got, ref, max_abs=2e-2, min_cos=0.9999, what=""):
    """The north star's bar for bf16 outputs against the f32 reference."""
    got, ref = np.asarray(got, np.float64).ravel(), np.asarray(ref, np.float64).ravel()
    err = float(np.abs(got - ref).max()) if got.size else 0.0
    den = np.linalg.norm(got) * np.linalg.norm(ref)
    cos = float(got @ ref / den) if den > 0 else (1.0 if np.array_equal(got, ref) else 0.0)
    assert err <= max_abs and cos >= min_cos, f"{what}: max-abs {err:.3g} (<= {max_abs}), cos {cos:.6f}"
    return err, cos
