"""The CPU oracle (oracle/liboracle.so) pinned against the golden vectors: the reference tests' float64 oracles,
executed from the reference's own source by tests/golden/make_golden.py, on the reference tests' own seeded inputs,
with the reference tests' tolerances. Also: the generated inputs still hash to the digests stored with the goldens,
the goldens record which reference source made them, and a mistake planted in the oracle is caught."""
import numpy as np
import pytest

import cases
import checks
import oracle


@pytest.fixture(scope="module")
def g():
    return checks.golden()


def test_goldens_come_from_the_reference_source(g):
    """The vectors were made by executing the reference tests' functions (not a restatement): the generator stores
    the functions it ran and the sha256 of the files it took them from."""
    assert "test_attn.ref" in str(g["source.functions"]) and "test_gdn_cuda.py:ref" in str(g["source.functions"])
    for f in ("source.test_cpu_kern.sha256", "source.test_gdn_cuda.sha256"):
        assert len(str(g[f])) == 64


def test_float64_restatements_agree_with_the_goldens(g):
    """oracle.attn_ref64 / gdn_ref64 (used by other tests as float64 checkers) give the same vectors as the
    reference's executed functions, to float32 storage."""
    for c in cases.attn_cases():
        q, k, v = (cases.to64(c[n], c["dt"]) for n in ("q", "k", "v"))
        for kind, m in (("none", None), ("causal", oracle.causal_mask(c["T"], c["N"])), ("array", c["rnd"])):
            checks.golden_close(oracle.attn_ref64(q, k, v, c["scale"], m), f"attn{c['case']}.{kind}", 1e-7,
                                what="attn_ref64")
    for i in range(len(cases.GDN_CUDA_CASES)):
        c = cases.gdn_cuda_case(i)
        y, s = oracle.gdn_ref64(cases.to64(c["q"], c["dt"]), cases.to64(c["k"], c["dt"]),
                                cases.to64(c["v"], c["dt"]), c["g"], cases.to64(c["beta"], c["b_dt"]), c["state"],
                                c["mask"])
        checks.golden_close(y, f"gdncuda{i}.y", 1e-7, what="gdn_ref64 y")
        checks.golden_close(s, f"gdncuda{i}.s", 1e-7, what="gdn_ref64 state")


def test_digests_match(g):
    for c in cases.attn_cases():
        assert str(g[f"attn{c['case']}.digest"]) == cases.digest(c["q"], c["kc"], c["vc"], c["rnd"])
    c = cases.gdn_cpu_case()
    assert str(g["gdncpu.digest"]) == cases.digest(c["q"], c["k"], c["v"], c["g"], c["beta"], c["state"])
    for i in range(len(cases.GDN_CUDA_CASES)):
        c = cases.gdn_cuda_case(i)
        assert str(g[f"gdncuda{i}.digest"]) == cases.digest(c["q"], c["k"], c["v"], c["g"], c["beta"], c["state"],
                                                            c["mask"])


@pytest.mark.parametrize("kind", ["none", "causal", "array"])
def test_oracle_attn_golden(kind):
    """tests/test_cpu_kern.py:151-169 against liboracle.so: decode (split keys), causal rows, array mask, K/V as
    slices of a longer cache buffer."""
    for c in cases.attn_cases():
        mk = {"none": oracle.MASK_NONE, "causal": oracle.MASK_CAUSAL, "array": oracle.MASK_ARRAY}[kind]
        for threads in (2, 0):
            o = oracle.attn(c["q"], c["k"], c["v"], c["scale"], c["dt"], mk, c["rnd"], threads=threads)
            got = oracle.to_f32(o, c["dt"])
            checks.golden_close(got, f"attn{c['case']}.{kind}", 1e-5, ulp=checks.ULP[c["dt"]],
                                what=f"case {c['case']} threads {threads}")


def test_oracle_gdn_cpu_golden():
    """tests/test_cpu_kern.py:103-134: state rel err < 1e-5, y within 2^-8 |Y| + 1e-5 max|Y|."""
    c = cases.gdn_cpu_case()
    y, s = oracle.gdn(c["q"], c["k"], c["v"], c["g"], c["beta"], c["state"], c["dt"], g_dt=c["g_dt"], b_dt=c["b_dt"])
    checks.golden_close(oracle.to_f32(y, c["dt"]), "gdncpu.y", 1e-5, ulp=2.0 ** -8, what="y")
    checks.golden_close(s, "gdncpu.s", 1e-5, what="state")


@pytest.mark.parametrize("i", range(len(cases.GDN_CUDA_CASES)))
def test_oracle_gdn_cuda_cases_golden(i):
    """tests/test_gdn_cuda.py:95-99's cases (scalar and per-Dk gate, masks, GQA) against the float64 recurrence,
    with the CPU kernel's bar; a masked position writes y = 0."""
    c = cases.gdn_cuda_case(i)
    y, s = oracle.gdn(c["q"], c["k"], c["v"], c["g"], c["beta"], c["state"], c["dt"], g_dt=c["g_dt"],
                      b_dt=c["b_dt"], mask=c["mask"])
    yf = oracle.to_f32(y, c["dt"])
    checks.golden_close(yf, f"gdncuda{i}.y", 1e-5, ulp=2.0 ** -8, what=f"case {i} y")
    checks.golden_close(s, f"gdncuda{i}.s", 1e-5, what=f"case {i} state")
    if c["mask"] is not None:
        assert not yf[~c["mask"]].any(), "a masked position wrote y"


def test_planted_mistake_is_caught():
    """A mistake planted in the oracle (scale off by 1%, then the GQA head map shifted) fails the golden check."""
    c = next(cases.attn_cases())
    o = oracle.attn(c["q"], c["k"], c["v"], c["scale"] * 1.01, c["dt"], oracle.MASK_NONE)
    with pytest.raises(AssertionError):
        checks.golden_close(oracle.to_f32(o, c["dt"]), "attn0.none", 1e-5, ulp=checks.ULP[c["dt"]])
    k2 = np.ascontiguousarray(c["k"][:, ::-1])
    v2 = np.ascontiguousarray(c["v"][:, ::-1])
    o = oracle.attn(c["q"], k2, v2, c["scale"], c["dt"], oracle.MASK_NONE)
    with pytest.raises(AssertionError):
        checks.golden_close(oracle.to_f32(o, c["dt"]), "attn0.none", 1e-5, ulp=checks.ULP[c["dt"]])


def test_fully_masked_leading_block_is_finite():
    """A key range whose first 32-key block is fully masked: the oracle adds nothing for it (the reference's
    CpuAttn would carry -inf into its accumulator there, cpu_kern.cpp:583, :601)."""
    rng = np.random.default_rng(7)
    q = rng.normal(0, 1, (1, 2, 2, 64)).astype(np.float32)
    k = rng.normal(0, 1, (1, 1, 96, 64)).astype(np.float32)
    v = rng.normal(0, 1, (1, 1, 96, 64)).astype(np.float32)
    m = np.zeros((2, 96), bool)
    m[:, 40:] = True
    o = oracle.attn(q, k, v, 0.125, oracle.F32, oracle.MASK_ARRAY, m, threads=1)
    ref = oracle.attn_ref64(q, k, v, 0.125, m)
    assert np.isfinite(o).all()
    checks.attn_close(o, ref, oracle.F32)


def test_glue_oracle_against_float64_definitions():
    """The CPU restatement of the reference's qk / agate kernels against the plain definitions in float64 (RMSNorm
    with weight, rotate-half RoPE on the first R dims, sigmoid gate), the restatement's bf16 roundings being the only
    difference."""
    rng = np.random.default_rng(11)
    B, S, NQ, NK, D, R = 2, 4, 3, 2, 128, 64
    qg = oracle.f32_to_bf16(rng.standard_normal((B, S, NQ * 2 * D)).astype(np.float32))
    kr = oracle.f32_to_bf16(rng.standard_normal((B, S, NK * D)).astype(np.float32))
    w = oracle.f32_to_bf16((1 + 0.1 * rng.standard_normal(D)).astype(np.float32))
    ang = np.arange(S)[:, None] * 10000.0 ** (-np.arange(R // 2) * 2.0 / R)[None]
    cs, sn = np.cos(np.concatenate([ang, ang], 1)), np.sin(np.concatenate([ang, ang], 1))
    q, k = oracle.qk_norm_rope(qg, kr, w, w, 1e-6, cs.astype(np.float32), sn.astype(np.float32), NQ, NK)

    def ref(x, heads):
        """(result, the magnitude the roundings scale with: each RoPE product is rounded before the sum)."""
        x = x.reshape(B, S, heads, -1)[..., :D].astype(np.float64)
        o = x / np.sqrt((x * x).mean(-1, keepdims=True) + 1e-6) * oracle.bf16_to_f32(w).astype(np.float64)
        rot = np.concatenate([-o[..., R // 2:R], o[..., :R // 2]], -1)
        mag = np.abs(o).copy()
        mag[..., :R] = np.abs(o[..., :R] * cs[None, :, None]) + np.abs(rot * sn[None, :, None])
        o[..., :R] = o[..., :R] * cs[None, :, None] + rot * sn[None, :, None]
        return o.transpose(0, 2, 1, 3), mag.transpose(0, 2, 1, 3)

    for got, x, heads in ((q, oracle.bf16_to_f32(qg), NQ), (k, oracle.bf16_to_f32(kr), NK)):
        r, mag = ref(x, heads)
        # up to five bf16 roundings stack (x inv, w, cos / sin, each product, the sum): a semantic pin (norm formula,
        # rotate-half pairing), which a wrong convention misses by order one
        assert np.all(np.abs(oracle.bf16_to_f32(got) - r) <= 8 * 2.0 ** -8 * mag + 1e-6)
    o = oracle.f32_to_bf16(rng.standard_normal((S, NQ * D)).astype(np.float32))
    g = oracle.f32_to_bf16(rng.standard_normal((S, NQ * 2 * D)).astype(np.float32))
    gate = oracle.bf16_to_f32(g).reshape(S, NQ, 2 * D)[..., D:].astype(np.float64)
    want = oracle.bf16_to_f32(o).reshape(S, NQ, D) / (1 + np.exp(-gate))
    got = oracle.bf16_to_f32(oracle.out_gate(o, g, NQ)).reshape(S, NQ, D)
    assert np.all(np.abs(got - want) <= 2 * 2.0 ** -8 * np.abs(want) + 1e-30)
