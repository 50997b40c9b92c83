"""Seeded inputs of the reference's own hot-path tests, regenerated with numpy.

The reference draws every test input from seeded numpy generators (no stored golden vectors exist upstream), so the
same draws are reproduced here in the same order:

  * attention: tests/test_cpu_kern.py:137-170 -- default_rng(4); per case q, the K and V cache buffers of N + 16
    positions (K/V are their first N rows, so the head stride is not N * D), then a random [T, N] mask with
    column 0 kept; masks none / causal / array.
  * GDN, CPU kernel: tests/test_cpu_kern.py:103-134 -- default_rng(3), B, T, Hk, Hv, D = 1, 5, 4, 8, 128 from a
    non-zero state.
  * GDN, CUDA kernel: tests/test_gdn_cuda.py:48-63, :95-99 -- default_rng(i) per case i; q, k rms-normalised and
    scaled by Dk^-1 / Dk^-0.5, g from compute_g, beta = sigmoid, a non-zero state, an optional [B, T] mask.
    MLX's bf16 rounding of rms_norm and of the scale products is restated (float32 math, then round to bf16),
    so these inputs are the reference test's draws with this build's rounding, not MLX's bits.

Arrays come back in storage form: float32, or uint16 bit patterns for bf16 / f16 (oracle.BF16 / oracle.F16).
"""
import hashlib
import os
import sys

import numpy as np

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))
import oracle  # noqa: E402

F32, BF16, F16 = oracle.F32, oracle.BF16, oracle.F16

# (B, Hq, Hkv, T, N, D, dtype) of tests/test_cpu_kern.py:151-152.
ATTN_CASES = ((1, 16, 2, 1, 700, 256, BF16), (1, 16, 2, 9, 300, 256, BF16),
              (2, 4, 4, 3, 40, 64, F32), (1, 8, 1, 1, 5000, 128, F16))
# (B, T, Hk, Hv, Dk, Dv, vec, masked) of tests/test_gdn_cuda.py:95-98.
GDN_CUDA_CASES = ((1, 1, 2, 6, 128, 128, False, False), (1, 37, 2, 6, 128, 128, False, False),
                  (2, 37, 2, 6, 128, 64, False, True), (1, 37, 4, 4, 64, 32, True, False),
                  (2, 7, 2, 4, 128, 128, True, True), (1, 37, 16, 48, 128, 128, False, False))


def _cast(x32, dt):
    return oracle.from_f32(np.asarray(x32, dtype=np.float32), dt)


def digest(*arrays):
    h = hashlib.sha256()
    for a in arrays:
        if a is None:
            continue
        a = np.ascontiguousarray(a)
        h.update(str(a.dtype).encode() + str(a.shape).encode())
        h.update(a.tobytes())
    return h.hexdigest()[:32]


def attn_cases():
    """Yields dict(case, B, Hq, Hkv, T, N, D, dt, q, kc, vc, k, v, scale, rnd) in test_cpu_kern.py's draw order."""
    rng = np.random.default_rng(4)
    for i, (B, Hq, Hkv, T, N, D, dt) in enumerate(ATTN_CASES):
        q = _cast(rng.normal(0, 1, (B, Hq, T, D)).astype(np.float32), dt)
        kc = _cast(rng.normal(0, 1, (B, Hkv, N + 16, D)).astype(np.float32), dt)
        vc = _cast(rng.normal(0, 1, (B, Hkv, N + 16, D)).astype(np.float32), dt)
        rnd = rng.random((T, N)) < 0.7
        rnd[:, 0] = True
        yield dict(case=i, B=B, Hq=Hq, Hkv=Hkv, T=T, N=N, D=D, dt=dt, q=q, kc=kc, vc=vc, k=kc[:, :, :N],
                   v=vc[:, :, :N], scale=D ** -0.5, rnd=rnd)


def gdn_cpu_case():
    """tests/test_cpu_kern.py:107-115: q, k, v, g, beta, s0 (bf16 q/k/v/beta, f32 g and state)."""
    rng = np.random.default_rng(3)
    B, T, Hk, Hv, D = 1, 5, 4, 8, 128

    def f(*s):
        return rng.normal(0, 1, s).astype(np.float32)
    q = _cast(f(B, T, Hk, D) * np.float32(0.1), BF16)
    k = _cast(f(B, T, Hk, D) * np.float32(0.1), BF16)
    v = _cast(f(B, T, Hv, D), BF16)
    g = rng.uniform(0.5, 1.0, (B, T, Hv)).astype(np.float32)
    beta = _cast(rng.uniform(0, 1, (B, T, Hv)).astype(np.float32), BF16)
    s0 = f(B, Hv, D, D)
    return dict(q=q, k=k, v=v, g=g, beta=beta, state=s0, mask=None, dt=BF16, g_dt=F32, b_dt=BF16)


def _bf(x32):
    return oracle.from_f32(x32, BF16)


def _bf_f(x32):
    """Round float32 to bf16 and back (the value an MLX bf16 op leaves)."""
    return oracle.bf16_to_f32(_bf(x32))


def gdn_cuda_case(i):
    """tests/test_gdn_cuda.py:48-60 for case i of GDN_CUDA_CASES."""
    B, T, Hk, Hv, Dk, Dv, vec, masked = GDN_CUDA_CASES[i]
    rng = np.random.default_rng(i)

    def bf(*s):
        return _bf_f(rng.normal(0, 1, s).astype(np.float32))
    qn = _bf_f(oracle.rms_norm(bf(B, T, Hk, Dk)))
    q = _bf(qn * _bf_f(np.float32(Dk ** -1.0)))
    kn = _bf_f(oracle.rms_norm(bf(B, T, Hk, Dk)))
    k = _bf(kn * _bf_f(np.float32(Dk ** -0.5)))
    v = _bf(bf(B, T, Hv, Dv))
    a = bf(B, T, Hv, Dk) if vec else bf(B, T, Hv)
    A_log = rng.normal(0, 0.5, (Hv, Dk) if vec else Hv).astype(np.float32)
    dt_bias = rng.normal(0, 0.5, (Hv, Dk) if vec else Hv).astype(np.float32)
    g = oracle.compute_g(A_log, a, dt_bias)
    beta = _bf(oracle.sigmoid(bf(B, T, Hv)))
    state = rng.normal(0, 0.3, (B, Hv, Dv, Dk)).astype(np.float32)
    mask = (rng.random((B, T)) > 0.3) if masked else None
    return dict(q=q, k=k, v=v, g=g, beta=beta, state=state, mask=mask, dt=BF16, g_dt=F32, b_dt=BF16,
                shape=(B, T, Hk, Hv, Dk, Dv, vec, masked))


def to64(a, dt):
    return oracle.to_f32(a, dt).astype(np.float64)


def projection(shape_last, seed=12345, cols=8):
    """A fixed random projection [last, cols] used to store large expected outputs compactly."""
    return np.random.default_rng(seed).normal(0, 1, (shape_last, cols))


MAX_FULL = 16384  # expected arrays with more elements than this are stored as projections onto `projection`
