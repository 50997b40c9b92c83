"""GPU parity of the attention kernels (split-KV decode and tcgen05 prefill) against the CPU oracle and the golden
vectors. Bar (the build's): outputs within max-abs 2e-2 and cosine >= 0.9999 of the f32 reference, computed by the
oracle (CpuAttn's arithmetic) on the same rounded inputs; masks and causal limits must agree exactly (a wrong mask
fails these bounds by orders of magnitude)."""
import numpy as np
import pytest
import torch

import cases
import checks
import oracle
from gpu_util import f32, to_np, to_torch, randn
from larder_b200 import ops

pytestmark = pytest.mark.gpu
DEV = "cuda"


def oracle_ref(q, k, v, scale, mask_kind=oracle.MASK_NONE, mask=None):
    """f32 oracle on torch tensors (any strides: the oracle takes the same views)."""
    dt = {torch.bfloat16: oracle.BF16, torch.float16: oracle.F16, torch.float32: oracle.F32}[q.dtype]
    qn, kn, vn = (to_np(t) for t in (q, k, v))
    m = None if mask is None else mask.cpu().numpy().reshape(q.shape[2], k.shape[2])
    return oracle.attn(qn, kn, vn, scale, dt, mask_kind, m, out_dt=oracle.F32)


@pytest.fixture(autouse=True)
def _status_clean():
    yield
    assert ops.status() == 0, "a device wait gave up"


# ------------------------------------------------------------------------------------------------ decode

@pytest.mark.parametrize("case", [0, 3])
def test_decode_reference_cases(case):
    """tests/test_cpu_kern.py's decode cases (one query, long keys, K/V slices of a longer cache buffer)."""
    c = [c for c in cases.attn_cases()][case]
    dt = c["dt"]
    q, kc, vc = (to_torch(c[n], dt) for n in ("q", "kc", "vc"))
    k, v = kc[:, :, :c["N"]], vc[:, :, :c["N"]]
    out = f32(ops.attn_decode(q, k, v, c["scale"]))
    ref = oracle_ref(q, k, v, c["scale"])
    checks.grading_close(out, ref, what=f"decode case {case}")
    checks.golden_close(out, f"attn{case}.none", 2e-3, ulp=2 ** -7, what="decode vs golden")


def test_decode_config2_ragged():
    """Config 2: B=16, 32/4 heads x 128, bf16, lengths U[1024, 8192] in a capacity-padded cache."""
    gen = torch.Generator().manual_seed(2)
    B, Hq, Hkv, D, cap = 16, 32, 4, 128, 8192
    lens = torch.randint(1024, 8193, (B,), generator=gen)
    q = randn((B, Hq, 1, D), oracle.BF16, gen)
    k = randn((B, Hkv, cap, D), oracle.BF16, gen)
    v = randn((B, Hkv, cap, D), oracle.BF16, gen)
    out = f32(ops.attn_decode(q, k, v, D ** -0.5, kv_len=lens.to(torch.int32).to(DEV)))
    for b in range(B):
        n = int(lens[b])
        ref = oracle_ref(q[b:b + 1], k[b:b + 1, :, :n], v[b:b + 1, :, :n], D ** -0.5)
        checks.grading_close(out[b:b + 1], ref, what=f"seq {b} len {n}")


@pytest.mark.parametrize("T,Hkv", [(2, 8), (3, 8), (4, 8), (3, 4), (4, 4)])
def test_decode_causal_verify_rows(T, Hkv):
    """foldattn's multi-row verify semantics: T rows, bottom-right causal, G*T rows folded (8 to 32 of them); q a
    transposed view."""
    gen = torch.Generator().manual_seed(10 + T + Hkv)
    B, Hq, D, N = 2, 32, 128, 4100
    q = randn((B, T, Hq, D), oracle.BF16, gen).transpose(1, 2)
    kb = randn((B, Hkv, N + 200, D), oracle.BF16, gen)
    vb = randn((B, Hkv, N + 200, D), oracle.BF16, gen)
    k, v = kb[:, :, :N], vb[:, :, :N]
    out = f32(ops.attn_decode(q, k, v, D ** -0.5, causal=True))
    ref = oracle_ref(q, k, v, D ** -0.5, oracle.MASK_CAUSAL)
    checks.grading_close(out, ref, what=f"verify T={T}")


@pytest.mark.parametrize("D,dt", [(64, oracle.F16), (128, oracle.BF16), (256, oracle.BF16)])
def test_decode_head_dims(D, dt):
    """Each head dim with 8 and 16 folded rows (one and two 8-row tiles), both schedules."""
    gen = torch.Generator().manual_seed(D)
    for Hq in (16, 32):
        q = randn((1, Hq, 1, D), dt, gen)
        k = randn((1, 2, 3000, D), dt, gen)
        v = randn((1, 2, 3000, D), dt, gen)
        for split in (0, 64, 1024):
            out = f32(ops.attn_decode(q, k, v, D ** -0.5, split=split))
            checks.grading_close(out, oracle_ref(q, k, v, D ** -0.5), what=f"D={D} Hq={Hq} split={split}")


def test_decode_partial_combine_equals_whole():
    """KV-range shards: per-range partial (o, lse), then the log-sum-exp combine equals one call over all keys."""
    gen = torch.Generator().manual_seed(5)
    B, Hq, Hkv, D, N, R = 4, 32, 4, 128, 4096, 4
    q = randn((B, Hq, 1, D), oracle.BF16, gen)
    k = randn((B, Hkv, N, D), oracle.BF16, gen)
    v = randn((B, Hkv, N, D), oracle.BF16, gen)
    parts = [ops.attn_decode_partial(q, k[:, :, r * N // R:(r + 1) * N // R], v[:, :, r * N // R:(r + 1) * N // R],
                                     D ** -0.5) for r in range(R)]
    po = torch.stack([p[0] for p in parts])
    pl = torch.stack([p[1] for p in parts])
    out = f32(ops.attn_combine(po, pl, torch.bfloat16))
    whole = f32(ops.attn_decode(q, k, v, D ** -0.5))
    checks.grading_close(out, oracle_ref(q, k, v, D ** -0.5), what="combined shards")
    assert np.abs(out - whole).max() <= 2e-2


def test_decode_balanced_runs_cross_pairs():
    """The balanced schedule (split = 0) on many short, ragged sequences (zero-length and sub-tile ones among them):
    a CTA's tile run crosses many (b, hk) pairs and a long pair spans many CTAs; both modes match the oracle."""
    gen = torch.Generator().manual_seed(8)
    B, Hq, Hkv, D, cap = 300, 8, 2, 128, 704
    lens = torch.randint(0, cap + 1, (B,), generator=gen)
    lens[:5] = torch.tensor([0, 1, 63, 64, 65])
    lens[-1] = cap
    q = randn((B, Hq, 1, D), oracle.BF16, gen)
    k = randn((B, Hkv, cap, D), oracle.BF16, gen)
    v = randn((B, Hkv, cap, D), oracle.BF16, gen)
    kv_len = lens.to(torch.int32).to(DEV)
    bal = f32(ops.attn_decode(q, k, v, D ** -0.5, kv_len=kv_len))
    spl = f32(ops.attn_decode(q, k, v, D ** -0.5, kv_len=kv_len, split=128))
    for b in range(B):
        n = int(lens[b])
        if n == 0:
            assert np.all(bal[b] == 0) and np.all(spl[b] == 0), f"seq {b}: zero length must give zeros"
            continue
        ref = oracle_ref(q[b:b + 1], k[b:b + 1, :, :n], v[b:b + 1, :, :n], D ** -0.5)
        checks.grading_close(bal[b:b + 1], ref, what=f"balanced seq {b} len {n}")
        checks.grading_close(spl[b:b + 1], ref, what=f"split seq {b} len {n}")
    # one long sequence over few heads: the pair's tiles spread over many CTAs (many partials a row)
    q1 = randn((1, 8, 1, D), oracle.BF16, gen)
    k1 = randn((1, 1, 8192, D), oracle.BF16, gen)
    v1 = randn((1, 1, 8192, D), oracle.BF16, gen)
    checks.grading_close(f32(ops.attn_decode(q1, k1, v1, D ** -0.5)), oracle_ref(q1, k1, v1, D ** -0.5),
                         what="one pair over many CTAs")


def test_decode_repeated_shapes_and_graph_replay():
    """Calls of different shapes (and grid sizes) in turn on one shared workspace, then the decode (persistent kernel
    and its programmatically dependent combine) captured in a CUDA graph and replayed with new inputs: all match the
    oracle."""
    gen = torch.Generator().manual_seed(9)
    D = 128
    shapes = [(16, 32, 4, 4096), (1, 8, 1, 300), (16, 32, 4, 4096), (3, 16, 2, 2000)]
    for B, Hq, Hkv, N in shapes:
        q = randn((B, Hq, 1, D), oracle.BF16, gen)
        k = randn((B, Hkv, N, D), oracle.BF16, gen)
        v = randn((B, Hkv, N, D), oracle.BF16, gen)
        checks.grading_close(f32(ops.attn_decode(q, k, v, D ** -0.5)), oracle_ref(q, k, v, D ** -0.5),
                             what=f"B={B} Hkv={Hkv} N={N}")
    B, Hq, Hkv, N = 8, 32, 4, 3000
    q = randn((B, Hq, 1, D), oracle.BF16, gen)
    k = randn((B, Hkv, N, D), oracle.BF16, gen)
    v = randn((B, Hkv, N, D), oracle.BF16, gen)
    lens = torch.randint(1, N + 1, (B,), generator=gen).to(torch.int32).to(DEV)
    out = torch.empty_like(q)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        ops.attn_decode(q, k, v, D ** -0.5, kv_len=lens, out=out)  # workspace allocated outside the capture
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        ops.attn_decode(q, k, v, D ** -0.5, kv_len=lens, out=out)
    ln = lens.cpu()
    for rep in range(3):
        q.copy_(randn((B, Hq, 1, D), oracle.BF16, gen))
        graph.replay()
        torch.cuda.synchronize()
        got = f32(out)
        for b in range(B):
            n = int(ln[b])
            ref = oracle_ref(q[b:b + 1], k[b:b + 1, :, :n], v[b:b + 1, :, :n], D ** -0.5)
            checks.grading_close(got[b:b + 1], ref, what=f"replay {rep} seq {b}")
    del graph


def test_decode_empty_and_short_sequences():
    """A zero-length sequence gives zeros; lengths shorter than one tile and than T work."""
    gen = torch.Generator().manual_seed(6)
    q = randn((3, 8, 1, 128), oracle.BF16, gen)
    k = randn((3, 2, 256, 128), oracle.BF16, gen)
    v = randn((3, 2, 256, 128), oracle.BF16, gen)
    lens = torch.tensor([0, 1, 37], dtype=torch.int32, device=DEV)
    out = f32(ops.attn_decode(q, k, v, 128 ** -0.5, kv_len=lens))
    assert np.all(out[0] == 0)
    for b, n in ((1, 1), (2, 37)):
        checks.grading_close(out[b:b + 1], oracle_ref(q[b:b + 1], k[b:b + 1, :, :n], v[b:b + 1, :, :n], 128 ** -0.5))


# ------------------------------------------------------------------------------------------------ prefill

@pytest.mark.parametrize("kind", ["none", "causal", "array"])
def test_prefill_reference_case(kind):
    """tests/test_cpu_kern.py's prefill case (T=9 over 300 keys, 16/2 x 256, bf16, cache-slice K/V)."""
    c = [c for c in cases.attn_cases()][1]
    q, kc, vc = (to_torch(c[n], c["dt"]) for n in ("q", "kc", "vc"))
    k, v = kc[:, :, :c["N"]], vc[:, :, :c["N"]]
    mask = {"none": None, "causal": "causal", "array": torch.from_numpy(c["rnd"]).to(DEV)}[kind]
    out = f32(ops.attn_prefill(q, k, v, c["scale"], mask))
    mk = {"none": oracle.MASK_NONE, "causal": oracle.MASK_CAUSAL, "array": oracle.MASK_ARRAY}[kind]
    ref = oracle_ref(q, k, v, c["scale"], mk, None if kind != "array" else torch.from_numpy(c["rnd"]))
    checks.grading_close(out, ref, what=f"prefill {kind}")
    checks.golden_close(out, f"attn1.{kind}", 2e-3, ulp=2 ** -7, what="prefill vs golden")


@pytest.mark.parametrize("D,Hq,Hkv,T,N,dt", [(256, 16, 2, 256, 512, oracle.BF16), (128, 32, 4, 300, 300, oracle.BF16),
                                             (64, 8, 8, 130, 1000, oracle.F16), (256, 4, 2, 2048, 2048, oracle.BF16),
                                             (128, 8, 1, 77, 4000, oracle.F16)])
def test_prefill_causal_shapes(D, Hq, Hkv, T, N, dt):
    gen = torch.Generator().manual_seed(D + T)
    q = randn((1, T, Hq, D), dt, gen).transpose(1, 2)  # mlx_lm hands q over as a transposed view
    kb = randn((1, Hkv, N + 64, D), dt, gen)
    vb = randn((1, Hkv, N + 64, D), dt, gen)
    k, v = kb[:, :, :N], vb[:, :, :N]
    out = f32(ops.attn_prefill(q, k, v, D ** -0.5, "causal"))
    checks.grading_close(out, oracle_ref(q, k, v, D ** -0.5, oracle.MASK_CAUSAL), what=f"D={D} T={T} N={N}")


def test_prefill_gate_epilogue():
    """Config 3's gated output: attn * sigmoid(gate), gate [B, T, Hq*D] seen as [B, Hq, T, D]."""
    gen = torch.Generator().manual_seed(33)
    B, Hq, Hkv, D, T, N = 1, 16, 2, 256, 256, 768
    q = randn((B, T, Hq, D), oracle.BF16, gen).transpose(1, 2)
    k = randn((B, Hkv, N, D), oracle.BF16, gen)
    v = randn((B, Hkv, N, D), oracle.BF16, gen)
    gate = randn((B, T, Hq * D), oracle.BF16, gen)
    g4 = gate.view(B, T, Hq, D).transpose(1, 2)
    out = f32(ops.attn_prefill(q, k, v, D ** -0.5, "causal", gate=g4))
    ref = oracle_ref(q, k, v, D ** -0.5, oracle.MASK_CAUSAL) * (1 / (1 + np.exp(-f32(g4))))
    checks.grading_close(out, ref, what="gated")


def test_prefill_t_greater_than_n_rows_without_keys():
    """Rows that see no key (T > N under bottom-right causal) come out as zeros."""
    gen = torch.Generator().manual_seed(44)
    q = randn((1, 4, 200, 128), oracle.BF16, gen)
    k = randn((1, 4, 150, 128), oracle.BF16, gen)
    v = randn((1, 4, 150, 128), oracle.BF16, gen)
    out = f32(ops.attn_prefill(q, k, v, 128 ** -0.5, "causal"))
    ref = oracle_ref(q, k, v, 128 ** -0.5, oracle.MASK_CAUSAL)
    assert np.all(out[:, :, :50] == 0)
    checks.grading_close(out, ref)
