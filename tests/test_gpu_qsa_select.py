"""QSA indexer block selection on the GPU (qwen4_exp_vendor.py:271-292; stream_fast.py:6243-6305): scores and the
top-k against the CPU oracle. Indices are integer work: the picks must be the same set as the oracle's, in
ascending order (the `tb` order of stream_fast.py:6478-6491); where the k-th and (k+1)-th scores lie closer than the
measured fp32 summation error, only such boundary blocks may trade places. Ties at the threshold go to the lowest
index."""
import math

import numpy as np
import pytest
import torch

import oracle
from gpu_util import to_torch
from larder_b200 import ops, qsa

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _status_clean():
    yield
    assert ops.status() == 0, "a device wait gave up"


def bf16(a):
    return oracle.f32_to_bf16(np.asarray(a, dtype=np.float32))


@pytest.mark.parametrize("B, S, H, D, nb, cr, k, offset_from_end", [
    (1, 1, 4, 128, 32768, 4, 512, 1),   # Flash-Next decode at 131072 tokens: 4 heads x 128, CR 4, budget 2048
    (4, 1, 4, 128, 3000, 4, 512, 3),    # a batch of decode rows, a partial trailing block
    (2, 3, 8, 64, 1501, 4, 256, 3),     # verify rows, 8 heads x 64, a block count that is not a multiple of 4
    (1, 2, 4, 64, 40001, 4, 2048, 2),   # a cluster of 8 CTAs a row
    (1, 1, 4, 64, 140001, 4, 2048, 1),  # more blocks than a cluster holds in registers: the streamed passes
    (3, 2, 2, 128, 5000, 4, 300, 0),    # two heads (MMA columns 2-7 zero), complete blocks only
    (1, 4, 1, 64, 777, 8, 64, 5),       # one head, compress ratio 8
])
def test_qsa_select_matches_oracle(B, S, H, D, nb, cr, k, offset_from_end):
    rng = np.random.default_rng(nb + S)
    q = bf16(rng.standard_normal((B, S, H, D)))
    pooled = bf16(rng.standard_normal((B, nb, D)))
    offset = nb * cr + offset_from_end - S  # the rows sit after every complete block
    top_ref, sc_ref = oracle.qsa_select(q, pooled, offset, cr, k, math.sqrt(D))
    top, sc = qsa.qsa_select(to_torch(q, oracle.BF16), to_torch(pooled, oracle.BF16), offset, cr, k, scores_out=True)
    sc = sc.cpu().numpy().astype(np.float64)
    fin = np.isfinite(sc_ref)
    assert np.array_equal(fin, np.isfinite(sc))
    err = np.max(np.abs(sc[fin] - sc_ref[fin]))
    assert err <= 1e-5 * np.abs(sc_ref[fin]).max()  # fp32 sums against float64
    top = top.cpu().numpy()
    for b in range(B):
        for s in range(S):
            assert np.all(np.diff(top[b, s][top[b, s] < nb]) > 0)
            srt = np.sort(sc_ref[b, s][np.isfinite(sc_ref[b, s])])[::-1]
            if len(srt) <= k or srt[k - 1] - srt[k] > 2 * err:
                assert np.array_equal(top[b, s], top_ref[b, s])
            else:  # two scores closer than the summation error at the boundary: only they may trade places
                kth = srt[k - 1]
                for n in set(top[b, s].tolist()) ^ set(top_ref[b, s].tolist()):
                    assert abs(sc_ref[b, s, n] - kth) <= 2 * err


def test_qsa_select_rows_with_fewer_candidates_and_ties():
    """Early rows see fewer than k complete blocks: all of them are picked, then n_blocks. Equal keys give equal
    scores: the lowest indices win."""
    B, S, H, D, nb, cr, k = 1, 4, 4, 128, 64, 4, 16
    rng = np.random.default_rng(7)
    q = bf16(rng.standard_normal((B, S, H, D)))
    row = rng.standard_normal(D)
    pooled = bf16(np.broadcast_to(row, (B, nb, D)))  # every block the same key: every score equal
    offset = 30  # rows at positions 30..33: 7, 7, 8, 8 complete blocks
    top_ref, _ = oracle.qsa_select(q, pooled, offset, cr, k, math.sqrt(D))
    top = qsa.qsa_select(to_torch(q, oracle.BF16), to_torch(pooled, oracle.BF16), offset, cr, k).cpu().numpy()
    assert np.array_equal(top, top_ref)
    assert list(top[0, 0]) == list(range(7)) + [nb] * 9
    pooled2 = bf16(np.broadcast_to(row, (B, 1000, D)))
    top2 = qsa.qsa_select(to_torch(q, oracle.BF16), to_torch(pooled2, oracle.BF16), 4000, cr, k).cpu().numpy()
    assert list(top2[0, 0]) == list(range(k))  # 1000 equal candidates: the first k
