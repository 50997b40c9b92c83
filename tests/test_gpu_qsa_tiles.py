"""QSA tile-sparse prefill (qsa_tiles.py's role) on the GPU: the tile-skipping kernel against the CPU oracle with the
same mask, and bit-equal to the masked kernel that visits every tile, for QSA-style masks (the causal rule, a local
window, and randomly picked 16-key blocks per 16-row group, as the reference's tile test builds them), on both
prefill kernels (CTA pairs for 256 rows at head dims 128 / 256, one CTA otherwise), with rows and whole row blocks
that keep nothing; install() routes chunkattn's array-masked calls to it."""
import numpy as np
import pytest
import torch

import checks
import oracle
from gpu_util import f32, to_np
from larder_b200 import chunkattn, ops, qsa_tiles

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _status_clean():
    yield
    assert ops.status() == 0, "a device wait gave up"


def qsa_mask(T, N, density, g, window=64, empty_rows=()):
    """Causal (bottom-right), the last `window` keys of each row, and a random share of 16-key blocks per 16-row
    group; rows in empty_rows keep nothing."""
    off = N - T
    r = torch.arange(T)[:, None]
    c = torch.arange(N)[None, :]
    causal = c <= off + r
    local = c > off + r - window
    picks = torch.rand(-(-T // 16), -(-N // 16), generator=g) < density
    blocks = picks.repeat_interleave(16, 0)[:T].repeat_interleave(16, 1)[:, :N]
    m = causal & (local | blocks)
    for i in empty_rows:
        m[i] = False
    return m


def rnd(g, *shape):
    return torch.randn(*shape, generator=g).to(torch.bfloat16).cuda()


@pytest.mark.parametrize("Hq,Hkv,D,T,N,density", [(24, 2, 256, 512, 4096, 0.05), (8, 2, 128, 600, 2000, 0.2),
                                                   (8, 2, 128, 100, 3000, 0.1), (4, 4, 64, 300, 1200, 0.3),
                                                   (24, 2, 256, 96, 4096, 0.05)])
def test_tiled_matches_oracle_and_masked_kernel(Hq, Hkv, D, T, N, density):
    g = torch.Generator().manual_seed(T + N)
    q, k, v = rnd(g, 1, Hq, T, D), rnd(g, 1, Hkv, N, D), rnd(g, 1, Hkv, N, D)
    m = qsa_mask(T, N, density, g, empty_rows=(3,)).cuda()
    out = ops.attn_prefill_tiled(q, k, v, D ** -0.5, m)
    dense = ops.attn_prefill(q, k, v, D ** -0.5, m)
    assert torch.equal(out, dense), "tile skipping changed the result"
    ref = oracle.attn(to_np(q), to_np(k), to_np(v), D ** -0.5, oracle.BF16, oracle.MASK_ARRAY, m.cpu().numpy(),
                      out_dt=oracle.F32)
    checks.grading_close(f32(out), ref, what=f"tiled {Hq}/{Hkv}x{D} T={T} N={N}")
    assert not f32(out)[0, :, 3].any(), "a row that keeps nothing gives zeros"
    if density <= 0.05:  # sparse enough that whole tiles were skipped
        assert qsa_tiles.group_flags(m, D).float().mean().item() < 1.0


def test_mask_view_with_padded_rows():
    """A mask that is a column slice of a wider one (row stride 2016, a multiple of 16; N = 2001, not): the tile
    listing reads 16 keys a load and the last tile's short piece bytewise."""
    g = torch.Generator().manual_seed(6)
    Hq, Hkv, D, T, N = 8, 2, 128, 300, 2001
    q, k, v = rnd(g, 1, Hq, T, D), rnd(g, 1, Hkv, N, D), rnd(g, 1, Hkv, N, D)
    wide = torch.zeros(T, 2016, dtype=torch.bool)
    wide[:, :N] = qsa_mask(T, N, 0.1, g)
    wide[:, N:] = True  # columns past N must not be read
    m = wide.cuda()[:, :N]
    out = ops.attn_prefill_tiled(q, k, v, D ** -0.5, m)
    assert torch.equal(out, ops.attn_prefill(q, k, v, D ** -0.5, m))


def test_whole_row_blocks_without_keys_and_the_gate():
    g = torch.Generator().manual_seed(5)
    Hq, Hkv, D, T, N = 16, 2, 256, 640, 2048
    q, k, v = rnd(g, 1, Hq, T, D), rnd(g, 1, Hkv, N, D), rnd(g, 1, Hkv, N, D)
    gate = rnd(g, 1, T, Hq * D).view(1, T, Hq, D).transpose(1, 2)
    m = qsa_mask(T, N, 0.05, g)
    m[256:512] = False  # a whole CTA-pair row block keeps nothing: its items have no tiles
    m = m.cuda()
    out = ops.attn_prefill_tiled(q, k, v, D ** -0.5, m, gate=gate)
    assert torch.equal(out, ops.attn_prefill(q, k, v, D ** -0.5, m, gate=gate))
    assert not f32(out)[0, :, 256:512].any()


def test_install_routes_array_masked_calls():
    g = torch.Generator().manual_seed(6)
    Hq, Hkv, D, T, N = 8, 2, 128, 300, 1500
    q, k, v = rnd(g, 1, Hq, T, D), rnd(g, 1, Hkv, N, D), rnd(g, 1, Hkv, N, D)
    m = qsa_mask(T, N, 0.1, g).cuda()
    try:
        assert qsa_tiles.install(on=True)
        assert chunkattn.chunked is qsa_tiles.chunked and chunkattn.array_prefill is ops.attn_prefill_tiled
        a = chunkattn.chunked(q, k, v, D ** -0.5, 128, 128, mask=m[None, None])
        b = chunkattn._wrap(None)(q, k, v, None, D ** -0.5, m[None, None])
        c = qsa_tiles.tile_chunk(q, k, v, D ** -0.5, m, 0, T, N)
        ref = ops.attn_prefill(q, k, v, D ** -0.5, m)
        assert torch.equal(a, ref) and torch.equal(b, ref) and torch.equal(c, ref)
        assert qsa_tiles.STATS["calls"] >= 1
    finally:
        qsa_tiles.uninstall()
    assert chunkattn.chunked is not qsa_tiles.chunked
