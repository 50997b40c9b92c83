"""QSA tile-sparse prefill attention on B200: the drop-in for the reference's qsa_tiles.py (qsa_tiles.py:28-42,
:144-292, :434-458).

A QSA mask keeps, for each query row, only the key blocks its indexer picked (plus the local window), so most of an
array-masked prefill's (row block, key tile) pairs hold no kept key. The reference runs each 16-row group's QK^T and
PV over only the 16-key tiles one of its rows keeps. Here the prefill kernel does the same at its own tile sizes:
lb2_attn_prefill_tiled lists, on the device, the key tiles each row block keeps (a row block is the rows one kernel
item takes: 256 on CTA pairs, 128 on one CTA; a key tile is the kernel's, 128 keys on CTA pairs), and the kernel
loads and multiplies only those. Every element is still masked as given, so the result is the masked attention's
(bit-equal to ops.attn_prefill with the same mask), at a cost that falls with the mask's tile density.

Surface kept: `chunked(q, k, v, scale, rows, min_rows, floor=0, mask=None)`, `tile_chunk(...)`, `install()`, `ON`,
`STATS`, and `group_flags` / `plan` in the kernel's granularity.
"""
import os

import torch

from . import chunkattn, ops

ON = os.environ.get("MOE_QSA_TILES", "0") == "1"
STATS = {"calls": 0, "tiles_kept": 0, "tiles_total": 0}
_STOCK_CHUNKED = chunkattn.chunked


def tile_shape(T, D):
    """(rows a row block, keys a key tile) of the kernel a prefill of T rows at head dim D runs on."""
    if D in (128, 256) and T > 128:
        return 256, 128
    return 128, 128 if D == 128 else 64 if D == 256 else 128


def group_flags(mask2, D):
    """[row blocks, key tiles] bool (device): which key tiles a row of each block keeps -- the lists the kernel
    builds, at its granularity (the reference's group_flags, qsa_tiles.py:351-359, at 16 x 16)."""
    T, N = mask2.shape[-2:]
    rb, bn = tile_shape(T, D)
    m = mask2.reshape(T, N)
    pad = torch.zeros(-(-T // rb) * rb, -(-N // bn) * bn, dtype=torch.bool, device=m.device)
    pad[:T, :N] = m
    return pad.view(pad.shape[0] // rb, rb, pad.shape[1] // bn, bn).any(dim=3).any(dim=1)


def plan(flags):
    """[(row block, kept key tiles ascending)] from group_flags (the reference's plan, qsa_tiles.py:28-35)."""
    return [(i, torch.nonzero(f).flatten().tolist()) for i, f in enumerate(flags)]


def tile_chunk(q, k, v, scale, mask2, c0, c1, nk, flags=None, budget=None, copies=None, gate=None):
    """Rows c0 .. c1 of the masked call over keys :nk, running only the key tiles each row block keeps
    (qsa_tiles.py:216-247's contract: [1, Hq, c1 - c0, D]). `flags`, `budget` and `copies` are the reference's
    knobs and change nothing here: the kept tiles are found on the device and nothing is materialised."""
    g = None if gate is None else gate[:, :, c0:c1]
    return ops.attn_prefill_tiled(q[:, :, c0:c1], k[:, :, :nk], v[:, :, :nk], scale, mask2[c0:c1, :nk], gate=g)


def chunked(q, k, v, scale, rows, min_rows, floor=0, mask=None, fused=False, gate=None):
    """chunkattn.chunked with an array-masked call's chunks on the tile-skipping kernel (qsa_tiles.py:266-292): the
    whole call in one launch (the fused kernel keeps no score buffer, so no row chunking is needed); calls without
    an array mask go to chunkattn's own chunked."""
    if mask is None:
        return _STOCK_CHUNKED(q, k, v, scale, rows, min_rows, floor, None, fused, gate)
    T, N = q.shape[2], k.shape[2]
    STATS["calls"] += 1
    return ops.attn_prefill_tiled(q, k, v, scale, mask.reshape(T, N), gate=gate)


def install(cache_gb=0.05, on=None):
    """With MOE_QSA_TILES=1 (or on=True): array-masked prefill calls take the tile-skipping kernel --
    chunkattn.chunked and chunkattn's array-mask route are rebound, as the reference rebinds chunkattn.chunked
    (qsa_tiles.py:434-458). The reference times the tile form against stock per shape and keeps the faster; here
    the tiled kernel is the masked kernel minus the empty tiles, never slower by more than its listing pass, so no
    calibration is kept. Returns whether it is on."""
    on = ON if on is None else on
    if not on:
        return False
    chunkattn.chunked = chunked
    chunkattn.array_prefill = ops.attn_prefill_tiled
    return True


def uninstall():
    chunkattn.chunked = _STOCK_CHUNKED
    chunkattn.array_prefill = None
