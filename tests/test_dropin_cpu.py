"""The drop-in installers on the CPU (no kernel runs): kv_host.install / make_class rebinding a model module's
attention cache class (kv_host.py:516-799), and gdn_cuda.install_glue patching a GatedDeltaNet class
(gdn_cuda.py:271-315) -- which calls reach the fused path and which stay on the layer's own lines."""
import types

import pytest
import torch

from dropin_models import KVCache
from larder_b200 import gdn_cuda, kv_host


@pytest.fixture
def q4():
    mod = types.SimpleNamespace(_AttnCache=KVCache)
    yield mod
    kv_host.uninstall(mod)


def test_install_rebinds_the_cache_class_once(q4, monkeypatch):
    monkeypatch.delenv("MOE_KV_HOST_FROM", raising=False)
    assert kv_host.install(q4, 1000, 512, 4, 2, 256, torch.bfloat16)
    cls = q4._AttnCache
    assert cls is not KVCache and issubclass(cls, KVCache) and cls.__name__ == "KVCache"
    assert kv_host.H == max(1000, 2 * kv_host.lru_slots(512) * 4)  # the LRU's own positions, twice
    assert kv_host.ROW_BYTES == 2 * 2 * 256 * 2
    assert kv_host.install(q4, 5, 8, 4, 2, 256, torch.bfloat16) and q4._AttnCache is cls  # idempotent
    kv_host.uninstall(q4)
    assert q4._AttnCache is KVCache


def test_install_refuses_more_picks_than_the_plan_takes(q4):
    assert not kv_host.install(q4, 1000, 1025, 4, 2, 256, torch.bfloat16)
    assert q4._AttnCache is KVCache


def test_switch_from_environment(q4, monkeypatch):
    monkeypatch.setenv("MOE_KV_HOST_FROM", "300")
    kv_host.install(q4, 100000, 16, 4, 2, 128, torch.bfloat16)
    assert kv_host.H == 300


def test_below_the_line_the_class_is_its_base(q4):
    """Under H positions the subclass runs the base's own update_and_fetch (same buffer, same growth)."""
    kv_host.install(q4, 1 << 20, 16, 4, 2, 64, torch.float32)
    c, ref = q4._AttnCache(), KVCache()
    g = torch.Generator().manual_seed(1)
    for s in (3, 300, 1):
        k, v = torch.randn(1, 2, s, 64, generator=g), torch.randn(1, 2, s, 64, generator=g)
        a, b = c.update_and_fetch(k, v), ref.update_and_fetch(k, v)
        assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])
        assert c.keys.shape == ref.keys.shape and c.offset == ref.offset
    assert not c.kv_host and c.decode(k[:, :, :1], v[:, :, :1], torch.zeros(1, dtype=torch.int32), 4) is None


class _Layer:
    num_k_heads, num_v_heads, head_k_dim, head_v_dim = 2, 4, 128, 128
    training = False

    def __init__(self):
        self.norm = types.SimpleNamespace(weight=torch.ones(128, dtype=torch.bfloat16), eps=1e-6)
        self.calls = 0

    def __call__(self, inputs, mask=None, cache=None):
        self.calls += 1
        return "own"


def test_install_glue_leaves_other_calls_on_the_layer():
    cls = type("GDN", (_Layer,), {})
    assert gdn_cuda.install_glue(rows=1, cls=cls) is cls and cls._gdn_glue
    orig = cls._gdn_glue_orig
    assert gdn_cuda.install_glue(rows=1, cls=cls) is cls and cls._gdn_glue_orig is orig  # once
    lay = cls()
    x = torch.zeros(1, 1, 16, dtype=torch.bfloat16)
    cache = [None, torch.zeros(1, 4, 128, 128)]
    assert lay(x, None, cache) == "own"                      # a CPU tensor: not the kernels' call
    assert lay(torch.zeros(1, 2, 16, dtype=torch.bfloat16), None, cache) == "own"   # more rows than installed
    assert lay(x, torch.ones(1, 1, dtype=torch.bool), cache) == "own"               # a mask
    assert lay(x, None, [None, None]) == "own"               # no state yet (a prefill comes first)
    assert lay.calls == 4


def test_install_glue_needs_a_class_when_mlx_lm_is_absent():
    with pytest.raises(ValueError, match="GatedDeltaNet class"):
        gdn_cuda.install_glue()


def test_qsa_tiles_install_is_off_unless_asked():
    from larder_b200 import chunkattn, ops, qsa_tiles
    assert not qsa_tiles.install(on=False)
    assert chunkattn.chunked is not qsa_tiles.chunked and chunkattn.array_prefill is None


def test_qsa_tiles_flags_and_plan_on_cpu_tensors():
    from larder_b200 import qsa_tiles
    m = torch.zeros(300, 700, dtype=torch.bool)
    m[10, 5] = True       # row block 0 (256 rows at D=256), key tile 0 (128 keys)
    m[299, 699] = True    # row block 1, key tile 5
    f = qsa_tiles.group_flags(m, 256)
    assert f.shape == (2, 6) and f.sum().item() == 2 and f[0, 0] and f[1, 5]
    assert qsa_tiles.plan(f) == [(0, [0]), (1, [5])]
    assert qsa_tiles.tile_shape(100, 256) == (128, 64) and qsa_tiles.tile_shape(300, 64) == (128, 128)
