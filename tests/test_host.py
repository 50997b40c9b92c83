"""Host-side logic of the drop-in modules, on CPU: chunk bounds and key cuts as the reference defines them, routing
of calls to the right kernel (recorded by spies instead of run), module-attribute rebinding by install(), and the
gated_delta_update signature. No kernel runs here."""
import types

import pytest
import torch

from larder_b200 import chunkattn, foldattn, gdn_cuda, ops


def test_bounds_fold_short_tail():
    # chunkattn.py:350-356: `rows` apart, a last chunk under min_rows folded into the one before
    assert chunkattn._bounds(300, 128, 128) == [0, 128, 300]
    assert chunkattn._bounds(8192, 2048, 128) == [0, 2048, 4096, 6144, 8192]
    assert chunkattn._bounds(100, 128, 128) == [0, 100]
    assert chunkattn._bounds(260, 128, 2) == [0, 128, 256, 260]
    assert chunkattn._bounds(258, 64, 128) == [0, 128, 258]  # rows raised to min_rows first


def test_cut_rounds_and_floors():
    # chunkattn.py:318-322
    assert chunkattn._cut(100, 5000, 4097) == 4160      # floored to 4097, then rounded up to 64
    assert chunkattn._cut(100, 3000, 4097) == 128       # n below the floor: only the rounding
    assert chunkattn._cut(2990, 3000, 0) == 3000         # capped at n
    assert chunkattn._cut(4200, 9000, 4097) == 4224


class Spy:
    def __init__(self):
        self.calls = []

    def __call__(self, name):
        def f(*a, **kw):
            self.calls.append((name, a, kw))
            return "out"
        return f


@pytest.fixture
def spy(monkeypatch):
    s = Spy()
    monkeypatch.setattr(ops, "attn_decode", s("decode"))
    monkeypatch.setattr(ops, "attn_prefill", s("prefill"))
    return s


def test_routing_few_rows_to_decode_many_to_prefill(spy):
    q1 = torch.zeros(1, 32, 1, 128, dtype=torch.bfloat16)
    q4 = torch.zeros(1, 32, 4, 128, dtype=torch.bfloat16)
    q9 = torch.zeros(1, 16, 9, 256, dtype=torch.bfloat16)
    kv = torch.zeros(1, 4, 500, 128, dtype=torch.bfloat16)
    kv2 = torch.zeros(1, 2, 500, 256, dtype=torch.bfloat16)
    chunkattn.attend(q1, kv, kv, 0.1, None)                # G*T = 8: decode
    chunkattn.attend(q4, kv, kv, 0.1, "causal")            # G*T = 32: decode, causal
    chunkattn.attend(q9, kv2, kv2, 0.1, "causal")          # G*T = 72 > 16 at D=256: prefill
    m = torch.ones(1, 1, 1, 500, dtype=torch.bool)
    chunkattn.attend(q1, kv, kv, 0.1, m)                   # an array mask: prefill
    assert [c[0] for c in spy.calls] == ["decode", "decode", "prefill", "prefill"]
    assert spy.calls[1][2]["causal"] is True and spy.calls[0][2]["causal"] is False


def test_wrapper_refuses_what_it_cannot_serve(spy):
    f = chunkattn._wrap(stock=None)
    q = torch.zeros(1, 8, 1, 64)
    with pytest.raises(NotImplementedError):
        f(q, q, q, None, 0.1, None, sinks=torch.zeros(8))
    with pytest.raises(NotImplementedError):
        f(q, q, q, types.SimpleNamespace(bits=4), 0.1, None)
    with pytest.raises(ValueError):
        f(q, q, q, None, 0.1, "sliding")
    assert spy.calls == []


def test_ops_refuse_host_tensors():
    """No op has a CPU path: handed host tensors, each raises before it touches the library or allocates."""
    from larder_b200 import layer_glue

    bf = torch.bfloat16
    q, kv = torch.zeros(1, 8, 4, 128, dtype=bf), torch.zeros(1, 2, 16, 128, dtype=bf)
    g, beta = torch.ones(1, 4, 8), torch.ones(1, 4, 8, dtype=bf)
    gq, gv = torch.zeros(1, 4, 4, 128, dtype=bf), torch.zeros(1, 4, 8, 128, dtype=bf)
    calls = [
        lambda: ops.attn_prefill(q, kv, kv, 0.1, "causal"),
        lambda: ops.attn_decode(q[:, :, :1], kv, kv, 0.1),
        lambda: ops.gdn_recurrent(gq, gq, gv, g, beta),
        lambda: ops.gdn_chunked(gq, gq, gv, g, beta),
        lambda: ops.kv_gather_picks(kv[0], kv[0], torch.zeros(2, dtype=torch.int32), 4),
        lambda: layer_glue.out_gate(torch.zeros(1, 2, 256, dtype=bf), torch.zeros(1, 2, 512, dtype=bf), 2),
    ]
    for call in calls:
        with pytest.raises(ValueError, match="CUDA"):
            call()


def test_chunked_runs_all_rows_in_one_launch(spy):
    """The fused kernel keeps no score buffer, so the wide cut's row chunks become one launch over all T rows and
    all N keys (bottom-right causal), whatever `rows`, `min_rows` and `floor` say."""
    B, Hq, Hkv, D, T, N = 1, 16, 2, 256, 300, 1000
    q = torch.zeros(B, Hq, T, D, dtype=torch.bfloat16)
    k = torch.zeros(B, Hkv, N, D, dtype=torch.bfloat16)
    chunkattn.chunked(q, k, k, 0.0625, 128, 128, floor=512)
    calls = [(c[0], c[1][0].shape[2], c[1][1].shape[2], c[1][4]) for c in spy.calls]
    assert calls == [("prefill", T, N, "causal")]


def test_install_rebinds_module_attribute():
    mod = types.ModuleType("fake_model_module")
    mod.scaled_dot_product_attention = lambda *a, **k: "stock"
    import sys
    sys.modules["fake_model_module"] = mod

    class Attn:
        n_heads, n_kv_heads, scale = 16, 2, 256 ** -0.5
    Attn.__module__ = "fake_model_module"

    class Model:
        def modules(self):
            return [Attn()]
    try:
        table = chunkattn.install(Model())
        assert table == {(16, 2, 256): (0.0, 1, 0)}
        assert getattr(mod.scaled_dot_product_attention, "chunkattn", False)
        first = mod.scaled_dot_product_attention
        chunkattn.install(Model())                       # idempotent: not wrapped twice
        assert mod.scaled_dot_product_attention is first
        foldattn.install(Model())                        # composes on top, keeps chunkattn underneath
        assert mod.scaled_dot_product_attention.stock is first
    finally:
        del sys.modules["fake_model_module"]


def test_gdn_install_matches_signature_only():
    good = types.ModuleType("fake_gd")

    def gated_delta_update(q, k, v, a, b, A_log, dt_bias, state=None, mask=None, *, use_kernel=True,
                           lower_bound=None, allow_neg_eigval=False):
        return "ops"
    good.gated_delta_update = gated_delta_update
    other = types.ModuleType("fake_other")
    other.gated_delta_update = lambda q, k, v: None
    done = gdn_cuda.install([good, other])
    assert done == [good] and good.gated_delta_update is gdn_cuda.gated_delta_update
    assert other.gated_delta_update is not gdn_cuda.gated_delta_update
    assert list(__import__("inspect").signature(gdn_cuda.gated_delta_update).parameters) == gdn_cuda._PARAMS


def test_compute_g_matches_formula():
    A_log = torch.tensor([0.3, -1.0])
    a = torch.tensor([[0.5, 2.0]])
    dt = torch.tensor([0.1, -0.2])
    g = gdn_cuda.compute_g(A_log, a, dt)
    ref = torch.exp(-torch.exp(A_log) * torch.log1p(torch.exp(a + dt)))
    assert torch.allclose(g, ref, rtol=1e-6)


def test_fold_split_from_chunks(spy):
    q = torch.zeros(1, 32, 4, 128, dtype=torch.bfloat16)
    k = torch.zeros(1, 8, 5000, 128, dtype=torch.bfloat16)
    foldattn.fold(q, k, k, 0.1, 8)
    assert spy.calls[0][2]["split"] == 640 and spy.calls[0][2]["causal"] is True
