"""Gated-DeltaNet on B200: the drop-in for the reference's gdn_cuda.py (gdn_cuda.py:88-99, :318-360).

recurrence(q, k, v, g, beta, state, mask=None) keeps the reference's contract: q, k [B, T, Hk, Dk], v [B, T, Hv, Dv],
g [B, T, Hv] (one gate a head) or [B, T, Hv, Dk] (per-Dk gate), beta [B, T, Hv], state [B, Hv, Dv, Dk] fp32, mask
[B, T] or None -> (y [B, T, Hv, Dv] in q's dtype, the new state). g is the multiplicative decay (the state is
multiplied by g, gdn_cuda.py:43). Long passes with a scalar gate and no mask run the chunked tensor-core scan
(lb2_gdn_chunked, chunks of 64 positions); everything else -- decode steps, short verify passes, vector gates,
masks -- runs the position-by-position kernel (lb2_gdn_recurrent). Both are CUDA; there is no ops-loop fallback.

install_glue(rows) routes a GatedDeltaNet layer's decode rows through step_glue + norm_gate (gdn_cuda.py:271-315).

gated_delta_update keeps mlx_lm 0.32's parameter list (gdn_cuda.py:318-319) and its gating: beta = sigmoid(b)
(doubled with allow_neg_eigval), g = compute_g(A_log, a, dt_bias) = exp(-exp(A_log) * softplus(a + dt_bias))
(the expression gdn_cuda.py:146-149 spells out), a zero state when none is given.
"""
import inspect
import sys

import torch

from . import ops

_PARAMS = ["q", "k", "v", "a", "b", "A_log", "dt_bias", "state", "mask", "use_kernel", "lower_bound",
           "allow_neg_eigval"]
CHUNK_MIN_T = 64  # passes at least this long (scalar gate, no mask, Dk = Dv = 128) take the chunked scan


def recurrence(q, k, v, g, beta, state, mask=None):
    """The gated delta recurrence over all T positions in one launch (gdn_cuda.py:88-99's contract)."""
    if q.shape[1] >= CHUNK_MIN_T and ops.gdn_chunked_supported(q, v, g, mask):
        return ops.gdn_chunked(q, k, v, g, beta, state)
    return ops.gdn_recurrent(q, k, v, g, beta, state, mask)


def compute_g(A_log, a, dt_bias):
    """g = exp(-exp(A_log) * softplus(a + dt_bias)) in fp32 (mlx_lm's compute_g, as gdn_cuda.py:146-149 spells it)."""
    return torch.exp(-torch.exp(A_log.float()) * torch.nn.functional.softplus(a.float() + dt_bias.float()))


def gated_delta_update(q, k, v, a, b, A_log, dt_bias, state=None, mask=None, *, use_kernel=True, lower_bound=None,
                       allow_neg_eigval=False):
    """mlx_lm's gated_delta_update with this package's kernels (gdn_cuda.py:336-353)."""
    if lower_bound is not None:
        raise NotImplementedError("gated_delta_update: lower_bound gating (compute_lower_bound_g) is not built")
    beta = torch.sigmoid(b.float())
    if allow_neg_eigval:
        beta = beta * 2.0
    g = compute_g(A_log, a, dt_bias)
    if state is None:
        B, _, Hk, Dk = q.shape
        Hv, Dv = v.shape[-2:]
        state = torch.zeros((B, Hv, Dv, Dk), dtype=torch.float32, device=q.device)
    return recurrence(q, k, v, g, beta, state, mask)


gated_delta_update._gdn_cuda = True


def step_glue(conv, a, b, A_log, dt_bias, state, Hk, Dk, Hv, Dv):
    """T positions of qwen3_5's GatedDeltaNet from the conv output (before silu): conv [1, T, 2 Hk Dk + Hv Dv], a / b
    [1, T, Hv], A_log / dt_bias [Hv], state [1, Hv, Dv, Dk] -> (y [1, T, Hv, Dv] in conv's dtype, the new state)
    (gdn_cuda.py:235-254's contract), one fused kernel."""
    if conv.shape[0] != 1 or Dk not in (64, 128) or Hv % Hk:
        raise ValueError("step_glue: B = 1, Dk in {64, 128}, Hv a multiple of Hk")
    y, s = ops.gdn_step_glue(conv, a, b, A_log, dt_bias, state.reshape(Hv, Dv, Dk), Hk, Dk, Hv, Dv)
    return y, s.reshape(state.shape)


def norm_gate(x, z, weight, eps):
    """Qwen3NextRMSNormGated(x, z): rms_norm with `weight`, then silu(z) times it (gdn_cuda.py:257-268)."""
    if z.shape != x.shape or weight.dtype != x.dtype:
        raise ValueError("norm_gate: z must match x and weight x's dtype")
    return ops.gdn_norm_gate(x, z, weight, eps)


def install_glue(rows=1, cls=None):
    """Route a GatedDeltaNet layer's decode rows -- and passes of up to `rows` positions -- through step_glue and
    norm_gate, every other call through the layer's own __call__ (gdn_cuda.py:271-315). `cls` is the layer class
    (default: mlx_lm.models.qwen3_5.GatedDeltaNet when that module is loaded); its instances carry qwen3_5's
    attributes (in_proj_qkv, in_proj_z, in_proj_a, in_proj_b, conv1d taking channels-last [B, L, C] and returning the
    conv output before silu, A_log, dt_bias, norm with weight / eps, out_proj, num_k_heads, head_k_dim, num_v_heads,
    head_v_dim, conv_kernel_size, conv_dim) and the cache holds [conv_state, recurrent state] with advance(S). The
    fused path is taken for B = 1, S <= rows, no mask, a cache whose state exists, bf16 activations and norm weight,
    Dk in {64, 128} and Hv a multiple of Hk; the rest falls to the layer's own lines, as in the reference."""
    if cls is None:
        mod = sys.modules.get("mlx_lm.models.qwen3_5")
        if mod is None:
            raise ValueError("install_glue: give the GatedDeltaNet class (mlx_lm.models.qwen3_5 is not loaded)")
        cls = mod.GatedDeltaNet
    if getattr(cls, "_gdn_glue", False):
        return cls
    orig = cls.__call__

    def __call__(self, inputs, mask=None, cache=None):
        B, S, _ = inputs.shape
        if not (B == 1 and S <= rows and mask is None and cache is not None and cache[1] is not None
                and getattr(cache, "lengths", None) is None and not getattr(self, "training", False)
                and inputs.dtype == torch.bfloat16 and inputs.is_cuda and self.head_k_dim in (64, 128)
                and self.num_v_heads % self.num_k_heads == 0 and self.norm.weight.dtype == torch.bfloat16):
            return orig(self, inputs, mask, cache)
        qkv = self.in_proj_qkv(inputs)
        z = self.in_proj_z(inputs).reshape(B, S, self.num_v_heads, self.head_v_dim)
        b = self.in_proj_b(inputs)
        a = self.in_proj_a(inputs)
        conv_state = cache[0] if cache[0] is not None else torch.zeros(
            (B, self.conv_kernel_size - 1, self.conv_dim), dtype=inputs.dtype, device=inputs.device)
        conv_input = torch.cat([conv_state, qkv], dim=1)
        cache[0] = conv_input[:, -(self.conv_kernel_size - 1):, :].contiguous()
        conv = self.conv1d(conv_input)
        out, state = step_glue(conv, a, b, self.A_log, self.dt_bias, cache[1], self.num_k_heads, self.head_k_dim,
                               self.num_v_heads, self.head_v_dim)
        cache[1] = state
        cache.advance(S)
        out = norm_gate(out, z, self.norm.weight, self.norm.eps)
        return self.out_proj(out.reshape(B, S, -1))

    cls.__call__ = __call__
    cls._gdn_glue = True
    cls._gdn_glue_orig = orig
    return cls


def install(modules=None):
    """Route `gated_delta_update` to this package wherever a module holds the name, as the reference rebinds it in
    gated_delta and in every model module that already imported it (gdn_cuda.py:322-360). `modules` defaults to
    every loaded module whose attribute of that name takes mlx_lm's parameter list; returns the modules rebound."""
    done = []
    cands = modules if modules is not None else [m for m in list(sys.modules.values()) if m is not None]
    for mod in cands:
        fn = getattr(mod, "gated_delta_update", None)
        if fn is None or fn is gated_delta_update or getattr(fn, "_gdn_cuda", False):
            continue
        try:
            params = list(inspect.signature(fn).parameters)
        except (TypeError, ValueError):
            continue
        if params != _PARAMS:
            continue
        mod.gated_delta_update = gated_delta_update
        done.append(mod)
    return done
