"""Stand-ins for the third-party classes the reference's drop-in surface attaches to, in torch (MLX and mlx_lm are not
installed here). Test infrastructure only.

  * KVCache: mlx-lm 0.32's KVCache contract as the reference's kv_host.make_class relies on it -- `keys` / `values`
    buffers [B, Hk, capacity, D] grown in steps of `step` (256) positions, `offset`, and update_and_fetch(keys, values)
    returning views of the first `offset` rows (the growth rule restated in kv_host.py:448-453's `_grown`).
  * GatedDeltaNet: qwen3_5's layer with the attributes gdn_cuda.install_glue reads, its own __call__ a plain torch
    composition of the reference's operations (projections, causal conv over [conv_state, x], silu, q / k RMSNorm
    scaled by Dk^-1 / Dk^-0.5, sigmoid(b), compute_g, the recurrence, the gated RMSNorm, out_proj).
"""
import torch


class KVCache:
    step = 256

    def __init__(self):
        self.keys = self.values = None
        self.offset = 0

    def update_and_fetch(self, keys, values):
        prev = self.offset
        if self.keys is None or prev + keys.shape[2] > self.keys.shape[2]:
            B, H, _, D = keys.shape
            n = (self.step + keys.shape[2] - 1) // self.step * self.step
            nk = torch.zeros((B, H, n, D), dtype=keys.dtype, device=keys.device)
            nv = torch.zeros((B, H, n, values.shape[3]), dtype=values.dtype, device=values.device)
            if self.keys is not None:
                if prev % self.step:
                    self.keys, self.values = self.keys[..., :prev, :], self.values[..., :prev, :]
                self.keys, self.values = torch.cat([self.keys, nk], 2), torch.cat([self.values, nv], 2)
            else:
                self.keys, self.values = nk, nv
        self.offset += keys.shape[2]
        self.keys[..., prev:self.offset, :] = keys
        self.values[..., prev:self.offset, :] = values
        return self.keys[..., :self.offset, :], self.values[..., :self.offset, :]

    @property
    def nbytes(self):
        return 0 if self.keys is None else 2 * self.keys.numel() * self.keys.element_size()


class ArraysCache(list):
    """[conv_state, recurrent state] with advance(S), as mlx_lm's ArraysCache for a GatedDeltaNet layer."""

    def __init__(self, state):
        super().__init__([None, state])
        self.advanced = 0

    def advance(self, s):
        self.advanced += s


def _silu16(x):
    """silu in the activation dtype: sigmoid rounded, then the product rounded (MLX's Multiply(x, Sigmoid(x)))."""
    sg = torch.sigmoid(x.float()).to(x.dtype)
    return (x.float() * sg.float()).to(x.dtype)


class GatedDeltaNet:
    def __init__(self, Hk, Hv, Dk, Dv, hidden, kernel=4, device="cuda", seed=0):
        g = torch.Generator().manual_seed(seed)
        self.num_k_heads, self.num_v_heads, self.head_k_dim, self.head_v_dim = Hk, Hv, Dk, Dv
        self.conv_kernel_size = kernel
        self.conv_dim = 2 * Hk * Dk + Hv * Dv
        self.training = False

        def lin(o, i):
            w = (torch.randn(o, i, generator=g) / i ** 0.5).to(torch.bfloat16).to(device)
            return lambda x: (x.float() @ w.float().t()).to(torch.bfloat16)
        self.in_proj_qkv = lin(self.conv_dim, hidden)
        self.in_proj_z = lin(Hv * Dv, hidden)
        self.in_proj_a = lin(Hv, hidden)
        self.in_proj_b = lin(Hv, hidden)
        self.out_proj = lin(hidden, Hv * Dv)
        cw = (torch.randn(self.conv_dim, kernel, generator=g) * 0.5).to(torch.bfloat16).to(device)

        def conv1d(x):  # depthwise causal conv over channels-last [B, L, C], valid outputs only (L - K + 1)
            L = x.shape[1]
            out = sum(x[:, i:L - kernel + 1 + i, :].float() * cw[:, i].float() for i in range(kernel))
            return out.to(torch.bfloat16)
        self.conv1d = conv1d
        self.A_log = (torch.randn(Hv, generator=g) * 0.5).to(device)
        self.dt_bias = (torch.randn(Hv, generator=g) * 0.5).to(device)
        norm_w = (1 + 0.1 * torch.randn(Dv, generator=g)).to(torch.bfloat16).to(device)
        self.norm = type("Norm", (), {"weight": norm_w, "eps": 1e-6})()

    def __call__(self, inputs, mask=None, cache=None):
        from larder_b200 import gdn_cuda, ops
        B, S, _ = inputs.shape
        Hk, Hv, Dk, Dv = self.num_k_heads, self.num_v_heads, self.head_k_dim, self.head_v_dim
        qkv = self.in_proj_qkv(inputs)
        z = self.in_proj_z(inputs).reshape(B, S, Hv, Dv)
        b = self.in_proj_b(inputs)
        a = self.in_proj_a(inputs)
        conv_state = cache[0] if cache[0] is not None else torch.zeros(
            (B, self.conv_kernel_size - 1, self.conv_dim), dtype=inputs.dtype, device=inputs.device)
        conv_input = torch.cat([conv_state, qkv], dim=1)
        cache[0] = conv_input[:, -(self.conv_kernel_size - 1):, :].contiguous()
        conv = _silu16(self.conv1d(conv_input))
        q = conv[..., :Hk * Dk].reshape(B, S, Hk, Dk)
        k = conv[..., Hk * Dk:2 * Hk * Dk].reshape(B, S, Hk, Dk)
        v = conv[..., 2 * Hk * Dk:].reshape(B, S, Hv, Dv)
        eps = 1e-6 / Dk

        def rms(x):
            xf = x.float()
            return (xf * torch.rsqrt((xf * xf).mean(-1, keepdim=True) + eps)).to(torch.bfloat16)
        sq = torch.tensor(Dk ** -1.0, dtype=torch.bfloat16).float()
        sk = torch.tensor(Dk ** -0.5, dtype=torch.bfloat16).float()
        q = (rms(q).float() * sq).to(torch.bfloat16)
        k = (rms(k).float() * sk).to(torch.bfloat16)
        beta = torch.sigmoid(b.float()).to(torch.bfloat16)
        g = gdn_cuda.compute_g(self.A_log, a, self.dt_bias)
        y, state = ops.gdn_recurrent(q, k, v, g, beta, cache[1])
        cache[1] = state
        cache.advance(S)
        xf = y.float()
        n = (self.norm.weight.float() * (xf * torch.rsqrt((xf * xf).mean(-1, keepdim=True) + self.norm.eps))
             .to(torch.bfloat16).float()).to(torch.bfloat16)
        out = (torch.nn.functional.silu(z.float()) * n.float()).to(torch.bfloat16)
        return self.out_proj(out.reshape(B, S, -1))
