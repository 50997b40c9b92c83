"""Helpers shared by the GPU parity tests: move numpy storage (oracle form) to torch CUDA tensors and back."""
import numpy as np
import torch

import oracle

TORCH_DT = {oracle.F32: torch.float32, oracle.BF16: torch.bfloat16, oracle.F16: torch.float16}


def to_torch(a, dt, device="cuda"):
    """numpy storage (float32 or uint16 bits) -> torch tensor of dtype code dt on device."""
    a = np.ascontiguousarray(a)
    if dt == oracle.F32:
        return torch.from_numpy(a.astype(np.float32)).to(device)
    return torch.from_numpy(a.view(np.int16)).view(TORCH_DT[dt]).to(device)


def to_np(t, dt=None):
    """torch tensor -> numpy storage in dtype code dt (default: the tensor's)."""
    t = t.detach().contiguous().cpu()
    if t.dtype == torch.float32:
        return t.numpy()
    return t.view(torch.int16).numpy().view(np.uint16)


def f32(t):
    return t.detach().float().cpu().numpy()


def np_store(t):
    """A torch tensor's values as oracle storage + its dtype code (strides kept by going through a contiguous copy
    of the same logical view)."""
    dt = {torch.float32: oracle.F32, torch.bfloat16: oracle.BF16, torch.float16: oracle.F16}[t.dtype]
    return to_np(t), dt


def randn(shape, dt, gen, device="cuda", scale=1.0):
    x = torch.randn(*shape, generator=gen, dtype=torch.float32) * scale
    return x.to(TORCH_DT[dt]).to(device)
