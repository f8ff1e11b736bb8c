"""Shared helpers for the GPU parity tests: seeded CPU inputs, bf16 bit views."""
import numpy as np
import torch


def gen(seed):
    return torch.Generator().manual_seed(seed)


def randn_bf16(shape, seed, scale=1.0):
    return (torch.randn(*shape, generator=gen(seed)) * scale).to(torch.bfloat16)


def bits(t):
    """bf16 tensor (any device) -> numpy uint16 bit patterns."""
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def from_bits(a, device=None):
    t = torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16)
    return t if device is None else t.to(device)


def adversarial_rows(S, D, seed):
    """Row magnitudes over logspace(-2, 3), first 7 columns x50 (the reference's
    tests/test_rmsnorm_exact.py:122-123 recipe)."""
    g = gen(seed)
    x = torch.randn(S, D, generator=g) * torch.logspace(-2, 3, S)[:, None]
    x[:, :7] *= 50
    return x.to(torch.bfloat16)


def ulp_step(f, k):
    """float32 value k ulps away from f (f > 0)."""
    u = np.array([f], dtype=np.float32).view(np.int32)[0] + k
    return np.array([u], dtype=np.int32).view(np.float32)[0]
