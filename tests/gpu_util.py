"""Helpers shared by the GPU parity tests (torch <-> oracle numpy formats)."""

import numpy as np
import torch


def bits(t: torch.Tensor) -> np.ndarray:
    """bf16 tensor -> uint16 bit patterns (numpy, CPU)."""
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def from_bits(b: np.ndarray, device="cuda") -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(b, dtype=np.uint16).view(np.int16)).view(torch.bfloat16).to(device)


def rel_l2(a, b) -> float:
    a = torch.as_tensor(a).double().cpu()
    b = torch.as_tensor(b).double().cpu()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


def cosine(a, b) -> float:
    a = torch.as_tensor(a).double().cpu().reshape(-1)
    b = torch.as_tensor(b).double().cpu().reshape(-1)
    return float(a @ b / (a.norm() * b.norm()).clamp_min(1e-30))


def outlier_activations(g, m, k, frac=0.01, mult=20.0):
    """Activations with outlier channels, as the INT8 GEMM benchmark uses: N(0,1) with 1% of
    channels scaled by 20."""
    x = torch.randn(m, k, generator=g)
    nout = max(1, int(round(k * frac)))
    cols = torch.randperm(k, generator=g)[:nout]
    x[:, cols] *= mult
    return x
