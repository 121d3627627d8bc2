"""Fused LayerNorm / RMSNorm modules with torchpp's signatures
(torchpp/dlops/normalization.py:7-50), backed by the sm_100a kernels in
csrc/norm.cu.  fp16 and bf16 are accepted (the reference is fp16-only)."""
from __future__ import annotations

import torch
import torch.nn as nn

from .. import ops


class LayerNormFused(nn.Module):
    """(x - mean) * rsqrt(var + eps) * weight over the last dim (no beta, as
    the reference; normalization.py:7-27)."""

    def __init__(self, normalize_dim_shape: int, eps: float = 1e-6,
                 dtype: torch.dtype = torch.float16,
                 device: torch.device = torch.device("cuda")):
        super().__init__()
        self.shape = normalize_dim_shape
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(self.shape, dtype=dtype, device=device))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return ops.layernorm(x, self.weight, None, self.eps)


class RmsNormFused(nn.Module):
    """x * rsqrt(mean(x^2) + eps) * weight over the last dim
    (normalization.py:30-50)."""

    def __init__(self, normalize_dim_shape: int, eps: float = 1e-6,
                 dtype: torch.dtype = torch.float16,
                 device: torch.device = torch.device("cuda")):
        super().__init__()
        self.shape = normalize_dim_shape
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(self.shape, dtype=dtype, device=device))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return ops.rmsnorm(x, self.weight, self.eps)


class LayerNorm4D(nn.Module):
    """Unfused reference module kept for API parity (normalization.py:57-78):
    normalises over dims (2, 3) of a 4-D tensor with gamma/beta.  Not on the
    inference hot path, so it stays plain torch."""

    def __init__(self, num_features: int):
        super().__init__()
        self.gamma = nn.Parameter(torch.ones(1, 1, 1, num_features))
        self.beta = nn.Parameter(torch.zeros(1, 1, 1, num_features))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        mean = x.mean(dim=[2, 3], keepdim=True)
        var = x.var(dim=[2, 3], keepdim=True, unbiased=False)
        return (x - mean) / torch.sqrt(var + 1e-6) * self.gamma + self.beta
