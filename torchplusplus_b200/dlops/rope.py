"""RoPE API of torchpp (torchpp/dlops/rope.py:6-54) on the sm_100a kernels."""
from __future__ import annotations

import torch

from .. import ops


def rope_apply(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Applies NeoX RoPE to x [batch, heads, seq_len, head_dim] using the first
    seq_len rows of cos/sin [>= seq_len, head_dim] (rope.py:6-21)."""
    return ops.rope(x, cos, sin)


def qkrope_apply(q: torch.Tensor, k: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor):
    """RoPE on Q and K (rope.py:24-41).  Unlike the reference kernel
    (qkrope_binding.cu:52-55), Q and K may have different head counts (GQA)."""
    return ops.qkrope(q, k, cos, sin)


def compute_rope_params(head_dim, theta_base, context_length, device="cuda",
                        dtype=torch.float32):
    """cos/sin tables [context_length, head_dim] = cat(theta, theta), angles in
    `dtype` (fp32 by default), tables returned in fp16 exactly as rope.py:43-54."""
    assert head_dim % 2 == 0, "head dim must be divisible by 2"
    ar = torch.arange(0, head_dim, 2, device=device, dtype=dtype)
    inv_freq = 1.0 / (theta_base ** (ar / head_dim))
    pos = torch.arange(context_length, device=device, dtype=dtype)
    angles = pos[:, None] * inv_freq[None, :]
    angles = torch.cat([angles, angles], dim=1)
    cos = torch.cos(angles).to(torch.float16).contiguous()
    sin = torch.sin(angles).to(torch.float16).contiguous()
    return cos, sin
