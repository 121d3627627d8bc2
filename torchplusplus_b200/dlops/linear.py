"""Linear layers of torchpp (torchpp/dlops/linear.py:8-144) on the sm_100a
kernels: M <= 64 rows run the streaming decode kernel, larger M the tcgen05
tensor-core GEMM; the activation is fused into the epilogue."""
from __future__ import annotations

import torch
import torch.nn as nn

from .. import ops


class _LinearAct(nn.Module):
    act = "none"

    def __init__(self, in_features: int, out_features: int, bias: bool = False,
                 dtype: torch.dtype = torch.float16, device=None):
        super().__init__()
        # reference init: weight = randn(out, in) fp16 (linear.py:18-20, 38-40)
        self.weight = nn.Parameter(torch.randn(out_features, in_features, dtype=dtype,
                                               device=device))
        self.bias = nn.Parameter(torch.zeros(out_features, dtype=dtype, device=device)) if bias else None

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return ops.linear(x, self.weight, self.bias, act=self.act)


class LinearGELU(_LinearAct):
    """y = gelu_tanh(x W^T (+ b))  (linear.py:8-25; activation.cuh:26-43)."""
    act = "gelu"


class LinearSILU(_LinearAct):
    """y = silu(x W^T (+ b))  (linear.py:28-45; activation.cuh:45-56)."""
    act = "silu"


class LinearReLU(_LinearAct):
    """y = relu(x W^T (+ b))  (binding LinearRelu, activation/binding.cu:112-160)."""
    act = "relu"


class Dense(nn.Module):
    """Contraction over arbitrary axes via tensordot (linear.py:47-101).  Not a
    hot-path op; kept in plain torch for API parity."""

    def __init__(self, in_featrues: tuple, out_features: tuple, axis: tuple = (-1,),
                 weight_dtype: torch.dtype = torch.float16,
                 device: torch.device = torch.device("cuda")):
        super().__init__()
        self.in_features = in_featrues
        self.out_features = out_features
        self.axis = axis
        self.kernel_shape = self.in_features + self.out_features
        self.weight = nn.Parameter(torch.empty(self.kernel_shape, dtype=weight_dtype, device=device))
        nn.init.normal_(self.weight, std=0.02)

    def _normalize_axes(self, axes, ndim):
        return tuple(a if a >= 0 else ndim + a for a in axes)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        norm_axis = self._normalize_axes(self.axis, x.ndim)
        contract = tuple(range(len(norm_axis)))
        return torch.tensordot(x.to(self.weight.dtype), self.weight,
                               dims=(norm_axis, contract)).to(x.dtype)


class _LinearNB(nn.Module):
    dtype = torch.float16

    def __init__(self, in_features: int, out_features: int, device=None):
        super().__init__()  # (the reference forgets this call, linear.py:112-145)
        self.weight = nn.Parameter(torch.empty(out_features, in_features, dtype=self.dtype,
                                               device=device))
        nn.init.kaiming_uniform_(self.weight, a=5 ** 0.5)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return ops.linear(x, self.weight)


class LinearNBFp16(_LinearNB):
    """Bias-free fp16 linear (linear.py:106-125)."""
    dtype = torch.float16


class LinearNBBf16(_LinearNB):
    """Bias-free bf16 linear (linear.py:128-144)."""
    dtype = torch.bfloat16
