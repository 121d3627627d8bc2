"""Alias module: examples/LLM/fastqwen3.py:7 imports LinearSILU from
``torchpp.dlops.fused_linear``, which the reference never shipped."""
from .linear import LinearGELU, LinearReLU, LinearSILU  # noqa: F401
