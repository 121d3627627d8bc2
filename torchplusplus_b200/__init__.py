"""torchplusplus_b200: torchpp's transformer-inference hot path, rebuilt for
NVIDIA B200 (sm_100a).

Module layout mirrors torchpp (``dlops``, ``attention``, ``llmops``).  Call
:func:`install_as_torchpp` to make ``import torchpp...`` (and the reference's
top-level extension modules ``rmsnormFused``, ``layernormFused``,
``ropeApplyFunction``, ``qkropeApplyFunction``, ``linearActvationFp16``)
resolve to this package, so code written against torchpp -- e.g.
examples/LLM/fastqwen3.py -- runs unchanged.
"""
from __future__ import annotations

import sys
import types

__version__ = "0.1.0"

from . import ops  # noqa: E402,F401
from ._native import LIB_PATH, TppError, lib  # noqa: E402,F401


def _extension_shims() -> dict[str, types.ModuleType]:
    """Modules with the reference's pybind function names (csrc/*/binding.cu)."""
    from . import ops as _o

    def mk(name: str, **fns) -> types.ModuleType:
        m = types.ModuleType(name)
        m.__dict__.update(fns)
        return m

    return {
        "rmsnormFused": mk("rmsnormFused",
                           rmsnormFused=lambda x, w, eps=1e-6: _o.rmsnorm(x, w, eps)),
        "layernormFused": mk("layernormFused",
                             applyLayernorm=lambda x, w, eps=1e-6: _o.layernorm(x, w, None, eps)),
        "ropeApplyFunction": mk("ropeApplyFunction",
                                rope_apply_cuda=lambda x, cos_cache, sin_cache:
                                _o.rope(x, cos_cache, sin_cache)),
        "qkropeApplyFunction": mk("qkropeApplyFunction",
                                  qkrope_apply_cuda=lambda q, k, cos_cache, sin_cache:
                                  list(_o.qkrope(q, k, cos_cache, sin_cache))),
        "linearActvationFp16": mk("linearActvationFp16",
                                  LinearGelu=lambda x, w: _o.linear(x, w, act="gelu"),
                                  LinearSilu=lambda x, w: _o.linear(x, w, act="silu"),
                                  LinearRelu=lambda x, w: _o.linear(x, w, act="relu")),
    }


def install_as_torchpp() -> None:
    """Registers this package under torchpp's module names in sys.modules."""
    import importlib

    names = [
        "dlops", "dlops.normalization", "dlops.rope", "dlops.linear", "dlops.fused_linear",
        "attention", "attention.gqa", "attention.mqa", "attention.mha", "attention.swa",
        "attention.ca", "llmops", "llmops.kvcache", "llmops.llm",
    ]
    sys.modules["torchpp"] = sys.modules[__name__]
    for n in names:
        sys.modules["torchpp." + n] = importlib.import_module(f"{__name__}.{n}")
    for name, mod in _extension_shims().items():
        sys.modules.setdefault(name, mod)
