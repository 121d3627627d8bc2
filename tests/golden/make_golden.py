"""Generates the golden fixtures under tests/golden/ from the REFERENCE's own
Python code (torchpp), run on the CPU in the build container.

The reference's compiled extensions (rmsnormFused, ropeApplyFunction, ...) and
the third-party flash_attn kernel cannot run without a GPU, so they are
replaced by the fp32 oracle restatements (oracle/ops.py) while everything else
-- module wiring, projections, q/k norms, transposes, repeat_interleave,
KVCache bookkeeping, compute_rope_params -- is the reference's unmodified
code, loaded straight from its source files.

Usage (needs the reference checkout; the GPU box does not have it and only
reads the committed .pt files):
    python tests/golden/make_golden.py --reference /path/to/TorchPlusPlus
"""
from __future__ import annotations

import argparse
import importlib.util
import sys
import types
from pathlib import Path

import torch
import torch.nn as nn

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))
from oracle import ops as O  # noqa: E402


def _stub_extensions() -> None:
    """Stand-ins for the reference's pybind modules and flash_attn (CPU)."""
    def mod(name, **fns):
        m = types.ModuleType(name)
        for k, v in fns.items():
            setattr(m, k, v)
        sys.modules[name] = m

    def rope_apply_cuda(x, cos, sin):
        return O.rope(x, cos, sin).to(x.dtype)

    def qkrope_apply_cuda(q, k, cos, sin):
        return [O.rope(q, cos, sin).to(q.dtype), O.rope(k, cos, sin).to(k.dtype)]

    mod("ropeApplyFunction", rope_apply_cuda=rope_apply_cuda)
    mod("qkropeApplyFunction", qkrope_apply_cuda=qkrope_apply_cuda)
    mod("rmsnormFused", rmsnormFused=lambda x, w, eps: O.rmsnorm(x, w, eps).to(x.dtype))
    mod("layernormFused", applyLayernorm=lambda x, w, eps: O.layernorm(x, w, None, eps).to(x.dtype))
    mod("linearActvationFp16",
        LinearSilu=lambda x, w: O.linear(x, w, None, "silu").to(x.dtype),
        LinearGelu=lambda x, w: O.linear(x, w, None, "gelu").to(x.dtype),
        LinearRelu=lambda x, w: O.linear(x, w, None, "relu").to(x.dtype))

    def flash_attn_func(q, k, v, causal=False, window_size=(-1, -1), **_):
        return O.attention(q, k, v, causal=causal, window_left=window_size[0]).to(q.dtype)

    mod("flash_attn", flash_attn_func=flash_attn_func)


def _load(ref: Path, dotted: str, rel: str):
    """Loads one reference source file as module `dotted` (parents stubbed;
    the reference's package __init__ files use broken absolute imports)."""
    parts = dotted.split(".")
    for i in range(1, len(parts)):
        name = ".".join(parts[:i])
        if name not in sys.modules:
            pkg = types.ModuleType(name)
            pkg.__path__ = []
            sys.modules[name] = pkg
    spec = importlib.util.spec_from_file_location(dotted, ref / rel)
    m = importlib.util.module_from_spec(spec)
    sys.modules[dotted] = m
    spec.loader.exec_module(m)
    return m


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=str(ROOT.parent / "reference"))
    a = ap.parse_args()
    ref = Path(a.reference)
    _stub_extensions()
    rope_m = _load(ref, "torchpp.dlops.rope", "torchpp/dlops/rope.py")
    kv_m = _load(ref, "torchpp.llmops.kvcache", "torchpp/llmops/kvcache.py")
    gqa_m = _load(ref, "torchpp.attention.gqa", "torchpp/attention/gqa.py")

    g = torch.Generator().manual_seed(0)
    out: dict[str, torch.Tensor] = {}

    # 1. compute_rope_params (torchpp/dlops/rope.py:43-54), head_dim 128, theta 1e6.
    cos, sin = rope_m.compute_rope_params(128, 1e6, 64, device="cpu")
    out["rope_cos"], out["rope_sin"] = cos, sin

    # 2. Known answers the reference's own tests check against (tests/rmsnorm_test.py,
    #    tests/layernorm_test.py): nn.RMSNorm / nn.LayerNorm(bias=0), eps 1e-6.
    x = torch.randn(4, 8, 512, generator=g).half()
    w = (1 + 0.1 * torch.randn(512, generator=g)).half()
    rn = nn.RMSNorm(512, eps=1e-6)
    rn.weight.data = w.float()
    ln = nn.LayerNorm(512, eps=1e-6)
    ln.weight.data = w.float()
    ln.bias.data.zero_()
    with torch.no_grad():
        out["norm_x"], out["norm_w"] = x, w
        out["rmsnorm_y"] = rn(x.float())
        out["layernorm_y"] = ln(x.float())

    # 3. KVCache index path (kvcache.py:83-108) -- decode writes at index 0 and
    #    1 (the second write triggers the first grow, the last one that works).
    cache = kv_m.KVCache(max_seq_len=16, n_kv_heads=2, head_dim=8, dtype=torch.float32,
                         device=torch.device("cpu"))
    k0, v0 = torch.randn(1, 2, 1, 8, generator=g), torch.randn(1, 2, 1, 8, generator=g)
    k1, v1 = torch.randn(1, 2, 1, 8, generator=g), torch.randn(1, 2, 1, 8, generator=g)
    cache.update(k0, v0, index=0)
    kk, vv = cache.update(k1, v1, index=1)
    out.update(kv_k0=k0, kv_v0=v0, kv_k1=k1, kv_v1=v1, kv_k=kk, kv_v=vv)

    # 4. GroupedQueryAttention.forward (gqa.py:70-131) without and with a cache
    #    (prefill of 6 tokens at cache_pos 0 through the index-free path is
    #    broken in the reference, so the module is run cache-free; the
    #    cache-free call applies rope over positions 0..S-1 and a causal mask).
    torch.manual_seed(1)
    attn = gqa_m.GroupedQueryAttention(d_in=128, num_heads=4, n_kv_heads=2, head_dim=64,
                                       qk_norm=True, dtype=torch.float32)
    for p in attn.parameters():
        p.data = (0.1 * torch.randn(p.shape, generator=g)).half().float()
    attn.q_norm.weight.data = (1 + 0.1 * torch.randn(64, generator=g)).half().float()
    attn.k_norm.weight.data = (1 + 0.1 * torch.randn(64, generator=g)).half().float()
    xg = torch.randn(2, 6, 128, generator=g).half().float()
    c16, s16 = rope_m.compute_rope_params(64, 1e6, 6, device="cpu")
    with torch.no_grad():
        yg = attn(xg, c16, s16)
    out["gqa_x"], out["gqa_y"] = xg, yg
    out["gqa_cos"], out["gqa_sin"] = c16, s16
    for k, v in attn.state_dict().items():
        out["gqa_sd." + k] = v

    torch.save(out, HERE / "golden_ref.pt")
    print("wrote", HERE / "golden_ref.pt", sorted(out))


if __name__ == "__main__":
    main()
