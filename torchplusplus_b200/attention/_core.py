"""Shared attention-block path: fused QKV projection -> fused per-head q/k
RMSNorm + RoPE + K/V write -> flash attention (prefill) or split-KV decode
attention -> output projection.  All on the sm_100a kernels.

Replaces, per forward, the reference's 3 nn.Linear + 2 nn.RMSNorm + 2
rope_apply launches + KVCache slice copies + 2 repeat_interleave copies +
transposes + flash_attn_func (torchpp/attention/gqa.py:80-131)."""
from __future__ import annotations

import torch

from .. import ops


def _version(t: torch.Tensor) -> int:
    try:
        return t._version
    except RuntimeError:  # inference tensors carry no version counter
        return -1


class FusedQKV:
    """Caches cat(Wq, Wk, Wv) so one GEMM produces q, k and v; rebuilt when any
    weight changes (tracked through the tensors' version counters)."""

    def __init__(self):
        self._key = None
        self._w = None

    def get(self, *ws: torch.Tensor) -> torch.Tensor:
        key = tuple((w.data_ptr(), _version(w), w.shape) for w in ws)
        if key != self._key:
            self._w = torch.cat([w.detach() for w in ws], dim=0).contiguous()
            self._key = key
        return self._w


def attention_block(x: torch.Tensor, wqkv: torch.Tensor, wo: torch.Tensor,
                    bo: torch.Tensor | None, Hq: int, Hkv: int, D: int,
                    qn_w: torch.Tensor | None, kn_w: torch.Tensor | None, eps: float,
                    cos: torch.Tensor | None, sin: torch.Tensor | None, kv_cache=None,
                    cache_pos: int | None = None, causal: bool = True,
                    window_left: int = -1, residual: torch.Tensor | None = None) -> torch.Tensor:
    B, S, _ = x.shape
    qkv = ops.linear(x, wqkv)                                  # [B, S, (Hq+2Hkv) D]
    if cos is None:  # no rotary embedding: identity tables
        cos = torch.ones((1, D), dtype=x.dtype, device=x.device).expand(1 << 20, D)
        sin = torch.zeros((1, D), dtype=x.dtype, device=x.device).expand(1 << 20, D)
    if kv_cache is not None:
        start = int(cache_pos) if cache_pos is not None else kv_cache.cache_len
        kv_cache._ensure_allocated(B)
        if start + S > kv_cache.max_seq_len:
            raise ValueError("KV cache overflow")
        kc, vc = kv_cache.k_cache[:B], kv_cache.v_cache[:B]
        positions = torch.full((B,), start, dtype=torch.int32, device=x.device)
        q = ops.qk_norm_rope_cache(qkv, qn_w, kn_w, eps, cos, sin, positions, kc, vc, Hq, Hkv)
        kv_cache.cache_len = max(kv_cache.cache_len, start + S)
        L = start + S
        if S == 1:
            o = ops.attention_decode(q[:, 0], kc, vc, None, L, window_left=window_left)
        else:
            o = ops.attention(q, kc[:, :, :L].transpose(1, 2), vc[:, :, :L].transpose(1, 2),
                              causal=causal, window_left=window_left)
    else:
        kbuf = torch.empty((B, Hkv, S, D), dtype=x.dtype, device=x.device)
        vbuf = torch.empty_like(kbuf)
        positions = torch.zeros((B,), dtype=torch.int32, device=x.device)
        q = ops.qk_norm_rope_cache(qkv, qn_w, kn_w, eps, cos, sin, positions, kbuf, vbuf, Hq, Hkv)
        o = ops.attention(q, kbuf.transpose(1, 2), vbuf.transpose(1, 2), causal=causal,
                          window_left=window_left)
    return ops.linear(o.reshape(B, S, Hq * D), wo, bo, residual=residual)


def norm_eps(m) -> float:
    e = getattr(m, "eps", None)
    return 1e-6 if e is None else float(e)
