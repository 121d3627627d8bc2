"""CrossAttention (torchpp/attention/ca.py:10-87): queries from x, keys and
values from a context y, no mask, no rotary embedding.  The reference
unpacks y as 2-D (ca.py:49) although it projects it as [B, S, cross_dim];
here y is [B, S_kv, cross_dim].  An optional KVCache holds the projected
context (written once, then reused)."""
from __future__ import annotations

from typing import Optional

import torch
import torch.nn as nn

from .. import ops
from ..llmops.kvcache import KVCache


class CrossAttention(nn.Module):

    def __init__(self, embed_dim: int, cross_dim: int, n_heads: int, qknorm: bool = True,
                 dtype: torch.dtype = torch.float16):
        super().__init__()
        assert embed_dim % n_heads == 0, "embed dimension should be divisible by number of heads"
        self.embed_dim = embed_dim
        self.cross_dim = cross_dim
        self.n_heads = n_heads
        self.head_dim = embed_dim // n_heads
        self.qknorm = qknorm
        self.dtype = dtype
        self.hidden_dim = self.head_dim * self.n_heads
        self.Wq = nn.Linear(embed_dim, self.hidden_dim, bias=False, dtype=dtype)
        self.Wk = nn.Linear(cross_dim, self.hidden_dim, bias=False, dtype=dtype)
        self.Wv = nn.Linear(cross_dim, self.hidden_dim, bias=False, dtype=dtype)
        self.out_projection = nn.Linear(self.hidden_dim, embed_dim, dtype=dtype)

    def forward(self, x: torch.Tensor, y: torch.Tensor,
                kv_cache: Optional[KVCache] = None) -> torch.Tensor:
        B, Sq, _ = x.shape
        H, D = self.n_heads, self.head_dim
        q = ops.linear(x, self.Wq.weight).view(B, Sq, H, D)
        if kv_cache is not None and kv_cache.cache_len > 0:
            L = kv_cache.cache_len
            k = kv_cache.k_cache[:B, :, :L].transpose(1, 2)
            v = kv_cache.v_cache[:B, :, :L].transpose(1, 2)
        else:
            Skv = y.shape[1]
            k = ops.linear(y, self.Wk.weight).view(B, Skv, H, D)
            v = ops.linear(y, self.Wv.weight).view(B, Skv, H, D)
            if kv_cache is not None:
                kk, vv = kv_cache.update(k.transpose(1, 2), v.transpose(1, 2), index=0)
                k, v = kk.transpose(1, 2), vv.transpose(1, 2)
        o = ops.attention(q, k, v, causal=False)
        return ops.linear(o.reshape(B, Sq, self.hidden_dim), self.out_projection.weight,
                          self.out_projection.bias)
