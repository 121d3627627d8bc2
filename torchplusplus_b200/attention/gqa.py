"""GroupedQueryAttention with torchpp's constructor/forward signature and
parameter names (torchpp/attention/gqa.py:11-131)."""
from __future__ import annotations

from typing import Optional

import torch
import torch.nn as nn

from ..llmops.kvcache import KVCache
from ._core import FusedQKV, attention_block, norm_eps


class GroupedQueryAttention(nn.Module):

    def __init__(self, d_in: int, num_heads: int, n_kv_heads: int, head_dim: int | None = None,
                 qk_norm: bool = True, dtype: torch.dtype = torch.float16, DEBUG: bool = False):
        super().__init__()
        assert num_heads % n_kv_heads == 0, "Num heads is not divisible by num kv grps"
        self.num_heads = num_heads
        self.n_kv_heads = n_kv_heads
        self.num_kv_grps = num_heads // n_kv_heads
        if head_dim is None:
            assert d_in % num_heads == 0, "in dimension must be divisible by number of heads"
            head_dim = d_in // num_heads
        self.head_dim: int = head_dim
        self.d_out = self.head_dim * self.num_heads
        self.Wq = nn.Linear(d_in, self.d_out, bias=False, dtype=dtype)
        self.Wk = nn.Linear(d_in, n_kv_heads * head_dim, bias=False, dtype=dtype)
        self.Wv = nn.Linear(d_in, n_kv_heads * head_dim, bias=False, dtype=dtype)
        self.out_projection = nn.Linear(self.d_out, d_in, bias=False, dtype=dtype)
        if qk_norm:
            self.q_norm = nn.RMSNorm(self.head_dim, eps=1e-6, dtype=dtype)
            self.k_norm = nn.RMSNorm(self.head_dim, eps=1e-6, dtype=dtype)
        else:
            self.q_norm = self.k_norm = None
        self.DEBUG = DEBUG
        self._qkv = FusedQKV()

    def forward(self, x, cos, sin, kv_cache: Optional[KVCache] = None,
                cache_pos: Optional[int] = None, residual: Optional[torch.Tensor] = None):
        """As gqa.py:70-131.  `residual` (an extension) is added to the output
        inside the output projection's epilogue."""
        if self.DEBUG:
            print(f"\nGQA Input x shape: {x.shape}")
        w = self._qkv.get(self.Wq.weight, self.Wk.weight, self.Wv.weight)
        return attention_block(
            x, w, self.out_projection.weight, self.out_projection.bias, self.num_heads,
            self.n_kv_heads, self.head_dim,
            self.q_norm.weight if self.q_norm is not None else None,
            self.k_norm.weight if self.k_norm is not None else None,
            norm_eps(self.q_norm) if self.q_norm is not None else 1e-6, cos, sin,
            kv_cache=kv_cache, cache_pos=cache_pos, causal=True, residual=residual)
