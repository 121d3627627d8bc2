"""MultiHeadAttention (torchpp/attention/mha.py:7-97): causal MHA with
optional per-head q/k RMSNorm and RoPE.  The reference omits
nn.Module.__init__ and sizes its q/k norms embed_dim while applying them per
head (mha.py:9-10, 39-41); both are fixed here (per-head norms)."""
from __future__ import annotations

from typing import Optional

import torch
import torch.nn as nn

from ._core import FusedQKV, attention_block, norm_eps


class MultiHeadAttention(nn.Module):

    def __init__(self, embed_dim: int, n_heads: int, qknorm: bool = True,
                 dtype: torch.dtype = torch.float16):
        super().__init__()
        assert embed_dim % n_heads == 0, "embed dimension should be divisible by number of heads"
        self.embed_dim = embed_dim
        self.n_heads = n_heads
        self.head_dim = embed_dim // n_heads
        self.qknorm = qknorm
        self.dtype = dtype
        self.Wq = nn.Linear(embed_dim, embed_dim, bias=False, dtype=dtype)
        self.Wk = nn.Linear(embed_dim, embed_dim, bias=False, dtype=dtype)
        self.Wv = nn.Linear(embed_dim, embed_dim, bias=False, dtype=dtype)
        self.out_projection = nn.Linear(embed_dim, embed_dim, dtype=dtype)
        if qknorm:
            self.q_norm = nn.RMSNorm(self.head_dim, eps=1e-6, dtype=dtype)
            self.k_norm = nn.RMSNorm(self.head_dim, eps=1e-6, dtype=dtype)
        else:
            self.q_norm = self.k_norm = None
        self._qkv = FusedQKV()

    def forward(self, x: torch.Tensor, cos, sin, kv_cache=None, cache_pos: Optional[int] = None):
        w = self._qkv.get(self.Wq.weight, self.Wk.weight, self.Wv.weight)
        return attention_block(
            x, w, self.out_projection.weight, self.out_projection.bias, self.n_heads,
            self.n_heads, self.head_dim,
            self.q_norm.weight if self.q_norm is not None else None,
            self.k_norm.weight if self.k_norm is not None else None,
            norm_eps(self.q_norm) if self.q_norm is not None else 1e-6, cos, sin,
            kv_cache=kv_cache, cache_pos=cache_pos, causal=True)
