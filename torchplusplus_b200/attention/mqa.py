"""MultiQueryAttention (torchpp/attention/mqa.py:9-93): one shared K/V head.
The reference rotates Q into K (`K = rope_apply(Q, ...)`, mqa.py:81); here K
gets its own rotation, which is what multi-query attention means."""
from __future__ import annotations

from typing import Optional

import torch
import torch.nn as nn

from ._core import FusedQKV, attention_block, norm_eps


class MultiQueryAttention(nn.Module):

    def __init__(self, num_q_heads: int, embed_dim: int, qk_norm: bool = True,
                 dtype: torch.dtype = torch.float16):
        super().__init__()
        self.embed_dim = embed_dim
        self.num_q_head = num_q_heads
        self.head_dim = embed_dim // num_q_heads
        self.Wq = nn.Linear(embed_dim, embed_dim, dtype=dtype, bias=False)
        self.Wk = nn.Linear(embed_dim, self.head_dim, dtype=dtype, bias=False)
        self.Wv = nn.Linear(embed_dim, self.head_dim, dtype=dtype, bias=False)
        self.out_projection = nn.Linear(embed_dim, embed_dim, dtype=dtype, bias=False)
        self.qk_norm = qk_norm
        self.q_norm = nn.RMSNorm(self.head_dim, eps=1e-6, dtype=dtype)
        self.k_norm = nn.RMSNorm(self.head_dim, eps=1e-6, dtype=dtype)
        self._qkv = FusedQKV()

    def forward(self, x, cos, sin, kv_cache=None, cache_pos: Optional[int] = None):
        w = self._qkv.get(self.Wq.weight, self.Wk.weight, self.Wv.weight)
        return attention_block(
            x, w, self.out_projection.weight, None, self.num_q_head, 1, self.head_dim,
            self.q_norm.weight if self.qk_norm else None,
            self.k_norm.weight if self.qk_norm else None, norm_eps(self.q_norm), cos, sin,
            kv_cache=kv_cache, cache_pos=cache_pos, causal=True)
