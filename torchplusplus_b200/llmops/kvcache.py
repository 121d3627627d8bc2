"""KV cache with torchpp's API and BHSD layout (torchpp/llmops/kvcache.py:6-117).

Layout: k_cache / v_cache are [batch, n_kv_heads, max_seq_len, head_dim]
(BHSD, the reference's layout with the batch generalised from 1).  The
storage is allocated once, at its full capacity, on the first update (the
reference allocates lazily too, kvcache.py:34-48, but then grows by 100 slots
and copies, kvcache.py:84-100).  Appends write in place with the kv_append
kernel; `update` returns views of the valid prefix instead of the
reference's `.contiguous()` copies of the whole cache (kvcache.py:76-81,
104-108), so an update costs O(new tokens), not O(cache length).

Reference bugs not reproduced: the append path returned a single slot
(kvcache.py:76-79) and the index path failed on its second grow.
"""
from __future__ import annotations

from typing import Tuple

import torch

from .. import ops


class KVCache:
    """KV cache management class."""

    def __init__(self, max_seq_len: int, n_kv_heads: int, head_dim: int,
                 dtype: torch.dtype = torch.float16,
                 device: torch.device = torch.device("cuda"), batch_size: int | None = None):
        self.max_seq_len = max_seq_len
        self.n_kv_heads = n_kv_heads
        self.head_dim = head_dim
        self.dtype = dtype
        self.device = torch.device(device)
        self.batch_size = batch_size
        self.k_cache: torch.Tensor | None = None
        self.v_cache: torch.Tensor | None = None
        self.cache_len = 0
        if batch_size is not None:
            self._ensure_allocated(batch_size)

    def _ensure_allocated(self, batch_size: int) -> None:
        if self.k_cache is not None and self.k_cache.shape[0] >= batch_size:
            return
        shape = (batch_size, self.n_kv_heads, self.max_seq_len, self.head_dim)
        self.k_cache = torch.zeros(shape, dtype=self.dtype, device=self.device)
        self.v_cache = torch.zeros(shape, dtype=self.dtype, device=self.device)
        self.batch_size = batch_size

    def update(self, k: torch.Tensor, v: torch.Tensor,
               index: int | None = None) -> Tuple[torch.Tensor, torch.Tensor]:
        """Writes k, v [B, Hkv, S, D] at row `index` (default: append at
        cache_len) and returns views [B, Hkv, new_len, D] of the valid cache."""
        B, H, S, D = k.shape
        if H != self.n_kv_heads or D != self.head_dim:
            raise ValueError("k/v head count or head dim does not match the cache")
        self._ensure_allocated(B)
        start = self.cache_len if index is None else int(index)
        if start < 0 or start + S > self.max_seq_len:
            raise ValueError(f"KV cache overflow: rows [{start}, {start + S}) exceed "
                             f"max_seq_len={self.max_seq_len}")
        ops.kv_append(k, v, self.k_cache, self.v_cache, start_pos=start)
        self.cache_len = max(self.cache_len, start + S)
        return self.k_cache[:B, :, :self.cache_len], self.v_cache[:B, :, :self.cache_len]

    def advance(self, n: int) -> None:
        """Marks n more rows valid (used when a kernel wrote them directly)."""
        self.cache_len = min(self.max_seq_len, self.cache_len + n)

    def reset(self) -> None:
        self.cache_len = 0
        if self.k_cache is not None:
            self.k_cache.zero_()
            self.v_cache.zero_()


class PagedKVCache:
    """Paged K/V storage for decode: block pools [num_blocks, Hkv, 64, D]
    shared by all sequences, and a block table [batch, max_blocks] (int32,
    on the device) mapping each sequence's 64-key blocks to pool blocks.
    Blocks are handed out from a host-side free list, so sequences of very
    different lengths share one pool instead of each reserving max_seq_len.
    The reference lists a paged cache as a TODO (todo.md:8); the decode
    kernels read it through tpp_attention_decode(_qkv)_paged."""

    BLOCK = 64

    def __init__(self, num_blocks: int, n_kv_heads: int, head_dim: int, dtype: torch.dtype,
                 device, batch_size: int, max_seq_len: int):
        self.k_pool = torch.zeros(num_blocks, n_kv_heads, self.BLOCK, head_dim, dtype=dtype,
                                  device=device)
        self.v_pool = torch.zeros_like(self.k_pool)
        self.max_blocks = (max_seq_len + self.BLOCK - 1) // self.BLOCK
        self.block_table = torch.full((batch_size, self.max_blocks), -1, dtype=torch.int32,
                                      device=device)
        self._table = [[] for _ in range(batch_size)]  # host copy of each row
        self._free = list(range(num_blocks))
        self.max_seq_len = max_seq_len

    @property
    def free_blocks(self) -> int:
        return len(self._free)

    def reserve(self, b: int, length: int) -> None:
        """Make sure sequence b owns blocks for positions < length."""
        if length > self.max_seq_len:
            raise ValueError("length exceeds max_seq_len")
        need = (length + self.BLOCK - 1) // self.BLOCK - len(self._table[b])
        if need <= 0:
            return
        if need > len(self._free):
            raise RuntimeError("paged KV cache: out of blocks")
        new = [self._free.pop() for _ in range(need)]
        start = len(self._table[b])
        self._table[b].extend(new)
        self.block_table[b, start:start + need] = torch.tensor(new, dtype=torch.int32)

    def release(self, b: int) -> None:
        """Return sequence b's blocks to the pool."""
        self._free.extend(reversed(self._table[b]))
        self._table[b] = []
        self.block_table[b].fill_(-1)

    def append(self, k: torch.Tensor, v: torch.Tensor, start_pos: int = 0) -> None:
        """k, v [B, Hkv, S, D] written at positions start_pos .. start_pos + S - 1."""
        from .. import ops
        B, _, S, _ = k.shape
        for b in range(B):
            self.reserve(b, start_pos + S)
        ops.kv_append_paged(k, v, self.k_pool, self.v_pool, self.block_table,
                            start_pos=start_pos)
