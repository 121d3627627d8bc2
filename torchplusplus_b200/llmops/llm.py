"""LLMInference: torchpp's abstract inference driver (torchpp/llmops/llm.py:9-333)
with the same public methods, on the B200 kernels.

Differences from the reference, all fixes of code that cannot run as shipped:
  * setup_kv_cache + reset_kv_cache work before the first update
    (kvcache.py:112-116 zeroes tensors that were never allocated);
  * clear_kv_cache / get_cache_info use the same attribute
    (llm.py:87, 291-301 use `kv_caches`, which is never set);
  * greedy decoding takes the argmax on the device (tpp_argmax) and only
    synchronises with the host when a stop/eos token has to be checked
    (the reference calls token.item() every step, llm.py:212);
  * top-p keeps the first token above the threshold (the intended shift of
    llm.py:134-137, which indexes with `... : -1`).
"""
from __future__ import annotations

from abc import ABC, abstractmethod
from typing import Callable, List, Optional

import torch
import torch.nn as nn

from .. import ops
from .kvcache import KVCache


class LLMInference(nn.Module, ABC):

    def __init__(self):
        super().__init__()
        self.kv_cache_array: Optional[List[KVCache]] = None

    @abstractmethod
    def forward_impl(self, input_ids: torch.Tensor, kv_caches: Optional[List[KVCache]] = None,
                     cache_position: Optional[int] = None) -> torch.Tensor:
        """Core forward pass: input ids [bs, seq_len] -> logits [bs, seq_len, vocab]."""

    @abstractmethod
    def get_num_layers(self) -> int: ...

    @abstractmethod
    def get_kv_heads(self) -> int: ...

    @abstractmethod
    def get_head_dim(self) -> int: ...

    @abstractmethod
    def get_dtype(self) -> torch.dtype: ...

    # ---------------------------------------------------------------- cache
    def setup_kv_cache(self, max_seq_len: int, batch_size: int | None = None):
        device = next(self.parameters()).device
        self.kv_cache_array = [
            KVCache(max_seq_len=max_seq_len, n_kv_heads=self.get_kv_heads(),
                    head_dim=self.get_head_dim(), dtype=self.get_dtype(), device=device,
                    batch_size=batch_size)
            for _ in range(self.get_num_layers())
        ]

    def reset_kv_cache(self):
        if self.kv_cache_array:
            for cache in self.kv_cache_array:
                cache.cache_len = 0

    def clear_kv_cache(self):
        """Drops the KV caches and frees their memory."""
        self.kv_cache_array = None
        if torch.cuda.is_available():
            torch.cuda.empty_cache()

    @property
    def kv_caches(self):  # name used by the reference's info helpers
        return self.kv_cache_array

    def forward(self, input_ids: torch.Tensor, use_cache: bool = False,
                cache_position: Optional[int] = None) -> torch.Tensor:
        if use_cache and self.kv_cache_array is None:
            raise ValueError(
                "KV cache is not initialized , call setup_kv_cache() or use normal nn.Module")
        return self.forward_impl(input_ids, self.kv_cache_array if use_cache else None,
                                 cache_position)

    # ---------------------------------------------------------------- sampling
    def sample_top_p(self, logits: torch.Tensor, top_p: float = 0.9, temp: float = 1.0,
                     filter_value: float = -float("inf")) -> torch.Tensor:
        logits = logits.float() / temp
        if top_p < 1.0:
            sorted_logits, sorted_idx = torch.sort(logits, descending=True)
            cum = torch.cumsum(torch.softmax(sorted_logits, dim=-1), dim=-1)
            remove = cum > top_p
            remove[..., 1:] = remove[..., :-1].clone()
            remove[..., 0] = False
            logits = logits.masked_fill(remove.scatter(1, sorted_idx, remove), filter_value)
        return torch.multinomial(torch.softmax(logits, dim=-1), num_samples=1)

    def sample_top_k(self, logits: torch.Tensor, top_k: int = 50, temp: float = 1.0,
                     filter_value: float = -float("inf")) -> torch.Tensor:
        logits = logits.float() / temp
        top_k = min(top_k, logits.size(-1))
        values, indices = torch.topk(logits, top_k)
        filt = torch.full_like(logits, filter_value).scatter_(1, indices, values)
        return torch.multinomial(torch.softmax(filt, dim=-1), num_samples=1)

    def sample_greedy(self, logits: torch.Tensor) -> torch.Tensor:
        return ops.argmax(logits).unsqueeze(-1)

    def _sample_token(self, logits: torch.Tensor, temperature: float, top_p: float,
                      top_k: Optional[int], strategy: str) -> torch.Tensor:
        if strategy == "greedy":
            return self.sample_greedy(logits)
        if strategy == "top_k" and top_k is not None:
            return self.sample_top_k(logits, top_k, temperature)
        if strategy == "top_p":
            return self.sample_top_p(logits, top_p, temperature)
        raise ValueError(f"Unknown sampling strategy: {strategy}")

    def _should_stop(self, token: torch.Tensor, stop_token_ids: List[int],
                     eos_token_id: Optional[int]) -> bool:
        ids = token.flatten().tolist()
        if eos_token_id is not None and all(t == eos_token_id for t in ids):
            return True
        return bool(stop_token_ids) and all(t in stop_token_ids for t in ids)

    # ---------------------------------------------------------------- generate
    @torch.inference_mode()
    def generate(self, input_ids: torch.Tensor, max_new_token: int = 100, temp: float = 1.0,
                 top_p: float = 0.9, top_k: Optional[int] = None,
                 sampling_strategy: str = "top_p", stop_token_ids: Optional[List[int]] = None,
                 eos_token_id: Optional[int] = None, stream: bool = False,
                 stream_callback: Optional[Callable[[torch.Tensor], None]] = None):
        device = next(self.parameters()).device
        input_ids = input_ids.to(device, non_blocking=True)
        batch_size, seq_len = input_ids.shape
        max_seq_len = seq_len + max_new_token
        caches = self.kv_cache_array
        if (caches is None or caches[0].max_seq_len < max_seq_len
                or (caches[0].batch_size or 0) < batch_size):
            self.setup_kv_cache(max_seq_len, batch_size)
        self.reset_kv_cache()
        stop_token_ids = stop_token_ids or []
        check_stop = eos_token_id is not None or bool(stop_token_ids)

        logits = self.forward(input_ids, use_cache=True, cache_position=0)
        next_token = self._sample_token(logits[:, -1, :], temp, top_p, top_k, sampling_strategy)
        if stream and stream_callback:
            stream_callback(next_token)
        generated = [next_token]
        if check_stop and self._should_stop(next_token, stop_token_ids, eos_token_id):
            return torch.cat([input_ids] + generated, dim=1)
        for i in range(max_new_token - 1):
            logits = self.forward(next_token, use_cache=True, cache_position=seq_len + i)
            next_token = self._sample_token(logits[:, -1, :], temp, top_p, top_k,
                                            sampling_strategy)
            if stream and stream_callback:
                stream_callback(next_token)
            generated.append(next_token)
            if check_stop and self._should_stop(next_token, stop_token_ids, eos_token_id):
                break
        return torch.cat([input_ids] + generated, dim=1)

    # ---------------------------------------------------------------- info
    def get_cache_info(self) -> dict:
        if not self.kv_cache_array:
            return {"initialized": False}
        c = self.kv_cache_array[0]
        return {
            "initialized": True,
            "num_layers": len(self.kv_cache_array),
            "cache_length": c.cache_len,
            "max_seq_len": c.max_seq_len,
            "n_kv_heads": c.n_kv_heads,
            "head_dim": c.head_dim,
        }

    def estimate_memory_usage(self, max_seq_len: int, batch_size: int = 1) -> dict:
        bytes_per_element = torch.empty(0, dtype=self.get_dtype()).element_size()
        per_layer = 2 * batch_size * self.get_kv_heads() * max_seq_len * self.get_head_dim() \
            * bytes_per_element
        total = self.get_num_layers() * per_layer
        return {
            "total_bytes": total,
            "total_mb": total / (1024 ** 2),
            "total_gb": total / (1024 ** 3),
            "per_layer_mb": per_layer / (1024 ** 2),
            "num_layers": self.get_num_layers(),
        }
