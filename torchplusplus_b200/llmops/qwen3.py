"""Qwen3-shaped decoder built from the torchpp modules of this package.

Structure follows examples/LLM/fastqwen3.py:15-189 of the reference
(embedding -> n x [RMSNorm -> GQA(q/k norm, RoPE) -> residual -> RMSNorm ->
FFN -> residual] -> RMSNorm -> untied LM head), with the FFN written as the
SwiGLU the reference intends (down(silu(gate(x)) * up(x)), as the Dia MLP of
examples/TTS/dia/model.py:104-116) -- the shipped FFN applies its 1024->3072
`linear_layerP` to the 3072-wide SiLU output (fastqwen3.py:71-75), a shape
error.  Parameter names match the reference's (`fused_linear_layer1` is the
gate, `linear_layerP` the up projection, `linear_layer2` the down projection).

`Qwen3.generate(..., sampling_strategy="greedy")` runs through
:class:`~torchplusplus_b200.llmops.engine.DecodeEngine` (CUDA-graph decode
step, on-device argmax); other strategies use LLMInference.generate.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional

import torch
import torch.nn as nn

from .. import ops
from ..attention._core import FusedQKV
from ..attention.gqa import GroupedQueryAttention
from ..dlops.linear import LinearSILU
from ..dlops.normalization import RmsNormFused
from ..dlops.rope import compute_rope_params
from .kvcache import KVCache
from .llm import LLMInference


@dataclass
class Qwen3Config:
    vocab_size: int = 151936
    context_length: int = 40960
    embed_dim: int = 1024
    n_heads: int = 16
    n_layers: int = 28
    head_dim: int = 128
    n_kv_heads: int = 8
    hidden_dim: int = 3072
    qk_norm: bool = True
    rope_base: float = 1e6
    dtype: torch.dtype = torch.bfloat16


class SwiGLUFFN(nn.Module):
    """y = down(silu(gate(x)) * up(x)); gate and up run as ONE GEMM with the
    SwiGLU product in its epilogue."""

    def __init__(self, in_dim: int, hidden_dim: int, dtype: torch.dtype, device=None):
        super().__init__()
        self.fused_linear_layer1 = LinearSILU(in_dim, hidden_dim, dtype=dtype, device=device)
        self.linear_layerP = nn.Linear(in_dim, hidden_dim, bias=False, dtype=dtype, device=device)
        self.linear_layer2 = nn.Linear(hidden_dim, in_dim, bias=False, dtype=dtype, device=device)
        self._gu = FusedQKV()

    def gate_up_weight(self) -> torch.Tensor:
        return self._gu.get(self.fused_linear_layer1.weight, self.linear_layerP.weight)

    def forward(self, x: torch.Tensor, residual: torch.Tensor | None = None) -> torch.Tensor:
        h = ops.linear(x, self.gate_up_weight(), act="swiglu")
        return ops.linear(h, self.linear_layer2.weight, residual=residual)


class Transformer(nn.Module):
    def __init__(self, cfg: Qwen3Config, device=None):
        super().__init__()
        self.attn = GroupedQueryAttention(d_in=cfg.embed_dim, num_heads=cfg.n_heads,
                                          head_dim=cfg.head_dim, n_kv_heads=cfg.n_kv_heads,
                                          qk_norm=cfg.qk_norm, dtype=cfg.dtype)
        self.rms_norm1 = RmsNormFused(cfg.embed_dim, eps=1e-6, dtype=cfg.dtype, device=device)
        self.rms_norm2 = RmsNormFused(cfg.embed_dim, eps=1e-6, dtype=cfg.dtype, device=device)
        self.ffn = SwiGLUFFN(cfg.embed_dim, cfg.hidden_dim, cfg.dtype, device)

    def forward(self, x, cos, sin, kv_cache: Optional[KVCache] = None,
                cache_position: Optional[int] = None):
        h = self.rms_norm1(x)
        x = self.attn(h, cos, sin, kv_cache, cache_position, residual=x)
        h = self.rms_norm2(x)
        return self.ffn(h, residual=x)


class Qwen3(LLMInference):

    def __init__(self, cfg: Qwen3Config, device=None):
        super().__init__()
        self.cfg = cfg
        self.tok_embed = nn.Embedding(cfg.vocab_size, cfg.embed_dim, dtype=cfg.dtype, device=device)
        self.transformer_blocs = nn.ModuleList([Transformer(cfg, device) for _ in range(cfg.n_layers)])
        self.final_rmsnorm = RmsNormFused(cfg.embed_dim, dtype=cfg.dtype, device=device)
        self.out_head = nn.Linear(cfg.embed_dim, cfg.vocab_size, bias=False, dtype=cfg.dtype,
                                  device=device)
        cos, sin = compute_rope_params(cfg.head_dim, cfg.rope_base, cfg.context_length,
                                       device=device if device is not None else "cpu")
        self.register_buffer("cos", cos, persistent=False)
        self.register_buffer("sin", sin, persistent=False)
        self._engine = None
        if device is not None:
            self.to(device)

    @torch.no_grad()
    def init_weights(self, std: float = 0.02, seed: int = 0) -> "Qwen3":
        """Random init used by the benchmarks: every matrix ~ N(0, std), norm
        weights 1 (generated on the parameters' device)."""
        g = torch.Generator(device=self.out_head.weight.device).manual_seed(seed)
        for _, p in self.named_parameters():
            if p.dim() >= 2:
                p.copy_(torch.randn(p.shape, generator=g, device=p.device, dtype=torch.float32)
                        .mul_(std).to(p.dtype))
            else:
                p.fill_(1.0)
        return self

    def get_num_layers(self) -> int:
        return self.cfg.n_layers

    def get_kv_heads(self) -> int:
        return self.cfg.n_kv_heads

    def get_head_dim(self) -> int:
        return self.cfg.head_dim

    def get_dtype(self) -> torch.dtype:
        return self.cfg.dtype

    def forward_impl(self, input_ids: torch.Tensor, kv_caches: Optional[List[KVCache]] = None,
                     cache_position: Optional[int] = None, last_only: bool = False) -> torch.Tensor:
        x = ops.embedding(input_ids, self.tok_embed.weight)
        for i, blk in enumerate(self.transformer_blocs):
            x = blk(x, self.cos, self.sin, kv_caches[i] if kv_caches is not None else None,
                    cache_position)
        if last_only:
            x = x[:, -1:]
        x = self.final_rmsnorm(x)
        return ops.linear(x, self.out_head.weight)

    def engine(self, batch_size: int, max_seq_len: int, weight_format: str | None = None):
        """The model's decode engine (rebuilt when the batch, capacity or
        weight format changes).  weight_format: "native" or "fp8" (decode
        projections on e4m3 weights); None keeps self.decode_weight_format."""
        from .engine import DecodeEngine
        fmt = weight_format or getattr(self, "decode_weight_format", "native")
        pers = getattr(self, "decode_persistent", None)
        e = self._engine
        if e is None or e.batch_size != batch_size or e.max_seq_len < max_seq_len or \
                e.weight_format != fmt or (pers is not None and (e.persistent is not None) != pers):
            self._engine = e = DecodeEngine(self, batch_size, max_seq_len, weight_format=fmt,
                                            persistent=pers)
        return e

    @torch.inference_mode()
    def generate(self, input_ids: torch.Tensor, max_new_token: int = 100, temp: float = 1.0,
                 top_p: float = 0.9, top_k: Optional[int] = None,
                 sampling_strategy: str = "top_p", stop_token_ids=None, eos_token_id=None,
                 stream: bool = False, stream_callback=None):
        if stream or sampling_strategy not in ("greedy", "top_p", "top_k") or \
                (sampling_strategy == "top_k" and top_k is None):
            return super().generate(input_ids, max_new_token, temp, top_p, top_k,
                                    sampling_strategy, stop_token_ids, eos_token_id, stream,
                                    stream_callback)
        B, S = input_ids.shape
        eng = self.engine(B, S + max_new_token)
        if sampling_strategy == "greedy":
            eng.set_greedy()
        else:
            # the reference's strategies are exclusive (llm.py:107-116); the
            # draw seed comes from torch's generator, so torch.manual_seed
            # makes a run reproducible
            eng.set_sampling(temperature=temp,
                             top_k=top_k if sampling_strategy == "top_k" else 0,
                             top_p=top_p if sampling_strategy == "top_p" else 1.0,
                             seed=int(torch.randint(0, 2 ** 62, (1,)).item()))
        return eng.generate(input_ids, max_new_token, eos_token_id=eos_token_id,
                            stop_token_ids=stop_token_ids)
