"""fp32 CPU forward of the Qwen3-shaped decoder (test oracle only).

Restates examples/LLM/fastqwen3.py:81-189 of the reference with the SwiGLU
FFN of examples/TTS/dia/model.py:104-116: embedding -> per layer
[x += o_proj(attn(q/k-norm, RoPE, causal GQA)(rmsnorm1(x)));
 x += down(silu(gate(h)) * up(h)), h = rmsnorm2(x)] -> rmsnorm -> LM head.
Parameters are read from a state dict with the names the torchpp modules use.
"""
from __future__ import annotations

import torch

from . import ops as O


@torch.no_grad()
def _storer(store_dtype):
    """Identity for the fp32 oracle; with a dtype, rounds a tensor to it (and
    back to fp32) -- where the reference's eager model run in that dtype
    stores each module's output."""
    if store_dtype is None:
        return lambda t: t
    return lambda t: t.to(store_dtype).float()


@torch.no_grad()
def forward(sd: dict, cfg, ids: torch.Tensor, last_only: bool = False,
            store_dtype: torch.dtype | None = None) -> torch.Tensor:
    """ids [B, S] -> logits [B, S, V] (fp32), full causal attention, no cache;
    last_only: the LM head on the last position only -> [B, 1, V].
    store_dtype (e.g. bf16): the reference's eager forward in that dtype --
    every module output (norms, projections, attention, activations, residual
    sums, logits) rounded to it, arithmetic inside a module in fp32."""
    r = _storer(store_dtype)
    f = {k: v.detach().float().cpu() for k, v in sd.items()}
    B, S = ids.shape
    Hq, Hkv, D = cfg.n_heads, cfg.n_kv_heads, cfg.head_dim
    cos, sin = O.compute_rope_params(D, cfg.rope_base, S)
    pos = torch.arange(S)[None, :, None]
    x = f["tok_embed.weight"][ids.cpu()]
    for i in range(cfg.n_layers):
        p = f"transformer_blocs.{i}."
        h = r(O.rmsnorm(x, f[p + "rms_norm1.weight"], 1e-6))
        q = r(h @ f[p + "attn.Wq.weight"].T).view(B, S, Hq, D)
        k = r(h @ f[p + "attn.Wk.weight"].T).view(B, S, Hkv, D)
        v = r(h @ f[p + "attn.Wv.weight"].T).view(B, S, Hkv, D)
        q = r(O.qk_norm_rope(q, f.get(p + "attn.q_norm.weight"), 1e-6, cos, sin, pos))
        k = r(O.qk_norm_rope(k, f.get(p + "attn.k_norm.weight"), 1e-6, cos, sin, pos))
        o = r(O.attention(q, k, v, causal=True)).reshape(B, S, Hq * D)
        x = r(x + r(o @ f[p + "attn.out_projection.weight"].T))
        h = r(O.rmsnorm(x, f[p + "rms_norm2.weight"], 1e-6))
        g = r(torch.nn.functional.silu(h @ f[p + "ffn.fused_linear_layer1.weight"].T))
        u = r(h @ f[p + "ffn.linear_layerP.weight"].T)
        x = r(x + r(r(g * u) @ f[p + "ffn.linear_layer2.weight"].T))
    if last_only:
        x = x[:, -1:]
    x = r(O.rmsnorm(x, f["final_rmsnorm.weight"], 1e-6))
    return r(x @ f["out_head.weight"].T)


@torch.no_grad()
def decode_step_cached(f: dict, cfg, tok: torch.Tensor, kc: list, vc: list, pos: int) -> torch.Tensor:
    """One greedy decode step with a KV cache (fp32 CPU): tok [B] at position
    `pos`; kc/vc per layer [B, Hkv, cap, D] are written at row pos.  Returns
    the next tokens [B].  Same arithmetic as forward() restricted to one row."""
    return decode_logits_cached(f, cfg, tok, kc, vc, pos).argmax(-1)


@torch.no_grad()
def decode_logits_cached(f: dict, cfg, tok: torch.Tensor, kc: list, vc: list,
                         pos: int, store_dtype: torch.dtype | None = None) -> torch.Tensor:
    """decode_step_cached's logits [B, V] (fp32) before the argmax;
    store_dtype as in forward() (the cache rows written are rounded too)."""
    r = _storer(store_dtype)
    B = tok.shape[0]
    Hq, Hkv, D = cfg.n_heads, cfg.n_kv_heads, cfg.head_dim
    cos, sin = O.compute_rope_params(D, cfg.rope_base, pos + 1)
    p_idx = torch.full((1, 1, 1), pos)
    x = f["tok_embed.weight"][tok][:, None]                       # [B,1,E]
    for i in range(cfg.n_layers):
        p = f"transformer_blocs.{i}."
        h = r(O.rmsnorm(x, f[p + "rms_norm1.weight"], 1e-6))
        q = r(h @ f[p + "attn.Wq.weight"].T).view(B, 1, Hq, D)
        k = r(h @ f[p + "attn.Wk.weight"].T).view(B, 1, Hkv, D)
        v = r(h @ f[p + "attn.Wv.weight"].T).view(B, 1, Hkv, D)
        q = r(O.qk_norm_rope(q, f.get(p + "attn.q_norm.weight"), 1e-6, cos, sin, p_idx))
        k = r(O.qk_norm_rope(k, f.get(p + "attn.k_norm.weight"), 1e-6, cos, sin, p_idx))
        kc[i][:, :, pos] = k[:, 0]
        vc[i][:, :, pos] = v[:, 0]
        K = kc[i][:, :, :pos + 1].repeat_interleave(Hq // Hkv, dim=1)   # [B,Hq,L,D]
        V = vc[i][:, :, :pos + 1].repeat_interleave(Hq // Hkv, dim=1)
        s = torch.einsum("bhd,bhld->bhl", q[:, 0], K) / D ** 0.5
        o = r(torch.einsum("bhl,bhld->bhd", torch.softmax(s, -1), V)).reshape(B, 1, Hq * D)
        x = r(x + r(o @ f[p + "attn.out_projection.weight"].T))
        h = r(O.rmsnorm(x, f[p + "rms_norm2.weight"], 1e-6))
        g = r(torch.nn.functional.silu(h @ f[p + "ffn.fused_linear_layer1.weight"].T))
        u = r(h @ f[p + "ffn.linear_layerP.weight"].T)
        x = r(x + r(r(g * u) @ f[p + "ffn.linear_layer2.weight"].T))
    x = r(O.rmsnorm(x, f["final_rmsnorm.weight"], 1e-6))
    return r(x[:, 0] @ f["out_head.weight"].T)


def random_state_dict(cfg, std: float = 0.02, seed: int = 0) -> dict:
    """fp32 CPU weights of the Qwen3 shape: matrices ~ N(0, std), norms 1."""
    g = torch.Generator().manual_seed(seed)
    E, Hq, Hkv, D, F = cfg.embed_dim, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, cfg.hidden_dim
    r = lambda *s: torch.randn(*s, generator=g) * std  # noqa: E731
    sd = {"tok_embed.weight": r(cfg.vocab_size, E), "final_rmsnorm.weight": torch.ones(E),
          "out_head.weight": r(cfg.vocab_size, E)}
    for i in range(cfg.n_layers):
        p = f"transformer_blocs.{i}."
        sd.update({p + "rms_norm1.weight": torch.ones(E), p + "rms_norm2.weight": torch.ones(E),
                   p + "attn.Wq.weight": r(Hq * D, E), p + "attn.Wk.weight": r(Hkv * D, E),
                   p + "attn.Wv.weight": r(Hkv * D, E), p + "attn.out_projection.weight": r(E, Hq * D),
                   p + "attn.q_norm.weight": torch.ones(D), p + "attn.k_norm.weight": torch.ones(D),
                   p + "ffn.fused_linear_layer1.weight": r(F, E),
                   p + "ffn.linear_layerP.weight": r(F, E), p + "ffn.linear_layer2.weight": r(E, F)})
    return sd
