"""fp32 PyTorch-eager restatements of each hot-path op (CPU).  Test oracle only."""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F


def f32(t: torch.Tensor) -> torch.Tensor:
    return t.detach().to("cpu", torch.float32)


def rmsnorm(x, w, eps=1e-6):
    """nn.RMSNorm semantics, as tests/rmsnorm_test.py:19 uses for the check of
    csrc/dlops/rmsnorm/rmsnorm_fp16.cuh:95-107 (x * rsqrt(mean(x^2)+eps) * w)."""
    x, w = f32(x), f32(w)
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w


def layernorm(x, w, b=None, eps=1e-6):
    """nn.LayerNorm with beta = 0 (tests/layernorm_test.py:19-21) -- the
    reference kernel csrc/dlops/layernorm/layernorm_fp16.cuh:46-144 has no beta;
    the optional b here is the extension this build adds."""
    x, w = f32(x), f32(w)
    mu = x.mean(-1, keepdim=True)
    var = (x - mu).pow(2).mean(-1, keepdim=True)
    y = (x - mu) * torch.rsqrt(var + eps) * w
    return y if b is None else y + f32(b)


def compute_rope_params(head_dim, theta_base, context_length, dtype=torch.float16):
    """torchpp/dlops/rope.py:43-54: fp32 angles, cos/sin = cat(theta, theta)
    cast to fp16 (the reference always returns fp16 tables)."""
    ar = torch.arange(0, head_dim, 2, dtype=torch.float32)
    inv_freq = 1.0 / (theta_base ** (ar / head_dim))
    pos = torch.arange(context_length, dtype=torch.float32)
    ang = pos[:, None] * inv_freq[None, :]
    ang = torch.cat([ang, ang], dim=1)
    return torch.cos(ang).to(dtype).contiguous(), torch.sin(ang).to(dtype).contiguous()


def rotate_half(x):
    h = x.shape[-1] // 2
    return torch.cat([-x[..., h:], x[..., :h]], dim=-1)


def rope(x, cos, sin, pos_offset=0):
    """x [B,H,S,D]: x*cos + rotate_half(x)*sin, cos/sin rows pos_offset.. --
    the arithmetic of csrc/dlops/rope/apply_rope.cuh:15-46 (verified equal to
    rotate_half), rows sliced as torchpp/attention/gqa.py:108-112 does."""
    x = f32(x)
    S = x.shape[-2]
    c = f32(cos)[pos_offset:pos_offset + S]
    s = f32(sin)[pos_offset:pos_offset + S]
    return x * c + rotate_half(x) * s


def act(y, kind):
    """csrc/activation/activation.cuh:26-67: tanh-GeLU, SiLU, ReLU."""
    if kind == "none":
        return y
    if kind == "silu":
        return F.silu(y)
    if kind == "gelu":
        return F.gelu(y, approximate="tanh")
    if kind == "relu":
        return F.relu(y)
    raise ValueError(kind)


def linear(x, w, b=None, kind="none", residual=None):
    """act(x @ W^T + b) (+ residual): what LinearSilu/LinearGelu are meant to
    compute (csrc/activation/binding.cu:11-109 with the epilogue of
    fused_gemm.cuh:79-105); swiglu = silu(x Wg^T) * (x Wu^T) as the SwiGLU MLP
    of examples/TTS/dia/model.py:104-116."""
    x, w = f32(x), f32(w)
    if kind == "swiglu":
        n = w.shape[0] // 2
        g = x @ w[:n].T
        u = x @ w[n:].T
        if b is not None:
            bb = f32(b)
            g, u = g + bb[:n], u + bb[n:]
        y = F.silu(g) * u
    else:
        y = x @ w.T
        if b is not None:
            y = y + f32(b)
        y = act(y, kind)
    if residual is not None:
        y = y + f32(residual)
    return y


def hgemv(W, x):
    """y = A x: the CPU reference of csrc/blas/hgemv/hgemv_bench.cpp:10-24."""
    return f32(W) @ f32(x)


def attention(q, k, v, causal=False, window_left=-1, scale=None):
    """Explicit softmax(Q K^T * scale + mask) V in fp32 on [B,S,H,D] tensors:
    flash_attn_func semantics as called at torchpp/attention/gqa.py:128 and
    swa.py:85-89 -- causal mask aligned bottom-right (query i at key position
    i + Sk - Sq), window (w-1, 0) => keys in [p - window_left, p], GQA via the
    repeat_interleave of gqa.py:120-121."""
    q, k, v = f32(q), f32(k), f32(v)
    B, Sq, Hq, D = q.shape
    Sk, Hkv = k.shape[1], k.shape[2]
    g = Hq // Hkv
    k = k.repeat_interleave(g, dim=2)
    v = v.repeat_interleave(g, dim=2)
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    s = torch.einsum("bqhd,bkhd->bhqk", q, k) * scale
    qpos = torch.arange(Sq)[:, None] + (Sk - Sq)
    kpos = torch.arange(Sk)[None, :]
    mask = torch.zeros(Sq, Sk, dtype=torch.bool)
    if causal:
        mask |= kpos > qpos
    if window_left >= 0:
        mask |= kpos < qpos - window_left
    s = s.masked_fill(mask, float("-inf"))
    p = torch.softmax(s, dim=-1)
    p = torch.nan_to_num(p, nan=0.0)  # fully masked rows -> zeros
    return torch.einsum("bhqk,bkhd->bqhd", p, v)


def attention_decode(q, k_cache, v_cache, seqlens, window_left=-1, scale=None):
    """q [B,Hq,D] at position seqlens[b]-1 against BHSD caches (KVCache layout
    of torchpp/llmops/kvcache.py:34-48)."""
    q, kc, vc = f32(q), f32(k_cache), f32(v_cache)
    B, Hq, D = q.shape
    out = torch.zeros(B, Hq, D)
    for b in range(B):
        L = int(seqlens[b])
        if L == 0:
            continue
        qb = q[b][None, None]                       # [1,1,Hq,D]
        kb = kc[b, :, :L].transpose(0, 1)[None]     # [1,L,Hkv,D]
        vb = vc[b, :, :L].transpose(0, 1)[None]
        out[b] = attention(qb, kb, vb, causal=True, window_left=window_left, scale=scale)[0, 0]
    return out


def qk_norm_rope(x, w, eps, cos, sin, pos):
    """Per-head q/k RMSNorm (nn.RMSNorm(head_dim), gqa.py:62-64,90-94) then RoPE
    at the token's absolute position (gqa.py:108-112).  x [..., D]; pos int
    tensor broadcastable to x.shape[:-1]."""
    x = f32(x)
    if w is not None:
        x = rmsnorm(x, w, eps)
    c = f32(cos)[pos]
    s = f32(sin)[pos]
    return x * c + rotate_half(x) * s


# ---- fp8 (e4m3) decode weights -------------------------------------------
# The reference lists quantized GEMMs as future work (todo.md:24-29) and has
# no implementation; the format is this build's: per-output-row scale =
# amax / 448, bytes = e4m3(w / scale) (round to nearest even, saturated), and
# inside each 64-wide k-block byte 16c + 4s + j holds k = 16s + {2c, 2c+1,
# 2c+8, 2c+9}[j].  The tolerance of the fp8 linear is defined against the
# dequantized weight (a weight-only format: activations stay bf16/fp16).

def fp8_k_order(K):
    """Logical k held by each stored byte position of a row (length K)."""
    pos = torch.arange(64)
    c, s, j = pos // 16, (pos // 4) % 4, pos % 4
    blk = 16 * s + 2 * c + (j % 2) + (j // 2) * 8
    return (torch.arange(0, K, 64)[:, None] + blk[None, :]).reshape(-1)


def _group_rows(q):
    """[rows, K] bytes (k already in stored order) -> the grouped storage
    [ceil(rows/32)][K/64][32][64] as one flat uint8 tensor."""
    rows, K = q.shape
    G = (rows + 31) // 32
    pad = torch.zeros(G * 32, K, dtype=torch.uint8)
    pad[:rows] = q
    return pad.view(G, 32, K // 64, 64).permute(0, 2, 1, 3).contiguous().view(-1)


def _ungroup_rows(flat, rows, K):
    G = (rows + 31) // 32
    return flat.view(G, K // 64, 32, 64).permute(0, 2, 1, 3).reshape(G * 32, K)[:rows]


def quantize_weight_fp8(w):
    """w [rows, K] -> (flat uint8 storage, scale fp32 [rows]); the storage is
    32-row groups [ceil(rows/32)][K/64][32][64 B], rows past `rows` zero."""
    w = f32(w)
    amax = w.abs().amax(dim=1)
    scale = torch.where(amax > 0, amax / 448.0, torch.ones_like(amax))
    q = (w / scale[:, None]).clamp(-448.0, 448.0).to(torch.float8_e4m3fn)
    q = q[:, fp8_k_order(w.shape[1])].view(torch.uint8)
    return _group_rows(q), scale


def dequantize_weight_fp8(q, scale, K):
    """Inverse of quantize_weight_fp8, fp32 [rows, K] in natural k order."""
    q, scale = q.detach().cpu(), f32(scale)
    rows = scale.shape[0]
    vals = _ungroup_rows(q, rows, K).view(torch.float8_e4m3fn).to(torch.float32)
    vals = vals * scale[:, None]
    out = torch.empty_like(vals)
    out[:, fp8_k_order(K)] = vals
    return out
