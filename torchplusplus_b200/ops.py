"""Tensor-level wrappers over the C-ABI kernels.

Every function here takes CUDA tensors, allocates its outputs with torch (the
caching allocator), launches on ``torch.cuda.current_stream()`` and raises on
any error.  CPU tensors are rejected: there is no CPU fallback.
"""
from __future__ import annotations

import math

import torch

from . import _native as N

_HALF = (torch.float16, torch.bfloat16)


def _cuda(*ts: torch.Tensor | None) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RuntimeError("torchplusplus_b200 ops need CUDA tensors (there is no CPU path)")


def _half(t: torch.Tensor, what: str) -> int:
    if t.dtype not in _HALF:
        raise TypeError(f"{what} must be float16 or bfloat16, got {t.dtype}")
    return N.dtype_code(t.dtype)


def _same_dtype(ref: torch.Tensor, *ts: torch.Tensor | None) -> None:
    for t in ts:
        if t is not None and t.dtype != ref.dtype:
            raise TypeError(f"dtype mismatch: {t.dtype} vs {ref.dtype}")


# ---------------------------------------------------------------- norms
def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6,
            out: torch.Tensor | None = None) -> torch.Tensor:
    """y = x * rsqrt(mean(x^2, -1) + eps) * weight over the last dim."""
    _cuda(x, weight)
    dt = _half(x, "x")
    _same_dtype(x, weight)
    if x.dim() < 1:
        raise ValueError("x must have at least one dim")
    n = x.shape[-1]
    if weight.dim() != 1 or weight.shape[0] != n:
        raise ValueError("weight must be 1-D with length == x.shape[-1]")
    if x.stride(-1) != 1:
        x = x.contiguous()
    x2 = x.reshape(-1, n) if x.is_contiguous() else x.contiguous().view(-1, n)
    weight = weight.contiguous()
    y = torch.empty(x.shape, dtype=x.dtype, device=x.device) if out is None else out
    y2 = y.view(-1, n)
    N.call("tpp_rmsnorm", x2.data_ptr(), x2.stride(0) if x2.shape[0] > 0 else n,
           weight.data_ptr(), y2.data_ptr(), y2.stride(0) if y2.shape[0] > 0 else n,
           x2.shape[0], n, float(eps), dt, N.stream_of(x))
    return y


def add_rmsnorm(x: torch.Tensor | None, residual: torch.Tensor, weight: torch.Tensor,
                eps: float = 1e-6, out: torch.Tensor | None = None) -> torch.Tensor:
    """residual += x (in place); returns rmsnorm(residual) * weight."""
    _cuda(x, residual, weight)
    dt = _half(residual, "residual")
    _same_dtype(residual, x, weight)
    if not residual.is_contiguous() or (x is not None and not x.is_contiguous()):
        raise ValueError("add_rmsnorm needs contiguous x/residual")
    n = residual.shape[-1]
    y = torch.empty_like(residual) if out is None else out
    N.call("tpp_add_rmsnorm", N.ptr(x), residual.data_ptr(), weight.data_ptr(), y.data_ptr(),
           residual.numel() // n, n, float(eps), dt, N.stream_of(residual))
    return y


def layernorm(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None = None,
              eps: float = 1e-6) -> torch.Tensor:
    """(x - mean) * rsqrt(var + eps) * weight (+ bias) over the last dim."""
    _cuda(x, weight, bias)
    dt = _half(x, "x")
    _same_dtype(x, weight, bias)
    n = x.shape[-1]
    if weight.numel() != n:
        raise ValueError("weight size must match the last dimension of x")
    x = x.contiguous()
    y = torch.empty_like(x)
    N.call("tpp_layernorm", x.data_ptr(), weight.contiguous().data_ptr(),
           N.ptr(bias.contiguous() if bias is not None else None), y.data_ptr(),
           x.numel() // n, n, float(eps), dt, N.stream_of(x))
    return y


# ---------------------------------------------------------------- rope
def _table(cos: torch.Tensor, sin: torch.Tensor, D: int) -> tuple[torch.Tensor, torch.Tensor, int, int]:
    if cos.dim() != 2 or sin.shape != cos.shape or cos.shape[1] != D:
        raise ValueError(f"cos/sin must both be [S, {D}]")
    if cos.dtype != sin.dtype:
        raise TypeError("cos and sin must share a dtype")
    if cos.stride(1) != 1 or sin.stride(1) != 1 or cos.stride(0) != sin.stride(0):
        cos, sin = cos.contiguous(), sin.contiguous()
    return cos, sin, cos.stride(0), N.dtype_code(cos.dtype)


def rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, pos_offset: int = 0) -> torch.Tensor:
    """NeoX RoPE on x [B,H,S,D] (any strides, D contiguous); cos/sin rows
    pos_offset .. pos_offset+S-1 are used.  Returns contiguous [B,H,S,D]."""
    _cuda(x, cos, sin)
    dt = _half(x, "x")
    if x.dim() != 4:
        raise ValueError("x must be 4-D [batch, heads, seq_len, head_dim]")
    B, H, S, D = x.shape
    if D % 2:
        raise ValueError("head dim must be even")
    if x.stride(3) != 1:
        x = x.contiguous()
    cos, sin, cs_stride, cs_dt = _table(cos, sin, D)
    if cos.shape[0] < pos_offset + S:
        raise ValueError("cos/sin table shorter than pos_offset + seq_len")
    out = torch.empty((B, H, S, D), dtype=x.dtype, device=x.device)
    N.call("tpp_rope", x.data_ptr(), x.stride(0), x.stride(1), x.stride(2), cos.data_ptr(),
           sin.data_ptr(), cs_stride, cs_dt, out.data_ptr(), B, H, S, D, int(pos_offset), dt,
           N.stream_of(x))
    return out


def qkrope(q: torch.Tensor, k: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
           pos_offset: int = 0) -> tuple[torch.Tensor, torch.Tensor]:
    """RoPE on Q [B,Hq,S,D] and K [B,Hk,S,D]; Hq may differ from Hk."""
    _cuda(q, k, cos, sin)
    dt = _half(q, "q")
    _same_dtype(q, k)
    if q.dim() != 4 or k.dim() != 4:
        raise ValueError("q and k must be 4-D [batch, heads, seq_len, head_dim]")
    B, Hq, S, D = q.shape
    if k.shape[0] != B or k.shape[2] != S or k.shape[3] != D:
        raise ValueError("k must match q in batch, seq_len and head_dim")
    q, k = q.contiguous(), k.contiguous()
    cos, sin, cs_stride, cs_dt = _table(cos, sin, D)
    if cos.shape[0] < pos_offset + S:
        raise ValueError("cos/sin table shorter than pos_offset + seq_len")
    qo, ko = torch.empty_like(q), torch.empty_like(k)
    N.call("tpp_qkrope", q.data_ptr(), k.data_ptr(), cos.data_ptr(), sin.data_ptr(), cs_stride,
           cs_dt, qo.data_ptr(), ko.data_ptr(), B, Hq, k.shape[1], S, D, int(pos_offset), dt,
           N.stream_of(q))
    return qo, ko


# ---------------------------------------------------------------- linear
def linear(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None = None,
           act: str = "none", residual: torch.Tensor | None = None,
           out: torch.Tensor | None = None) -> torch.Tensor:
    """y = act(x @ weight.T + bias) + residual over the last dim of x.

    act: none | silu | gelu (tanh) | relu | swiglu.  For swiglu, weight is
    [2N, K] = cat(gate, up) and y = silu(x Wg^T + bg) * (x Wu^T + bu)."""
    _cuda(x, weight, bias, residual, out)
    dt = _half(x, "x")
    _same_dtype(x, weight, bias, residual)
    K = x.shape[-1]
    if weight.dim() != 2 or weight.shape[1] != K:
        raise ValueError(f"weight must be [N, {K}]")
    code = N.ACT_CODE[act]
    Nout = weight.shape[0] // 2 if act == "swiglu" else weight.shape[0]
    if act == "swiglu" and weight.shape[0] % 2:
        raise ValueError("swiglu weight needs an even number of rows (gate; up)")
    lead = x.shape[:-1]
    if x.stride(-1) != 1:
        x = x.contiguous()
    x2 = x.reshape(-1, K)
    if x2.shape[0] > 1 and x2.stride(0) % 8 != 0:
        x2 = x2.contiguous()
    M = x2.shape[0]
    weight = weight.contiguous()
    if out is None:
        out = torch.empty((*lead, Nout), dtype=x.dtype, device=x.device)
    y2 = out.view(-1, Nout)
    r2 = None
    if residual is not None:
        if residual.shape != out.shape:
            raise ValueError("residual must have the output's shape")
        r2 = residual.contiguous().view(-1, Nout)
    ldx = x2.stride(0) if M > 1 else K
    N.call("tpp_linear", x2.data_ptr(), ldx, weight.data_ptr(),
           N.ptr(bias.contiguous() if bias is not None else None), N.ptr(r2), y2.data_ptr(),
           Nout, M, Nout, K, code, dt, N.stream_of(x))
    return out


def fold_rmsnorm_weight(weight: torch.Tensor, gamma: torch.Tensor) -> torch.Tensor:
    """W' = W * gamma[None, :] (rounded once to W's dtype): the matrix
    rmsnorm_linear expects.  One-time preparation, not a hot-path op."""
    return (weight.float() * gamma.float()[None, :]).to(weight.dtype).contiguous()


def rmsnorm_linear(x: torch.Tensor, w_folded: torch.Tensor, eps: float = 1e-6,
                   bias: torch.Tensor | None = None, act: str = "none",
                   residual: torch.Tensor | None = None,
                   out: torch.Tensor | None = None) -> torch.Tensor:
    """linear(rmsnorm(x, gamma), W) for decode shapes (<= 64 rows) in one
    kernel; `w_folded` = fold_rmsnorm_weight(W, gamma)."""
    _cuda(x, w_folded, bias, residual, out)
    dt = _half(x, "x")
    _same_dtype(x, w_folded, bias, residual)
    K = x.shape[-1]
    code = N.ACT_CODE[act]
    Nout = w_folded.shape[0] // 2 if act == "swiglu" else w_folded.shape[0]
    x2 = x.reshape(-1, K)
    if x2.stride(-1) != 1 or (x2.shape[0] > 1 and x2.stride(0) % 8):
        x2 = x2.contiguous()
    M = x2.shape[0]
    if out is None:
        out = torch.empty((*x.shape[:-1], Nout), dtype=x.dtype, device=x.device)
    y2 = out.view(-1, Nout)
    r2 = residual.contiguous().view(-1, Nout) if residual is not None else None
    N.call("tpp_rmsnorm_linear", x2.data_ptr(), x2.stride(0) if M > 1 else K,
           w_folded.data_ptr(), N.ptr(bias), N.ptr(r2), y2.data_ptr(), Nout, M, Nout, K,
           float(eps), code, dt, N.stream_of(x))
    return out


class PackedWeight:
    """A decode-linear weight re-laid out once (tpp_pack_weight) into the
    per-CTA, swizzled tiles the packed kernel copies with contiguous bulk
    loads.  `n` = outputs, `k` = inputs, `act` as for linear()."""

    def __init__(self, weight: torch.Tensor, act: str = "none"):
        _cuda(weight)
        dt = _half(weight, "weight")
        rows, K = weight.shape
        Nout = rows // 2 if act == "swiglu" else rows
        code = N.ACT_CODE[act]
        nbytes = N.lib().tpp_packed_weight_bytes(Nout, K, code)
        if nbytes <= 0:
            raise ValueError("layer does not fit the packed decode form "
                             "(K must be a multiple of 64, N at most 256 per SM)")
        w = weight.contiguous()
        self.data = torch.empty(nbytes, dtype=torch.uint8, device=weight.device)
        N.call("tpp_pack_weight", w.data_ptr(), Nout, K, code, dt, self.data.data_ptr(),
               N.stream_of(weight))
        self.n, self.k, self.act, self.dtype = Nout, K, act, weight.dtype

    @staticmethod
    def supported(n: int, k: int, act: str = "none") -> bool:
        return N.lib().tpp_packed_weight_bytes(n, k, N.ACT_CODE[act]) > 0


def packed_activation_bytes(M: int, K: int) -> int:
    return int(N.lib().tpp_packed_activation_bytes(M, K))


def pack_activation(x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """x [M, K] (M <= 64) -> packed activation bytes for linear_packed."""
    _cuda(x, out)
    dt = _half(x, "x")
    M, K = x.shape
    nbytes = packed_activation_bytes(M, K)
    if nbytes <= 0:
        raise ValueError("need 0 < M <= 64 and K a multiple of 64")
    if out is None:
        out = torch.empty(nbytes, dtype=torch.uint8, device=x.device)
    x2 = x if x.stride(-1) == 1 and x.stride(0) % 8 == 0 else x.contiguous()
    N.call("tpp_pack_activation", x2.data_ptr(), x2.stride(0), M, K, dt, out.data_ptr(),
           N.stream_of(x))
    return out


def linear_packed(x_packed: torch.Tensor, M: int, w: PackedWeight,
                  bias: torch.Tensor | None = None, residual: torch.Tensor | None = None,
                  eps: float | None = None, out: torch.Tensor | None = None,
                  out_packed: torch.Tensor | None = None) -> torch.Tensor:
    """Decode linear on packed operands: y[M, n] = act(scale * x.W^T + bias)
    + residual, scale = rsqrt(mean(x^2) + eps) when eps is given (w packed from
    the norm-folded matrix).  out_packed receives y packed for the next layer."""
    _cuda(x_packed, bias, residual, out, out_packed)
    dt = 1 if w.dtype == torch.bfloat16 else 0
    if out is None:
        out = torch.empty((M, w.n), dtype=w.dtype, device=x_packed.device)
    N.call("tpp_linear_packed", x_packed.data_ptr(), w.data.data_ptr(), N.ptr(bias),
           N.ptr(residual), out.data_ptr(), out.stride(0), N.ptr(out_packed), M, w.n, w.k,
           -1.0 if eps is None else float(eps), N.ACT_CODE[w.act], dt, N.stream_of(x_packed))
    return out


class Fp8Weight:
    """A linear weight quantized once to fp8 e4m3 with one fp32 scale per
    output row (tpp_quantize_weight_fp8), in the decode kernel's k order.
    `n` = outputs, `k` = inputs, `act` as for linear() (swiglu: [2N, K])."""

    def __init__(self, weight: torch.Tensor, act: str = "none"):
        _cuda(weight)
        dt = _half(weight, "weight")
        rows, K = weight.shape
        if K % 64:
            raise ValueError("fp8 weights need K a multiple of 64")
        w = weight.contiguous()
        # 32-row groups [ceil(rows/32)][K/64][32][64 B] (tpp_fp8_weight_bytes)
        self.q = torch.empty(int(N.lib().tpp_fp8_weight_bytes(rows, K)), dtype=torch.uint8,
                             device=weight.device)
        self.scale = torch.empty(rows, dtype=torch.float32, device=weight.device)
        N.call("tpp_quantize_weight_fp8", w.data_ptr(), rows, K, dt, self.q.data_ptr(),
               self.scale.data_ptr(), N.stream_of(weight))
        self.rows = rows
        self.n = rows // 2 if act == "swiglu" else rows
        self.k, self.act, self.dtype = K, act, weight.dtype

    def dequantize(self) -> torch.Tensor:
        """The weight this format represents, [rows, K] in self.dtype."""
        out = torch.empty((self.rows, self.k), dtype=self.dtype, device=self.q.device)
        N.call("tpp_dequantize_weight_fp8", self.q.data_ptr(), self.scale.data_ptr(),
               self.rows, self.k, N.dtype_code(self.dtype), out.data_ptr(),
               N.stream_of(self.q))
        return out


def linear_fp8(x: torch.Tensor, w: Fp8Weight, bias: torch.Tensor | None = None,
               residual: torch.Tensor | None = None, eps: float | None = None,
               out: torch.Tensor | None = None) -> torch.Tensor:
    """y = act(r * (x . W^T) + bias) + residual with W the fp8 weight;
    r = rsqrt(mean(x^2) + eps) when eps is given (norm weight folded into W
    before quantizing).  Up to 32 tokens run the fp8 decode kernel; more go
    through the dequantized weight and the GEMM path."""
    _cuda(x, bias, residual, out)
    dt = _half(x, "x")
    if x.dtype != w.dtype:
        raise TypeError("x and the fp8 weight's compute dtype differ")
    K = w.k
    x2 = x.reshape(-1, K)
    M = x2.shape[0]
    if M > 32:
        wd = w.dequantize()
        if eps is not None:
            ones = torch.ones(K, dtype=x.dtype, device=x.device)
            x = rmsnorm(x, ones, eps)
        return linear(x, wd, bias, w.act, residual, out)
    if x2.stride(-1) != 1 or (M > 1 and x2.stride(0) % 8):
        x2 = x2.contiguous()
    if out is None:
        out = torch.empty((*x.shape[:-1], w.n), dtype=x.dtype, device=x.device)
    y2 = out.view(-1, w.n)
    r2 = residual.contiguous().view(-1, w.n) if residual is not None else None
    N.call("tpp_linear_fp8", x2.data_ptr(), x2.stride(0) if M > 1 else K, w.q.data_ptr(),
           w.scale.data_ptr(), N.ptr(bias), N.ptr(r2), y2.data_ptr(), w.n, M, w.n, K,
           -1.0 if eps is None else float(eps), N.ACT_CODE[w.act], dt, N.stream_of(x))
    return out


def l2_prefetch(t: torch.Tensor) -> None:
    """Bulk-prefetch a (contiguous) tensor's bytes into L2 on the current stream."""
    _cuda(t)
    n = t.numel() * t.element_size()
    N.call("tpp_l2_prefetch", t.data_ptr(), n - n % 16, N.stream_of(t))


PERSISTENT_ROW_PAD = 32  # TPP_PERSISTENT_ROW_PAD (include/tpp_b200.h)


class PersistentDecode:
    """Operands of tpp_decode_step_persistent for one sequence: the per-layer
    pointer table (tpp_decode_layer records, in device memory) and the
    zero-initialised workspace.  `layers` holds per layer the folded QKV
    weight, q/k norm weights, o-proj weight, folded gate/up weight, down
    weight and the layer's [Hkv, Smax, D] K and V caches.  The projection
    and LM-head weights are copied once into the kernel's padded layout (row
    pitch in + PERSISTENT_ROW_PAD elements)."""

    def __init__(self, layers: list, emb: torch.Tensor, lm_head_folded: torch.Tensor,
                 cos: torch.Tensor, sin: torch.Tensor, Hq: int, Hkv: int, D: int, Smax: int,
                 eps: float = 1e-6):
        _cuda(emb, lm_head_folded, cos, sin)
        self.dt = _half(emb, "embedding")
        if cos.dtype != torch.float16 or sin.dtype != torch.float16 or cos.shape[1] != D:
            raise ValueError("RoPE tables must be fp16 [ctx, D]")
        dev = emb.device
        nbytes = int(N.lib().tpp_decode_step_persistent_workspace(
            emb.shape[1], Hq, Hkv, D, layers[0]["wgu"].shape[0] // 2, Smax))
        if nbytes <= 0:
            raise ValueError("model shape outside the persistent decode plan")
        # weights in the kernel's layout: row pitch in + TPP_PERSISTENT_ROW_PAD
        pad = lambda w: torch.nn.functional.pad(w, (0, PERSISTENT_ROW_PAD)).contiguous()
        lm_head_folded = pad(lm_head_folded)
        self.keep = [emb, lm_head_folded, cos, sin]
        ptrs = []
        for L in layers:
            L = dict(L, wqkv=pad(L["wqkv"]), wo=pad(L["wo"]), wgu=pad(L["wgu"]),
                     wdown=pad(L["wdown"]))
            for t in (L["wqkv"], L["qn"], L["kn"], L["wo"], L["wgu"], L["wdown"], L["kc"], L["vc"]):
                if t is not None:
                    _same_dtype(emb, t)
                    if not t.is_contiguous() or t.data_ptr() % 16:
                        raise ValueError("persistent decode operands must be contiguous and "
                                         "16-byte aligned (they are bulk-copied)")
                    self.keep.append(t)
                ptrs.append(0 if t is None else t.data_ptr())
        self.table = torch.tensor(ptrs, dtype=torch.int64).to(dev)
        self.n_layers = len(layers)
        self.E = emb.shape[1]
        self.V = lm_head_folded.shape[0]
        self.F = layers[0]["wgu"].shape[0] // 2
        self.Hq, self.Hkv, self.D, self.Smax, self.eps = Hq, Hkv, D, Smax, eps
        self.ws = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
        self.emb, self.lm_head, self.cos, self.sin = emb, lm_head_folded, cos, sin

    def step(self, tokens: torch.Tensor, positions: torch.Tensor, seqlens: torch.Tensor | None,
             out_ids: torch.Tensor | None, logits: torch.Tensor) -> None:
        """One greedy decode step (see tpp_decode_step_persistent)."""
        N.call("tpp_decode_step_persistent", self.table.data_ptr(), self.n_layers,
               self.emb.data_ptr(), self.lm_head.data_ptr(), self.cos.data_ptr(),
               self.sin.data_ptr(), self.cos.stride(0), tokens.data_ptr(), positions.data_ptr(),
               N.ptr(seqlens), N.ptr(out_ids), 0 if out_ids is None else out_ids.shape[-1],
               logits.data_ptr(), self.ws.data_ptr(), self.ws.numel(), self.E, self.Hq,
               self.Hkv, self.D, self.F, self.V, self.Smax, float(self.eps), self.dt,
               N.stream_of(logits))


def set_sm_budget(sms: int) -> None:
    """Decode launches made next from this thread plan their grids for `sms`
    SMs (0 = the whole device); see tpp_set_sm_budget."""
    N.call("tpp_set_sm_budget", int(sms))


def hgemv(weight: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
    """y[N] = weight[N,K] @ x[K] with fp32 accumulation."""
    _cuda(weight, x)
    dt = _half(x, "x")
    _same_dtype(x, weight)
    Nn, K = weight.shape
    if x.numel() != K:
        raise ValueError("x must have K elements")
    y = torch.empty(Nn, dtype=x.dtype, device=x.device)
    N.call("tpp_hgemv", weight.contiguous().data_ptr(), x.contiguous().data_ptr(), y.data_ptr(),
           Nn, K, dt, N.stream_of(x))
    return y


# ---------------------------------------------------------------- attention
def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool = False,
              window_left: int = -1, scale: float | None = None,
              out: torch.Tensor | None = None) -> torch.Tensor:
    """flash_attn_func semantics on [B,S,H,D] tensors (any batch/seq/head
    strides, D contiguous).  Causal masking is bottom-right aligned; GQA/MQA
    when Hq is a multiple of Hkv."""
    _cuda(q, k, v)
    dt = _half(q, "q")
    _same_dtype(q, k, v)
    B, Sq, Hq, D = q.shape
    Bk, Sk, Hkv, Dk = k.shape
    if Bk != B or Dk != D or v.shape != k.shape:
        raise ValueError("k/v must be [B, Sk, Hkv, D] matching q")
    if Hq % Hkv:
        raise ValueError("number of query heads must be a multiple of kv heads")
    q, k, v = (t if t.stride(3) == 1 else t.contiguous() for t in (q, k, v))
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    if out is None:
        out = torch.empty((B, Sq, Hq, D), dtype=q.dtype, device=q.device)
    N.call("tpp_attention_prefill", q.data_ptr(), q.stride(0), q.stride(1), q.stride(2),
           k.data_ptr(), k.stride(0), k.stride(1), k.stride(2), v.data_ptr(), v.stride(0),
           v.stride(1), v.stride(2), out.data_ptr(), out.stride(0), out.stride(1), out.stride(2),
           B, Sq, Sk, Hq, Hkv, D, int(bool(causal)), int(window_left), float(scale), dt,
           N.stream_of(q))
    return out


def decode_workspace_bytes(B: int, Hq: int, max_seqlen: int, D: int) -> int:
    return int(N.lib().tpp_attention_decode_workspace(B, Hq, max_seqlen, D))


def attention_decode(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                     seqlens: torch.Tensor | None, max_seqlen: int, window_left: int = -1,
                     scale: float | None = None, out: torch.Tensor | None = None,
                     workspace: torch.Tensor | None = None) -> torch.Tensor:
    """One query token per sequence.  q [B,Hq,D]; caches [B,Hkv,Smax,D] (BHSD,
    the KVCache layout); seqlens int32 [B] on the device (valid rows; the query
    is at position seqlens[b]-1) or None for max_seqlen everywhere."""
    _cuda(q, k_cache, v_cache, seqlens)
    dt = _half(q, "q")
    _same_dtype(q, k_cache, v_cache)
    B, Hq, D = q.shape
    Bc, Hkv, Smax, Dc = k_cache.shape
    if Bc != B or Dc != D or v_cache.shape != k_cache.shape or k_cache.stride() != v_cache.stride():
        raise ValueError("caches must be [B, Hkv, Smax, D] with identical layouts")
    if max_seqlen > Smax:
        raise ValueError("max_seqlen exceeds the cache capacity")
    if seqlens is not None and (seqlens.dtype != torch.int32 or seqlens.numel() != B):
        raise ValueError("seqlens must be int32 [B]")
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    if out is None:
        out = torch.empty((B, Hq, D), dtype=q.dtype, device=q.device)
    need = decode_workspace_bytes(B, Hq, max_seqlen, D)
    if workspace is None and need > 0:
        workspace = torch.empty(need, dtype=torch.uint8, device=q.device)
    N.call("tpp_attention_decode", q.data_ptr(), q.stride(0), q.stride(1), k_cache.data_ptr(),
           v_cache.data_ptr(), k_cache.stride(0), k_cache.stride(1), k_cache.stride(2),
           N.ptr(seqlens), int(max_seqlen), out.data_ptr(), out.stride(0), out.stride(1), B, Hq,
           Hkv, D, int(window_left), float(scale), N.ptr(workspace),
           0 if workspace is None else workspace.numel(), dt, N.stream_of(q))
    return out


def attention_decode_qkv(qkv: torch.Tensor, q_norm_w: torch.Tensor | None,
                         k_norm_w: torch.Tensor | None, eps: float, cos: torch.Tensor,
                         sin: torch.Tensor, positions: torch.Tensor, k_cache: torch.Tensor,
                         v_cache: torch.Tensor, seqlens: torch.Tensor, max_seqlen: int,
                         Hq: int, Hkv: int, window_left: int = -1, scale: float | None = None,
                         out: torch.Tensor | None = None,
                         workspace: torch.Tensor | None = None) -> torch.Tensor:
    """Decode step in one launch: qkv [B, 1, (Hq+2Hkv)*D] raw projection rows ->
    q/k RMSNorm + RoPE at positions[b], new k/v written into the caches at row
    positions[b], attention over keys up to it -> o [B, Hq, D].  Requires
    positions == seqlens - 1 (int32 [B] each); fp16 RoPE tables."""
    _cuda(qkv, q_norm_w, k_norm_w, cos, sin, positions, k_cache, v_cache, seqlens)
    dt = _half(qkv, "qkv")
    _same_dtype(qkv, k_cache, v_cache, q_norm_w, k_norm_w)
    B = qkv.shape[0]
    D = k_cache.shape[-1]
    if qkv.shape[-1] != (Hq + 2 * Hkv) * D or qkv.stride(-1) != 1:
        raise ValueError("qkv must be [B, 1, (Hq+2Hkv)*D]")
    if k_cache.shape[:2] != (B, Hkv) or v_cache.shape != k_cache.shape \
            or k_cache.stride() != v_cache.stride():
        raise ValueError("caches must be [B, Hkv, Smax, D] with identical layouts")
    for t, nm in ((positions, "positions"), (seqlens, "seqlens")):
        if t.dtype != torch.int32 or t.numel() != B:
            raise ValueError(f"{nm} must be int32 [B]")
    cos, sin, cs_stride, cs_dt = _table(cos, sin, D)
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    if out is None:
        out = torch.empty((B, Hq, D), dtype=qkv.dtype, device=qkv.device)
    need = decode_workspace_bytes(B, Hq, max_seqlen, D)
    if workspace is None and need > 0:
        workspace = torch.empty(need, dtype=torch.uint8, device=qkv.device)
    N.call("tpp_attention_decode_qkv", qkv.data_ptr(), qkv.stride(0), N.ptr(q_norm_w),
           N.ptr(k_norm_w), float(eps), cos.data_ptr(), sin.data_ptr(), cs_stride, cs_dt,
           positions.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), k_cache.stride(0),
           k_cache.stride(1), k_cache.stride(2), seqlens.data_ptr(), int(max_seqlen),
           out.data_ptr(), out.stride(0), out.stride(1), B, Hq, Hkv, D, int(window_left),
           float(scale), N.ptr(workspace), 0 if workspace is None else workspace.numel(), dt,
           N.stream_of(qkv))
    return out


def _paged_args(k_pool, v_pool, block_table, B):
    NB, Hkv, blk, D = k_pool.shape
    if blk != 64 or v_pool.shape != k_pool.shape or not k_pool.is_contiguous() \
            or not v_pool.is_contiguous():
        raise ValueError("pools must be contiguous [num_blocks, Hkv, 64, D]")
    if block_table.dtype != torch.int32 or block_table.dim() != 2 or block_table.shape[0] != B \
            or block_table.stride(1) != 1:
        raise ValueError("block_table must be int32 [B, max_blocks] with unit column stride")
    return NB, Hkv, D


def attention_decode_paged(q: torch.Tensor, k_pool: torch.Tensor, v_pool: torch.Tensor,
                           block_table: torch.Tensor, seqlens: torch.Tensor, max_seqlen: int,
                           window_left: int = -1, scale: float | None = None,
                           out: torch.Tensor | None = None,
                           workspace: torch.Tensor | None = None) -> torch.Tensor:
    """attention_decode over a paged cache: pools [num_blocks, Hkv, 64, D],
    key k of sequence b in block block_table[b, k // 64], row k % 64."""
    _cuda(q, k_pool, v_pool, block_table, seqlens)
    dt = _half(q, "q")
    _same_dtype(q, k_pool, v_pool)
    B, Hq, D = q.shape
    NB, Hkv, Dc = _paged_args(k_pool, v_pool, block_table, B)
    if Dc != D or seqlens.dtype != torch.int32 or seqlens.numel() != B:
        raise ValueError("head dims must match; seqlens int32 [B]")
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    if out is None:
        out = torch.empty((B, Hq, D), dtype=q.dtype, device=q.device)
    need = decode_workspace_bytes(B, Hq, max_seqlen, D)
    if workspace is None and need > 0:
        workspace = torch.empty(need, dtype=torch.uint8, device=q.device)
    N.call("tpp_attention_decode_paged", q.data_ptr(), q.stride(0), q.stride(1),
           k_pool.data_ptr(), v_pool.data_ptr(), NB, block_table.data_ptr(),
           block_table.stride(0), seqlens.data_ptr(), int(max_seqlen), out.data_ptr(),
           out.stride(0), out.stride(1), B, Hq, Hkv, D, int(window_left), float(scale),
           N.ptr(workspace), 0 if workspace is None else workspace.numel(), dt, N.stream_of(q))
    return out


def attention_decode_qkv_paged(qkv: torch.Tensor, q_norm_w: torch.Tensor | None,
                               k_norm_w: torch.Tensor | None, eps: float, cos: torch.Tensor,
                               sin: torch.Tensor, positions: torch.Tensor, k_pool: torch.Tensor,
                               v_pool: torch.Tensor, block_table: torch.Tensor,
                               seqlens: torch.Tensor, max_seqlen: int, Hq: int, Hkv: int,
                               window_left: int = -1, scale: float | None = None,
                               out: torch.Tensor | None = None,
                               workspace: torch.Tensor | None = None) -> torch.Tensor:
    """attention_decode_qkv over a paged cache (the new k/v rows are written
    into the pools)."""
    _cuda(qkv, q_norm_w, k_norm_w, cos, sin, positions, k_pool, v_pool, block_table, seqlens)
    dt = _half(qkv, "qkv")
    _same_dtype(qkv, k_pool, v_pool, q_norm_w, k_norm_w)
    B = qkv.shape[0]
    NB, Hkv_p, D = _paged_args(k_pool, v_pool, block_table, B)
    if Hkv_p != Hkv or qkv.shape[-1] != (Hq + 2 * Hkv) * D or qkv.stride(-1) != 1:
        raise ValueError("qkv must be [B, 1, (Hq+2Hkv)*D] matching the pools")
    for t, nm in ((positions, "positions"), (seqlens, "seqlens")):
        if t.dtype != torch.int32 or t.numel() != B:
            raise ValueError(f"{nm} must be int32 [B]")
    cos, sin, cs_stride, cs_dt = _table(cos, sin, D)
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    if out is None:
        out = torch.empty((B, Hq, D), dtype=qkv.dtype, device=qkv.device)
    need = decode_workspace_bytes(B, Hq, max_seqlen, D)
    if workspace is None and need > 0:
        workspace = torch.empty(need, dtype=torch.uint8, device=qkv.device)
    N.call("tpp_attention_decode_qkv_paged", qkv.data_ptr(), qkv.stride(0), N.ptr(q_norm_w),
           N.ptr(k_norm_w), float(eps), cos.data_ptr(), sin.data_ptr(), cs_stride, cs_dt,
           positions.data_ptr(), k_pool.data_ptr(), v_pool.data_ptr(), NB,
           block_table.data_ptr(), block_table.stride(0), seqlens.data_ptr(), int(max_seqlen),
           out.data_ptr(), out.stride(0), out.stride(1), B, Hq, Hkv, D, int(window_left),
           float(scale), N.ptr(workspace), 0 if workspace is None else workspace.numel(), dt,
           N.stream_of(qkv))
    return out


def kv_append_paged(k: torch.Tensor, v: torch.Tensor, k_pool: torch.Tensor, v_pool: torch.Tensor,
                    block_table: torch.Tensor, positions: torch.Tensor | None = None,
                    start_pos: int = 0) -> None:
    """k, v [B, Hkv, S, D] -> pools at positions (positions[b] or start_pos) + s."""
    _cuda(k, v, k_pool, v_pool, block_table, positions)
    dt = _half(k, "k")
    _same_dtype(k, v, k_pool, v_pool)
    B, Hkv, S, D = k.shape
    NB, Hkv_p, Dp = _paged_args(k_pool, v_pool, block_table, B)
    if v.shape != k.shape or Hkv_p != Hkv or Dp != D:
        raise ValueError("k/v must be [B, Hkv, S, D] matching the pools")
    if positions is not None and (positions.dtype != torch.int32 or positions.numel() != B):
        raise ValueError("positions must be int32 [B]")
    N.call("tpp_kv_append_paged", k.data_ptr(), k.stride(0), k.stride(1), k.stride(2),
           v.data_ptr(), v.stride(0), v.stride(1), v.stride(2), k_pool.data_ptr(),
           v_pool.data_ptr(), NB, block_table.data_ptr(), block_table.stride(0),
           N.ptr(positions), int(start_pos), B, Hkv, S, D, dt, N.stream_of(k))


# ---------------------------------------------------------------- cache / step helpers
def qk_norm_rope_cache(qkv: torch.Tensor, q_norm_w: torch.Tensor | None,
                       k_norm_w: torch.Tensor | None, eps: float, cos: torch.Tensor,
                       sin: torch.Tensor, positions: torch.Tensor, k_cache: torch.Tensor,
                       v_cache: torch.Tensor, Hq: int, Hkv: int,
                       q_out: torch.Tensor | None = None) -> torch.Tensor:
    """qkv [B,S,(Hq+2Hkv)*D] -> q [B,S,Hq,D] (normed + rotated); k (normed +
    rotated) and v are written into the caches at rows positions[b] + s."""
    _cuda(qkv, q_norm_w, k_norm_w, cos, sin, positions, k_cache, v_cache)
    dt = _half(qkv, "qkv")
    B, S, W = qkv.shape
    D = k_cache.shape[-1]
    if W != (Hq + 2 * Hkv) * D or qkv.stride(2) != 1 or qkv.stride(0) != S * qkv.stride(1):
        raise ValueError("qkv must be [B, S, (Hq+2Hkv)*D] with packed token rows")
    if positions.dtype != torch.int32 or positions.numel() != B:
        raise ValueError("positions must be int32 [B]")
    cos, sin, cs_stride, cs_dt = _table(cos, sin, D)
    if q_out is None:
        q_out = torch.empty((B, S, Hq, D), dtype=qkv.dtype, device=qkv.device)
    N.call("tpp_qk_norm_rope_cache", qkv.data_ptr(), qkv.stride(1), N.ptr(q_norm_w),
           N.ptr(k_norm_w), float(eps), cos.data_ptr(), sin.data_ptr(), cs_stride, cs_dt,
           positions.data_ptr(), q_out.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(),
           k_cache.stride(0), k_cache.stride(1), k_cache.stride(2), B, S, Hq, Hkv, D, dt,
           N.stream_of(qkv))
    return q_out


def kv_append(k: torch.Tensor, v: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
              start_pos: int = 0, positions: torch.Tensor | None = None) -> None:
    """Writes k/v [B,Hkv,S,D] into the BHSD caches at rows start_pos + s (or
    positions[b] + s)."""
    _cuda(k, v, k_cache, v_cache, positions)
    dt = _half(k, "k")
    _same_dtype(k, v, k_cache, v_cache)
    B, H, S, D = k.shape
    if v.shape != k.shape or k_cache.shape[0] < B or k_cache.shape[1] != H or k_cache.shape[3] != D:
        raise ValueError("k/v/cache shapes disagree")
    if positions is None and start_pos + S > k_cache.shape[2]:
        raise ValueError("KV cache overflow")
    N.call("tpp_kv_append", k.data_ptr(), k.stride(0), k.stride(1), k.stride(2), v.data_ptr(),
           v.stride(0), v.stride(1), v.stride(2), k_cache.data_ptr(), v_cache.data_ptr(),
           k_cache.stride(0), k_cache.stride(1), k_cache.stride(2), B, H, S, D, int(start_pos),
           N.ptr(positions), dt, N.stream_of(k))


def argmax(logits: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """Greedy token per row of logits [B, V] -> int64 [B]."""
    _cuda(logits)
    if logits.stride(-1) != 1:
        logits = logits.contiguous()
    B, V = logits.shape
    if out is None:
        out = torch.empty(B, dtype=torch.int64, device=logits.device)
    N.call("tpp_argmax", logits.data_ptr(), logits.stride(0), B, V, out.data_ptr(),
           N.dtype_code(logits.dtype), N.stream_of(logits))
    return out


def sample(logits: torch.Tensor, temperature: float = 1.0, top_k: int = 0, top_p: float = 1.0,
           seed: int = 0, counters: torch.Tensor | None = None,
           out: torch.Tensor | None = None) -> torch.Tensor:
    """One token per row of logits [B, V] from softmax(logits / temperature)
    restricted to the top_k largest logits and the top_p nucleus, on the
    device (see tpp_sample).  counters (int32 [B], e.g. positions) select the
    random draw per row."""
    _cuda(logits, counters)
    if logits.stride(-1) != 1:
        logits = logits.contiguous()
    B, V = logits.shape
    if counters is not None and (counters.dtype != torch.int32 or counters.numel() != B):
        raise ValueError("counters must be int32 [B]")
    if out is None:
        out = torch.empty(B, dtype=torch.int64, device=logits.device)
    N.call("tpp_sample", logits.data_ptr(), logits.stride(0), B, V, float(temperature),
           int(top_k), float(top_p), int(seed) & 0xFFFFFFFFFFFFFFFF, N.ptr(counters),
           out.data_ptr(), N.dtype_code(logits.dtype), N.stream_of(logits))
    return out


def embedding(ids: torch.Tensor, table: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    _cuda(ids, table)
    dt = _half(table, "table")
    if ids.dtype != torch.int64:
        ids = ids.long()
    ids = ids.contiguous()
    V, D = table.shape
    if out is None:
        out = torch.empty((*ids.shape, D), dtype=table.dtype, device=table.device)
    N.call("tpp_embedding", ids.data_ptr(), ids.numel(), table.contiguous().data_ptr(), V, D,
           out.data_ptr(), dt, N.stream_of(table))
    return out


def decode_advance(next_tokens: torch.Tensor, out_ids: torch.Tensor | None,
                   positions: torch.Tensor, seqlens: torch.Tensor | None) -> None:
    """positions += 1; out_ids[b, positions[b]] = next_tokens[b]; seqlens = positions + 1."""
    _cuda(next_tokens, out_ids, positions, seqlens)
    B = positions.numel()
    N.call("tpp_decode_advance", next_tokens.data_ptr(), N.ptr(out_ids),
           0 if out_ids is None else out_ids.stride(0), 0 if out_ids is None else out_ids.shape[1],
           positions.data_ptr(), N.ptr(seqlens), B, N.stream_of(positions))


def device_error() -> int:
    """Reads and clears the device flag raised when a bounded wait expires."""
    return int(N.lib().tpp_device_error(N.stream_of(torch.empty(0, device="cuda"))))
