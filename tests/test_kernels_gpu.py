"""GPU parity tests: every sm_100a kernel, called through the C-ABI (via the
thin ctypes wrappers in torchplusplus_b200.ops), against the fp32 CPU oracle
on the same seeded inputs.

Tolerance (the project's parity bar): fp16/bf16 outputs must satisfy
max |err| <= 2e-2 * max(1, |ref|) against the fp32 reference (absolute for
unit-scale values; relative above 1, where one bf16 ulp alone exceeds 2e-2),
and mean |err| <= 1e-3 against
the fp32 reference rounded once to the output dtype.  (The second comparison
is against the rounded reference because storing a unit-scale value in bf16
alone costs a mean error of ulp/4 ~ 1e-3-2e-3; the bound then measures the
kernel's own error, not the storage format's.)
"""
import math

import pytest
import torch

from oracle import ops as O
from torchplusplus_b200 import ops

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-2
MEAN_ABS = 1e-3
DEV = "cuda"
DTYPES = [torch.float16, torch.bfloat16]


def gen(seed=0):
    return torch.Generator().manual_seed(seed)


def rnd(*shape, g, std=1.0, mean=0.0, dtype=torch.float16):
    return (mean + std * torch.randn(*shape, generator=g)).to(dtype)


def check(y, ref, max_abs=MAX_ABS, mean_abs=MEAN_ABS):
    dt = y.dtype
    y = y.detach().float().cpu()
    ref = ref.float()
    assert y.shape == ref.shape, (y.shape, ref.shape)
    assert torch.isfinite(y).all()
    err = (y - ref).abs() / ref.abs().clamp(min=1.0)
    assert err.max().item() <= max_abs, f"max abs err {err.max().item():.3g}"
    err_r = (y - ref.to(dt).float()).abs()
    assert err_r.mean().item() <= mean_abs, f"mean abs err {err_r.mean().item():.3g}"


# ------------------------------------------------------------------ norms
@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("shape", [(2048, 1024), (32, 128, 512), (3, 100), (5, 4104), (1, 8192),
                                   (4, 16, 1, 128)])
def test_rmsnorm(dtype, shape):
    g = gen(1)
    x = rnd(*shape, g=g, dtype=dtype)
    w = rnd(shape[-1], g=g, mean=1.0, std=0.1, dtype=dtype)
    y = ops.rmsnorm(x.to(DEV), w.to(DEV), 1e-6)
    check(y, O.rmsnorm(x, w, 1e-6))


def test_rmsnorm_strided_rows_and_empty():
    g = gen(2)
    base = rnd(64, 2048, g=g)
    x = base[:, :1024]  # row stride 2048
    w = rnd(1024, g=g, mean=1.0, std=0.1)
    check(ops.rmsnorm(x.to(DEV), w.to(DEV)), O.rmsnorm(x, w))
    e = ops.rmsnorm(torch.empty(0, 1024, dtype=torch.float16, device=DEV), w.to(DEV))
    assert e.shape == (0, 1024)


@pytest.mark.parametrize("dtype", DTYPES)
def test_add_rmsnorm(dtype):
    g = gen(3)
    x, r = rnd(32, 1024, g=g, dtype=dtype), rnd(32, 1024, g=g, dtype=dtype)
    w = rnd(1024, g=g, mean=1.0, std=0.1, dtype=dtype)
    rd = r.to(DEV)
    y = ops.add_rmsnorm(x.to(DEV), rd, w.to(DEV), 1e-6)
    s = (x.float() + r.float()).to(dtype)
    check(rd, s.float(), max_abs=0, mean_abs=0)
    check(y, O.rmsnorm(s, w, 1e-6))


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("bias", [False, True])
@pytest.mark.parametrize("shape", [(32, 128, 512), (7, 1000), (2048, 1024)])
def test_layernorm(dtype, bias, shape):
    g = gen(4)
    x = rnd(*shape, g=g, dtype=dtype, mean=3.0)  # large mean: checks the two-pass variance
    w = rnd(shape[-1], g=g, mean=1.0, std=0.1, dtype=dtype)
    b = rnd(shape[-1], g=g, std=0.1, dtype=dtype) if bias else None
    y = ops.layernorm(x.to(DEV), w.to(DEV), None if b is None else b.to(DEV), 1e-6)
    check(y, O.layernorm(x, w, b, 1e-6))


# ------------------------------------------------------------------ rope
@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("D", [128, 64, 10])
def test_rope(dtype, D):
    g = gen(5)
    x = rnd(2, 4, 96, D, g=g, dtype=dtype)
    cos, sin = O.compute_rope_params(D, 1e6, 200)
    y = ops.rope(x.to(DEV), cos.to(DEV), sin.to(DEV))
    check(y, O.rope(x, cos, sin))
    y = ops.rope(x.to(DEV), cos.to(DEV), sin.to(DEV), pos_offset=57)
    check(y, O.rope(x, cos, sin, pos_offset=57))


def test_rope_strided_bshd_view_and_fp32_tables():
    g = gen(6)
    xs = rnd(2, 33, 8, 128, g=g)           # [B,S,H,D] buffer
    x = xs.transpose(1, 2)                  # [B,H,S,D] view, not contiguous
    cos, sin = O.compute_rope_params(128, 1e6, 64, dtype=torch.float32)
    y = ops.rope(x.to(DEV), cos.to(DEV), sin.to(DEV))
    check(y, O.rope(x, cos, sin))


@pytest.mark.parametrize("dtype", DTYPES)
def test_qkrope_gqa_heads(dtype):
    g = gen(7)
    q, k = rnd(4, 16, 128, 128, g=g, dtype=dtype), rnd(4, 8, 128, 128, g=g, dtype=dtype)
    cos, sin = O.compute_rope_params(128, 1e6, 128)
    qo, ko = ops.qkrope(q.to(DEV), k.to(DEV), cos.to(DEV), sin.to(DEV))
    check(qo, O.rope(q, cos, sin))
    check(ko, O.rope(k, cos, sin))


# ------------------------------------------------------------------ linear
def _linear_case(M, N, K, act, dtype, bias=False, residual=False, seed=8):
    g = gen(seed)
    x = rnd(M, K, g=g, dtype=dtype)
    rows = 2 * N if act == "swiglu" else N
    w = rnd(rows, K, g=g, std=0.02, dtype=dtype)
    b = rnd(rows, g=g, std=0.1, dtype=dtype) if bias else None
    r = rnd(M, N, g=g, dtype=dtype) if residual else None
    y = ops.linear(x.to(DEV), w.to(DEV), None if b is None else b.to(DEV), act=act,
                   residual=None if r is None else r.to(DEV))
    check(y, O.linear(x, w, b, act, r))


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("M", [1, 7, 17, 20, 31, 32, 64])
@pytest.mark.parametrize("act", ["none", "silu", "gelu", "relu", "swiglu"])
def test_linear_decode_shapes(dtype, M, act):
    # 17..32 tokens exercise the two-tile (16 + up to 16 tokens) decode grids
    _linear_case(M, 3072, 1024, act, dtype)


@pytest.mark.parametrize("MNK", [(32, 1024, 3072), (20, 1024, 2048), (32, 4096, 1024),
                                 (9, 6144, 1024), (32, 640, 4096)])
def test_linear_decode_planned_shapes_bias_residual(MNK):
    """Slice widths, token split and single- vs multi-chunk plans of the
    x-stationary decode linear, with bias and residual."""
    M, N, K = MNK
    _linear_case(M, N, K, "none", torch.bfloat16, bias=True, residual=True, seed=21)


def test_l2_prefetch_leaves_data_unchanged():
    g = gen(22)
    w = rnd(4096, 1024, g=g, dtype=torch.bfloat16).to(DEV)
    before = w.clone()
    ops.l2_prefetch(w)
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    assert torch.equal(w, before)


@pytest.mark.parametrize("MNK", [(1, 1024, 3072), (5, 1000, 200), (32, 2048, 2048),
                                 (16, 24, 4096), (2, 4096, 1024)])
def test_linear_decode_ragged_bias_residual(MNK):
    M, N, K = MNK
    _linear_case(M, N, K, "silu", torch.bfloat16, bias=True, residual=True)
    _linear_case(M, N, K, "swiglu", torch.float16, bias=True, residual=True)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("act", ["none", "silu", "gelu", "swiglu"])
@pytest.mark.parametrize("MNK", [(2048, 3072, 1024), (65, 256, 64), (300, 1000, 200), (200, 384, 128),
                                 (512, 2048, 3072)])
def test_linear_tensor_core(dtype, act, MNK):
    M, N, K = MNK
    _linear_case(M, N, K, act, dtype)


@pytest.mark.parametrize("MNK", [(300, 1000, 200), (200, 384, 128), (2048, 3072, 1024)])
def test_linear_tensor_core_bias_residual(MNK):
    """Bias + residual epilogue on the 256-row-tile path (and its ragged last
    tile: one half partly or wholly past M)."""
    M, N, K = MNK
    _linear_case(M, N, K, "gelu", torch.bfloat16, bias=True, residual=True)


def test_linear_tensor_core_bias_residual():
    _linear_case(384, 1024, 1024, "gelu", torch.bfloat16, bias=True, residual=True)
    _linear_case(200, 3072, 1024, "swiglu", torch.float16, bias=True, residual=True)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("act", ["none", "swiglu", "silu"])
@pytest.mark.parametrize("MNK", [(32, 4096, 1024), (1, 1024, 1024), (64, 151936, 1024),
                                 (7, 1000, 200), (17, 3072, 1024)])
def test_rmsnorm_linear_fused(dtype, act, MNK):
    M, N, K = MNK
    g = gen(17)
    x = rnd(M, K, g=g, dtype=dtype)
    gamma = rnd(K, g=g, mean=1.0, std=0.1, dtype=dtype)
    rows = 2 * N if act == "swiglu" else N
    w = rnd(rows, K, g=g, std=0.02, dtype=dtype)
    r = rnd(M, N, g=g, dtype=dtype)
    wf = ops.fold_rmsnorm_weight(w.to(DEV), gamma.to(DEV))
    y = ops.rmsnorm_linear(x.to(DEV), wf, 1e-6, act=act, residual=r.to(DEV))
    h = O.rmsnorm(x, gamma, 1e-6)
    check(y, O.linear(h, w, None, act, r))


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("case", [
    # (M, N, K, act, fused norm, bias, residual)
    (32, 4096, 1024, "none", True, False, False),    # Qwen3-0.6B qkv
    (32, 1024, 2048, "none", False, False, True),    # o-proj + residual
    (32, 3072, 1024, "swiglu", True, False, False),  # gate/up
    (32, 1024, 3072, "none", False, False, True),    # down + residual
    (1, 1000, 512, "silu", False, True, True),       # ragged N, batch 1
    (20, 640, 192, "gelu", True, True, False),       # BN 32 with 20 tokens
    (32, 2048, 1024, "swiglu", False, True, True),   # full 32-token tile
    (9, 9000, 128, "none", False, False, False),     # 64 rows per CTA
    (3, 4736, 64, "relu", True, False, True),        # one k-block
])
def test_linear_packed(dtype, case):
    M, N, K, act, norm, bias, residual = case
    g = gen(31)
    x = rnd(M, K, g=g, dtype=dtype)
    rows = 2 * N if act == "swiglu" else N
    w = rnd(rows, K, g=g, std=0.02, dtype=dtype)
    b = rnd(rows, g=g, std=0.1, dtype=dtype) if bias else None
    r = rnd(M, N, g=g, dtype=dtype) if residual else None
    gamma = rnd(K, g=g, mean=1.0, std=0.1, dtype=dtype)
    wd = w.to(DEV)
    if norm:
        wd = ops.fold_rmsnorm_weight(wd, gamma.to(DEV))
    if not ops.PackedWeight.supported(N, K, act):
        pytest.skip("layer too wide for the packed form on this device")
    pw = ops.PackedWeight(wd, act)
    xp = ops.pack_activation(x.to(DEV))
    yp = torch.zeros(ops.packed_activation_bytes(M, N), dtype=torch.uint8, device=DEV) \
        if N % 64 == 0 else None
    y = ops.linear_packed(xp, M, pw, None if b is None else b.to(DEV),
                          None if r is None else r.to(DEV), 1e-6 if norm else None,
                          out_packed=yp)
    h = O.rmsnorm(x, gamma, 1e-6) if norm else x
    check(y, O.linear(h, w, b, act, r))
    if yp is not None:
        # the packed second output is exactly pack_activation(y)
        assert torch.equal(yp.cpu(), ops.pack_activation(y).cpu())


@pytest.mark.parametrize("KN", [(1024, 2048), (1024, 3072), (3072, 1024), (1024, 151936)])
def test_hgemv_sweep(KN):
    K, N = KN
    g = gen(9)
    x = rnd(K, g=g)
    W = rnd(N, K, g=g, std=0.02)
    y = ops.hgemv(W.to(DEV), x.to(DEV))
    check(y, O.hgemv(W, x))


def test_hgemv_known_answer_small():
    # csrc/blas/hgemv/hgemv_bench.cpp:69-73 recipe (A[i]=i+1, x[i]=i+1) at a size
    # that stays exact in fp16 inputs and fp32 accumulation.
    M, K = 4, 16
    A = torch.arange(1, M * K + 1, dtype=torch.float32).view(M, K)
    x = torch.arange(1, K + 1, dtype=torch.float32)
    y = ops.hgemv(A.half().to(DEV), x.half().to(DEV)).float().cpu()
    exp = O.hgemv(A, x)
    torch.testing.assert_close(y, exp.half().float(), atol=0, rtol=1e-3)


# ------------------------------------------------------------------ attention
def _attn_case(B, Sq, Sk, Hq, Hkv, D, causal, window, dtype, seed=10):
    g = gen(seed)
    q = rnd(B, Sq, Hq, D, g=g, dtype=dtype)
    k = rnd(B, Sk, Hkv, D, g=g, dtype=dtype)
    v = rnd(B, Sk, Hkv, D, g=g, dtype=dtype)
    y = ops.attention(q.to(DEV), k.to(DEV), v.to(DEV), causal=causal, window_left=window)
    check(y, O.attention(q, k, v, causal=causal, window_left=window))


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("case", [
    (1, 256, 256, 16, 8, 128, True, -1),     # config-2 shape family (GQA, causal)
    (2, 200, 200, 4, 4, 64, True, -1),       # ragged, MHA, D=64
    (1, 130, 130, 8, 2, 128, False, -1),     # non-causal
    (1, 300, 300, 4, 1, 128, True, 63),      # MQA + sliding window 64
    (2, 17, 301, 8, 4, 128, True, -1),       # chunked prefill: Sq < Sk, bottom-right
    (1, 1, 77, 4, 2, 128, True, -1),         # single query row
])
def test_attention_prefill(dtype, case):
    _attn_case(*case, dtype=dtype)


def test_attention_prefill_reads_bhsd_cache_views():
    g = gen(11)
    B, Hkv, Smax, D, L = 2, 4, 512, 128, 300
    kc = rnd(B, Hkv, Smax, D, g=g)
    vc = rnd(B, Hkv, Smax, D, g=g)
    q = rnd(B, L, 8, D, g=g)
    k = kc[:, :, :L].transpose(1, 2)
    v = vc[:, :, :L].transpose(1, 2)
    kd, vd = kc.to(DEV), vc.to(DEV)
    y = ops.attention(q.to(DEV), kd[:, :, :L].transpose(1, 2), vd[:, :, :L].transpose(1, 2),
                      causal=True)
    check(y, O.attention(q, k, v, causal=True))


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("case", [
    (4, 16, 8, 128, [1, 100, 1000, 5000], -1),
    (8, 16, 8, 128, [700, 1, 64, 65, 513, 2000, 129, 300], -1),  # splits merged in a cluster
    (3, 16, 8, 128, [4096, 4097, 9000], 4095),   # sliding window 4096
    (2, 16, 1, 128, [33, 700], -1),               # MQA
    (2, 8, 8, 64, [64, 1], -1),                   # MHA, D=64
    (1, 32, 2, 128, [2048], -1),                  # G=16 query heads per kv head
])
def test_attention_decode(dtype, case):
    B, Hq, Hkv, D, lens, window = case
    g = gen(12)
    Smax = max(lens) + 3
    q = rnd(B, Hq, D, g=g, dtype=dtype)
    kc = rnd(B, Hkv, Smax, D, g=g, dtype=dtype)
    vc = rnd(B, Hkv, Smax, D, g=g, dtype=dtype)
    sl = torch.tensor(lens, dtype=torch.int32)
    y = ops.attention_decode(q.to(DEV), kc.to(DEV), vc.to(DEV), sl.to(DEV), max(lens),
                             window_left=window)
    check(y, O.attention_decode(q, kc, vc, sl, window_left=window))


def test_attention_decode_uniform_lengths_without_seqlens():
    g = gen(13)
    q = rnd(2, 16, 128, g=g)
    kc = rnd(2, 8, 600, 128, g=g)
    vc = rnd(2, 8, 600, 128, g=g)
    y = ops.attention_decode(q.to(DEV), kc.to(DEV), vc.to(DEV), None, 513)
    check(y, O.attention_decode(q, kc, vc, torch.tensor([513, 513])))


# ------------------------------------------------------------------ cache helpers
@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("S", [1, 37])
def test_qk_norm_rope_cache(dtype, S):
    g = gen(14)
    B, Hq, Hkv, D, Smax = 3, 16, 8, 128, 128
    qkv = rnd(B, S, (Hq + 2 * Hkv) * D, g=g, dtype=dtype)
    qn = rnd(D, g=g, mean=1.0, std=0.1, dtype=dtype)
    kn = rnd(D, g=g, mean=1.0, std=0.1, dtype=dtype)
    cos, sin = O.compute_rope_params(D, 1e6, 256)
    pos = torch.tensor([0, 5, 90], dtype=torch.int32)
    kc = torch.zeros(B, Hkv, Smax, D, dtype=dtype, device=DEV)
    vc = torch.zeros_like(kc)
    q = ops.qk_norm_rope_cache(qkv.to(DEV), qn.to(DEV), kn.to(DEV), 1e-6, cos.to(DEV),
                               sin.to(DEV), pos.to(DEV), kc, vc, Hq, Hkv)
    x = qkv.view(B, S, Hq + 2 * Hkv, D)
    p = (pos[:, None] + torch.arange(S)[None, :])[:, :, None]     # [B,S,1]
    check(q, O.qk_norm_rope(x[:, :, :Hq], qn, 1e-6, cos, sin, p))
    kref = O.qk_norm_rope(x[:, :, Hq:Hq + Hkv], kn, 1e-6, cos, sin, p)
    for b in range(B):
        rows = slice(int(pos[b]), int(pos[b]) + S)
        check(kc[b, :, rows].transpose(0, 1), kref[b])
        check(vc[b, :, rows].transpose(0, 1), x[b, :, Hq + Hkv:].float(), max_abs=0, mean_abs=0)
    # rows outside the written range stay untouched
    assert kc[0, :, S:].abs().sum().item() == 0


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("case", [
    # B, Hq, Hkv, D, lens (new token at lens-1), window, norms
    (4, 16, 8, 128, [1, 64, 65, 700], -1, True),       # Qwen3-0.6B heads; first token
    (3, 16, 8, 128, [513, 2000, 40], 255, True),       # sliding window
    (2, 8, 1, 64, [129, 5], -1, False),                # MQA, D 64, no q/k norm
    (8, 32, 4, 128, [300] * 8, -1, True),              # 8 query heads per kv head
    (1, 64, 2, 128, [9000], -1, True),                 # G = 32: two head passes, many splits
])
def test_attention_decode_qkv_fused(dtype, case):
    """One launch = q/k norm + RoPE + KV append + attention; checked against
    the fp32 oracle and against the unfused two-kernel path."""
    B, Hq, Hkv, D, lens, window, norms = case
    g = gen(41)
    Smax = max(lens) + 5
    qkv = rnd(B, 1, (Hq + 2 * Hkv) * D, g=g, dtype=dtype)
    qn = rnd(D, g=g, mean=1.0, std=0.1, dtype=dtype) if norms else None
    kn = rnd(D, g=g, mean=1.0, std=0.1, dtype=dtype) if norms else None
    cos, sin = O.compute_rope_params(D, 1e6, Smax)
    kc0 = rnd(B, Hkv, Smax, D, g=g, dtype=dtype)
    vc0 = rnd(B, Hkv, Smax, D, g=g, dtype=dtype)
    sl = torch.tensor(lens, dtype=torch.int32)
    pos = sl - 1
    d = lambda t: None if t is None else t.to(DEV)
    kc, vc = kc0.to(DEV), vc0.to(DEV)
    y = ops.attention_decode_qkv(qkv.to(DEV), d(qn), d(kn), 1e-6, cos.to(DEV), sin.to(DEV),
                                 pos.to(DEV), kc, vc, sl.to(DEV), Smax, Hq, Hkv,
                                 window_left=window)
    # oracle: q/k normed + rotated, caches with the new row, decode attention
    x = qkv.view(B, 1, Hq + 2 * Hkv, D)
    p = pos[:, None, None]
    qref = O.qk_norm_rope(x[:, :, :Hq], qn, 1e-6, cos, sin, p)
    kref = O.qk_norm_rope(x[:, :, Hq:Hq + Hkv], kn, 1e-6, cos, sin, p)
    kref_c, vref_c = kc0.float().clone(), vc0.float().clone()
    for b in range(B):
        kref_c[b, :, int(pos[b])] = kref[b, 0].to(dtype).float()
        vref_c[b, :, int(pos[b])] = x[b, 0, Hq + Hkv:].float()
    check(y, O.attention_decode(qref[:, 0].to(dtype), kref_c.to(dtype), vref_c.to(dtype), sl,
                                window_left=window))
    # the cache rows written by the fused launch match the oracle; others untouched
    for b in range(B):
        check(kc[b, :, int(pos[b])], kref[b, 0])
        assert torch.equal(vc[b, :, int(pos[b])].cpu(), x[b, 0, Hq + Hkv:])
        keep = torch.ones(Smax, dtype=torch.bool)
        keep[int(pos[b])] = False
        assert torch.equal(kc[b][:, keep].cpu(), kc0[b][:, keep])
    # and the unfused path agrees
    kc2, vc2 = kc0.to(DEV), vc0.to(DEV)
    q2 = ops.qk_norm_rope_cache(qkv.to(DEV), d(qn), d(kn), 1e-6, cos.to(DEV), sin.to(DEV),
                                pos.to(DEV), kc2, vc2, Hq, Hkv)
    y2 = ops.attention_decode(q2.view(B, Hq, D), kc2, vc2, sl.to(DEV), Smax, window_left=window)
    check(y, y2.float().cpu())


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("case", [(32, 300), (4, 2000), (1, 9000)])   # (B, L): few .. many splits
@pytest.mark.parametrize("fused", [False, True])
def test_attention_decode_rising_scores(dtype, case, fused):
    """Scores that rise steadily along the key range (key j aligned with q,
    scaled by 40 j / L): each tile raises the row maximum a little, so the
    lazy O rescale (base kept until the maximum grows by more than 2^8) and
    the per-warp / per-split merges see stale bases grow step by step; the
    new key of the fused mode carries the largest score."""
    B, L = case
    Hq, Hkv, D = 16, 8, 128
    G = Hq // Hkv
    g = gen(61)
    cos, sin = O.compute_rope_params(D, 1e6, L + 1)
    qraw = torch.randn(B, 1, Hq + 2 * Hkv, D, generator=g)
    pos = torch.full((B,), L - 1, dtype=torch.int32)
    # direction each kv head's keys align with: its first query head, as the
    # kernel sees it (rotated at the new position in fused mode)
    qdir = O.qk_norm_rope(qraw[:, :, :Hq], None, 1e-6, cos, sin, pos[:, None, None])[:, 0] \
        if fused else qraw[:, 0, :Hq]
    qdir = qdir[:, ::G]                                                   # [B, Hkv, D]
    coef = 40.0 * torch.arange(L).float() / L * math.sqrt(D)              # score ~ 40 j / L
    kc0 = coef[None, None, :, None] * (qdir / qdir.norm(dim=-1, keepdim=True) ** 2)[:, :, None]
    kc0 = (kc0 + 0.3 * torch.randn(B, Hkv, L, D, generator=g)).to(dtype)
    vc0 = torch.randn(B, Hkv, L, D, generator=g).to(dtype)
    sl = torch.full((B,), L, dtype=torch.int32)
    kc, vc = kc0.to(DEV), vc0.to(DEV)
    if fused:
        # the new key continues the ramp: raw k = the ramp's next row
        qkv = qraw.clone()
        qkv[:, 0, Hq:Hq + Hkv] = kc0[:, :, L - 1].float()
        qkv = qkv.to(dtype)
        y = ops.attention_decode_qkv(qkv.view(B, 1, -1).to(DEV), None, None, 1e-6, cos.to(DEV),
                                     sin.to(DEV), pos.to(DEV), kc, vc, sl.to(DEV), L, Hq, Hkv)
        x = qkv.view(B, 1, Hq + 2 * Hkv, D)
        qref = O.qk_norm_rope(x[:, :, :Hq], None, 1e-6, cos, sin, pos[:, None, None])[:, 0]
        kref = O.qk_norm_rope(x[:, :, Hq:Hq + Hkv], None, 1e-6, cos, sin, pos[:, None, None])
        kr, vr = kc0.float().clone(), vc0.float().clone()
        kr[:, :, L - 1] = kref[:, 0].to(dtype).float()
        vr[:, :, L - 1] = x[:, 0, Hq + Hkv:].float()
        ref = O.attention_decode(qref.to(dtype), kr.to(dtype), vr.to(dtype), sl)
    else:
        q = qraw[:, 0, :Hq].to(dtype)
        y = ops.attention_decode(q.to(DEV), kc, vc, sl.to(DEV), L)
        ref = O.attention_decode(q, kc0, vc0, sl)
    check(y, ref)
    if B == 1:   # the many-split case really goes through the split merge
        from torchplusplus_b200 import _native as N
        assert N.lib().tpp_attention_decode_workspace_exact(B, Hq, Hkv, L, D, -1) > 0


def test_kv_append_and_kvcache():
    from torchplusplus_b200.llmops.kvcache import KVCache
    g = gen(15)
    c = KVCache(max_seq_len=64, n_kv_heads=2, head_dim=128, dtype=torch.bfloat16, device=DEV)
    k1, v1 = rnd(3, 2, 10, 128, g=g, dtype=torch.bfloat16), rnd(3, 2, 10, 128, g=g, dtype=torch.bfloat16)
    k2, v2 = rnd(3, 2, 1, 128, g=g, dtype=torch.bfloat16), rnd(3, 2, 1, 128, g=g, dtype=torch.bfloat16)
    c.update(k1.to(DEV), v1.to(DEV))
    kk, vv = c.update(k2.to(DEV), v2.to(DEV))
    assert c.cache_len == 11 and kk.shape == (3, 2, 11, 128)
    assert torch.equal(kk.cpu(), torch.cat([k1, k2], 2))
    assert torch.equal(vv.cpu(), torch.cat([v1, v2], 2))
    kk, vv = c.update(k2.to(DEV), v2.to(DEV), index=3)   # index path overwrites row 3
    assert torch.equal(kk[:, :, 3].cpu(), k2[:, :, 0]) and c.cache_len == 11
    with pytest.raises(ValueError):
        c.update(k1.to(DEV), v1.to(DEV), index=60)


def test_argmax_and_embedding():
    g = gen(16)
    logits = rnd(4, 151936, g=g, dtype=torch.bfloat16)
    logits[1, 7] = 100.0
    logits[1, 9] = 100.0     # tie -> first index
    logits[2].fill_(0.5)     # all equal -> 0
    got = ops.argmax(logits.to(DEV)).cpu()
    assert torch.equal(got, torch.argmax(logits.float(), dim=-1))
    table = rnd(1000, 1024, g=g)
    ids = torch.tensor([[3, 999, 0], [5, 5, 17]])
    emb = ops.embedding(ids.to(DEV), table.to(DEV)).cpu()
    assert torch.equal(emb, table[ids])


@pytest.mark.parametrize("V,ld,dtype", [(5, 5, torch.bfloat16), (37, 40, torch.float16),
                                         (64, 64, torch.bfloat16), (1003, 1003, torch.float16),
                                         (151936, 151936, torch.float32),
                                         (151937, 151944, torch.bfloat16)])
def test_argmax_row_slices(V, ld, dtype):
    """Rows are split over a CTA cluster: ties across slices resolve to the
    first index, NaN wins, a maximum in the vector tail is found."""
    g = gen(31)
    base = rnd(6, ld, g=g, dtype=dtype)
    logits = base[:, :V]
    logits[1, V - 1] = 50.0                  # max in the last element (tail)
    logits[2, V // 2] = 50.0
    logits[2, V - 1] = 50.0                  # tie across slices -> first
    logits[3].fill_(-1.0)                    # all equal -> 0
    logits[4, V // 3] = float("nan")         # NaN is the max
    logits[5, 0] = 50.0
    logits[5, V - 1] = 50.0
    got = ops.argmax(base.to(DEV)[:, :V]).cpu()
    assert torch.equal(got, torch.argmax(logits.float(), dim=-1))


def test_no_bounded_wait_expired():
    assert ops.device_error() == 0


def test_bounded_wait_expiry_is_reported_and_the_gpu_stays_usable():
    """A device wait that runs out (an mbarrier nothing arrives on, no copy in
    flight, 256 polls) returns instead of hanging: the kernel exits, the flag
    carries the site code, reading it clears it, and later kernels run."""
    from torchplusplus_b200 import _native as N
    assert ops.device_error() == 0
    st = torch.cuda.current_stream().cuda_stream
    assert N.lib().tpp_debug_expire_wait(256, 0x5A, st) == 0, N.lib().tpp_last_error()
    torch.cuda.synchronize()
    assert ops.device_error() == 0x5A
    assert ops.device_error() == 0
    x = torch.randn(8, 1024, device=DEV, dtype=torch.bfloat16)
    w = torch.ones(1024, device=DEV, dtype=torch.bfloat16)
    check(ops.rmsnorm(x, w), O.rmsnorm(x.cpu(), w.cpu()))
    assert N.lib().tpp_debug_expire_wait(0, 1, st) != 0    # rejected on the host
