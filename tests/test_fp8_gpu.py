"""fp8 (e4m3) decode weights: the quantizer against the oracle's restatement
(bit-exact bytes and scales) and the fp8 decode linear against the fp32
product with the dequantized weight (the weight-only format's reference),
under the suite's tolerance: max |err| <= 2e-2 * max(1, |ref|), mean |err|
<= 1e-3 against the reference rounded to the output dtype."""
import pytest
import torch

from oracle import ops as O
from torchplusplus_b200 import ops

from .test_kernels_gpu import DEV, DTYPES, check, gen, rnd

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("rows,K", [(8, 64), (37, 1024), (6144, 1024), (3, 3072)])
def test_quantize_matches_oracle(dtype, rows, K):
    g = gen(41)
    w = rnd(rows, K, g=g, std=0.05, dtype=dtype)
    w[0].zero_()                                    # zero row: scale 1, bytes 0
    if rows > 2:
        w[1, :8] = torch.tensor([1e-6, -3e-4, 0.5, -0.25, 2.0, 7.0, -7.0, 0.0]).to(dtype)
        w[2] *= 1e-3                                # small row: subnormal e4m3 codes
    fw = ops.Fp8Weight(w.to(DEV))
    q_ref, s_ref = O.quantize_weight_fp8(w)
    assert torch.equal(fw.scale.cpu(), s_ref)
    assert torch.equal(fw.q.cpu(), q_ref)
    # the dequantized weight is the oracle's, rounded once to the dtype
    assert torch.equal(fw.dequantize().cpu(), O.dequantize_weight_fp8(q_ref, s_ref, K).to(dtype))


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("case", [
    # M, N, K, act, norm, bias, residual
    (1, 4096, 1024, "none", True, False, False),     # qkv projection (norm fused)
    (32, 4096, 1024, "none", True, False, False),
    (17, 1024, 2048, "none", False, False, True),    # o projection + residual
    (32, 3072, 1024, "swiglu", True, False, False),  # gate/up
    (7, 1024, 3072, "none", False, True, True),      # down + bias + residual
    (16, 200, 128, "gelu", False, True, False),      # ragged N
    (5, 8, 64, "silu", False, False, False),         # tiny (weight part < 1 KB)
    (3, 24, 64, "swiglu", False, False, False),      # tiny SwiGLU (8-row slices)
    (4, 40, 128, "swiglu", False, True, False),      # SwiGLU, up rows mid-group
    (32, 151936, 1024, "none", True, False, False),  # LM head (persistent form)
    (5, 20000, 512, "silu", False, True, True),      # persistent, 16-token tile
    (32, 30016, 1024, "none", True, False, True),    # persistent, partial last group
    (9, 19003, 256, "gelu", False, True, False),     # persistent, N % 8 != 0
    (3, 40000, 2048, "none", False, False, False),   # too wide a K: slice plan
])
def test_linear_fp8(dtype, case):
    M, N, K, act, norm, bias, residual = case
    g = gen(43)
    x = rnd(M, K, g=g, dtype=dtype)
    rows = 2 * N if act == "swiglu" else N
    w = rnd(rows, K, g=g, std=0.02, dtype=dtype)
    b = rnd(rows, g=g, std=0.1, dtype=dtype) if bias else None
    r = rnd(M, N, g=g, dtype=dtype) if residual else None
    gamma = rnd(K, g=g, mean=1.0, std=0.1, dtype=dtype)
    wd = w.to(DEV)
    if norm:
        wd = ops.fold_rmsnorm_weight(wd, gamma.to(DEV))
    fw = ops.Fp8Weight(wd, act)
    y = ops.linear_fp8(x.to(DEV), fw, None if b is None else b.to(DEV),
                       None if r is None else r.to(DEV), 1e-6 if norm else None)
    w_ref = O.dequantize_weight_fp8(fw.q, fw.scale, K)
    h = O.rmsnorm(x, torch.ones(K), 1e-6) if norm else x
    check(y, O.linear(h, w_ref, b, act, r))


def test_linear_fp8_many_tokens_uses_dequantized_gemm():
    g = gen(47)
    x = rnd(100, 1024, g=g, dtype=torch.bfloat16)
    w = rnd(512, 1024, g=g, std=0.02, dtype=torch.bfloat16)
    fw = ops.Fp8Weight(w.to(DEV))
    y = ops.linear_fp8(x.to(DEV), fw)
    check(y, O.linear(x, O.dequantize_weight_fp8(fw.q, fw.scale, 1024)))


def test_fp8_halves_weight_bytes_and_tracks_bf16():
    """The fp8 product stays within the quantization error of the bf16 one."""
    g = gen(53)
    x = rnd(32, 1024, g=g, dtype=torch.bfloat16).to(DEV)
    w = rnd(4096, 1024, g=g, std=0.02, dtype=torch.bfloat16).to(DEV)
    fw = ops.Fp8Weight(w)
    assert fw.q.numel() * 2 == w.numel() * w.element_size()   # 4096 rows: whole groups
    y8 = ops.linear_fp8(x, fw).float()
    y16 = ops.linear(x, w).float()
    rel = (y8 - y16).norm() / y16.norm()
    assert rel.item() < 0.05, rel.item()
