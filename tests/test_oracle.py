"""Pins the CPU oracle (oracle/ops.py) against the reference's own known
answers and golden vectors (tests/golden/golden_ref.pt, generated from the
reference's Python by tests/golden/make_golden.py)."""
from pathlib import Path

import torch
import torch.nn.functional as F

from oracle import ops as O

G = torch.load(Path(__file__).resolve().parent / "golden" / "golden_ref.pt")


def test_rope_tables_match_reference_compute_rope_params():
    cos, sin = O.compute_rope_params(128, 1e6, 64)
    assert torch.equal(cos, G["rope_cos"]) and torch.equal(sin, G["rope_sin"])


def test_rmsnorm_matches_nn_rmsnorm_known_answer():
    # tests/rmsnorm_test.py: nn.RMSNorm(512, eps=1e-6) is the ground truth
    y = O.rmsnorm(G["norm_x"], G["norm_w"], 1e-6)
    torch.testing.assert_close(y, G["rmsnorm_y"], atol=1e-5, rtol=1e-5)


def test_layernorm_matches_nn_layernorm_known_answer():
    # tests/layernorm_test.py: nn.LayerNorm with bias zeroed is the ground truth
    y = O.layernorm(G["norm_x"], G["norm_w"], None, 1e-6)
    torch.testing.assert_close(y, G["layernorm_y"], atol=1e-5, rtol=1e-5)


def test_rope_is_rotate_half_form():
    x = torch.randn(1, 2, 5, 8)
    cos, sin = O.compute_rope_params(8, 1e4, 5, dtype=torch.float32)
    y = O.rope(x, cos, sin)
    # position 0 is the identity
    torch.testing.assert_close(y[:, :, 0], x[:, :, 0])
    # rotation preserves the norm of each (i, i + D/2) pair
    n0 = x[..., :4] ** 2 + x[..., 4:] ** 2
    n1 = y[..., :4] ** 2 + y[..., 4:] ** 2
    torch.testing.assert_close(n0, n1, atol=1e-5, rtol=1e-5)


def test_attention_oracle_matches_sdpa():
    g = torch.Generator().manual_seed(0)
    q = torch.randn(2, 7, 4, 16, generator=g)
    k = torch.randn(2, 7, 2, 16, generator=g)
    v = torch.randn(2, 7, 2, 16, generator=g)
    ref = F.scaled_dot_product_attention(
        q.transpose(1, 2), k.repeat_interleave(2, 2).transpose(1, 2),
        v.repeat_interleave(2, 2).transpose(1, 2), is_causal=True).transpose(1, 2)
    torch.testing.assert_close(O.attention(q, k, v, causal=True), ref, atol=1e-5, rtol=1e-5)


def test_attention_window_and_bottom_right_alignment():
    g = torch.Generator().manual_seed(1)
    q = torch.randn(1, 2, 1, 8, generator=g)
    k = torch.randn(1, 6, 1, 8, generator=g)
    v = torch.randn(1, 6, 1, 8, generator=g)
    # query rows sit at absolute positions 4 and 5; window 2 => keys [p-1, p]
    y = O.attention(q, k, v, causal=True, window_left=1)
    for i, p in enumerate((4, 5)):
        s = (q[0, i, 0] @ k[0, p - 1:p + 1, 0].T) / 8 ** 0.5
        ref = torch.softmax(s, -1) @ v[0, p - 1:p + 1, 0]
        torch.testing.assert_close(y[0, i, 0], ref, atol=1e-5, rtol=1e-5)


def test_linear_activations():
    g = torch.Generator().manual_seed(2)
    x, w = torch.randn(3, 8, generator=g), torch.randn(4, 8, generator=g)
    torch.testing.assert_close(O.linear(x, w, kind="silu"), F.silu(x @ w.T))
    torch.testing.assert_close(O.linear(x, w, kind="gelu"),
                               0.5 * (x @ w.T) * (1 + torch.tanh(0.7978845608028654 * (
                                   (x @ w.T) + 0.044715 * (x @ w.T) ** 3))), atol=1e-6, rtol=1e-6)
    w2 = torch.randn(8, 8, generator=g)
    torch.testing.assert_close(O.linear(x, w2, kind="swiglu"),
                               F.silu(x @ w2[:4].T) * (x @ w2[4:].T))


def test_hgemv_known_answer_recipe():
    # csrc/blas/hgemv/hgemv_bench.cpp:69-73 fills A[i] = i + 1, x[i] = i + 1
    M, K = 4, 8
    A = torch.arange(1, M * K + 1, dtype=torch.float32).view(M, K)
    x = torch.arange(1, K + 1, dtype=torch.float32)
    exp = torch.tensor([sum((r * K + j + 1) * (j + 1) for j in range(K)) for r in range(M)],
                       dtype=torch.float32)
    torch.testing.assert_close(O.hgemv(A, x), exp)


def test_kvcache_golden_matches_reference_index_path():
    k = torch.cat([G["kv_k0"], G["kv_k1"]], dim=2)
    v = torch.cat([G["kv_v0"], G["kv_v1"]], dim=2)
    torch.testing.assert_close(G["kv_k"], k)
    torch.testing.assert_close(G["kv_v"], v)


def test_gqa_golden_is_consistent_with_oracle_composition():
    sd = {k[len("gqa_sd."):]: v for k, v in G.items() if k.startswith("gqa_sd.")}
    x = G["gqa_x"]
    B, S, _ = x.shape
    q = (x @ sd["Wq.weight"].T).view(B, S, 4, 64)
    k = (x @ sd["Wk.weight"].T).view(B, S, 2, 64)
    v = (x @ sd["Wv.weight"].T).view(B, S, 2, 64)
    pos = torch.arange(S)[None, :, None]
    q = O.qk_norm_rope(q, sd["q_norm.weight"], 1e-6, G["gqa_cos"], G["gqa_sin"], pos)
    k = O.qk_norm_rope(k, sd["k_norm.weight"], 1e-6, G["gqa_cos"], G["gqa_sin"], pos)
    o = O.attention(q, k, v, causal=True).reshape(B, S, 256)
    y = o @ sd["out_projection.weight"].T
    torch.testing.assert_close(y, G["gqa_y"], atol=2e-3, rtol=2e-3)


# ---- fp8 weight format (oracle restatement) --------------------------------
def test_fp8_k_order_is_a_permutation_of_each_block():
    order = O.fp8_k_order(192)
    assert sorted(order.tolist()) == list(range(192))
    # byte 16c + 4s + j holds k = 16s + {2c, 2c+1, 2c+8, 2c+9}[j]
    assert order[:8].tolist() == [0, 1, 8, 9, 16, 17, 24, 25]
    assert order[16:20].tolist() == [2, 3, 10, 11]
    assert order[64:68].tolist() == [64, 65, 72, 73]


def test_fp8_rounding_known_answers():
    # e4m3: 3 mantissa bits, max 448; ties round to even
    w = torch.zeros(1, 64)
    w[0, :8] = torch.tensor([448.0, 34.0, 38.0, -0.0625, 0.0, 1.0, -1.5, 100.0])
    q, s = O.quantize_weight_fp8(w)
    assert s.item() == 1.0
    deq = O.dequantize_weight_fp8(q, s, 64)[0, :8]
    assert deq.tolist() == [448.0, 32.0, 40.0, -0.0625, 0.0, 1.0, -1.5, 96.0]
    # raw codes in the stored order (k = 0, 1 sit at bytes 0, 1)
    assert q[0].item() == 0x7E and q[1].item() == 0x60
    # one row pads to a 32-row group: 32 x 64 bytes, rows 1..31 zero
    assert q.numel() == 32 * 64 and int(q[64:].sum()) == 0


def test_fp8_round_trip_error_bound():
    g = torch.Generator().manual_seed(5)
    w = torch.randn(64, 1024, generator=g) * 0.02
    w[3].zero_()
    q, s = O.quantize_weight_fp8(w)
    assert q.dtype == torch.uint8 and q.numel() == 64 * 1024
    back = O.dequantize_weight_fp8(q, s, 1024)
    assert torch.equal(back[3], torch.zeros(1024))
    # relative spacing of e4m3 normals is 2^-3: error <= half an ulp of the
    # value, or half the subnormal step 2^-10 * scale near zero
    err = (back - w).abs()
    bound = torch.maximum(w.abs() * 2.0 ** -4, s[:, None] * 2.0 ** -10)
    assert (err <= bound * 1.0001).all()


def test_fp8_grouped_storage_round_trip_ragged_rows():
    # 37 rows: two 32-row groups, the second padded with 27 zero rows
    g = torch.Generator().manual_seed(6)
    w = torch.randn(37, 128, generator=g)
    q, s = O.quantize_weight_fp8(w)
    assert q.numel() == 64 * 128
    # group 1, k-block 0 holds rows 32..63; rows 37..63 are zero
    blk = q.view(2, 2, 32, 64)
    assert int(blk[1, :, 5:].abs().sum()) == 0
    back = O.dequantize_weight_fp8(q, s, 128)
    assert back.shape == (37, 128)
    assert ((back - w).abs() <= torch.maximum(w.abs() * 2.0 ** -4, s[:, None] * 2.0 ** -10)
            * 1.0001).all()
